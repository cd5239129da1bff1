"""Decode attention + KV append throughput on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config5|config1|config2|config3|config4]

Default workload (`config5`, the box-scale request partition): 512 independent sequences,
cached contexts log-uniform in [128, 8192] (seed 4), 32q/8kv x 128, bf16 paged cache with
block size 16 (the vLLM Triton-backend layout), one query token per sequence with in-kernel
q/k normalisation and K/V append.  Sequences are split over the N GPUs by a greedy
token-balanced assignment; each GPU owns its block pools; nothing crosses NVLink on the hot
path and NCCL only gathers the timings.  A step is one decode token for every sequence
through the 36 attention layers of a Dory-shaped step (8 input + 20 shared + 8 output), each
layer reading its own cache pool (distinct pools, cycled when HBM cannot hold 36; every pool
is far larger than L2, so nothing is reused from L2 between layers).

Our arm: the 36 layer calls are captured in one CUDA graph; K replays are timed with CUDA
events between barriers (max over ranks).  `e2e` times the same step through the public
API with host buffers: every layer's q/k/v/gate are copied from pinned host memory and its
output back, overlapped with the kernels on a second stream.  The reference arm
(`--impl reference`) times the reference semantics on the host CPU (PyTorch eager FP32,
all cores) on a bounded sample of the same workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dory-vllm-experiments_b200"))

import torch  # noqa: E402

import workloads as W  # noqa: E402

NH, NKV, HD, BLOCK = W.NH, W.NKV, W.HD, W.BLOCK
KV_ROW_BYTES = NKV * HD * 2 * 2           # K and V of one position, all KV heads: 4096 B
TOKEN_IO_BYTES = ((NH + NKV) * HD + NKV * HD + NH * HD + NH * HD) * 4  # qk, v, gate, out
METRIC = ("decode-attn+KV-append µs/layer-step, HBM GB/s vs peak; seqs/s at 1/2/4/8 GPU")
DORY_LAYERS = 36
DECODE_ORDER_2_LOOPS = list(range(8)) + list(range(8, 28)) * 2 + list(range(28, 36))


# ---------------------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------------------

def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return world, rank, local


def init_dist(world: int, local: int):
    if world == 1:
        return None
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    return dist


def barrier(dist, dev):
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)


def max_over_ranks(dist, value: float, dev) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(dist, value: float, dev) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------

REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """nvidia-smi samples of this GPU's SM clock and throttle reasons (read-only)."""

    def __init__(self, dev: torch.device, period_ms: int = 50):
        props = torch.cuda.get_device_properties(dev)
        ident = f"GPU-{props.uuid}" if getattr(props, "uuid", None) else str(dev.index or 0)
        fields = ["clocks.sm", "clocks.max.sm"] + [f"clocks_event_reasons.{r}" for r in REASONS]
        self.cmd = ["nvidia-smi", "-i", ident, f"--query-gpu={','.join(fields)}",
                    "--format=csv,noheader,nounits", "-lms", str(period_ms)]
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, smax, seen = [], [], set()
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 2 + len(REASONS):
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(REASONS, parts[2:]):
                if val.lower().startswith("active"):
                    seen.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax),
                "reasons": sorted(seen), "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# workloads on the device
# ---------------------------------------------------------------------------------------

def tuned_splits(workload: str, world: int):
    """(splits, min_blocks_per_split) measured fastest on B200 for each workload; config 5
    uses 4 splits once its 512 sequences are partitioned over 2+ GPUs (fewer, longer
    sequences per GPU: finer splits even out the last wave)."""
    if workload == "config5":
        return (2, 64) if world == 1 else (4, 64)
    return {"config1": (16, 1), "config2": (16, 1), "config3": (2, 32),
            "config4": (32, 1)}.get(workload, (2, 64))


def workload_spec(name: str):
    """(cached context lengths, tokens per sequence, shared, layer order, pool factor, notes)."""
    if name == "config5":
        return W.config5_lens(), 1, False, list(range(DORY_LAYERS)), 1.0, \
            "512 seqs, ctx log-uniform [128, 8192], seed 4"
    if name == "config3":
        return W.config3_lens(), 1, False, list(range(DORY_LAYERS)), 1.2, \
            "64 seqs, ctx uniform [128, 1152], seed 2, pool 1.2x tokens"
    if name == "config4":
        return [7936], 1, False, DECODE_ORDER_2_LOOPS, 1.0, \
            "1 seq, ctx 7936, 2 loops: 56 applications over 36 caches, seed 3"
    if name == "config1":
        return [640], 1, False, DECODE_ORDER_2_LOOPS, 1.0, \
            "1 seq, ctx 640, 2 loops: 56 applications over 36 caches, seed 0"
    if name == "config2":
        return [2560 + 150], 4, True, list(range(20)), 1.0, \
            "wavefront: 4 tokens at positions 2710..2713 (prompt 2560 + 150 generated), " \
            "20 shared layers, seed 1"
    raise SystemExit(f"unknown workload {name}")


class DeviceWorkload:
    """Per-rank device tensors: block pools, tables, per-layer inputs and outputs."""

    def __init__(self, lens, tokens_per_seq, shared, layers, pool_factor, dev, seed,
                 mem_fraction=0.5):
        self.dev = dev
        self.lens = lens
        self.shared = shared
        self.layers = layers
        self.num_layers = max(layers) + 1
        g = W.generator(seed)
        if shared:
            assert len(lens) == 1
            p = lens[0]
            self.seq_lens_list = [p + t + 1 for t in range(tokens_per_seq)]
            need = [-(-(p + tokens_per_seq) // BLOCK)]
            self.tokens = tokens_per_seq
        else:
            self.seq_lens_list = [n + 1 for n in lens]
            need = [-(-(n + 1) // BLOCK) for n in lens]
            self.tokens = len(lens)
        blocks = max(int(math.ceil(pool_factor * sum(need))), sum(need))
        perm = torch.randperm(blocks, generator=g).to(torch.int32)
        width = max(need)
        tables = torch.zeros(len(need), width, dtype=torch.int32)
        at = 0
        for i, k in enumerate(need):
            tables[i, :k] = perm[at:at + k]
            at += k
        self.tables = tables.to(dev)
        T = self.tokens
        rows = [0] * T if shared else list(range(T))
        self.table_offsets = torch.tensor([r * width for r in rows], dtype=torch.int64,
                                          device=dev)
        self.cache_offsets = torch.zeros(T, dtype=torch.int64, device=dev)
        self.seq_lens = torch.tensor(self.seq_lens_list, dtype=torch.int32, device=dev)
        # append slot of every token (its table entry at seq_len - 1, as vLLM's slot_mapping)
        self.slots = torch.tensor([int(tables[rows[t], (n - 1) // BLOCK]) * BLOCK + (n - 1) % BLOCK
                                   for t, n in enumerate(self.seq_lens_list)],
                                  dtype=torch.int64, device=dev)
        self.separate = False  # --path separate: q/k normalisation kernel, then __call__
        self.pool_blocks = blocks
        pool_bytes = blocks * BLOCK * KV_ROW_BYTES
        free, _ = torch.cuda.mem_get_info(dev)
        self.num_pools = max(1, min(self.num_layers, int(mem_fraction * free // pool_bytes)))
        gd = torch.Generator(device=dev).manual_seed(seed)
        self.raws, self.keys, self.values = [], [], []
        for _ in range(self.num_pools):
            raw, key, value = W.cache_views(blocks, BLOCK, NKV, HD, "triton", dev)
            raw.normal_(generator=gd)
            self.raws.append(raw)
            self.keys.append(key)
            self.values.append(value)
        L = self.num_layers
        self.qk = torch.randn(L, T, (NH + NKV) * HD, device=dev, generator=gd)
        self.v = torch.randn(L, T, NKV * HD, device=dev, generator=gd)
        self.gate = torch.sigmoid(torch.randn(L, T, NH * HD, device=dev, generator=gd))
        self.sqk = (torch.rand(NH * HD, device=dev, generator=gd) + 0.5).to(torch.bfloat16)
        self.out = torch.zeros(L, T, 8, NH * HD // 8, device=dev)
        self.q_out = torch.empty(T, NH * HD, dtype=torch.bfloat16, device=dev)
        self.sumsq = None  # --sumsq: [layers, T] FP32 sum of squared outputs per token

    def pool(self, layer: int):
        return self.keys[layer % self.num_pools], self.values[layer % self.num_pools]

    def algorithmic_bytes_per_application(self) -> int:
        """Unique attended positions x 4096 B (new rows written, the rest read) + per-token
        q/k/v/gate/out bytes + sqk + block-table entries + seq_lens."""
        if self.shared:
            unique = max(self.seq_lens_list)
            table = -(-unique // BLOCK) * 4
        else:
            unique = sum(self.seq_lens_list)
            table = sum(-(-n // BLOCK) for n in self.seq_lens_list) * 4
        return (unique * KV_ROW_BYTES + self.tokens * TOKEN_IO_BYTES + NH * HD * 2 + table
                + 4 * self.tokens)


def make_attention(wl: DeviceWorkload, args):
    from dory_decode_attention import DecodeAttention
    return DecodeAttention(NH, NKV, HD, wl.dev, splits=args.splits,
                           max_tokens=max(wl.tokens, 1),
                           min_blocks_per_split=args.min_blocks_per_split,
                           overlap_launch=getattr(args, "overlap_launch", False))


def layer_call(attn, wl: DeviceWorkload, app: int, layer: int, qk, v, gate, out):
    from dory_decode_attention import EPS
    key, value = wl.pool(layer)
    if wl.separate:
        # The reference's separate path (bench_decode_attention.py:144-152): the q/k
        # normalisation kernel writes the cache and the bf16 query, then __call__ attends.
        from dory_attention import qk_norm_cache
        qk_norm_cache(qk[0], v[0], wl.sqk, W.SQK_FACTOR, EPS, wl.q_out[0], NH, HD,
                      key_cache=key, value_cache=value, slot_mapping=wl.slots[0:1])
        attn(wl.q_out[0], key, value, wl.tables[0], wl.seq_lens[0:1], 0, HD ** -0.5, gate[0],
             out[0], out_sumsq=None if wl.sumsq is None else wl.sumsq[layer])
        return
    attn.multi_from_raw(qk, v, wl.sqk, W.SQK_FACTOR, EPS, wl.cache_offsets, key, value,
                        wl.tables, wl.table_offsets, wl.seq_lens, 0, HD ** -0.5, gate, out,
                        shared_cache=wl.shared,
                        out_sumsq=None if wl.sumsq is None else wl.sumsq[layer])


def run_step(attn, wl: DeviceWorkload):
    for app, layer in enumerate(wl.layers):
        layer_call(attn, wl, app, layer, wl.qk[layer], wl.v[layer], wl.gate[layer],
                   wl.out[layer])


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------

def subset(lens, k: int):
    """k sequences evenly spaced by length (keeps the workload's length distribution)."""
    if k <= 0 or k >= len(lens):
        return lens
    order = sorted(range(len(lens)), key=lambda i: lens[i])
    return [lens[order[int((i + 0.5) * len(order) / k)]] for i in range(k)]


def bench_profile(args):
    """Eager steps of the layer sequence for profilers (no graph, no e2e, no CPU leg)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lens_all, tps, shared, layers, pool_factor, notes = workload_spec(args.workload)
    lens_all = subset(lens_all, args.max_seqs)
    wl = DeviceWorkload(lens_all, tps, shared, layers, pool_factor, dev, 11,
                        mem_fraction=args.mem_fraction)
    attn = make_attention(wl, args)
    for _ in range(args.profile_steps):
        run_step(attn, wl)
    torch.cuda.synchronize(dev)
    attn.check_errors()
    print(json.dumps({"profile_steps": args.profile_steps, "launches": args.profile_steps *
                      len(layers), "sequences": len(lens_all), "pools": wl.num_pools,
                      "algorithmic_bytes_per_launch": wl.algorithmic_bytes_per_application()}),
          flush=True)


def bench_ours(args, world, rank, local):
    dist = init_dist(world, local)
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    lens_all, tps, shared, layers, pool_factor, notes = workload_spec(args.workload)
    if shared or len(lens_all) == 1:
        mine = list(range(len(lens_all)))  # a single sequence does not shard: replicas
        scaling = "replicas"
    else:
        mine = W.partition(lens_all, world)[rank]
        scaling = "strong"
    lens = [lens_all[i] for i in mine]
    seed = {"config5": 4, "config3": 2, "config4": 3, "config1": 0, "config2": 1}[args.workload]
    wl = DeviceWorkload(lens, tps, shared, layers, pool_factor, dev, seed + 1000 * rank)
    if args.sumsq:
        wl.sumsq = torch.zeros(wl.num_layers, wl.tokens, device=dev)
    if args.path == "separate":
        if wl.tokens != 1:
            raise SystemExit("--path separate takes single-sequence workloads (config1, config4)")
        wl.separate = True
    attn = make_attention(wl, args)
    apps = len(layers)

    # capture the step in a CUDA graph (the reference's time_graph idiom)
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        run_step(attn, wl)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    attn.check_errors()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run_step(attn, wl)
    for _ in range(args.warmup):
        graph.replay()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist, dev)
    with ClockSampler(dev) as clocks:
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        torch.cuda.synchronize(dev)
    barrier(dist, dev)
    ms_local = start.elapsed_time(end)
    ms = max_over_ranks(dist, ms_local, dev)
    attn.check_errors()

    total_seqs = len(lens_all) * (tps if shared else 1)
    bytes_rank = wl.algorithmic_bytes_per_application() * apps
    bytes_all = sum_over_ranks(dist, float(bytes_rank), dev)
    ms_per_step = ms / args.steps
    seqs_per_s = (total_seqs * (world if scaling == "replicas" else 1)) / (ms_per_step / 1e3)
    us_per_layer = ms_per_step * 1e3 / apps
    hbm_gbs = bytes_all / (ms_per_step / 1e3) / 1e9

    # roofline of the one kernel: this rank's bytes per launch / its average launch time
    peaks = load_peaks()
    per_launch_bytes = wl.algorithmic_bytes_per_application()
    launch_us = ms_local * 1e3 / (args.steps * apps)
    achieved = per_launch_bytes / (launch_us * 1e-6) / 1e9
    ratio = read_traffic_ratio(args.workload)
    traffic = int(ratio * per_launch_bytes) if ratio else None
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks[0],
                "unit": "GB/s", "frac": round(achieved / peaks[0], 4),
                "traffic": traffic, "peak_source": peaks[1],
                "algorithmic_bytes_per_launch": per_launch_bytes,
                "launch_us": round(launch_us, 3)}

    e2e = bench_e2e(attn, wl, args, dist, dev, total_seqs, world, scaling)
    del graph
    torch.cuda.synchronize(dev)

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(args.workload, lens_all, args.cpu_seconds)

    line = {
        "metric": METRIC, "value": round(seqs_per_s, 2), "unit": "seqs/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V, q/k/v, gate; random block-table permutations)",
        "config": {"workload": f"{args.workload}: {notes}", "global_batch": total_seqs,
                   "layers_per_step": apps, "num_heads": NH, "num_kv_heads": NKV,
                   "head_dim": HD, "block_size": BLOCK, "cache_layout": "vLLM Triton "
                   "[blocks, kv_heads, 16, 2*head_dim] viewed via transpose(1,2).split",
                   "parallelism": f"request partition over {world} GPU(s), no collectives",
                   "distinct_pools_per_rank": wl.num_pools,
                   "l2": "inputs larger than L2 (each pool > 126 MB; pools cycled per layer)",
                   "splits": args.splits, "min_blocks_per_split": args.min_blocks_per_split,
                   "overlap_launch": args.overlap_launch, "path": args.path,
                   "out_sumsq": bool(args.sumsq)},
        "us_per_layer_step": round(us_per_layer, 3),
        "hbm_gbs": round(hbm_gbs, 1),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps * apps * (2 if wl.separate else 1),
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def bench_e2e(attn, wl: DeviceWorkload, args, dist, dev, total_seqs, world, scaling):
    """The same step through the public API with host buffers: per layer, H2D of its q/k,
    v and gate from pinned memory and D2H of its output into pinned memory, overlapped with
    the kernels (copy stream + events)."""
    L = wl.num_layers
    host_in = [(wl.qk[l].cpu().pin_memory(), wl.v[l].cpu().pin_memory(),
                wl.gate[l].cpu().pin_memory()) for l in range(L)]
    host_out = [torch.empty_like(wl.out[l], device="cpu").pin_memory() for l in range(L)]
    apps = len(wl.layers)
    nbuf = 3  # device staging slots, rotated over the layer applications
    stage = [(torch.empty_like(wl.qk[0]), torch.empty_like(wl.v[0]),
              torch.empty_like(wl.gate[0]), torch.empty_like(wl.out[0])) for _ in range(nbuf)]
    compute = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    h2d_bytes = sum(t.numel() * t.element_size() for t in host_in[0]) * apps
    d2h_bytes = host_out[0].numel() * 4 * apps

    def step():
        loaded = [torch.cuda.Event() for _ in range(apps)]
        done = [torch.cuda.Event() for _ in range(apps)]
        freed = [torch.cuda.Event() for _ in range(apps)]
        h2d.wait_stream(compute)
        for a, layer in enumerate(wl.layers):
            buf = stage[a % nbuf]
            with torch.cuda.stream(h2d):
                if a >= nbuf:
                    h2d.wait_event(done[a - nbuf])  # inputs of this slot consumed
                for dst, src in zip(buf[:3], host_in[layer]):
                    dst.copy_(src, non_blocking=True)
                loaded[a].record(h2d)
            compute.wait_event(loaded[a])
            if a >= nbuf:
                compute.wait_event(freed[a - nbuf])  # output of this slot read back
            layer_call(attn, wl, a, layer, buf[0], buf[1], buf[2], buf[3])
            done[a].record(compute)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done[a])
                host_out[layer].copy_(buf[3], non_blocking=True)
                freed[a].record(d2h)
        compute.wait_stream(d2h)

    for _ in range(max(1, args.warmup)):
        step()
    steps = max(1, min(args.steps, args.e2e_steps))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist, dev)
    start.record(compute)
    for _ in range(steps):
        step()
    end.record(compute)
    torch.cuda.synchronize(dev)
    barrier(dist, dev)
    ms = max_over_ranks(dist, start.elapsed_time(end), dev) / steps
    value = (total_seqs * (world if scaling == "replicas" else 1)) / (ms / 1e3)
    return {"value": round(value, 2), "unit": "seqs/s", "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes, "steps": steps, "ms_per_step": round(ms, 4),
            "path": "DecodeAttention.multi_from_raw per layer, pinned host buffers, "
                    "copies overlapped on a second stream"}


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return 6650.0, "fallback (6.65 TB/s earlier pool measurement)"


def read_traffic_ratio(workload: str):
    """DRAM traffic / algorithmic bytes of one launch, from the committed ncu summary of this
    workload (profiles/decode_kernel_<workload>.txt), or None."""
    path = ROOT / "profiles" / f"decode_kernel_{workload}.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_ratio:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------------------
# CPU baseline / reference arm: the reference semantics in PyTorch eager FP32 on the host
# ---------------------------------------------------------------------------------------

def cpu_sample(workload: str, lens_all, budget_s: float):
    """A bounded sample of the workload for the CPU: a spread of sequences of one layer."""
    lens_sorted = sorted(range(len(lens_all)), key=lambda i: lens_all[i])
    if workload == "config2":
        return [lens_all[0]], True
    if len(lens_all) == 1:
        return [lens_all[0]], False
    # evenly spaced by length so the sample's mean matches the workload's
    k = max(2, min(len(lens_all), 64, int(budget_s * 4)))
    pick = [lens_sorted[int((i + 0.5) * len(lens_sorted) / k)] for i in range(k)]
    return [lens_all[i] for i in pick], False


class CpuSample:
    """A bounded sample of the workload on the host CPU: the reference semantics in PyTorch
    eager FP32 (oracle/dory_oracle.py) over a spread of the workload's sequences, one layer."""

    def __init__(self, workload: str, lens_all, budget_s: float):
        sys.path.insert(0, str(ROOT / "oracle"))
        import dory_oracle as O
        self.O = O
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.lens, shared = cpu_sample(workload, lens_all, budget_s)
        if shared:
            self.case = W.wavefront(seed=1, prompt=self.lens[0], generated=0, tokens=4)
        else:
            self.case = W.batched(seed=4, lens=self.lens)
        self.shared = shared
        self.key = self.case.key.to(torch.bfloat16)
        self.value = self.case.value.to(torch.bfloat16)
        _, _, _, layers, _, _ = workload_spec(workload)
        self.layers = len(layers)

    def once(self) -> float:
        """Seconds for one pass of the sample (one layer, the caches restored first)."""
        c, O = self.case, self.O
        k, v = self.key.clone(), self.value.clone()
        width = c.tables.shape[1]
        t0 = time.perf_counter()
        O.multi_from_raw(c.qk, c.v, c.sqk, c.sqk_factor, O.EPS,
                         torch.zeros(c.tokens, dtype=torch.int64), k.view(-1), v.view(-1),
                         tuple(k.shape), k.stride(), c.tables.reshape(-1),
                         torch.tensor([r * width for r in c.table_rows]), c.seq_lens,
                         c.window, c.scale, c.gate, NH, NKV, shared_cache=c.shared)
        return time.perf_counter() - t0

    def seqs_per_s(self, seconds: float) -> float:
        seqs = 1 if self.shared else len(self.lens)
        return seqs / (seconds * self.layers)

    def describe(self, seconds: float, reps: int) -> str:
        return (f"{len(self.lens)} sequence(s) (ctx {min(self.lens)}..{max(self.lens)}, mean "
                f"{sum(self.lens) / len(self.lens):.0f}) x 1 layer, {seconds:.3f} s each, {reps} "
                f"repetition(s), scaled to {self.layers} layers; PyTorch eager FP32 restatement "
                "of the reference semantics (oracle/dory_oracle.py)")


def cpu_baseline(workload: str, lens_all, budget_s: float):
    """Times the CPU sample, repeating it until `budget_s` seconds have passed."""
    sample = CpuSample(workload, lens_all, budget_s)
    sample.once()  # warm-up
    total, reps = 0.0, 0
    while total < budget_s or reps == 0:
        total += sample.once()
        reps += 1
    dt = total / reps
    return {"value": round(sample.seqs_per_s(dt), 4), "unit": "seqs/s", "cores": sample.threads,
            "kind": "port", "sample": sample.describe(dt, reps)}


def bench_reference(args, world, rank, local):
    if rank != 0:
        return
    lens_all, tps, shared, layers, _, notes = workload_spec(args.workload)
    # each step is one pass of a bounded sample, sized so the whole run takes minutes
    budget = max(0.05, min(args.cpu_seconds, 120.0 / max(1, args.steps + args.warmup)))
    sample = CpuSample(args.workload, lens_all, budget)
    for _ in range(args.warmup):
        sample.once()
    times = [sample.once() for _ in range(args.steps)]
    dt = statistics.mean(times)
    value = sample.seqs_per_s(dt)
    cpu = {"value": round(value, 4), "unit": "seqs/s", "cores": sample.threads, "kind": "port",
           "sample": sample.describe(dt, len(times))}
    total_seqs = len(lens_all) * (tps if shared else 1)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "seqs/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_seqs / value * 1e3, 3) if value else None,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded), bounded CPU sample",
            "config": {"workload": f"{args.workload}: {notes}", "global_batch": total_seqs,
                       "layers_per_step": len(layers)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(value, 4), "unit": "seqs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "the reference's path is Triton GPU code; its CPU implementation is its "
                    "eager PyTorch semantics, restated in oracle/dory_oracle.py"}
    print(json.dumps(line), flush=True)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="config5")
    ap.add_argument("--splits", type=int, default=None,
                    help="split count (default: the tuned setting of the workload and GPU count)")
    ap.add_argument("--min-blocks-per-split", type=int, default=None)
    ap.add_argument("--overlap-launch", action="store_true",
                    help="launch each layer call as a programmatic dependent of the previous one")
    ap.add_argument("--path", choices=("fused", "separate"), default="fused",
                    help="separate: the q/k normalisation kernel then the non-raw call "
                         "(single-sequence workloads; the reference's two-kernel path)")
    ap.add_argument("--sumsq", action="store_true",
                    help="also produce each token's sum of squared outputs (out_sumsq)")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="run this many eager steps for a profiler and exit")
    ap.add_argument("--max-seqs", type=int, default=0,
                    help="profile mode: a length-spread subset of the workload's sequences")
    ap.add_argument("--mem-fraction", type=float, default=0.5,
                    help="profile mode: share of free HBM for the cache pools")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world, rank, local = dist_env()
    tuned = tuned_splits(args.workload, world)
    if args.splits is None:
        args.splits = tuned[0]
    if args.min_blocks_per_split is None:
        args.min_blocks_per_split = tuned[1]
    if args.gpus != world and world > 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    if args.profile_steps > 0:
        bench_profile(args)
    elif args.impl == "reference":
        bench_reference(args, world, rank, local)
    else:
        bench_ours(args, world, rank, local)
    return 0


if __name__ == "__main__":
    sys.exit(main())
