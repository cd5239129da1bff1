"""Decode attention + KV append throughput on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config5|config1|config2|config3|config4|
                                dory640|dory2048|dory8192]

Default workload (`config5`, the box-scale request partition): 512 independent sequences,
cached contexts log-uniform in [128, 8192] (seed 4), 32q/8kv x 128, bf16 paged cache with
block size 16 (the vLLM Triton-backend layout), one query token per sequence with in-kernel
q/k normalisation and K/V append.  Sequences are split over the N GPUs by a greedy
token-balanced assignment; each GPU owns its block pools; nothing crosses NVLink on the hot
path and NCCL only gathers the timings.  A step is one decode token for every sequence
through the 36 attention layers of a Dory-shaped step (8 input + 20 shared + 8 output), each
layer reading its own cache pool (distinct pools, cycled when HBM cannot hold 36; every pool
is far larger than L2, so nothing is reused from L2 between layers).

The dory640/2048/8192 workloads are the reference benchmark's own shape (16q/4kv x 256, one
sequence, the 56 applications of the two-loop decode order each on its own cache, window
1024 on 3 of 4 layers).

Our arm: the step's layer calls are captured in one CUDA graph; K replays are timed with
CUDA events between barriers (max over ranks).  `e2e` times the same step through the
public API with host buffers: every application's q/k/v/gate are copied from pinned host
memory and its output back every step, in chunks overlapped with the kernels on two copy
streams, the step replayed as one CUDA graph (and, as `eager`, issued from Python).  The
reference arm
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
from dataclasses import dataclass, field
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dory-vllm-experiments_b200"))

NCCL_LOG = None
if int(os.environ.get("WORLD_SIZE", "1")) > 1 and "NCCL_DEBUG" not in os.environ:
    # NCCL's communicator set-up lines (ranks, devices) go to a per-process file that
    # init_dist copies to stderr once the communicator exists, so that a multi-GPU run shows
    # how many ranks joined while stdout keeps the one JSON line.  (NCCL opens its debug
    # file for writing, which would truncate a shared stderr file.)  NCCL reads these once,
    # when the library is first loaded, hence before torch is imported.
    import tempfile
    NCCL_LOG = os.path.join(tempfile.gettempdir(), f"dory_bench_nccl_{os.getpid()}.log")
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
    os.environ["NCCL_DEBUG_FILE"] = NCCL_LOG

import torch  # noqa: E402

import workloads as W  # noqa: E402

NH, NKV, HD, BLOCK = W.NH, W.NKV, W.HD, W.BLOCK
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
    dist.barrier()  # the communicator exists (and has logged its set-up) after this
    if NCCL_LOG is not None and os.path.exists(NCCL_LOG):
        with open(NCCL_LOG) as f:
            sys.stderr.write(f.read())
        sys.stderr.flush()
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

WORKLOADS = ("config5", "config1", "config2", "config3", "config4",
             "dory640", "dory2048", "dory8192")


def tuned_splits(workload: str, world: int, kv_dtype: str = "bf16"):
    """(splits, min_blocks_per_split) measured fastest on B200 for each workload; config 5
    uses 4 splits once its 512 sequences are partitioned over 2+ GPUs, and 3 splits at 8+
    GPUs, where each GPU's sequences run longest-first (`longest_first`; measured on one
    GPU's share of each partition).  With an FP8 cache on one GPU, config 5 measured
    fastest with 2 splits of at least 192 blocks (426 us, against 432 at 128 and 449 at 64
    blocks)."""
    if workload == "config5" and world == 1 and kv_dtype == "fp8":
        return (2, 192)
    if workload == "config5":
        return (2, 64) if world == 1 else (4, 64) if world < 8 else (3, 64)
    return {"config1": (16, 1), "config2": (16, 1), "config3": (2, 32),
            "config4": (32, 1), "dory640": (16, 1), "dory2048": (32, 1),
            "dory8192": (32, 1)}.get(workload, (2, 64))


def longest_first(workload: str, world: int) -> bool:
    """Whether a GPU's share of the request partition is launched longest sequence first.
    With 64 config-5 sequences per GPU (8 GPUs) the longest ones' splits then start in the
    first wave and the short ones fill the tail: 85.1 us per layer with 3 splits against
    90.9 us for the best setting in request order (8 splits of at least 96 blocks), one GPU
    running rank 0's share.  With 128 or more sequences per GPU it measured slower (2 GPUs:
    340 against 324 us; 4 GPUs: 172 against 168 us; 1 GPU: 5%), so request order stays."""
    return workload == "config5" and world >= 8


def rank_sequences(workload: str, lens_all: list, world: int, rank: int) -> list:
    """This rank's sequence indices of the request partition, in launch order."""
    mine = W.partition(lens_all, world)[rank]
    if longest_first(workload, world):
        mine = sorted(mine, key=lambda i: (-lens_all[i], i))
    return mine


@dataclass
class Spec:
    """One bench workload.  `layers[a]` is the cache/input set application `a` uses (a
    layer id; applications that share an id read the same pool); `windows[id]` is that
    layer's sliding window (0 = full context)."""
    lens: list            # cached context length of each sequence (the prompt if shared)
    tokens_per_seq: int
    shared: bool
    layers: list
    pool_factor: float
    notes: str
    seed: int
    nh: int = NH
    nkv: int = NKV
    hd: int = HD
    windows: dict = field(default_factory=dict)

    def window(self, layer: int) -> int:
        return self.windows.get(layer, 0)


def dory_spec(context: int) -> Spec:
    """The reference benchmark's own shape (kernels/bench_decode_attention.py: 16q/4kv x 256,
    one token, 56 applications of the two-loop decode order, each application with its own
    shuffled cache of context // 16 + 1 blocks, sliding window 1024 on the layers with
    layer % 4 != 3 of the Dory model)."""
    apps = len(DECODE_ORDER_2_LOOPS)
    windows = {a: (1024 if layer % 4 != 3 else 0) for a, layer in enumerate(DECODE_ORDER_2_LOOPS)}
    full = sum(1 for w in windows.values() if w == 0)
    return Spec([context], 1, False, list(range(apps)), 1.0,
                f"reference benchmark shape: 16q/4kv x 256, 1 seq, ctx {context}, {apps} "
                f"decode-order applications each on its own cache, window 1024 on "
                f"{apps - full} of them, seed 5", 5 + context, nh=16, nkv=4, hd=256,
                windows=windows)


def workload_spec(name: str) -> Spec:
    if name == "config5":
        return Spec(W.config5_lens(), 1, False, list(range(DORY_LAYERS)), 1.0,
                    "512 seqs, ctx log-uniform [128, 8192], seed 4", 4)
    if name == "config3":
        return Spec(W.config3_lens(), 1, False, list(range(DORY_LAYERS)), 1.2,
                    "64 seqs, ctx uniform [128, 1152], seed 2, pool 1.2x tokens", 2)
    if name == "config4":
        return Spec([7936], 1, False, DECODE_ORDER_2_LOOPS, 1.0,
                    "1 seq, ctx 7936, 2 loops: 56 applications over 36 caches, seed 3", 3)
    if name == "config1":
        return Spec([640], 1, False, DECODE_ORDER_2_LOOPS, 1.0,
                    "1 seq, ctx 640, 2 loops: 56 applications over 36 caches, seed 0", 0)
    if name == "config2":
        return Spec([2560 + 150], 4, True, list(range(20)), 1.0,
                    "wavefront: 4 tokens at positions 2710..2713 (prompt 2560 + 150 "
                    "generated), 20 shared layers, seed 1", 1)
    if name.startswith("dory") and name[4:] in ("640", "2048", "8192"):
        return dory_spec(int(name[4:]))
    raise SystemExit(f"unknown workload {name} (one of {', '.join(WORKLOADS)})")


def algorithmic_bytes(seq_lens, shared: bool, window: int, nh: int, nkv: int, hd: int,
                      split_k: int = 0, residual_hidden: int = 0, kv_bytes: int = 2) -> int:
    """Bytes one launch must move: unique attended positions x the K/V row bytes (the new
    rows written, the rest read) + per-token q/k/v/gate reads and out writes (FP32) + sqk
    + the block-table entries of the attended range + seq_lens.  With a sliding window w a
    token attends [max(seq_len - w, 0), seq_len); a shared-cache group reads the union of
    its tokens' ranges once.  split_k: the q/k/v/gate epilogue's I/O replaces the q/k/v/gate
    reads; residual_hidden: the residual update's I/O is added (the sublayer chain);
    kv_bytes: bytes per cache element (2 bf16, 1 e4m3)."""
    kv_row = nkv * hd * 2 * kv_bytes
    token_io = ((nh + nkv) * hd + nkv * hd + 2 * nh * hd) * 4
    extra = 0
    if split_k:
        # q/k/v/gate GEMV partials in (2 * (Q + KV) rows per split), output out, the token's
        # position and bf16 cos/sin row; the bf16 gate scales once per launch
        token_io = (split_k * 2 * (nh + nkv) * hd + nh * hd) * 4 + 8 + hd * 2
        extra = nh * hd * 2
    if residual_hidden:
        # the output GEMV's split-K partials, the sublayer input (bf16), h as bf16 and as
        # nibble-major FP32, the output statistic written and read; alpha (bf16) once
        H = residual_hidden
        token_io += RESIDUAL_SPLIT_K * H * 4 + H * 2 + H * 2 + H * 4 + 8
        extra += H * 2

    def span(n):
        return (max(n - window, 0) if window > 0 else 0), n

    def table_entries(first, last):
        return (last - 1) // BLOCK - first // BLOCK + 1 if last > first else 0

    if shared:
        firsts, lasts = zip(*(span(n) for n in seq_lens))
        spans = [(min(firsts), max(lasts))]
    else:
        spans = [span(n) for n in seq_lens]
    unique = sum(b - a for a, b in spans)
    table = sum(table_entries(a, b) for a, b in spans) * 4
    return (unique * kv_row + len(seq_lens) * token_io + nh * hd * 2 + table + 4 * len(seq_lens)
            + extra)


# Each graph replay must touch more than this many bytes of distinct cache pools, so that
# no step finds its K/V left in the 126 MB L2 by the step before: small workloads capture
# several steps per graph, each over its own pools.
L2_BYTES = 126e6
MIN_REPLAY_BYTES = 3 * L2_BYTES


class DeviceWorkload:
    """Per-rank device tensors: block pools, tables, per-layer inputs and outputs.

    One graph replay runs `reps` steps; step r's layer l reads pool (r * layers + l) modulo
    the pool count, and `reps` is the smallest count whose distinct pools exceed
    MIN_REPLAY_BYTES (1 for every workload whose layers alone exceed it)."""

    def __init__(self, spec: Spec, lens, dev, seed, mem_fraction=0.5, kv_dtype: str = "bf16"):
        tokens_per_seq, shared, layers = spec.tokens_per_seq, spec.shared, spec.layers
        pool_factor = spec.pool_factor
        self.spec = spec
        self.nh, self.nkv, self.hd = NH_, NKV_, HD_ = spec.nh, spec.nkv, spec.hd
        self.kv8 = kv_dtype == "fp8"
        self.kv_bytes = 1 if self.kv8 else 2
        self.kv_row_bytes = NKV_ * HD_ * 2 * self.kv_bytes  # K and V of one position
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
        # fused: from_raw / multi_from_raw; separate: the q/k normalisation kernel, then
        # __call__; call: __call__ alone on a prepared bf16 query (prepare_call_path)
        self.path = "fused"
        self.q_call = None
        self.pool_blocks = blocks
        self.pool_bytes = pool_bytes = blocks * BLOCK * self.kv_row_bytes
        free, _ = torch.cuda.mem_get_info(dev)
        fit = max(1, int(mem_fraction * free // pool_bytes))
        self.reps = max(1, math.ceil(MIN_REPLAY_BYTES / (pool_bytes * self.num_layers)))
        if self.reps * self.num_layers > fit:
            self.reps = 1
        self.num_pools = max(1, min(self.num_layers * self.reps, fit))
        gd = torch.Generator(device=dev).manual_seed(seed)
        self.raws, self.keys, self.values = [], [], []
        for _ in range(self.num_pools):
            if self.kv8:
                # e4m3 bytes of N(0, 1) values (scales 1), drawn in slices to bound the
                # temporary FP32 buffer
                raw, key, value = W.cache_views(blocks, BLOCK, NKV_, HD_, "triton", dev,
                                                torch.uint8)
                for i in range(0, blocks, 4096):
                    part = raw[i:i + 4096]
                    part.copy_(W.e4m3_bytes(torch.randn(part.shape, device=dev, generator=gd),
                                            1.0))
            else:
                raw, key, value = W.cache_views(blocks, BLOCK, NKV_, HD_, "triton", dev)
                raw.normal_(generator=gd)
            self.raws.append(raw)
            self.keys.append(key)
            self.values.append(value)
        L = self.num_layers
        self.qk = torch.randn(L, T, (NH_ + NKV_) * HD_, device=dev, generator=gd)
        self.v = torch.randn(L, T, NKV_ * HD_, device=dev, generator=gd)
        self.gate = torch.sigmoid(torch.randn(L, T, NH_ * HD_, device=dev, generator=gd))
        self.sqk = (torch.rand(NH_ * HD_, device=dev, generator=gd) + 0.5).to(torch.bfloat16)
        self.out = torch.zeros(L, T, 8, NH_ * HD_ // 8, device=dev)
        self.q_out = torch.empty(T, NH_ * HD_, dtype=torch.bfloat16, device=dev)
        self.sumsq = None  # --sumsq: [layers, T] FP32 sum of squared outputs per token

    def pool(self, layer: int, rep: int = 0):
        i = (rep * self.num_layers + layer) % self.num_pools
        return self.keys[i], self.values[i]

    def window(self, layer: int) -> int:
        return self.spec.window(layer)

    def algorithmic_bytes_per_application(self, layer: int = 0) -> int:
        return algorithmic_bytes(self.seq_lens_list, self.shared, self.window(layer),
                                 self.nh, self.nkv, self.hd,
                                 QKVG_SPLIT_K if self.path in ("qkvg", "sublayer") else 0,
                                 self.hidden if self.path == "sublayer" else 0,
                                 self.kv_bytes)

    def algorithmic_bytes_per_step(self) -> int:
        return sum(self.algorithmic_bytes_per_application(layer) for layer in self.layers)


def make_attention(wl: DeviceWorkload, args):
    from dory_decode_attention import DecodeAttention
    return DecodeAttention(wl.nh, wl.nkv, wl.hd, wl.dev, splits=args.splits,
                           max_tokens=max(wl.tokens, 1),
                           min_blocks_per_split=args.min_blocks_per_split,
                           overlap_launch=getattr(args, "overlap_launch", False),
                           prefetch_chunks=getattr(args, "prefetch_chunks", 0),
                           consumer=getattr(args, "consumer", "mma"),
                           kv_cache_dtype="fp8" if wl.kv8 else "auto")


def prepare_call_path(wl: DeviceWorkload):
    """`--path call`: each layer's bf16 queries from its raw q/k (the q/k normalisation kernel,
    which also appends the layer's new k/v), made once before timing; every timed call then
    finds its K/V already in the cache, as the reference's non-raw `__call__` expects."""
    from dory_sublayer_steps import qk_norm_cache
    from dory_decode_attention import EPS
    wl.q_call = torch.empty(wl.num_layers, wl.tokens, wl.nh * wl.hd, dtype=torch.bfloat16,
                            device=wl.dev)
    for rep in range(wl.reps):
        for layer in range(wl.num_layers):
            key, value = wl.pool(layer, rep)
            qk_norm_cache(wl.qk[layer], wl.v[layer], wl.sqk, W.SQK_FACTOR, EPS,
                          wl.q_call[layer], wl.nh, wl.hd, key_cache=key, value_cache=value,
                          slot_mapping=wl.slots)
    wl.path = "call"


QKVG_SPLIT_K = 2  # the reference's q/k/v/gate GEMV configuration (dory_multi_token.py:41)
RESIDUAL_SPLIT_K = 4  # its attention output GEMV configuration (dory_multi_token.py:42)


def prepare_qkvg_path(wl: DeviceWorkload):
    """`--path qkvg`: each layer's input is the multi-token path's q/k/v/gate GEMV output,
    split-K partial sums FP32 [split_k, T, 2 * (Q + KV)], with the tokens' rotary positions
    (seq_len - 1), a cos/sin table and the gate scales; a layer is the epilogue kernel, then
    multi_from_raw (the reference's two launches, dory_multi_token.py:196-205)."""
    T, L = wl.tokens, wl.num_layers
    rows = 2 * (wl.nh + wl.nkv) * wl.hd
    gd = torch.Generator(device=wl.dev).manual_seed(77)
    wl.partials = torch.randn(L, QKVG_SPLIT_K, T, rows, device=wl.dev, generator=gd) * 0.5
    wl.positions = (wl.seq_lens.to(torch.int64) - 1).clamp(min=0)
    wl.cos_sin = torch.randn(int(wl.seq_lens.max()) + 1, wl.hd, device=wl.dev,
                             generator=gd).to(torch.bfloat16)
    wl.s_gate = (torch.rand(wl.nh * wl.hd, device=wl.dev, generator=gd) + 0.5).to(torch.bfloat16)
    wl.qkvg_bufs = (torch.empty(T, (wl.nh + wl.nkv) * wl.hd, device=wl.dev),
                    torch.empty(T, wl.nkv * wl.hd, device=wl.dev),
                    torch.empty(T, wl.nh * wl.hd, device=wl.dev))
    wl.path = "qkvg"


def prepare_sublayer_path(wl: DeviceWorkload):
    """`--path sublayer`: the non-GEMM steps of the multi-token attention sublayer
    (MultiTokenSublayers.attention, dory_multi_token.py:183-210): the q/k/v/gate epilogue,
    multi_from_raw with the output statistic, then the residual update after the output
    GEMV (`_residual_tokens_kernel`, :109-131) fed that statistic instead of the output.
    Each layer's inputs are both GEMVs' split-K partials (the GEMVs themselves, NVFP4, are
    not part of this build).  Hidden size 2560 (the Dory model) for 256-dim heads, else
    heads x head_dim."""
    prepare_qkvg_path(wl)
    T, L = wl.tokens, wl.num_layers
    wl.hidden = H = 2560 if wl.hd == 256 else wl.nh * wl.hd
    gd = torch.Generator(device=wl.dev).manual_seed(78)
    wl.o_partials = torch.randn(L, RESIDUAL_SPLIT_K, T, H, device=wl.dev, generator=gd)
    a = torch.randn(T, H, device=wl.dev, generator=gd)
    wl.h_in = (a / a.norm(dim=1, keepdim=True)).to(torch.bfloat16)
    wl.alpha = (torch.randn(H, device=wl.dev, generator=gd) * 0.02).to(torch.bfloat16)
    wl.h_out = torch.empty(T, H, dtype=torch.bfloat16, device=wl.dev)
    wl.h_out_nm = torch.empty(T, 8, H // 8, device=wl.dev)
    if wl.sumsq is None:
        wl.sumsq = torch.zeros(L, T, device=wl.dev)
    wl.path = "sublayer"


def step_inputs(wl: DeviceWorkload):
    """The per-layer input tensors ([layers, T, ...]) the workload's path reads."""
    if wl.path == "call":
        return (wl.q_call, wl.gate)
    if wl.path == "sublayer":
        return (wl.partials, wl.o_partials)
    if wl.path == "qkvg":
        return (wl.partials,)
    return (wl.qk, wl.v, wl.gate)


def layer_call(attn, wl: DeviceWorkload, app: int, layer: int, ins, out, rep: int = 0):
    """One application: `ins` are this application's slices of step_inputs(); `rep` picks
    the step's pools within a multi-step replay."""
    from dory_decode_attention import EPS
    key, value = wl.pool(layer, rep)
    window, scale = wl.window(layer), wl.hd ** -0.5
    sumsq = None if wl.sumsq is None else wl.sumsq[layer]
    if wl.path == "call":
        q, gate = ins
        if hasattr(attn, "call_tokens"):  # a comparison leg that takes all tokens at once
            attn.call_tokens(q, key, value, window, scale, gate, out)
            return
        attn(q[0], key, value, wl.tables[0], wl.seq_lens[0:1], window, scale, gate[0], out[0],
             out_sumsq=sumsq)
        return
    if wl.path in ("qkvg", "sublayer"):
        from dory_sublayer_steps import qkvg_epilogue, residual_tokens
        qk_b, v_b, gate_b = wl.qkvg_bufs
        qkvg_epilogue(ins[0], wl.positions, wl.cos_sin, wl.s_gate, 0.9, qk_b, v_b, gate_b,
                      wl.nh, wl.nkv, wl.hd, overlap_launch=attn.overlap_launch)
        attn.multi_from_raw(qk_b, v_b, wl.sqk, W.SQK_FACTOR, EPS, wl.cache_offsets, key, value,
                            wl.tables, wl.table_offsets, wl.seq_lens, window, scale, gate_b, out,
                            shared_cache=wl.shared, out_sumsq=sumsq)
        if wl.path == "sublayer":
            residual_tokens(ins[1], None, wl.h_in, wl.alpha, 2.5, EPS, wl.h_out, wl.h_out_nm,
                            x_sumsq=sumsq, overlap_launch=attn.overlap_launch)
        return
    qk, v, gate = ins
    if wl.path == "separate":
        # The reference's separate path (bench_decode_attention.py:144-152): the q/k
        # normalisation kernel writes the cache and the bf16 query, then __call__ attends.
        from dory_sublayer_steps import qk_norm_cache
        qk_norm_cache(qk[0], v[0], wl.sqk, W.SQK_FACTOR, EPS, wl.q_out[0], wl.nh, wl.hd,
                      key_cache=key, value_cache=value, slot_mapping=wl.slots[0:1])
        attn(wl.q_out[0], key, value, wl.tables[0], wl.seq_lens[0:1], window, scale, gate[0],
             out[0], out_sumsq=sumsq)
        return
    attn.multi_from_raw(qk, v, wl.sqk, W.SQK_FACTOR, EPS, wl.cache_offsets, key, value,
                        wl.tables, wl.table_offsets, wl.seq_lens, window, scale, gate, out,
                        shared_cache=wl.shared, out_sumsq=sumsq)


def run_step(attn, wl: DeviceWorkload, rep: int = 0):
    for app, layer in enumerate(wl.layers):
        layer_call(attn, wl, app, layer, [t[layer] for t in step_inputs(wl)], wl.out[layer],
                   rep)


def run_replay(attn, wl: DeviceWorkload):
    """What one graph replay runs: wl.reps steps, each over its own pools."""
    for rep in range(wl.reps):
        run_step(attn, wl, rep)


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
    spec = workload_spec(args.workload)
    lens_all = subset(spec.lens, args.max_seqs)
    wl = DeviceWorkload(spec, lens_all, dev, 11, mem_fraction=args.mem_fraction,
                        kv_dtype=args.kv_dtype)
    attn = make_attention(wl, args)
    for _ in range(args.profile_steps):
        run_step(attn, wl)
    torch.cuda.synchronize(dev)
    attn.check_errors()
    print(json.dumps({"profile_steps": args.profile_steps, "launches": args.profile_steps *
                      len(spec.layers), "sequences": len(lens_all), "pools": wl.num_pools,
                      "algorithmic_bytes_per_launch":
                          wl.algorithmic_bytes_per_step() / len(spec.layers)}),
          flush=True)


def time_graph(attn, wl: DeviceWorkload, steps: int, warmup: int, dist, dev):
    """Eager warm-up and error check, then one graph replay (wl.reps steps) captured,
    `warmup` untimed replays, and `steps` workload steps timed with CUDA events between
    barriers while nvidia-smi samples the clocks.  `steps` must be a multiple of wl.reps.
    Returns (ms per step on this rank, clock summary)."""
    assert steps % wl.reps == 0
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        run_replay(attn, wl)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    attn.check_errors()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run_replay(attn, wl)
    for _ in range(warmup):
        graph.replay()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(dist, dev)
    with ClockSampler(dev) as clocks:
        start.record()
        for _ in range(steps // wl.reps):
            graph.replay()
        end.record()
        torch.cuda.synchronize(dev)
    barrier(dist, dev)
    attn.check_errors()
    del graph
    return start.elapsed_time(end) / steps, clocks.summary()


def roofline_of(wl: DeviceWorkload, workload: str, us_per_launch: float) -> dict:
    """Roofline of the kernel: algorithmic bytes per launch / average launch time against
    the measured copy bandwidth; traffic from the committed ncu summary when there is one."""
    peaks = load_peaks()
    per_launch = wl.algorithmic_bytes_per_step() / len(wl.layers)
    achieved = per_launch / (us_per_launch * 1e-6) / 1e9
    ratio = read_traffic_ratio(workload, "fp8" if wl.kv8 else "bf16")
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks[0], "unit": "GB/s",
            "frac": round(achieved / peaks[0], 4),
            "traffic": int(ratio * per_launch) if ratio else None, "peak_source": peaks[1],
            "algorithmic_bytes_per_launch": round(per_launch), "launch_us": round(us_per_launch, 3)}


def bench_ours(args, world, rank, local):
    dist = init_dist(world, local)
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    spec = workload_spec(args.workload)
    lens_all, tps, shared, layers, notes = (spec.lens, spec.tokens_per_seq, spec.shared,
                                            spec.layers, spec.notes)
    if shared or len(lens_all) == 1:
        mine = list(range(len(lens_all)))  # a single sequence does not shard: replicas
        scaling = "replicas"
    else:
        mine = rank_sequences(args.workload, lens_all, world, rank)
        scaling = "strong"
    lens = [lens_all[i] for i in mine]
    wl = DeviceWorkload(spec, lens, dev, spec.seed + 1000 * rank, kv_dtype=args.kv_dtype)
    if args.sumsq:
        wl.sumsq = torch.zeros(wl.num_layers, wl.tokens, device=dev)
    if args.kv_dtype == "fp8" and args.path != "fused":
        raise SystemExit("--kv-dtype fp8 takes the fused path")
    if args.path in ("separate", "call") and wl.tokens != 1:
        raise SystemExit(f"--path {args.path} takes single-sequence workloads "
                         "(config1, config4, dory*)")
    prepare_path(wl, args.path)
    attn = make_attention(wl, args)
    apps = len(layers)

    steps = -(-args.steps // wl.reps) * wl.reps
    ms_local, clocks = time_graph(attn, wl, steps, args.warmup, dist, dev)
    ms = max_over_ranks(dist, ms_local, dev)

    total_seqs = len(lens_all) * (tps if shared else 1)
    bytes_rank = wl.algorithmic_bytes_per_step()
    bytes_all = sum_over_ranks(dist, float(bytes_rank), dev)
    ms_per_step = ms
    seqs_per_s = (total_seqs * (world if scaling == "replicas" else 1)) / (ms_per_step / 1e3)
    us_per_layer = ms_per_step * 1e3 / apps
    hbm_gbs = bytes_all / (ms_per_step / 1e3) / 1e9
    # roofline of the one kernel: this rank's bytes per launch / its average launch time
    roofline = roofline_of(wl, args.workload, ms_local * 1e3 / apps)

    e2e = bench_e2e(attn, wl, args, dist, dev, total_seqs, world, scaling)
    launches_per_step = apps * {"separate": 2, "qkvg": 2, "sublayer": 3}.get(wl.path, 1)
    config = {"workload": f"{args.workload}: {notes}", "global_batch": total_seqs,
              "layers_per_step": apps, "num_heads": wl.nh, "num_kv_heads": wl.nkv,
              "head_dim": wl.hd, "block_size": BLOCK,
              "windows": sorted({wl.window(layer) for layer in layers}),
              "cache_layout": "vLLM Triton [blocks, kv_heads, 16, 2*head_dim] viewed "
              "via transpose(1,2).split",
              "parallelism": f"request partition over {world} GPU(s), no collectives",
              "distinct_pools_per_rank": wl.num_pools, "steps_per_replay": wl.reps,
              "l2": l2_note(wl),
              "splits": args.splits, "min_blocks_per_split": args.min_blocks_per_split,
              "overlap_launch": args.overlap_launch, "path": args.path,
              "consumer": args.consumer, "kv_dtype": args.kv_dtype,
              "out_sumsq": bool(args.sumsq)}
    del attn, wl
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()

    cpu, extra = None, None
    if rank == 0 and world == 1 and args.kv_dtype == "bf16":
        cpu = cpu_baseline(args.workload, args.cpu_seconds)
        if (args.all_configs and args.workload == "config5" and args.path == "fused"
                and args.consumer == "mma" and args.kv_dtype == "bf16"):
            extra = measure_other_configs(args, dev)

    line = {
        "metric": METRIC, "value": round(seqs_per_s, 2), "unit": "seqs/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        # an FP8 cache is read as e4m3 bytes and multiplied in f16 (fp32 accumulation)
        "dtype": "bf16" if args.kv_dtype == "bf16" else "fp8_e4m3",
        "data": "synthetic (seeded N(0,1) K/V, q/k/v, gate; random block-table permutations)",
        "config": config,
        "us_per_layer_step": round(us_per_layer, 3),
        "hbm_gbs": round(hbm_gbs, 1),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": steps * launches_per_step,
        "clocks": clocks,
    }
    if extra is not None:
        line["configs"] = extra
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def prepare_path(wl: DeviceWorkload, path: str):
    if path == "separate":
        wl.path = "separate"
    elif path == "call":
        prepare_call_path(wl)
    elif path == "qkvg":
        prepare_qkvg_path(wl)
    elif path == "sublayer":
        prepare_sublayer_path(wl)


# The other configurations of the metric, reported beside the config-5 headline at N = 1:
# the single-sequence and small-batch shapes (configs 1-4) and the reference benchmark's own
# 16q/4kv x 256 shape (dory640/2048/8192).
OTHER_CONFIGS = ("config1", "config2", "config3", "config4", "dory640", "dory2048", "dory8192")
OTHER_STEPS = 400  # timed steps per mode: 0.1-0.6 s of GPU time, several clock samples


def measure_other_configs(args, dev) -> dict:
    """Each other configuration on this GPU: µs per layer-step with plain launches and with
    programmatic dependent launches (`overlap_launch`), the roofline of the plain launches,
    the clocks during both and the CPU baseline of the same workload."""
    out = {}
    budget = max(1.0, min(3.0, args.cpu_seconds / 5))
    for name in OTHER_CONFIGS:
        spec = workload_spec(name)
        splits, mbps = tuned_splits(name, 1)
        entry = {"workload": f"{name}: {spec.notes}", "splits": splits,
                 "min_blocks_per_split": mbps, "layers_per_step": len(spec.layers)}
        wl = DeviceWorkload(spec, list(spec.lens), dev, spec.seed)
        steps = -(-OTHER_STEPS // wl.reps) * wl.reps
        entry.update({"steps": steps, "warmup": args.warmup, "steps_per_replay": wl.reps,
                      "distinct_pools": wl.num_pools, "l2": l2_note(wl)})
        seqs = len(spec.lens) * spec.tokens_per_seq
        for overlap in (False, True):
            a = argparse.Namespace(splits=splits, min_blocks_per_split=mbps, overlap_launch=overlap)
            attn = make_attention(wl, a)
            ms, clocks = time_graph(attn, wl, steps, args.warmup, None, dev)
            us = ms * 1e3 / len(spec.layers)
            res = {"us_per_layer_step": round(us, 3), "seqs_per_s": round(seqs / (ms / 1e3), 1),
                   "hbm_gbs": round(wl.algorithmic_bytes_per_step() / (ms / 1e3) / 1e9, 1),
                   "roofline": roofline_of(wl, name, us), "clocks": clocks,
                   "gpu_launches": steps * len(spec.layers)}
            if overlap:
                entry["overlap_launch"] = res
            else:
                entry.update(res)
            del attn
        if name in ("config1", "dory640"):
            entry["host_issue"] = measure_host_issue(args, wl, splits, mbps)
        del wl
        torch.cuda.empty_cache()
        entry["cpu_baseline"] = cpu_baseline(name, budget)
        if name == "config2":
            entry["wavefront_step"] = measure_wavefront_step(args, dev)
        out[name] = entry
    return out


def measure_host_issue(args, wl: DeviceWorkload, splits: int, mbps: int) -> dict:
    """Host cost of the Python boundary: the layer sequence issued eagerly (DecodeAttention
    from Python, ctypes into the C ABI, one kernel launch per call) `reps` times.  host_us is
    the wall time to issue one call (no synchronisation inside the loop); eager_us the time
    per call until the GPU has finished them all, against the graph replay's per-call time."""
    a = argparse.Namespace(splits=splits, min_blocks_per_split=mbps, overlap_launch=False)
    attn = make_attention(wl, a)
    run_step(attn, wl)
    torch.cuda.synchronize(wl.dev)
    reps = 10
    calls = reps * len(wl.layers)
    t0 = time.perf_counter()
    for _ in range(reps):
        run_step(attn, wl)
    t1 = time.perf_counter()
    torch.cuda.synchronize(wl.dev)
    t2 = time.perf_counter()
    attn.check_errors()
    return {"calls": calls, "host_us_per_call": round((t1 - t0) / calls * 1e6, 2),
            "eager_us_per_call": round((t2 - t0) / calls * 1e6, 2),
            "what": "DecodeAttention.multi_from_raw issued from Python per layer, no graph"}


def measure_wavefront_step(args, dev, layers: int = 20) -> dict:
    """A whole wavefront step of the recurrent block's attention sublayers at configuration
    2's shape, replayed as one CUDA graph (WavefrontRecurrentBlock): for each of the 20
    recurrent attention layers, the q/k/v/gate epilogue on seeded GEMV partials, the four
    rows' multi_from_raw on the layer's shared "last_loop" cache (loop pattern 3, 2, 1, 0)
    with the output statistic, and the residual update fed it (the NVFP4 GEMVs between
    them are not part of this build; their split-K partials are the seeded inputs).  Each
    layer reads its own 11 MB cache, 220 MB per step, more than L2."""
    from dory_decode_attention import EPS, DecodeAttention
    from wavefront_binding import AttentionSublayer, WavefrontLayer, WavefrontRecurrentBlock
    spec = workload_spec("config2")
    rows, position = spec.tokens_per_seq, spec.lens[0]
    need = -(-(position + rows) // BLOCK)
    gd = torch.Generator(device=dev).manual_seed(2027)
    table = torch.randperm(need + 8, device=dev, generator=gd)[:need].to(torch.int32)[None]
    cos_sin = torch.randn(position + rows + 4, HD, device=dev, generator=gd)
    subs = []
    for _ in range(layers):
        kv = torch.empty(need + 8, NKV, BLOCK, 2 * HD, dtype=torch.bfloat16, device=dev)
        kv.normal_(generator=gd)
        subs.append(AttentionSublayer(
            WavefrontLayer([kv] * rows, [0] * rows, table.shape[1], NKV, HD),
            (torch.rand(NH * HD, device=dev, generator=gd) + 0.5).to(torch.bfloat16),
            (torch.rand(NH * HD, device=dev, generator=gd) + 0.5).to(torch.bfloat16), cos_sin,
            (torch.randn(NH * HD, device=dev, generator=gd) * 0.02).to(torch.bfloat16), 0,
            HD ** -0.5))
    splits, mbps = tuned_splits("config2", 1)
    positions = torch.arange(position, position + rows, dtype=torch.int64, device=dev)
    seq_lens = (positions + 1).to(torch.int32)
    h_in = torch.randn(rows, NH * HD, device=dev, generator=gd).to(torch.bfloat16)
    lens = [position + t + 1 for t in range(rows)]
    per_layer = algorithmic_bytes(lens, True, 0, NH, NKV, HD, QKVG_SPLIT_K, NH * HD)
    out = {"what": "20 recurrent attention sublayers of one wavefront step (4 rows at loop "
                   "depths 3..0, positions 2710..2713): q/k/v/gate epilogue, multi_from_raw "
                   "on the shared cache with the output statistic, residual update; one CUDA "
                   "graph, GEMV partials seeded",
           "launches_per_step": 3 * layers}
    for overlap in (False, True):
        attn = DecodeAttention(NH, NKV, HD, dev, splits=splits, max_tokens=rows,
                               min_blocks_per_split=mbps, overlap_launch=overlap)
        block = WavefrontRecurrentBlock(attn, subs, table, NH * HD, W.SQK_FACTOR, 0.9, 2.5, EPS)
        for i in range(layers):
            block.qkvg_partials(i, rows).normal_(generator=gd)
            block.out_partials(i, rows).normal_(generator=gd)
        block.replay(rows, positions, seq_lens, h_in)  # plain launches, then the capture
        for _ in range(args.warmup):
            block.replay(rows, positions, seq_lens, h_in)
        steps = OTHER_STEPS
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        with ClockSampler(dev) as clocks:
            start.record()
            for _ in range(steps):
                block.replay(rows, positions, seq_lens, h_in)
            end.record()
            torch.cuda.synchronize(dev)
        attn.check_errors()
        us = start.elapsed_time(end) * 1e3 / steps
        res = {"us_per_wavefront_step": round(us, 3), "us_per_layer": round(us / layers, 3),
               "steps": steps, "hbm_gbs": round(per_layer * layers / (us * 1e-6) / 1e9, 1),
               "clocks": clocks.summary()}
        if overlap:
            out["overlap_launch"] = res  # the three kernels of each layer chained as PDL
        else:
            out.update(res)
        del block, attn
    return out


def l2_note(wl: DeviceWorkload) -> str:
    """How the step's inputs relate to the 126 MB L2 (nothing is flushed between steps)."""
    if wl.pool_bytes > L2_BYTES:
        return "inputs larger than L2 (each pool > 126 MB; pools cycled per layer)"
    per_replay = wl.pool_bytes * min(wl.num_pools, wl.num_layers * wl.reps)
    return (f"inputs larger than L2: each graph replay ({wl.reps} step(s)) reads "
            f"{min(wl.num_pools, wl.num_layers * wl.reps)} distinct pools of "
            f"{wl.pool_bytes / 1e6:.1f} MB ({per_replay / 1e6:.0f} MB > 126 MB)")


E2E_CHUNK_BYTES = 1 << 20  # smallest host->device copy of the end-to-end leg


def bench_e2e(attn, wl: DeviceWorkload, args, dist, dev, total_seqs, world, scaling):
    """The same step through the public API with host buffers.  Every step copies each
    application's q/k, v and gate from pinned host memory and reads each output back into
    pinned host memory.  Copies run on two copy streams, in chunks of consecutive
    applications of at least E2E_CHUNK_BYTES (one per application on large workloads), and
    overlap the kernels: a chunk's kernels wait only for its own inputs.  The reported
    value replays the step (copies and API calls) as one CUDA graph, as vLLM runs its
    decode step; `eager` issues the same step from Python every time."""
    apps = len(wl.layers)
    # inputs per application: an application that revisits a layer gets its own copy
    host_in = [torch.stack([t[layer].cpu() for layer in wl.layers]).pin_memory()
               for t in step_inputs(wl)]
    host_out = torch.empty((apps,) + tuple(wl.out.shape[1:])).pin_memory()
    dev_in = [torch.empty_like(h, device=dev) for h in host_in]
    dev_out = torch.empty(host_out.shape, device=dev)
    per_app = sum(h[0].numel() * h.element_size() for h in host_in)
    k = max(1, min(apps, -(-E2E_CHUNK_BYTES // per_app)))
    chunks = [(a, min(a + k, apps)) for a in range(0, apps, k)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    h2d_bytes = per_app * apps
    d2h_bytes = host_out.numel() * host_out.element_size()

    def step():
        compute = torch.cuda.current_stream(dev)
        h2d.wait_stream(compute)  # the previous step's kernels are done with the inputs
        d2h.wait_stream(compute)
        for a0, a1 in chunks:
            loaded, done = torch.cuda.Event(), torch.cuda.Event()
            with torch.cuda.stream(h2d):
                for dst, src in zip(dev_in, host_in):
                    dst[a0:a1].copy_(src[a0:a1], non_blocking=True)
                loaded.record(h2d)
            compute.wait_event(loaded)
            for a in range(a0, a1):
                layer_call(attn, wl, a, wl.layers[a], [t[a] for t in dev_in], dev_out[a])
            done.record(compute)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done)
                host_out[a0:a1].copy_(dev_out[a0:a1], non_blocking=True)
        compute.wait_stream(h2d)
        compute.wait_stream(d2h)  # the step ends when its outputs are in host memory

    def timed(run, steps):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(dist, dev)
        start.record()
        for _ in range(steps):
            run()
        end.record()
        torch.cuda.synchronize(dev)
        barrier(dist, dev)
        return max_over_ranks(dist, start.elapsed_time(end), dev) / steps

    steps = max(1, min(args.steps, args.e2e_steps))
    for _ in range(max(1, args.warmup)):
        step()
    ms_eager = timed(step, steps)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(1, args.warmup)):
        graph.replay()
    ms = timed(graph.replay, steps)
    torch.cuda.synchronize(dev)
    if not torch.equal(host_out, dev_out.cpu()):
        raise RuntimeError("end-to-end leg: host outputs differ from the device outputs")
    del graph
    seqs = total_seqs * (world if scaling == "replicas" else 1)
    return {"value": round(seqs / (ms / 1e3), 2), "unit": "seqs/s", "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes, "steps": steps, "ms_per_step": round(ms, 4),
            "copy_chunks": len(chunks),
            "eager": {"value": round(seqs / (ms_eager / 1e3), 2), "ms_per_step":
                      round(ms_eager, 4)},
            "path": "DecodeAttention.multi_from_raw per application, inputs from and outputs "
                    "to pinned host memory every step, chunked copies on two copy streams "
                    "overlapped with the kernels; value: the step as one CUDA graph"}


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return 6650.0, "fallback (6.65 TB/s earlier pool measurement)"


def read_traffic_ratio(workload: str, kv_dtype: str = "bf16"):
    """DRAM traffic / algorithmic bytes of one launch, from the committed ncu summary of this
    workload and cache type (profiles/decode_kernel_<workload>.txt, or
    decode_kernel_fp8_<workload>.txt for FP8 caches), or None."""
    kind = "fp8_" if kv_dtype == "fp8" else ""
    path = ROOT / "profiles" / f"decode_kernel_{kind}{workload}.txt"
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

class CpuSample:
    """The workload's CPU pass: the reference semantics in PyTorch eager FP32
    (oracle/dory_oracle.py) for one attention layer over ALL of the workload's sequences
    (the wavefront's four tokens for config 2).  One pass times one application per
    distinct sliding window of the step; the step's time is each application's time
    weighted by the number of applications with that window (36 full-context layers for
    configs 3 and 5).  Passes reuse the cache: the append writes the same rows at the same
    slots every time, so a pass after the first reads exactly what the first read."""

    def __init__(self, workload: str):
        sys.path.insert(0, str(ROOT / "oracle"))
        import dory_oracle as O
        self.O = O
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        spec = self.spec = workload_spec(workload)
        self.lens = list(spec.lens)
        self.shared = spec.shared
        self.layers = len(spec.layers)
        counts: dict[int, int] = {}
        for layer in spec.layers:
            w = spec.window(layer)
            counts[w] = counts.get(w, 0) + 1
        shape = dict(num_heads=spec.nh, num_kv_heads=spec.nkv, head_dim=spec.hd)
        self.cases = []  # (case, bf16 key, bf16 value, applications per step)
        for w, n in sorted(counts.items()):
            if spec.shared:
                case = W.wavefront(seed=spec.seed, prompt=self.lens[0], generated=0,
                                   tokens=spec.tokens_per_seq, window=w, **shape)
                key, value = case.key.to(torch.bfloat16), case.value.to(torch.bfloat16)
            else:
                # caches of several GB (config 5): filled by parallel seeded generators
                case = W.batched(seed=spec.seed, lens=self.lens, window=w, draw_cache=False,
                                 **shape)
                cshape = (case.num_blocks, case.block_size, case.num_kv_heads, case.head_dim)
                key = W.normal_bf16(cshape, 2 * spec.seed)
                value = W.normal_bf16(cshape, 2 * spec.seed + 1)
            self.cases.append((case, key, value, n))
        self.tokens = self.cases[0][0].tokens

    def once(self) -> tuple[float, float]:
        """(seconds measured for this pass, seconds of the whole step it stands for)."""
        O, measured, step = self.O, 0.0, 0.0
        for c, key, value, n in self.cases:
            width = c.tables.shape[1]
            t0 = time.perf_counter()
            O.multi_from_raw(c.qk, c.v, c.sqk, c.sqk_factor, O.EPS,
                             torch.zeros(c.tokens, dtype=torch.int64), key.view(-1),
                             value.view(-1), tuple(key.shape), key.stride(),
                             c.tables.reshape(-1),
                             torch.tensor([r * width for r in c.table_rows]), c.seq_lens,
                             c.window, c.scale, c.gate, c.num_heads, c.num_kv_heads,
                             shared_cache=c.shared)
            dt = time.perf_counter() - t0
            measured += dt
            step += n * dt
        return measured, step

    def seqs_per_s(self, step_seconds: float) -> float:
        """Query tokens served per second (a shared-cache group counts each of its tokens,
        as the GPU arm does)."""
        return self.tokens / step_seconds

    def describe(self, measured: float, step_seconds: float, reps: int) -> str:
        windows = ", ".join(f"{n} x window {c.window}" if c.window else f"{n} x full context"
                            for c, _, _, n in self.cases)
        what = (f"{self.tokens} wavefront tokens at {self.lens[0] + 1}.."
                f"{self.lens[0] + self.tokens}" if self.shared else
                f"all {len(self.lens)} sequence(s) (ctx {min(self.lens)}..{max(self.lens)}, "
                f"mean {sum(self.lens) / len(self.lens):.0f})")
        return (f"{what}: one application per distinct window, {measured:.3f} s per pass, "
                f"scaled to the step's {self.layers} layer applications ({windows}) = "
                f"{step_seconds:.3f} s per step, {reps} pass(es); PyTorch eager FP32 "
                "restatement of the reference semantics (oracle/dory_oracle.py)")


def cpu_baseline(workload: str, budget_s: float):
    """Times CPU passes of the workload (after one warm-up pass) until `budget_s` seconds
    have passed (at least one)."""
    sample = CpuSample(workload)
    sample.once()  # warm-up
    measured = step = 0.0
    reps = 0
    while measured < budget_s or reps == 0:
        m, st = sample.once()
        measured += m
        step += st
        reps += 1
    return {"value": round(sample.seqs_per_s(step / reps), 4), "unit": "seqs/s",
            "cores": sample.threads, "kind": "port",
            "sample": sample.describe(measured / reps, step / reps, reps)}


def bench_reference(args, world, rank, local):
    """The reference arm: the reference's CPU implementation of the path (its eager PyTorch
    semantics; the reference's own kernel is Triton GPU code) on the host cores, rank 0
    only.  A step is one CPU pass (one attention layer over all of the workload's
    sequences; `ms_per_step` is that measured pass), and the value scales it to the
    metric's whole step of `layers_per_step` applications."""
    if rank != 0:
        return
    spec = workload_spec(args.workload)
    sample = CpuSample(args.workload)
    for _ in range(args.warmup):
        sample.once()
    runs = [sample.once() for _ in range(args.steps)]
    measured = statistics.mean(m for m, _ in runs)
    step = statistics.mean(st for _, st in runs)
    value = sample.seqs_per_s(step)
    cpu = {"value": round(value, 4), "unit": "seqs/s", "cores": sample.threads, "kind": "port",
           "sample": sample.describe(measured, step, len(runs))}
    total_seqs = sample.tokens
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "seqs/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(measured * 1e3, 3),
            "step": "one CPU pass: one attention layer application per distinct window over "
                    "every sequence of the workload; value = sequences per second of the "
                    f"whole {len(spec.layers)}-application step ({step:.3f} s)",
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded); the full workload's sequences",
            "config": {"workload": f"{args.workload}: {spec.notes}", "global_batch": total_seqs,
                       "layers_per_step": len(spec.layers)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(value, 4), "unit": "seqs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "the reference's path is Triton GPU code; its CPU implementation is its "
                    "eager PyTorch semantics, restated in oracle/dory_oracle.py"}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
# comparison legs on the same GPU: the reference's own Triton kernel, vLLM's attention
# ---------------------------------------------------------------------------------------

class ReferenceTriton:
    """The reference's DecodeAttention (kernels/dory_decode_attention.py:225-331, Triton),
    installed unmodified under baseline/_ref, behind the layer calls bench.py makes."""
    overlap_launch = False

    def __init__(self, mod, wl: DeviceWorkload, splits: int):
        self.a = mod.DecodeAttention(wl.nh, wl.nkv, wl.hd, wl.dev, splits=splits,
                                     max_tokens=max(wl.tokens, 1))

    def __call__(self, *args, out_sumsq=None):
        self.a(*args)

    def multi_from_raw(self, *args, out_sumsq=None, **kw):
        self.a.multi_from_raw(*args, **kw)

    def check_errors(self):
        pass


class VllmUnified:
    """vLLM's Triton unified attention over the same paged cache, then the gate product:
    the comparison row of the reference's own benchmark (kernels/bench_decode_attention.py:
    71-97).  It takes normalised bf16 queries whose k/v are already cached (the non-raw
    call); a wavefront's tokens are one sequence's causal query block, a batch's tokens one
    query each."""
    overlap_launch = False
    SEGMENTS = 16  # the reference benchmark's NUM_PAR_SOFTMAX_SEGMENTS

    def __init__(self, wl: DeviceWorkload):
        from vllm.v1.attention.ops.triton_unified_attention import unified_attention
        self.fn = unified_attention
        T, dev = wl.tokens, wl.dev
        self.T, self.nh, self.hd = T, wl.nh, wl.hd
        f32 = dict(dtype=torch.float32, device=dev)
        if wl.shared:
            seqs = 1
            self.cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
            self.seqused = wl.seq_lens[-1:].clone()
            self.max_q = T
            self.table = wl.tables[0:1]
        else:
            seqs = T
            self.cu = torch.arange(T + 1, dtype=torch.int32, device=dev)
            self.seqused = wl.seq_lens
            self.max_q = 1
            self.table = wl.tables
        self.max_k = max(wl.seq_lens_list)
        self.segm_output = torch.empty(T, wl.nh, self.SEGMENTS, wl.hd, **f32)
        self.segm_max = torch.empty(T, wl.nh, self.SEGMENTS, **f32)
        self.segm_expsum = torch.empty(T, wl.nh, self.SEGMENTS, **f32)
        self.descale = torch.ones(seqs, wl.nkv, **f32)
        self.out = torch.empty(T, wl.nh, wl.hd, dtype=torch.bfloat16, device=dev)

    def call_tokens(self, q, key, value, window, scale, gate, out):
        self.fn(q=q.view(self.T, self.nh, self.hd), k=key, v=value, out=self.out,
                cu_seqlens_q=self.cu, max_seqlen_q=self.max_q, seqused_k=self.seqused,
                max_seqlen_k=self.max_k, softmax_scale=scale, causal=True,
                window_size=(window - 1, 0) if window else (-1, -1), block_table=self.table,
                softcap=0, q_descale=None, k_descale=self.descale, v_descale=self.descale,
                seq_threshold_3D=32, num_par_softmax_segments=self.SEGMENTS,
                softmax_segm_output=self.segm_output, softmax_segm_max=self.segm_max,
                softmax_segm_expsum=self.segm_expsum)
        torch.mul(self.out.view(self.T, -1), gate.view(self.T, -1), out=out.view(self.T, -1))

    def check_errors(self):
        pass


COMPARE_WORKLOADS = ("config1", "config2", "config3", "config4", "config5", "dory640",
                     "dory2048", "dory8192")
SINGLE_SEQUENCE = ("config1", "config4", "dory640", "dory2048", "dory8192")


def load_reference_triton():
    """The reference's decode-attention module from baseline/_ref, or (None, why not)."""
    path = ROOT / "baseline" / "_ref" / "dory_decode_attention.py"
    if not path.exists():
        return None, ("baseline/_ref is not installed here (python "
                      "baseline/install_reference.py, where the reference checkout is)")
    import importlib.util
    spec = importlib.util.spec_from_file_location("reference_dory_decode_attention", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, None


def bench_compare(args):
    """One JSON line per (implementation, workload, path): this build, the reference's own
    Triton kernel and vLLM's unified attention, each timed as CUDA-graph replays of the
    same layer sequence over the same pools on one GPU (µs per layer-step, the workload's
    algorithmic bytes over that time).  Paths: "fused" (raw q/k/v: normalisation, append,
    attention, gate; multi_from_raw) and "call" (normalised query, k/v cached beforehand;
    __call__), the latter for the single-sequence workloads, and for vLLM, whose attention
    has no raw mode, on every workload."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ref_mod, why = load_reference_triton()
    names = COMPARE_WORKLOADS if args.workload == "config5" else (args.workload,)
    impls = ("ours", "triton-reference", "vllm-unified")
    for name in names:
        spec = workload_spec(name)
        splits, mbps = tuned_splits(name, 1)
        for impl in impls:
            paths = ["fused", "call"] if name in SINGLE_SEQUENCE else ["fused"]
            if impl == "vllm-unified":
                paths = ["call"]
            for path in paths:
                line = {"impl": impl, "workload": name, "path": path,
                        "metric": "us per layer-step", "unit": "us"}
                if impl == "triton-reference" and ref_mod is None:
                    line["unavailable"] = why
                    print(json.dumps(line), flush=True)
                    continue
                wl = DeviceWorkload(spec, list(spec.lens), dev, spec.seed)
                if path == "call":
                    prepare_call_path(wl)
                if impl == "ours":
                    a = argparse.Namespace(splits=splits, min_blocks_per_split=mbps,
                                           overlap_launch=False, prefetch_chunks=0)
                    attn = make_attention(wl, a)
                    line["splits"] = splits
                elif impl == "triton-reference":
                    attn = ReferenceTriton(ref_mod, wl, 32)  # the reference's default split count
                    line["splits"] = 32
                else:
                    attn = VllmUnified(wl)
                    line["segments"] = VllmUnified.SEGMENTS
                steps = -(-max(50, args.steps) // wl.reps) * wl.reps
                ms, clocks = time_graph(attn, wl, steps, args.warmup, None, dev)
                us = ms * 1e3 / len(spec.layers)
                byts = wl.algorithmic_bytes_per_step() / len(spec.layers)
                line.update({"value": round(us, 3), "us_per_layer_step": round(us, 3),
                             "hbm_gbs": round(byts / (us * 1e-6) / 1e9, 1),
                             "frac_of_measured_peak": round(byts / (us * 1e-6) / 1e9 / load_peaks()[0], 4),
                             "steps": steps, "layers_per_step": len(spec.layers),
                             "clocks": clocks})
                print(json.dumps(line), flush=True)
                del attn, wl
                torch.cuda.empty_cache()


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference", "compare"), default="ours",
                    help="reference: the reference semantics on the host CPU (the driver's "
                         "reference arm); compare: this build, the reference's own Triton "
                         "kernel (baseline/_ref) and vLLM's unified attention on this GPU, "
                         "one JSON line each, for every workload (or --workload's)")
    ap.add_argument("--workload", default="config5", choices=WORKLOADS,
                    help="config1..5: the 32q/8kv x 128 configurations; dory640/2048/8192: "
                         "the reference benchmark's 16q/4kv x 256 shape")
    ap.add_argument("--splits", type=int, default=None,
                    help="split count (default: the tuned setting of the workload and GPU count)")
    ap.add_argument("--min-blocks-per-split", type=int, default=None)
    ap.add_argument("--overlap-launch", action="store_true",
                    help="launch each layer call as a programmatic dependent of the previous one")
    ap.add_argument("--path", choices=("fused", "separate", "call", "qkvg", "sublayer"),
                    default="fused",
                    help="qkvg: the multi-token q/k/v/gate epilogue kernel on the GEMV's "
                         "split-K partials, then multi_from_raw; sublayer: qkvg, then the "
                         "residual update on the output GEMV's partials, fed the attention "
                         "output's sum of squares; "
                         "call: the non-raw __call__ alone (q normalised and its k/v cached "
                         "beforehand); separate: the q/k normalisation kernel then the "
                         "non-raw call "
                         "(single-sequence workloads; the reference's two-kernel path)")
    ap.add_argument("--prefetch-chunks", type=int, default=0,
                    help="L2 prefetch distance ahead of each CTA's ring, in 16-row chunks "
                         "(0: automatic, < 0: none)")
    ap.add_argument("--consumer", choices=("mma", "fma"), default="mma",
                    help="dot products of the chunk step: mma.sync tensor-core tiles (the "
                         "product) or FP32 FMAs on the CUDA cores (the measured alternative; "
                         "128-dim heads, no shared cache)")
    ap.add_argument("--kv-dtype", choices=("bf16", "fp8"), default="bf16",
                    help="cache element type: bf16 (the reference's) or fp8 e4m3 (vLLM's fp8 "
                         "kv_cache_dtype, scales 1; single sequences and independent batches)")
    ap.add_argument("--sumsq", action="store_true",
                    help="also produce each token's sum of squared outputs (out_sumsq)")
    ap.add_argument("--all-configs", action=argparse.BooleanOptionalAction, default=True,
                    help="with the default config5 workload on one GPU, also time configs "
                         "1-4 and dory640/2048/8192 and report them under \"configs\"")
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
    tuned = tuned_splits(args.workload, world, args.kv_dtype)
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
    elif args.impl == "compare":
        if rank == 0:
            bench_compare(args)
    else:
        bench_ours(args, world, rank, local)
    return 0


if __name__ == "__main__":
    sys.exit(main())
