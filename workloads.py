"""Seeded synthetic decode workloads with the shapes of the reference's configurations.

The reference measures this path on no public dataset; every input here is drawn from
`torch.Generator().manual_seed(seed)` on the CPU (so values are identical on every host),
N(0, 1) for q, k, v, the gate's pre-activation and the cached K/V, with random block-table
permutations, as kernels/bench_decode_attention.py:46-55,104-115 builds its inputs
(sqk = bf16(U[0.5, 1.5)), sqk_factor = 0.7).  Large caches for throughput runs can be
filled on the device instead (`fill="device"`), where only the seed and shapes matter.

Cache layouts (all viewed as [blocks, block_size, kv_heads, head_dim] key/value tensors):
  "triton": vLLM Triton backend as the reference reads it, raw [blocks, kv_heads,
            block_size, 2 * head_dim] -> transpose(1, 2).split(head_dim, -1)
            (kernels/dory_fused_model.py:122-137)
  "unbind": vLLM 0.22 Triton backend, raw [blocks, 2, block_size, kv_heads, head_dim]
            -> unbind(1)
  "bench":  the reference benchmark's raw [blocks, block_size, kv_heads, 2 * head_dim]
            -> split(head_dim, -1) (kernels/bench_decode_attention.py:51-54)
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass, field

import torch

LAYOUTS = ("triton", "unbind", "bench")
NH, NKV, HD, BLOCK = 32, 8, 128, 16  # 32 query heads, 8 KV heads, head_dim 128, block size 16
SQK_FACTOR = 0.7


def generator(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def cache_views(num_blocks: int, block_size: int, kv_heads: int, head_dim: int, layout: str,
                device, storage_dtype=torch.bfloat16):
    """(raw storage, key view, value view) of an uninitialised cache in `layout`."""
    if layout == "triton":
        raw = torch.empty(num_blocks, kv_heads, block_size, 2 * head_dim, dtype=storage_dtype,
                          device=device)
        key, value = raw.transpose(1, 2).split(head_dim, dim=-1)
    elif layout == "unbind":
        raw = torch.empty(num_blocks, 2, block_size, kv_heads, head_dim, dtype=storage_dtype,
                          device=device)
        key, value = raw.unbind(1)
    elif layout == "bench":
        raw = torch.empty(num_blocks, block_size, kv_heads, 2 * head_dim, dtype=storage_dtype,
                          device=device)
        key, value = raw.split(head_dim, dim=-1)
    else:
        raise ValueError(f"unknown cache layout {layout!r}")
    return raw, key, value


@dataclass
class Token:
    """Per-token inputs of a raw-mode call (FP32 on CPU)."""
    qk: torch.Tensor      # [(NH + NKV) * HD]
    v: torch.Tensor       # [NKV * HD]
    gate: torch.Tensor    # [NH * HD], post-sigmoid


@dataclass
class Case:
    """A raw-mode decode call: T tokens over one cache pool (CPU tensors)."""
    num_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    key: torch.Tensor            # FP32 [num_blocks, B, NKV, HD] initial cache contents
    value: torch.Tensor
    tables: torch.Tensor         # int32 [rows, width] block tables
    table_rows: list[int]        # token t reads tables[table_rows[t]]
    seq_lens: list[int]          # per token
    qk: torch.Tensor             # FP32 [T, (NH + NKV) * HD]
    v: torch.Tensor              # FP32 [T, NKV * HD]
    gate: torch.Tensor           # FP32 [T, NH * HD]
    sqk: torch.Tensor            # bf16 [NH * HD]
    window: int = 0
    shared: bool = False
    sqk_factor: float = SQK_FACTOR
    meta: dict = field(default_factory=dict)

    @property
    def tokens(self) -> int:
        return len(self.seq_lens)

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    def slot(self, t: int) -> int:
        """Append slot of token t: its table entry at seq_len - 1 (vLLM slot_mapping)."""
        n = self.seq_lens[t]
        if n <= 0:
            return -1
        pos = n - 1
        return int(self.tables[self.table_rows[t], pos // self.block_size]) * self.block_size \
            + pos % self.block_size


def _draw_tokens(g: torch.Generator, T: int, nh: int, nkv: int, hd: int):
    qk = torch.randn(T, (nh + nkv) * hd, generator=g)
    v = torch.randn(T, nkv * hd, generator=g)
    gate = torch.sigmoid(torch.randn(T, nh * hd, generator=g))
    return qk, v, gate


def _draw_sqk(g: torch.Generator, nh: int, hd: int) -> torch.Tensor:
    return (torch.rand(nh * hd, generator=g) + 0.5).to(torch.bfloat16)


def _draw_cache(g: torch.Generator, num_blocks: int, block_size: int, nkv: int, hd: int):
    return (torch.randn(num_blocks, block_size, nkv, hd, generator=g),
            torch.randn(num_blocks, block_size, nkv, hd, generator=g))


def normal_bf16(shape, seed: int, threads: int = 0) -> torch.Tensor:
    """A bf16 tensor of N(0, 1) draws, filled in parallel chunks by NumPy generators spawned
    from `seed` (reproducible for a given seed and shape, whatever the thread count).  For
    caches of several GB, where torch.randn's single-threaded CPU generator takes a minute."""
    import concurrent.futures
    import numpy as np
    out = torch.empty(shape, dtype=torch.bfloat16)
    flat = out.view(-1)
    n = flat.numel()
    chunk = 1 << 24
    pieces = [(i, min(i + chunk, n)) for i in range(0, n, chunk)]
    seeds = np.random.SeedSequence(seed).spawn(len(pieces))

    def fill(job):
        (a, b), ss = job
        x = np.random.default_rng(ss).standard_normal(b - a, dtype=np.float32)
        flat[a:b].copy_(torch.from_numpy(x))

    workers = threads or (os.cpu_count() or 1)
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as ex:
        list(ex.map(fill, zip(pieces, seeds)))
    return out


def single(seed: int = 0, context: int = 640, pool_blocks: int = 64, window: int = 0,
           num_heads: int = NH, num_kv_heads: int = NKV, head_dim: int = HD,
           block_size: int = BLOCK) -> Case:
    """One token at position `context` (seq_len context + 1) over a permuted pool.

    Defaults are configuration 1 of the reference build's baseline: 32q/8kv x 128, block 16,
    640 cached tokens in a 64-block pool, seed 0, slot_mapping[0] at position 640."""
    g = generator(seed)
    qk, v, gate = _draw_tokens(g, 1, num_heads, num_kv_heads, head_dim)
    sqk = _draw_sqk(g, num_heads, head_dim)
    key, value = _draw_cache(g, pool_blocks, block_size, num_kv_heads, head_dim)
    table = torch.randperm(pool_blocks, generator=g).to(torch.int32)
    need = -(-(context + 1) // block_size)
    if need > pool_blocks:
        raise ValueError("pool too small for the context")
    return Case(num_heads, num_kv_heads, head_dim, block_size, pool_blocks, key, value,
                table[None], [0], [context + 1], qk, v, gate, sqk, window=window,
                meta={"kind": "single", "seed": seed, "context": context})


def wavefront(seed: int = 1, prompt: int = 2560, generated: int = 0, tokens: int = 4,
              window: int = 0, pool_blocks: int | None = None, num_heads: int = NH,
              num_kv_heads: int = NKV, head_dim: int = HD, block_size: int = BLOCK) -> Case:
    """Shared-KV wavefront step (configuration 2): `tokens` query tokens at consecutive
    positions p..p+T-1 (p = prompt + generated, loop depths T-1..0), one cache and one
    block table for all of them, causal among themselves (token t sees p..p+t)."""
    g = generator(seed)
    qk, v, gate = _draw_tokens(g, tokens, num_heads, num_kv_heads, head_dim)
    sqk = _draw_sqk(g, num_heads, head_dim)
    p = prompt + generated
    if pool_blocks is None:
        pool_blocks = -(-(prompt + 300 + tokens) // block_size) + 2
    key, value = _draw_cache(g, pool_blocks, block_size, num_kv_heads, head_dim)
    table = torch.randperm(pool_blocks, generator=g).to(torch.int32)
    lens = [p + t + 1 for t in range(tokens)]
    return Case(num_heads, num_kv_heads, head_dim, block_size, pool_blocks, key, value,
                table[None], [0] * tokens, lens, qk, v, gate, sqk, window=window, shared=True,
                meta={"kind": "wavefront", "seed": seed, "position": p})


def batched(seed: int = 2, lens: list[int] | None = None, num_seqs: int = 64, lo: int = 128,
            hi: int = 1152, pool_factor: float = 1.2, window: int = 0, num_heads: int = NH,
            num_kv_heads: int = NKV, head_dim: int = HD, block_size: int = BLOCK,
            draw_cache: bool = True) -> Case:
    """Independent sequences, one query token each, over one permuted block pool
    (configuration 3: 64 sequences, cached context uniform in [128, 1152], pool 1.2x the
    tokens).  `lens` are cached-context lengths; each sequence's seq_len is len + 1."""
    g = generator(seed)
    if lens is None:
        lens = torch.randint(lo, hi + 1, (num_seqs,), generator=g).tolist()
    T = len(lens)
    need = [-(-(n + 1) // block_size) for n in lens]
    pool_blocks = max(int(math.ceil(pool_factor * sum(n + 1 for n in lens) / block_size)),
                      sum(need))
    qk, v, gate = _draw_tokens(g, T, num_heads, num_kv_heads, head_dim)
    sqk = _draw_sqk(g, num_heads, head_dim)
    perm = torch.randperm(pool_blocks, generator=g).to(torch.int32)
    width = max(need)
    tables = torch.zeros(T, width, dtype=torch.int32)
    at = 0
    for t, k in enumerate(need):
        tables[t, :k] = perm[at:at + k]
        at += k
    if draw_cache:
        key, value = _draw_cache(g, pool_blocks, block_size, num_kv_heads, head_dim)
    else:
        key = value = None
    return Case(num_heads, num_kv_heads, head_dim, block_size, pool_blocks, key, value,
                tables, list(range(T)), [n + 1 for n in lens], qk, v, gate, sqk,
                window=window, meta={"kind": "batched", "seed": seed, "lens": lens})


def config3_lens(seed: int = 2) -> list[int]:
    return torch.randint(128, 1153, (64,), generator=generator(seed)).tolist()


def config5_lens(seed: int = 4, num_seqs: int = 512) -> list[int]:
    """512 contexts log-uniform in [128, 8192] (configuration 5)."""
    u = torch.rand(num_seqs, generator=generator(seed))
    return torch.exp(math.log(128) + u * (math.log(8192) - math.log(128))).round().long().tolist()


def partition(lens: list[int], parts: int) -> list[list[int]]:
    """Greedy token-balanced assignment (longest first, to the least-loaded part): the
    request partition of sequences over GPUs.  Returns the sequence indices of each part."""
    order = sorted(range(len(lens)), key=lambda i: (-lens[i], i))
    loads = [0] * parts
    out: list[list[int]] = [[] for _ in range(parts)]
    for i in order:
        j = min(range(parts), key=lambda k: (loads[k], k))
        out[j].append(i)
        loads[j] += lens[i] + 1
    return [sorted(part) for part in out]


def e4m3_bytes(x: torch.Tensor, scale: float) -> torch.Tensor:
    """Synthetic FP8 cache contents: e4m3 bytes (uint8) of x / scale, round to nearest even,
    saturating at +-448."""
    return (x.float() / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)


def to_device(case: Case, layout: str, device, copy_cache: bool = True, kv8=None):
    """Device tensors of a case: dict with raw/key/value caches (in `layout`), flat tables,
    offsets, seq_lens, qk, v, gate, sqk, outputs.  kv8 = (k_scale, v_scale): e4m3 caches
    (uint8 storage) holding the case's K / V quantised with those scales."""
    raw, key, value = cache_views(case.num_blocks, case.block_size, case.num_kv_heads,
                                  case.head_dim, layout, device,
                                  torch.uint8 if kv8 else torch.bfloat16)
    if copy_cache and kv8:
        key.copy_(e4m3_bytes(case.key, kv8[0]))
        value.copy_(e4m3_bytes(case.value, kv8[1]))
    elif copy_cache:
        key.copy_(case.key.to(torch.bfloat16))
        value.copy_(case.value.to(torch.bfloat16))
    width = case.tables.shape[1]
    T = case.tokens
    d = dict(raw=raw, key=key, value=value,
             tables=case.tables.contiguous().to(device),
             table_offsets=torch.tensor([r * width for r in case.table_rows], dtype=torch.int64,
                                        device=device),
             cache_offsets=torch.zeros(T, dtype=torch.int64, device=device),
             seq_lens=torch.tensor(case.seq_lens, dtype=torch.int32, device=device),
             qk=case.qk.contiguous().to(device), v=case.v.contiguous().to(device),
             gate=case.gate.contiguous().to(device), sqk=case.sqk.to(device),
             slots=torch.tensor([case.slot(t) for t in range(T)], dtype=torch.int64,
                                device=device),
             out=torch.full((T, 8, case.num_heads * case.head_dim // 8), float("nan"),
                            device=device))
    return d
