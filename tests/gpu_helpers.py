"""Shared helpers of the GPU parity tests: run a workloads.Case through DecodeAttention
(C ABI -> sm_100a kernel) and build the expected cache bytes."""

from __future__ import annotations

import torch

import dory_oracle as O
import workloads as W
from dory_decode_attention import EPS, DecodeAttention

# Parity bar for the bf16 path: 2e-2 absolute / 1e-2 relative.
ATOL, RTOL = 2e-2, 1e-2


def run(case: W.Case, layout: str = "triton", splits: int = 32, blocks_per_tile: int = 1,
        min_blocks_per_split: int = 1, single_entry: bool | None = None, attn=None,
        device: str = "cuda", prefetch_chunks: int = 0, consumer: str = "mma"):
    """Runs the case once; returns (out [T, 8, Q/8] on CPU, device dict, raw cache before)."""
    dev = torch.device(device)
    d = W.to_device(case, layout, dev)
    before = d["raw"].clone()
    T = case.tokens
    if attn is None:
        attn = DecodeAttention(case.num_heads, case.num_kv_heads, case.head_dim, dev,
                               splits=splits, blocks_per_tile=blocks_per_tile,
                               max_tokens=max(T, 1), min_blocks_per_split=min_blocks_per_split,
                               prefetch_chunks=prefetch_chunks, consumer=consumer)
    if single_entry is None:
        single_entry = T == 1 and not case.shared
    if single_entry:
        attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                      d["key"], d["value"], d["tables"][case.table_rows[0]], d["seq_lens"][0:1],
                      case.window, case.scale, d["gate"][0], d["out"][0])
    else:
        attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS,
                            d["cache_offsets"], d["key"], d["value"], d["tables"],
                            d["table_offsets"], d["seq_lens"], case.window, case.scale,
                            d["gate"], d["out"], shared_cache=case.shared)
    torch.cuda.synchronize()
    attn.check_errors()
    return d["out"].cpu(), d, before


def expected_raw(case: W.Case, layout: str, before: torch.Tensor, rows) -> torch.Tensor:
    """The raw cache bytes after the call: `before` with each token's slot holding its
    appended (k, v) rows — rows[t] = (k bf16 [NKV, HD], v bf16 [NKV, HD])."""
    raw = before.clone().cpu()
    # rebuild views of the CPU copy in the same layout
    if layout == "triton":
        key, value = raw.transpose(1, 2).split(case.head_dim, dim=-1)
    elif layout == "unbind":
        key, value = raw.unbind(1)
    else:
        key, value = raw.split(case.head_dim, dim=-1)
    B = case.block_size
    for t in range(case.tokens):
        slot = case.slot(t)
        if slot < 0:
            continue
        key[slot // B, slot % B] = rows[t][0]
        value[slot // B, slot % B] = rows[t][1]
    return raw


def oracle_rows(case: W.Case):
    rows = []
    for t in range(case.tokens):
        _, k, v = O.raw_qkv(case.qk[t], case.v[t], case.sqk, case.sqk_factor, EPS,
                            case.num_heads, case.num_kv_heads, case.head_dim)
        rows.append((k, v))
    return rows


def oracle_out(case: W.Case, second_rounding: bool = True) -> torch.Tensor:
    key = case.key.to(torch.bfloat16).clone()
    value = case.value.to(torch.bfloat16).clone()
    width = case.tables.shape[1]
    return O.multi_from_raw(
        case.qk, case.v, case.sqk, case.sqk_factor, EPS,
        torch.zeros(case.tokens, dtype=torch.int64), key.view(-1), value.view(-1),
        tuple(key.shape), key.stride(), case.tables.reshape(-1),
        torch.tensor([r * width for r in case.table_rows]), case.seq_lens, case.window,
        case.scale, case.gate, case.num_heads, case.num_kv_heads, shared_cache=case.shared,
        second_rounding=second_rounding)


def assert_close(out: torch.Tensor, ref: torch.Tensor, rel_l2: float = 1e-2):
    torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)
    assert O.relative_error(out, ref) < rel_l2, O.relative_error(out, ref)
