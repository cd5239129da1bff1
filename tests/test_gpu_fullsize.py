"""Parity at the benchmark configurations' full sizes (one layer each, the bench's split
settings), through DecodeAttention and the C ABI.

* Configurations 2 (4-token shared-cache wavefront at position 2710), 3 (64 sequences,
  39,362 cached tokens) and 4 (one 7,936-token sequence): every output against the oracle and
  the whole pool bit for bit after the append.
* Configuration 5 (512 sequences, 1,038,941 cached tokens, a 4.3 GB pool): the outputs of a
  length-stratified sample of 16 sequences against the oracle (their blocks copied back to
  the host), and on the device, that exactly the 512 appended rows changed and that they
  hold the oracle's normalised k and bf16 v (bit for bit).
"""

from __future__ import annotations

import pytest
import torch

import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows, run

pytestmark = pytest.mark.gpu


def check_cache(case, layout, d, before):
    exp = expected_raw(case, layout, before, oracle_rows(case))
    got = d["raw"].cpu()
    assert torch.equal(got.view(torch.int16), exp.view(torch.int16)), \
        f"{int((got.view(torch.int16) != exp.view(torch.int16)).sum())} cache elements differ"


def test_config2_full():
    case = W.wavefront(seed=1, prompt=2560, generated=150, tokens=4)
    out, d, before = run(case, "triton", splits=16)
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_config3_full():
    case = W.batched(seed=2, lens=W.config3_lens())
    assert sum(W.config3_lens()) == 39362
    out, d, before = run(case, "triton", splits=2, min_blocks_per_split=32)
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_config4_full():
    case = W.single(seed=3, context=7936, pool_blocks=500)
    out, d, before = run(case, "triton", splits=37)
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_config5_full_sampled():
    lens = W.config5_lens()
    assert sum(lens) == 1_038_941
    case = W.batched(seed=4, lens=lens, pool_factor=1.0, draw_cache=False)
    T, B, NH, NKV, HD = case.tokens, case.block_size, case.num_heads, case.num_kv_heads, 128
    d = W.to_device(case, "triton", "cuda", copy_cache=False)
    gen = torch.Generator(device="cuda").manual_seed(4)
    d["raw"].normal_(generator=gen)
    before = d["raw"].clone()
    attn = DecodeAttention(NH, NKV, HD, torch.device("cuda"), splits=2, max_tokens=T,
                           min_blocks_per_split=64)
    attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS, d["cache_offsets"],
                        d["key"], d["value"], d["tables"], d["table_offsets"], d["seq_lens"],
                        0, case.scale, d["gate"], d["out"])
    torch.cuda.synchronize()
    attn.check_errors()

    # Cache: the appended rows hold the oracle's rows; nothing else changed.
    rows = oracle_rows(case)
    slots = torch.tensor([case.slot(t) for t in range(T)], device="cuda")
    blk, row = slots // B, slots % B
    key_a = d["raw"].transpose(1, 2)[..., :HD]    # [blocks, B, NKV, HD] views of the layout
    value_a = d["raw"].transpose(1, 2)[..., HD:]
    k_exp = torch.stack([r[0] for r in rows]).cuda()
    v_exp = torch.stack([r[1] for r in rows]).cuda()
    assert torch.equal(key_a[blk, row].view(torch.int16), k_exp.view(torch.int16))
    assert torch.equal(value_a[blk, row].view(torch.int16), v_exp.view(torch.int16))
    changed = d["raw"].view(torch.int16) != before.view(torch.int16)
    changed[blk, :, row, :] = False
    assert not bool(changed.any()), "cache rows other than the appended ones changed"
    del changed

    # Outputs of a length-stratified sample against the oracle, on each sequence's own blocks.
    order = sorted(range(T), key=lambda t: lens[t])
    sample = sorted({order[round(i * (T - 1) / 15)] for i in range(16)})
    key_b = before.transpose(1, 2)[..., :HD]
    value_b = before.transpose(1, 2)[..., HD:]
    out = d["out"].cpu()
    for t in sample:
        need = -(-(lens[t] + 1) // B)
        ids = case.tables[t, :need].long().cuda()
        one = W.Case(NH, NKV, HD, B, need, key_b[ids].float().contiguous().cpu(),
                     value_b[ids].float().contiguous().cpu(),
                     torch.arange(need, dtype=torch.int32)[None], [0], [lens[t] + 1],
                     case.qk[t:t + 1], case.v[t:t + 1], case.gate[t:t + 1], case.sqk)
        assert_close(out[t:t + 1], oracle_out(one))
