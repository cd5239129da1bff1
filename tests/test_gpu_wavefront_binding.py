"""wavefront_binding on B200: the engine's recurrent-block calls through the binding.

* Per-loop caches carved out of one allocation with loop 1's cache lowest in memory (the
  binding's base) and loop 0's highest, each loop with its own block-table row, a 3-row
  recurrent call (row t at loop 2 - t): every row's output against the oracle of its own
  loop's cache and every loop's cache bit-exact after its row's append
  (kernels/dory_wavefront_engine.py:257-332, :393-420).
* A shared "last_loop" cache (the same tensor for every loop, shared_cache=True): the
  wavefront's rows against the oracle's write-all-first semantics, with bf16 and FP8 (e4m3)
  caches.
* Both vLLM cache layouts; `entry_slots` against the slots the oracle appends at.
"""

from __future__ import annotations

import pytest
import torch

import wavefront_binding as WB
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def fill(raw_loop: torch.Tensor, case: W.Case, layout: str):
    from vllm_binding import kv_cache_views
    k, v = kv_cache_views(raw_loop, case.num_kv_heads, case.head_dim)
    k.copy_(case.key.to(torch.bfloat16))
    v.copy_(case.value.to(torch.bfloat16))


@pytest.mark.parametrize("layout", ["pinned", "vllm"])
def test_per_loop_caches_recurrent_call(layout):
    L, P = 3, 40
    cases = [W.single(seed=300 + loop, context=400 + 37 * loop, pool_blocks=P)
             for loop in range(L)]
    NKV, HD, B = 8, 128, 16
    shape = (P, NKV, B, 2 * HD) if layout == "pinned" else (P, 2, B, NKV, HD)
    slot_of_loop = [2, 0, 1]  # loop 1's cache sits lowest, loop 0's highest
    buf = torch.empty((L,) + shape, dtype=torch.bfloat16, device=DEV)
    for loop, c in enumerate(cases):
        fill(buf[slot_of_loop[loop]], c, layout)
    width = cases[0].tables.shape[1]
    tables = torch.stack([c.tables[0] for c in cases]).to(DEV)  # row l: loop l's table
    layer = WB.WavefrontLayer([buf[slot_of_loop[loop]] for loop in range(L)], list(range(L)),
                              width, NKV, HD)
    assert min(layer.loop_offsets) == 0 and layer.key.data_ptr() == buf[0].data_ptr()
    pattern = WB.recurrent_pattern(L)
    rows = [cases[loop] for loop in pattern]
    for c in rows:
        c.sqk = cases[0].sqk
    qk = torch.stack([c.qk[0] for c in rows]).to(DEV)
    v = torch.stack([c.v[0] for c in rows]).to(DEV)
    gate = torch.stack([c.gate[0] for c in rows]).to(DEV)
    seq_lens = torch.tensor([c.seq_lens[0] for c in rows], dtype=torch.int32, device=DEV)
    out = torch.full((L, 8, 32 * HD // 8), float("nan"), device=DEV)
    before = buf.clone().cpu()
    attn = DecodeAttention(32, NKV, HD, DEV, splits=8, max_tokens=L)
    WB.WavefrontAttention(attn).attention_call(
        layer, pattern, qk, v, cases[0].sqk.to(DEV), cases[0].sqk_factor, EPS, tables, seq_lens,
        0, cases[0].scale, gate, out)
    torch.cuda.synchronize()
    attn.check_errors()
    for t, c in enumerate(rows):
        assert_close(out[t].cpu(), oracle_out(c)[0])
    if layout == "pinned":  # expected_raw speaks the [blocks, kv_heads, B, 2 * HD] layout
        for loop, c in enumerate(cases):
            exp = expected_raw(c, "triton", before[slot_of_loop[loop]], oracle_rows(c))
            got = buf[slot_of_loop[loop]].cpu()
            assert torch.equal(got.view(torch.int16), exp.view(torch.int16))
    else:  # every loop's cache: only its own row's slot changed
        for loop, c in enumerate(cases):
            changed = (buf[slot_of_loop[loop]].cpu() != before[slot_of_loop[loop]]).any(-1)
            changed = changed.any(-1).any(1)  # [blocks, B]
            slot = c.slot(0)
            assert not changed.flatten()[torch.arange(changed.numel()) != slot].any()


def test_shared_last_loop_cache():
    case = W.wavefront(seed=310, prompt=700, generated=4, tokens=3)
    d = W.to_device(case, "triton", DEV)
    before = d["raw"].clone()
    width = case.tables.shape[1]
    layer = WB.WavefrontLayer([d["raw"]] * 3, [0] * 3, width, case.num_kv_heads, case.head_dim)
    attn = DecodeAttention(case.num_heads, case.num_kv_heads, case.head_dim, DEV, max_tokens=3)
    WB.WavefrontAttention(attn).attention_call(
        layer, WB.recurrent_pattern(3), d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS,
        d["tables"], d["seq_lens"], case.window, case.scale, d["gate"], d["out"],
        shared_cache=True)
    torch.cuda.synchronize()
    attn.check_errors()
    assert_close(d["out"].cpu(), oracle_out(case))
    exp = expected_raw(case, "triton", before.cpu(), oracle_rows(case))
    assert torch.equal(d["raw"].cpu().view(torch.int16), exp.view(torch.int16))


def test_shared_last_loop_fp8_cache():
    """The same call over an e4m3 cache (kv_cache_dtype="fp8", the layer's scales passed
    through the binding): outputs and cache bytes against oracle.multi_from_raw_fp8."""
    import dory_oracle as O
    case = W.wavefront(seed=311, prompt=700, generated=4, tokens=3)
    ks, vs = 0.5, 0.25
    d = W.to_device(case, "triton", DEV, kv8=(ks, vs))
    width = case.tables.shape[1]
    layer = WB.WavefrontLayer([d["raw"]] * 3, [0] * 3, width, case.num_kv_heads, case.head_dim)
    attn = DecodeAttention(case.num_heads, case.num_kv_heads, case.head_dim, DEV, max_tokens=3,
                           kv_cache_dtype="fp8")
    WB.WavefrontAttention(attn).attention_call(
        layer, WB.recurrent_pattern(3), d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS,
        d["tables"], d["seq_lens"], case.window, case.scale, d["gate"], d["out"],
        shared_cache=True, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    attn.check_errors()
    key8, value8 = W.e4m3_bytes(case.key, ks), W.e4m3_bytes(case.value, vs)
    want = O.multi_from_raw_fp8(
        case.qk, case.v, case.sqk, case.sqk_factor, EPS, torch.zeros(3, dtype=torch.int64),
        key8.view(-1), value8.view(-1), tuple(key8.shape), key8.stride(),
        case.tables.reshape(-1), torch.zeros(3, dtype=torch.int64), case.seq_lens,
        case.window, case.scale, case.gate, case.num_heads, case.num_kv_heads, ks, vs,
        shared_cache=True)
    assert_close(d["out"].cpu(), want)
    assert torch.equal(d["key"].cpu(), key8)
    assert torch.equal(d["value"].cpu(), value8)


def test_entry_slots_on_the_device():
    case = W.single(seed=320, context=530, pool_blocks=50)
    tables = torch.stack([case.tables[0], case.tables[0].flip(0)]).to(DEV)
    position = torch.tensor([530], dtype=torch.int64, device=DEV)
    slots = WB.entry_slots(tables, position, case.block_size)
    torch.cuda.synchronize()
    assert slots[0].item() == case.slot(0)
    assert slots.dtype == torch.int64 and slots.shape == (2,)


def test_call_argument_errors():
    (case,) = [W.single(seed=321, context=100, pool_blocks=20)]
    d = W.to_device(case, "triton", DEV)
    width = case.tables.shape[1]
    layer = WB.WavefrontLayer([d["raw"]], [0], width, case.num_kv_heads, case.head_dim)
    wa = WB.WavefrontAttention(DecodeAttention(32, 8, 128, DEV, max_tokens=2))
    args = (d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS)
    with pytest.raises(ValueError):  # a pattern deeper than the layer's loops
        wa.attention_call(layer, (1,), *args, d["tables"], d["seq_lens"], 0, case.scale,
                          d["gate"], d["out"])
    with pytest.raises(ValueError):  # tables of another width
        wa.attention_call(layer, (0,), *args, d["tables"][:, :-1].contiguous(), d["seq_lens"],
                          0, case.scale, d["gate"], d["out"])
