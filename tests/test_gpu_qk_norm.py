"""Parity of the separate q/k normalisation step (the reference's _qk_norm_cache_kernel,
kernels/dory_attention.py:69-96) with the oracle, bit for bit, through the C ABI:

* q_out, the cached k / v rows (WRITE_CACHE) and k_out / v_out against the oracle's
  raw_qkv, for one token through the reference's launch form and for batches of tokens;
* the separate path (qk_norm_cache, then DecodeAttention.__call__) gives the same output and
  cache bits as the fused path (DecodeAttention.from_raw), as the reference's
  bench_decode_attention.py compares them (:144-157);
* padding slots write nothing; slots outside the cache are reported, not written;
* sqk in fp32 / bf16 / fp16 and head dims 64 / 128 / 256.
"""

from __future__ import annotations

import pytest
import torch

import dory_oracle as O
import workloads as W
from dory_sublayer_steps import _qk_norm_cache_kernel, qk_norm_cache
from dory_decode_attention import EPS, DecodeAttention

pytestmark = pytest.mark.gpu


def bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int16).cpu()


def oracle(qk, v, sqk, factor, NH, NKV, HD):
    return [O.raw_qkv(qk[t].cpu(), v[t].cpu(), sqk.cpu(), factor, EPS, NH, NKV, HD)
            for t in range(qk.shape[0])]


def test_reference_launch_form_writes_cache_bit_exact():
    case = W.single(seed=500, context=640, pool_blocks=64)
    d = W.to_device(case, "triton", "cuda")
    before = d["raw"].clone()
    NH, NKV, HD = 32, 8, 128
    q_out = torch.empty(NH * HD, dtype=torch.bfloat16, device="cuda")
    key, value = d["key"], d["value"]
    _qk_norm_cache_kernel[(NH + NKV,)](
        d["qk"][0], d["v"][0], d["sqk"], q_out, key, value, d["slots"][0:1], None, None,
        case.sqk_factor, EPS, key.stride(0), key.stride(1), key.stride(2), NUM_Q_HEADS=NH,
        HEAD_DIM=HD, CACHE_BLOCK=key.shape[1], WRITE_CACHE=True, num_warps=2)
    torch.cuda.synchronize()
    q, k, v = O.raw_qkv(case.qk[0], case.v[0], case.sqk, case.sqk_factor, EPS, NH, NKV, HD)
    assert torch.equal(bits(q_out.view(NH, HD)), bits(q))
    slot = case.slot(0)
    assert torch.equal(bits(key[slot // 16, slot % 16]), bits(k))
    assert torch.equal(bits(value[slot // 16, slot % 16]), bits(v))
    changed = d["raw"].view(torch.int16) != before.view(torch.int16)
    changed.transpose(1, 2)[slot // 16, slot % 16] = False
    assert not bool(changed.any())


@pytest.mark.parametrize("sqk_dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hd,nh,nkv", [(128, 32, 8), (64, 16, 4), (256, 16, 4)])
def test_batch_without_cache_write_matches_oracle(hd, nh, nkv, sqk_dtype):
    T = 9
    g = torch.Generator().manual_seed(hd + nh)
    qk = torch.randn(T, (nh + nkv) * hd, generator=g).cuda()
    v = torch.randn(T, nkv * hd, generator=g).cuda()
    sqk = (torch.rand(nh * hd, generator=g) + 0.5).to(sqk_dtype).cuda()
    q_out = torch.empty(T, nh * hd, dtype=torch.bfloat16, device="cuda")
    k_out = torch.empty(T, nkv * hd, dtype=torch.bfloat16, device="cuda")
    v_out = torch.empty_like(k_out)
    qk_norm_cache(qk, v, sqk, 0.7, EPS, q_out, nh, hd, k_out=k_out, v_out=v_out)
    torch.cuda.synchronize()
    for t, (q, k, vv) in enumerate(oracle(qk, v, sqk, 0.7, nh, nkv, hd)):
        assert torch.equal(bits(q_out[t].view(nh, hd)), bits(q))
        assert torch.equal(bits(k_out[t].view(nkv, hd)), bits(k))
        assert torch.equal(bits(v_out[t].view(nkv, hd)), bits(vv))


@pytest.mark.parametrize("layout", W.LAYOUTS)
def test_batch_cache_write_with_padding(layout):
    case = W.batched(seed=501, lens=[40, 0, 300, 17, 1025, 5, 64, 700])
    d = W.to_device(case, layout, "cuda")
    slots = d["slots"].clone()
    slots[3] = -1  # a padding token: nothing cached
    before = d["raw"].clone()
    T, NH, NKV, HD = case.tokens, 32, 8, 128
    q_out = torch.empty(T, NH * HD, dtype=torch.bfloat16, device="cuda")
    qk_norm_cache(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS, q_out, NH, HD,
                  key_cache=d["key"], value_cache=d["value"], slot_mapping=slots)
    torch.cuda.synchronize()
    rows = oracle(case.qk, case.v, case.sqk, case.sqk_factor, NH, NKV, HD)
    for t in range(T):
        assert torch.equal(bits(q_out[t].view(NH, HD)), bits(rows[t][0]))
    raw = before.cpu().clone()
    # the expected pool: `before` with each written slot holding the oracle rows
    exp_raw, exp_k, exp_v = W.cache_views(case.num_blocks, 16, NKV, HD, layout, "cpu")
    exp_raw.copy_(raw)
    for t in range(T):
        s = int(slots[t])
        if s >= 0:
            exp_k[s // 16, s % 16] = rows[t][1]
            exp_v[s // 16, s % 16] = rows[t][2]
    assert torch.equal(d["raw"].cpu().view(torch.int16), exp_raw.view(torch.int16))


def test_slot_outside_cache_is_reported_not_written():
    case = W.single(seed=502, context=100, pool_blocks=20)
    d = W.to_device(case, "triton", "cuda")
    before = d["raw"].clone()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    q_out = torch.empty(32 * 128, dtype=torch.bfloat16, device="cuda")
    slot = torch.tensor([20 * 16 + 3], dtype=torch.int64, device="cuda")
    qk_norm_cache(d["qk"][0], d["v"][0], d["sqk"], 0.7, EPS, q_out, 32, 128,
                  key_cache=d["key"], value_cache=d["value"], slot_mapping=slot, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 2  # DORY_DEVERR_SLOT_OOB
    assert torch.equal(d["raw"], before)


@pytest.mark.parametrize("window", [0, 256])
def test_separate_path_equals_fused_raw_path(window):
    """qk_norm_cache + DecodeAttention.__call__ against DecodeAttention.from_raw: the cache
    bit for bit; the outputs to within 1e-4 abs / 1e-3 rel (measured: 2e-5 at most, outputs
    of order 1e-2).  The fused raw path adds the new token's row to the merge from the k/v
    it normalises, with that row's softmax weight unrounded; the non-raw call reads the row
    from the cache inside the chunk loop, where P is rounded to bf16 for the P.V product as
    the reference does for every row: one weight differs by at most one bf16 rounding."""
    case = W.single(seed=503, context=900, pool_blocks=80, window=window)
    NH, HD = 32, 128
    results = []
    for separate in (False, True):
        d = W.to_device(case, "triton", "cuda")
        attn = DecodeAttention(NH, 8, HD, torch.device("cuda"), splits=16)
        if separate:
            q_out = torch.empty(NH * HD, dtype=torch.bfloat16, device="cuda")
            qk_norm_cache(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, q_out, NH, HD,
                          key_cache=d["key"], value_cache=d["value"], slot_mapping=d["slots"][0:1])
            attn(q_out, d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], window,
                 case.scale, d["gate"][0], d["out"][0])
        else:
            attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                          d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], window,
                          case.scale, d["gate"][0], d["out"][0])
        torch.cuda.synchronize()
        attn.check_errors()
        results.append((d["out"].cpu(), d["raw"].cpu()))
    (o0, r0), (o1, r1) = results
    torch.testing.assert_close(o0, o1, atol=1e-4, rtol=1e-3)
    assert torch.equal(r0.view(torch.int16), r1.view(torch.int16))
