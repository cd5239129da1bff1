"""The multi-token path's q/k/v/gate epilogue on B200.

* `qkvg_epilogue` (the reference's `_qkvg_epilogue_kernel`, kernels/dory_multi_token.py:53-80)
  against the golden vectors the reference's own kernel produced: qk and v to the bit, the
  gate within the sigmoid's rounding; the launch-form shim gives the same bits.
* The multi-token sublayer's two launches (the epilogue, then `multi_from_raw`, as
  MultiTokenSublayers.attention runs them, :196-205) against the oracle (its epilogue, then
  its attention) within the bf16 bar (2e-2 abs / 1e-2 rel), the cache pool bit-exact: single tokens, batches
  with padding, shared-cache wavefronts, head dims 64/128/256, split_k 1-4, int64/int32
  positions, FP32/BF16/FP16 cos-sin tables and gate scales, with out_sumsq.
* Positions outside the cos/sin table are reported in the error word, not dereferenced.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import dory_oracle as O
import specs
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from dory_sublayer_steps import _qkvg_epilogue_kernel, qkvg_epilogue
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda")


def run_epilogue(case, int32_positions=False):
    NH, NKV, HD, T = case.num_heads, case.num_kv_heads, case.head_dim, case.tokens
    qk = torch.full((T, (NH + NKV) * HD), float("nan"), device=DEV)
    v = torch.full((T, NKV * HD), float("nan"), device=DEV)
    gate = torch.full((T, NH * HD), float("nan"), device=DEV)
    pos = case.positions.to(torch.int32 if int32_positions else torch.int64).to(DEV)
    qkvg_epilogue(case.partials.to(DEV), pos, case.cos_sin.to(DEV), case.s_gate.to(DEV),
                  case.s_gate_factor, qk, v, gate, NH, NKV, HD)
    torch.cuda.synchronize()
    return qk.cpu(), v.cpu(), gate.cpu()


@pytest.mark.parametrize("name", sorted(specs.qkvg_specs()))
def test_epilogue_matches_reference_golden(name):
    case = specs.qkvg_specs()[name]()
    g = np.load(GOLDEN / f"{name}.npz")
    assert str(g["digest"]) == specs.qkvg_digest(case)
    for int32_positions in (False, True):
        qk, v, gate = run_epilogue(case, int32_positions)
        assert np.array_equal(qk.numpy().view(np.int32), g["qk"].view(np.int32))
        assert np.array_equal(v.numpy().view(np.int32), g["v"].view(np.int32))
        np.testing.assert_allclose(gate.numpy(), g["gate"], rtol=1e-6, atol=1e-7)


def test_launch_form_shim_gives_same_bits():
    case = specs.qkvg_specs()["qkvg_128"]()
    NH, NKV, HD, T = case.num_heads, case.num_kv_heads, case.head_dim, case.tokens
    Q, KV = NH * HD, NKV * HD
    qk, v, gate = run_epilogue(case)
    qk2 = torch.zeros(T, Q + KV, device=DEV)
    v2 = torch.zeros(T, KV, device=DEV)
    g2 = torch.zeros(T, Q, device=DEV)
    parts = case.partials.to(DEV)
    _qkvg_epilogue_kernel[(parts.shape[2] // HD, T)](
        parts, case.positions.to(DEV), case.cos_sin.to(DEV), case.s_gate.to(DEV), qk2, v2, g2,
        case.s_gate_factor, Q_ROWS=Q, KV_ROWS=KV, HEAD_DIM=HD, SPLIT_K=parts.shape[0], T=T,
        num_warps=4)
    torch.cuda.synchronize()
    assert torch.equal(qk2.cpu(), qk) and torch.equal(v2.cpu(), v) and torch.equal(g2.cpu(), gate)


# ---- the epilogue, then the attention ----

def with_partials(case: W.Case, seed: int, split_k: int, cos_dtype=torch.float32,
                  s_gate_dtype=torch.bfloat16):
    """Draws GEMV partials, positions (seq_len - 1), a cos/sin table and gate scales for a
    case, and replaces the case's qk / v / gate by the oracle's epilogue of them."""
    g = torch.Generator().manual_seed(seed)
    NH, NKV, HD, T = case.num_heads, case.num_kv_heads, case.head_dim, case.tokens
    rows = 2 * (NH + NKV) * HD
    ex = {"partials": torch.randn(split_k, T, rows, generator=g) * 0.7,
          "positions": torch.tensor([max(n - 1, 0) for n in case.seq_lens], dtype=torch.int64),
          "cos_sin": torch.randn(max(case.seq_lens) + 8, HD, generator=g).to(cos_dtype),
          "s_gate": (torch.rand(NH * HD, generator=g) + 0.5).to(s_gate_dtype),
          "s_gate_factor": 0.9}
    qk, v, gate = O.qkvg_epilogue(ex["partials"], ex["positions"], ex["cos_sin"], ex["s_gate"],
                                  ex["s_gate_factor"], NH, NKV, HD)
    case.qk, case.v, case.gate = qk, v, gate
    return ex


def run_sublayer(case: W.Case, ex, splits=8, sumsq=False, int32_positions=False):
    """The epilogue then multi_from_raw on the device: (out, sumsq, raw cache) on the CPU."""
    NH, NKV, HD, T = case.num_heads, case.num_kv_heads, case.head_dim, case.tokens
    d = W.to_device(case, "triton", DEV)
    attn = DecodeAttention(NH, NKV, HD, DEV, splits=splits, max_tokens=max(T, 1))
    ss = torch.full((T,), float("nan"), device=DEV) if sumsq else None
    pos = ex["positions"].to(torch.int32 if int32_positions else torch.int64).to(DEV)
    qk = torch.empty(T, (NH + NKV) * HD, device=DEV)
    v = torch.empty(T, NKV * HD, device=DEV)
    gate = torch.empty(T, NH * HD, device=DEV)
    qkvg_epilogue(ex["partials"].to(DEV), pos, ex["cos_sin"].to(DEV), ex["s_gate"].to(DEV),
                  ex["s_gate_factor"], qk, v, gate, NH, NKV, HD)
    attn.multi_from_raw(qk, v, d["sqk"], case.sqk_factor, EPS, d["cache_offsets"], d["key"],
                        d["value"], d["tables"], d["table_offsets"], d["seq_lens"], case.window,
                        case.scale, gate, d["out"], shared_cache=case.shared, out_sumsq=ss)
    torch.cuda.synchronize()
    attn.check_errors()
    return d["out"].cpu(), None if ss is None else ss.cpu(), d["raw"].cpu()


def check_against_oracle(case, out, raw):
    assert_close(out, oracle_out(case))
    before = W.to_device(case, "triton", "cpu")["raw"]
    exp = expected_raw(case, "triton", before, oracle_rows(case))
    assert torch.equal(raw.view(torch.int16), exp.view(torch.int16))


CASES = {
    "single_256": lambda: W.single(seed=900, context=1500, pool_blocks=100, window=1024,
                                   num_heads=16, num_kv_heads=4, head_dim=256),
    "single_128": lambda: W.single(seed=901, context=640, pool_blocks=64),
    "batched_padding": lambda: W.batched(seed=902, lens=[0, 15, 16, 700, 1030, 2]),
    "wavefront_128": lambda: W.wavefront(seed=903, prompt=700, generated=9, tokens=4),
    "wavefront_256": lambda: W.wavefront(seed=904, prompt=1200, generated=3, tokens=4,
                                         window=1024, num_heads=16, num_kv_heads=4,
                                         head_dim=256),
    "wavefront_16tok_64": lambda: W.wavefront(seed=905, prompt=300, tokens=16, num_heads=8,
                                              num_kv_heads=2, head_dim=64),
    "gqa16_128": lambda: W.batched(seed=906, lens=[333, 900], num_heads=32, num_kv_heads=2,
                                   head_dim=128),
}


@pytest.mark.parametrize("split_k", [1, 2, 4])
@pytest.mark.parametrize("name", sorted(CASES))
def test_epilogue_then_attention_matches_oracle(name, split_k):
    case = CASES[name]()
    if name == "batched_padding":
        case.seq_lens[0] = 0
    ex = with_partials(case, seed=910 + split_k, split_k=split_k)
    out, _, raw = run_sublayer(case, ex)
    check_against_oracle(case, out, raw)


@pytest.mark.parametrize("cos_dtype,s_gate_dtype,int32_positions",
                         [(torch.bfloat16, torch.float32, True),
                          (torch.float16, torch.bfloat16, False)])
def test_dtypes_and_sumsq(cos_dtype, s_gate_dtype, int32_positions):
    case = CASES["wavefront_256"]()
    ex = with_partials(case, seed=930, split_k=3, cos_dtype=cos_dtype, s_gate_dtype=s_gate_dtype)
    out, ss, raw = run_sublayer(case, ex, sumsq=True, int32_positions=int32_positions)
    check_against_oracle(case, out, raw)
    torch.testing.assert_close(ss.double(), out.double().reshape(case.tokens, -1).square().sum(1),
                               rtol=1e-5, atol=1e-6)


def test_position_outside_table_is_reported():
    case = W.single(seed=940, context=300, pool_blocks=30)
    ex = with_partials(case, seed=941, split_k=1)
    NH, NKV, HD = 32, 8, 128
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    qk = torch.full((1, (NH + NKV) * HD), float("nan"), device=DEV)
    v = torch.empty(1, NKV * HD, device=DEV)
    gate = torch.empty(1, NH * HD, device=DEV)
    qkvg_epilogue(ex["partials"].to(DEV), ex["positions"].to(DEV), ex["cos_sin"][:100].to(DEV),
                  ex["s_gate"].to(DEV), 0.9, qk, v, gate, NH, NKV, HD, error_word=err)
    torch.cuda.synchronize()
    assert int(err.item()) & 16  # DORY_DEVERR_POSITION_OOB: position 300 is past the table
    assert torch.equal(qk.cpu(), torch.zeros_like(qk.cpu()))


def test_argument_errors():
    NH, NKV, HD, T = 4, 2, 64, 2
    Q, KV = NH * HD, NKV * HD
    parts = torch.zeros(1, T, 2 * (Q + KV), device=DEV)
    pos = torch.zeros(T, dtype=torch.int64, device=DEV)
    cs = torch.zeros(8, HD, device=DEV)
    sg = torch.ones(Q, device=DEV)
    outs = (torch.empty(T, Q + KV, device=DEV), torch.empty(T, KV, device=DEV),
            torch.empty(T, Q, device=DEV))
    with pytest.raises(ValueError):  # wrong row count
        qkvg_epilogue(parts[:, :, :-64].contiguous(), pos, cs, sg, 1.0, *outs, NH, NKV, HD)
    with pytest.raises(ValueError):  # float positions
        qkvg_epilogue(parts, pos.float(), cs, sg, 1.0, *outs, NH, NKV, HD)
    with pytest.raises(ValueError):  # cos/sin of another head dim
        qkvg_epilogue(parts, pos, cs[:, :32].contiguous(), sg, 1.0, *outs, NH, NKV, HD)
    with pytest.raises(ValueError):  # output of the wrong size
        qkvg_epilogue(parts, pos, cs, sg, 1.0, outs[0][:1], outs[1], outs[2], NH, NKV, HD)


def test_overlapped_chain_reusing_buffers_in_a_graph():
    """Epilogue and attention of several layers, every launch a programmatic dependent of
    the one before, all layers sharing one set of qk / v / gate buffers (each epilogue
    rewrites them while the previous layer's attention may still be reading its gate):
    the same bits as plain launches."""
    cases = [CASES["wavefront_128"]() for _ in range(3)]
    exs = [with_partials(c, seed=970 + i, split_k=2) for i, c in enumerate(cases)]
    NH, NKV, HD, T = 32, 8, 128, cases[0].tokens
    devs = [W.to_device(c, "triton", DEV) for c in cases]
    bufs = (torch.empty(T, (NH + NKV) * HD, device=DEV), torch.empty(T, NKV * HD, device=DEV),
            torch.empty(T, NH * HD, device=DEV))
    parts = [e["partials"].to(DEV) for e in exs]
    pos = exs[0]["positions"].to(DEV)
    cos_sin, s_gate = exs[0]["cos_sin"].to(DEV), exs[0]["s_gate"].to(DEV)

    def step(attn, overlap):
        for d, part in zip(devs, parts):
            qkvg_epilogue(part, pos, cos_sin, s_gate, 0.9, *bufs, NH, NKV, HD,
                          overlap_launch=overlap)
            attn.multi_from_raw(bufs[0], bufs[1], d["sqk"], cases[0].sqk_factor, EPS,
                                d["cache_offsets"], d["key"], d["value"], d["tables"],
                                d["table_offsets"], d["seq_lens"], 0, cases[0].scale, bufs[2],
                                d["out"], shared_cache=True)

    plain = DecodeAttention(NH, NKV, HD, DEV, splits=8, max_tokens=T)
    step(plain, False)
    torch.cuda.synchronize()
    want = [d["out"].clone() for d in devs]
    over = DecodeAttention(NH, NKV, HD, DEV, splits=8, max_tokens=T, overlap_launch=True)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step(over, True)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(over, True)
    for _ in range(3):
        for d in devs:
            d["out"].fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        for d, w in zip(devs, want):
            assert torch.equal(d["out"], w)
    over.check_errors()
