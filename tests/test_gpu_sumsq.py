"""The optional out_sumsq output: sum over e of out[t][e]^2 per token (the statistic the
consumer's output GEMV normalises by, dory_attention.py:114-117), computed in the kernel's
epilogue.

* against the kernel's own output summed in FP64 (only the summation order differs) and
  against the oracle's output (1e-2 relative, the bf16 bar);
* every epilogue path: one split (direct store), split merge by the last CTA, padding
  requests (0), shared-cache token groups, 8-row and 16-row tiles, head dims 64/128/256;
* bit-identical on repeated calls and graph replays (fixed summation order, self-resetting
  per-token counters); the outputs themselves are unchanged by asking for it.
"""

from __future__ import annotations

import pytest
import torch

import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import oracle_out, run

pytestmark = pytest.mark.gpu


def own_sumsq(out: torch.Tensor) -> torch.Tensor:
    return out.double().reshape(out.shape[0], -1).square().sum(1)


def call(case, layout="triton", splits=16, min_bps=1, **kw):
    """Runs the case with out_sumsq; returns (out, sumsq) on the CPU."""
    d = W.to_device(case, layout, "cuda")
    T = case.tokens
    attn = DecodeAttention(case.num_heads, case.num_kv_heads, case.head_dim,
                           torch.device("cuda"), splits=splits, max_tokens=max(T, 1),
                           min_blocks_per_split=min_bps)
    ss = torch.full((T,), float("nan"), device="cuda")
    if T == 1 and not case.shared and kw.get("single", True):
        attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                      d["key"], d["value"], d["tables"][case.table_rows[0]],
                      d["seq_lens"][0:1], case.window, case.scale, d["gate"][0], d["out"][0],
                      out_sumsq=ss)
    else:
        attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS,
                            d["cache_offsets"], d["key"], d["value"], d["tables"],
                            d["table_offsets"], d["seq_lens"], case.window, case.scale,
                            d["gate"], d["out"], shared_cache=case.shared, out_sumsq=ss)
    torch.cuda.synchronize()
    attn.check_errors()
    return d["out"].cpu(), ss.cpu()


def check(case, out, ss):
    mine = own_sumsq(out)
    torch.testing.assert_close(ss.double(), mine, rtol=1e-5, atol=1e-6)
    ref = own_sumsq(oracle_out(case))
    torch.testing.assert_close(ss.double(), ref, rtol=2e-2, atol=1e-4)


@pytest.mark.parametrize("splits", [1, 3, 16, 148])
@pytest.mark.parametrize("name", ["config1", "window"])
def test_single_token_paths(name, splits):
    case = (W.single(seed=600, context=640, pool_blocks=64) if name == "config1"
            else W.single(seed=601, context=1500, pool_blocks=100, window=1024))
    out, ss = call(case, splits=splits)
    check(case, out, ss)


def test_batch_with_padding():
    case = W.batched(seed=602, lens=[0, 1, 15, 16, 17, 300, 1023, 1024, 1025, 2000, 31, 700,
                                     4000, 2, 64, 129])
    case.seq_lens[0] = 0
    case.seq_lens[7] = 0
    out, ss = call(case, splits=4)
    assert ss[0] == 0 and ss[7] == 0
    check(case, out, ss)


@pytest.mark.parametrize("tokens", [2, 4, 16])
def test_shared_wavefront_groups(tokens):
    case = W.wavefront(seed=603, prompt=900, generated=3, tokens=tokens)
    out, ss = call(case, splits=8)
    check(case, out, ss)


@pytest.mark.parametrize("nh,nkv,hd", [(64, 8, 128), (128, 8, 128), (32, 8, 64), (16, 4, 256)])
def test_head_shapes(nh, nkv, hd):
    case = W.batched(seed=604 + nh, lens=[100, 900, 2500], num_heads=nh, num_kv_heads=nkv,
                     head_dim=hd)
    out, ss = call(case, splits=8)
    check(case, out, ss)


def test_outputs_unchanged_and_repeat_bit_identical():
    case = W.batched(seed=605, lens=[50, 700, 3000, 1200])
    out_a, ss_a = call(case, splits=8)
    out_b, ss_b = call(case, splits=8)
    assert torch.equal(ss_a, ss_b)
    assert torch.equal(out_a, out_b)
    plain, _, _ = run(case, "triton", splits=8)
    assert torch.equal(plain, out_a)


def test_graph_replay_resets_counters():
    case = W.single(seed=606, context=800, pool_blocks=70)
    d = W.to_device(case, "triton", "cuda")
    attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=16)
    ss = torch.zeros(1, device="cuda")

    def step():
        attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                      d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], 0, case.scale,
                      d["gate"][0], d["out"][0], out_sumsq=ss)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = ss.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(3):
        ss.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(ss, eager)
    attn.check_errors()


def test_non_raw_call():
    case = W.single(seed=607, context=500, pool_blocks=50)
    d = W.to_device(case, "triton", "cuda")
    attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=16)
    attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                  d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], 0, case.scale,
                  d["gate"][0], d["out"][0])
    import dory_oracle as O
    q, _, _ = O.raw_qkv(case.qk[0], case.v[0], case.sqk, case.sqk_factor, EPS, 32, 8, 128)
    ss = torch.zeros(1, device="cuda")
    out = torch.zeros_like(d["out"][0])
    attn(q.reshape(-1).cuda(), d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], 0,
         case.scale, d["gate"][0], out, out_sumsq=ss)
    torch.cuda.synchronize()
    torch.testing.assert_close(ss.cpu().double(), own_sumsq(out.cpu()[None]), rtol=1e-5,
                               atol=1e-6)
