"""The residual update after an output GEMV on B200: the consumer of the attention output.

* `residual_tokens` / `residual_update` (the reference's `_residual_tokens_kernel`,
  kernels/dory_multi_token.py:109-131, and `residual_update`, kernels/dory_common.py:55-81)
  against the golden vectors the reference's kernels produced (FP32 within 5e-8 absolute +
  1e-6 relative, as the oracle) and against the oracle, whose arithmetic the kernel follows
  (FP64 sums of squares rounded once, correctly rounded inverse square roots, unfused FP32
  products and sums): the same bits on all but a rare element.  The BF16 output is the
  kernel's FP32 result rounded to nearest even; the launch-form shim gives the same bits.
* x_sumsq: the attention call's out_sumsq in place of its output x gives h within the
  golden tolerance of the oracle fed x itself (out_sumsq is an FP32 sum).
* Input dtypes, hidden sizes up to 16384 (four groups of 8 per thread), T = 0, argument,
  alias and alignment errors.
* The attention sublayer's chain in a CUDA graph: epilogue, attention with out_sumsq, an
  output projection (a plain matmul stand-in for the W4A16 GEMV, split-K partials), the
  residual update; overlapped launches give the bits of plain launches.
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
from dory_sublayer_steps import _residual_tokens_kernel, qkvg_epilogue, residual_tokens, residual_update

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
DEV = torch.device("cuda")
ATOL, RTOL = 5e-8, 1e-6


def run(partials, x, a, alpha, alpha_scale, x_sumsq=None, overlap=False):
    T, H = partials.shape[1], partials.shape[2]
    h = torch.full((T, H), float("nan"), dtype=torch.bfloat16, device=DEV)
    h_nm = torch.full((T, 8, H // 8), float("nan"), device=DEV)
    residual_tokens(partials.to(DEV), None if x is None else x.to(DEV), a.to(DEV),
                    alpha.to(DEV), alpha_scale, EPS, h, h_nm,
                    x_sumsq=None if x_sumsq is None else x_sumsq.to(DEV), overlap_launch=overlap)
    torch.cuda.synchronize()
    return h.cpu(), h_nm.cpu()


def natural(h_nm: torch.Tensor) -> torch.Tensor:
    return h_nm.transpose(1, 2).reshape(h_nm.shape[0], -1)


def check_against_oracle(h, h_nm, want_nm, exact_fraction=0.999):
    np.testing.assert_allclose(h_nm.numpy(), want_nm.numpy(), rtol=RTOL, atol=ATOL)
    assert (h_nm == want_nm).float().mean().item() >= exact_fraction
    assert torch.equal(h, natural(h_nm).to(torch.bfloat16))


@pytest.mark.parametrize("name", sorted(specs.residual_specs()))
def test_residual_matches_reference_golden(name):
    case = specs.residual_specs()[name]()
    g = np.load(GOLDEN / f"{name}.npz")
    assert str(g["digest"]) == specs.residual_digest(case)
    h, h_nm = run(case.partials, case.x, case.a, case.alpha, case.alpha_scale)
    np.testing.assert_allclose(h_nm.numpy(), g["h_nm"], rtol=RTOL, atol=ATOL)
    _, _, want_nm = O.residual_tokens(case.partials, case.x, None, case.a, case.alpha,
                                      case.alpha_scale)
    check_against_oracle(h, h_nm, want_nm)


def test_launch_form_shims_give_same_bits():
    case = specs.residual_specs()["residual_attn_dory"]()
    T, H, K = case.tokens, case.hidden, case.x.shape[1]
    h, h_nm = run(case.partials, case.x, case.a, case.alpha, case.alpha_scale)
    h2 = torch.zeros(T, H, dtype=torch.bfloat16, device=DEV)
    nm2 = torch.zeros(T, 8, H // 8, device=DEV)
    _residual_tokens_kernel[(T,)](case.partials.to(DEV), case.x.to(DEV), case.a.to(DEV),
                                  case.alpha.to(DEV), h2, nm2, case.alpha_scale, EPS, H=H,
                                  K_IN=K, SPLIT_K=case.partials.shape[0], T=T, W_BLOCK=512,
                                  X_BLOCK=4096, num_warps=8)
    torch.cuda.synchronize()
    assert torch.equal(h2.cpu(), h) and torch.equal(nm2.cpu(), h_nm)

    one = specs.residual_specs()["residual_update_dory"]()
    h, h_nm = run(one.partials, None, one.a, one.alpha, one.alpha_scale)
    h3 = torch.zeros(one.hidden, dtype=torch.bfloat16, device=DEV)
    nm3 = torch.zeros(8, one.hidden // 8, device=DEV)
    residual_update(one.a[0].to(DEV), one.partials[0, 0].to(DEV), one.alpha.to(DEV),
                    one.alpha_scale, h3, nm3)
    torch.cuda.synchronize()
    assert torch.equal(h3.cpu(), h[0]) and torch.equal(nm3.cpu(), h_nm[0])


@pytest.mark.parametrize("hidden,x_dim,split_k,tokens", [
    (8, 4, 1, 1), (2560, 4096, 4, 4), (8192, 7168, 2, 2), (8200, 64, 1, 3), (16384, 4096, 3, 2),
    (1000, 333, 2, 5)])
@pytest.mark.parametrize("a_dtype,alpha_dtype", [(torch.bfloat16, torch.bfloat16),
                                                 (torch.float32, torch.float32),
                                                 (torch.float16, torch.bfloat16)])
def test_shapes_and_dtypes_against_oracle(hidden, x_dim, split_k, tokens, a_dtype, alpha_dtype):
    g = torch.Generator().manual_seed(hidden * 7 + split_k)
    partials = torch.randn(split_k, tokens, hidden, generator=g)
    x = torch.randn(tokens, x_dim, generator=g) * 0.3
    a = torch.randn(tokens, hidden, generator=g)
    a = (a / a.norm(dim=1, keepdim=True)).to(a_dtype)
    alpha = (torch.randn(hidden, generator=g) * 0.05).to(alpha_dtype)
    h, h_nm = run(partials, x, a, alpha, 3.0)
    _, _, want_nm = O.residual_tokens(partials, x, None, a, alpha, 3.0)
    check_against_oracle(h, h_nm, want_nm, exact_fraction=0.8 if hidden == 8 else 0.999)


def test_given_sumsq_and_no_x():
    case = specs.residual_specs()["residual_mlp_dory"]()
    x64 = case.x.double()
    sumsq = (x64 * x64).sum(1).float()
    h, h_nm = run(case.partials, None, case.a, case.alpha, case.alpha_scale, x_sumsq=sumsq)
    h_x, h_nm_x = run(case.partials, case.x, case.a, case.alpha, case.alpha_scale)
    # the FP32 rounding of the exact sum is the kernel's own FP64 sum, rounded once
    assert (h_nm == h_nm_x).float().mean().item() >= 0.999
    _, _, want = O.residual_tokens(case.partials, None, None, case.a, case.alpha, case.alpha_scale)
    h0, nm0 = run(case.partials, None, case.a, case.alpha, case.alpha_scale)
    check_against_oracle(h0, nm0, want)


def test_zero_tokens_is_a_no_op():
    h = torch.full((0, 64), 1.0, dtype=torch.bfloat16, device=DEV)
    nm = torch.zeros(0, 8, 8, device=DEV)
    residual_tokens(torch.zeros(2, 0, 64, device=DEV), None, torch.zeros(0, 64, device=DEV),
                    torch.zeros(64, device=DEV), 1.0, EPS, h, nm)
    torch.cuda.synchronize()


def test_argument_errors():
    T, H = 2, 64
    parts = torch.zeros(1, T, H, device=DEV)
    a = torch.zeros(T, H, dtype=torch.bfloat16, device=DEV)
    alpha = torch.zeros(H, device=DEV)
    h = torch.zeros(T, H, dtype=torch.bfloat16, device=DEV)
    nm = torch.zeros(T, 8, H // 8, device=DEV)
    x = torch.ones(T, 16, device=DEV)
    with pytest.raises(ValueError):  # x and x_sumsq
        residual_tokens(parts, x, a, alpha, 1.0, EPS, h, nm, x_sumsq=torch.ones(T, device=DEV))
    with pytest.raises(ValueError):  # hidden not a multiple of 8
        residual_tokens(torch.zeros(1, T, 12, device=DEV), None,
                        torch.zeros(T, 12, device=DEV), torch.zeros(12, device=DEV), 1.0, EPS,
                        torch.zeros(T, 12, dtype=torch.bfloat16, device=DEV),
                        torch.zeros(T * 12, device=DEV))
    with pytest.raises(NotImplementedError):  # hidden above 16384
        Hb = 16392
        residual_tokens(torch.zeros(1, 1, Hb, device=DEV), None, torch.zeros(1, Hb, device=DEV),
                        torch.zeros(Hb, device=DEV), 1.0, EPS,
                        torch.zeros(1, Hb, dtype=torch.bfloat16, device=DEV),
                        torch.zeros(1, 8, Hb // 8, device=DEV))
    with pytest.raises(ValueError):  # h_out inside a
        buf = torch.zeros(2 * T * H, dtype=torch.bfloat16, device=DEV)
        residual_tokens(parts, None, buf[:T * H].view(T, H), alpha, 1.0, EPS,
                        buf[T * H // 2:T * H // 2 + T * H].view(T, H), nm)
    with pytest.raises(ValueError):  # a misaligned by one element
        buf = torch.zeros(T * H + 8, dtype=torch.bfloat16, device=DEV)
        residual_tokens(parts, None, buf[1:1 + T * H].view(T, H), alpha, 1.0, EPS, h, nm)
    torch.cuda.synchronize()


def test_sublayer_chain_with_sumsq_in_a_graph():
    """qkvg epilogue -> multi_from_raw (out_sumsq) -> output projection (matmul over the
    natural-order output, split-K partials) -> residual_tokens(x_sumsq=out_sumsq), for four
    wavefront rows of the Dory shape: h against the oracle fed the output itself; the
    overlapped chain captured in a graph gives the bits of plain launches."""
    case = W.wavefront(seed=990, prompt=900, generated=2, tokens=4, window=1024, num_heads=16,
                       num_kv_heads=4, head_dim=256)
    NH, NKV, HD, T = 16, 4, 256, case.tokens
    Q, KV, H, SPLIT = NH * HD, NKV * HD, 2560, 4
    g = torch.Generator().manual_seed(991)
    partials_qkvg = (torch.randn(2, T, 2 * (Q + KV), generator=g) * 0.7).to(DEV)
    positions = torch.tensor([n - 1 for n in case.seq_lens], dtype=torch.int64, device=DEV)
    cos_sin = torch.randn(max(case.seq_lens) + 8, HD, generator=g).to(DEV)
    s_gate = (torch.rand(Q, generator=g) + 0.5).to(torch.bfloat16).to(DEV)
    w_o = (torch.randn(H, Q, generator=g) / 64).to(DEV)
    a = torch.randn(T, H, generator=g)
    a = (a / a.norm(dim=1, keepdim=True)).to(torch.bfloat16).to(DEV)
    alpha = (torch.randn(H, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    d = W.to_device(case, "triton", DEV)
    qk = torch.empty(T, Q + KV, device=DEV)
    v = torch.empty(T, KV, device=DEV)
    gate = torch.empty(T, Q, device=DEV)
    sumsq = torch.empty(T, device=DEV)
    out_partials = torch.empty(SPLIT, T, H, device=DEV)
    h = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    h_nm = torch.empty(T, 8, H // 8, device=DEV)

    def step(attn, overlap):
        qkvg_epilogue(partials_qkvg, positions, cos_sin, s_gate, 0.9, qk, v, gate, NH, NKV, HD,
                      overlap_launch=overlap)
        attn.multi_from_raw(qk, v, d["sqk"], case.sqk_factor, EPS, d["cache_offsets"], d["key"],
                            d["value"], d["tables"], d["table_offsets"], d["seq_lens"],
                            case.window, case.scale, gate, d["out"], shared_cache=True,
                            out_sumsq=sumsq)
        x = d["out"].transpose(1, 2).reshape(T, Q)
        for k in range(SPLIT):
            c = slice(k * Q // SPLIT, (k + 1) * Q // SPLIT)
            torch.matmul(x[:, c], w_o[:, c].t(), out=out_partials[k])
        residual_tokens(out_partials, None, a, alpha, 2.5, EPS, h, h_nm, x_sumsq=sumsq,
                        overlap_launch=overlap)

    plain = DecodeAttention(NH, NKV, HD, DEV, splits=8, max_tokens=T)
    step(plain, False)
    torch.cuda.synchronize()
    plain.check_errors()
    _, _, want = O.residual_tokens(out_partials.cpu(), d["out"].cpu().reshape(T, Q), None,
                                   a.cpu(), alpha.cpu(), 2.5)
    np.testing.assert_allclose(h_nm.cpu().numpy(), want.numpy(), rtol=RTOL, atol=ATOL)
    assert torch.equal(h.cpu(), natural(h_nm.cpu()).to(torch.bfloat16))
    ref_h, ref_nm = h.clone(), h_nm.clone()

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
        h.fill_(float("nan"))
        h_nm.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(h, ref_h) and torch.equal(h_nm, ref_nm)
    over.check_errors()
