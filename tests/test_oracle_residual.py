"""The oracle's residual update against the reference's own kernels.

tests/golden/residual_*.npz hold the outputs of the reference's `_residual_tokens_kernel`
(kernels/dory_multi_token.py:109-131) and `residual_update` (kernels/dory_common.py:55-81)
on seeded inputs (tests/golden/make_golden_residual.py, run through Triton's interpreter,
which sums in FP32 in its own order and takes its inverse square roots in FP32).  The
regenerated inputs must hash to the stored digests; the FP32 nibble-major output must agree
within 5e-8 absolute + 1e-6 relative (the outputs are unit rows of 296-12288 elements,
|h| ~ 0.01-0.1; the orders of the FP32 sums differ); the BF16 output is the oracle's own FP32
result rounded to nearest even and within one BF16 step of the golden FP32 rounded the same
way.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import dory_oracle as O
import specs

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = specs.residual_specs()
ATOL, RTOL = 5e-8, 1e-6


def natural(h_nm: np.ndarray) -> torch.Tensor:
    """[T, 8, H / 8] nibble-major -> [T, H] natural order."""
    t = torch.from_numpy(np.ascontiguousarray(h_nm))
    return t.transpose(1, 2).reshape(t.shape[0], -1)


@pytest.mark.parametrize("name", sorted(CASES))
def test_residual_matches_reference(name):
    case = CASES[name]()
    g = np.load(GOLDEN / f"{name}.npz")
    assert str(g["digest"]) == specs.residual_digest(case)
    h, h_bf16, h_nm = O.residual_tokens(case.partials, case.x, None, case.a, case.alpha,
                                        case.alpha_scale)
    np.testing.assert_allclose(h_nm.numpy(), g["h_nm"], rtol=RTOL, atol=ATOL)
    assert torch.equal(natural(h_nm.numpy()), h)
    assert torch.equal(h_bf16, h.to(torch.bfloat16))
    golden_bf16 = natural(g["h_nm"]).to(torch.bfloat16)
    step = torch.finfo(torch.bfloat16).eps * golden_bf16.float().abs().clamp_min(1e-30)
    assert ((h_bf16.float() - golden_bf16.float()).abs() <= step).all()


def test_sumsq_input_equals_x_input():
    """r_x from a given sum of squares is the same number as from x when the sum is the
    FP32 rounding of the exact sum (the oracle's own sum)."""
    case = CASES["residual_attn_dory"]()
    x = case.x.numpy().astype(np.float64)
    sumsq = torch.from_numpy((x * x).sum(axis=1).astype(np.float32))
    via_x = O.residual_tokens(case.partials, case.x, None, case.a, case.alpha, case.alpha_scale)
    via_s = O.residual_tokens(case.partials, None, sumsq, case.a, case.alpha, case.alpha_scale)
    for u, v in zip(via_x, via_s):
        assert torch.equal(u, v)


def test_no_x_uses_the_partials_as_b():
    case = CASES["residual_ragged_f32"]()
    b = case.partials.sum(0, keepdim=True)  # any FP32 values
    h, _, _ = O.residual_tokens(b, None, None, case.a, case.alpha, case.alpha_scale)
    ya = O.normalize(case.a.float().numpy())
    yb = O.normalize(b[0].numpy())
    lr = np.abs(case.alpha.float().numpy() * np.float32(case.alpha_scale))
    z = (ya + (lr * (yb - ya))).astype(np.float32)
    np.testing.assert_allclose(h.numpy(), O.normalize(z), rtol=1e-6, atol=1e-9)


def test_rejects_bad_arguments():
    case = CASES["residual_ragged_f32"]()
    with pytest.raises(ValueError):
        O.residual_tokens(case.partials, case.x, torch.ones(case.tokens), case.a, case.alpha, 1.0)
    with pytest.raises(ValueError):
        O.residual_tokens(torch.zeros(1, 1, 12), None, None, torch.zeros(1, 12), torch.zeros(12),
                          1.0)


@pytest.mark.parametrize("seed,hidden", [(60, 64), (61, 2560), (62, 16384)])
def test_properties(seed, hidden):
    """Size-independent properties of h = n(n(a) + lr (n(b) - n(a))): unit rows; the
    partials and x enter only through b / |b|, so scaling the partials or x by a positive
    factor leaves h unchanged up to rounding while sum b^2 stays far above eps; lr = 0
    gives h = n(n(a)) and b parallel to a gives h = n(a)."""
    g = torch.Generator().manual_seed(seed)
    T = 3
    parts = torch.randn(2, T, hidden, generator=g)
    x = torch.randn(T, 300, generator=g)
    a = torch.randn(T, hidden, generator=g)
    a = (a / a.norm(dim=1, keepdim=True)).to(torch.bfloat16)
    alpha = (torch.randn(hidden, generator=g) * 0.05).to(torch.bfloat16)
    h, _, _ = O.residual_tokens(parts, x, None, a, alpha, 2.5)
    np.testing.assert_allclose(h.double().norm(dim=1).numpy(), 1.0, atol=1e-6)
    # scalings that keep sum b^2 far above eps (below it, eps breaks the invariance)
    for scaled in ((parts * 3.7, x), (parts, x * 0.01), (parts * 2.0, x * 0.5)):
        h2, _, _ = O.residual_tokens(scaled[0], scaled[1], None, a, alpha, 2.5)
        np.testing.assert_allclose(h2.numpy(), h.numpy(), atol=2e-7, rtol=0)
    h0, _, _ = O.residual_tokens(parts, x, None, a, torch.zeros(hidden), 2.5)
    na = O.normalize(O.normalize(a.float().numpy()))
    np.testing.assert_allclose(h0.numpy(), na, atol=1e-7, rtol=0)
    par = a.float()[None] * 0.5  # b = 0.5 a (one split), no x: n(b) = n(a)
    hp, _, _ = O.residual_tokens(par, None, None, a, alpha, 2.5)
    np.testing.assert_allclose(hp.numpy(), O.normalize(a.float().numpy()), atol=1e-7, rtol=0)
