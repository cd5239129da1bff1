"""The oracle's q/k/v/gate epilogue against the reference's own kernel.

tests/golden/qkvg_*.npz hold the outputs of the reference's `_qkvg_epilogue_kernel`
(kernels/dory_multi_token.py:53-80) on seeded inputs (tests/golden/make_golden_qkvg.py):
the regenerated inputs must hash to the stored digests, qk and v must match to the bit
(split-K sum in order, unfused FP32 products and sums) and the gate within 2 FP32 ulp (the
sigmoid's own rounding).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import dory_oracle as O
import specs

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = specs.qkvg_specs()


@pytest.mark.parametrize("name", sorted(CASES))
def test_epilogue_matches_reference(name):
    case = CASES[name]()
    g = np.load(GOLDEN / f"{name}.npz")
    assert str(g["digest"]) == specs.qkvg_digest(case)
    qk, v, gate = O.qkvg_epilogue(case.partials, case.positions, case.cos_sin, case.s_gate,
                                  case.s_gate_factor, case.num_heads, case.num_kv_heads,
                                  case.head_dim)
    assert np.array_equal(qk.numpy().view(np.int32), g["qk"].view(np.int32))
    assert np.array_equal(v.numpy().view(np.int32), g["v"].view(np.int32))
    np.testing.assert_allclose(gate.numpy(), g["gate"], rtol=2.5e-7, atol=1.2e-7)


def test_epilogue_rejects_wrong_row_count():
    case = CASES["qkvg_64_t1"]()
    with pytest.raises(ValueError):
        O.qkvg_epilogue(case.partials[:, :, :-64], case.positions, case.cos_sin, case.s_gate,
                        case.s_gate_factor, case.num_heads, case.num_kv_heads, case.head_dim)


def test_rotary_pairs_are_adjacent_rows():
    """Row 2i / 2i + 1 of a head are rotary dims i / i + half (the reference's row order,
    rotary_pair_order, kernels/dory_attention.py:126-130): with cos = 1, sin = 0 the
    epilogue de-interleaves the rows."""
    NH, NKV, HD = 2, 1, 64
    rows = 2 * (NH + NKV) * HD
    p = torch.arange(rows, dtype=torch.float32)[None, None, :]
    cos_sin = torch.cat([torch.ones(1, HD // 2), torch.zeros(1, HD // 2)], dim=1)
    qk, v, _ = O.qkvg_epilogue(p, [0], cos_sin, torch.ones(NH * HD), 1.0, NH, NKV, HD)
    head0 = qk[0, :HD]
    assert torch.equal(head0[:HD // 2], torch.arange(0, HD, 2, dtype=torch.float32))
    assert torch.equal(head0[HD // 2:], torch.arange(1, HD, 2, dtype=torch.float32))
    assert torch.equal(v[0], torch.arange((NH + NKV) * HD, (NH + 2 * NKV) * HD,
                                          dtype=torch.float32))


@pytest.mark.parametrize("head_dim,split_k", [(64, 1), (128, 2), (256, 3)])
def test_rotation_preserves_head_norms(head_dim, split_k):
    """With a true rotation table (cos = cos(theta), sin = sin(theta)), the rotary step keeps
    every q and k head's norm (each (i, i + half) pair is rotated by theta), and v and the
    gate do not depend on the table."""
    NH, NKV, T = 4, 2, 3
    Q, KV = NH * head_dim, NKV * head_dim
    g = torch.Generator().manual_seed(head_dim + split_k)
    parts = torch.randn(split_k, T, 2 * (Q + KV), generator=g)
    theta = torch.rand(50, head_dim // 2, generator=g, dtype=torch.float64) * 6.283
    cos_sin = torch.cat([theta.cos(), theta.sin()], dim=1).float()
    pos = torch.randint(0, 50, (T,), generator=g)
    s_gate = torch.rand(Q, generator=g) + 0.5
    qk, v, gate = O.qkvg_epilogue(parts, pos, cos_sin, s_gate, 0.9, NH, NKV, head_dim)
    y = parts.double().sum(0)[:, :Q + KV].reshape(T, NH + NKV, head_dim)
    got = qk.double().reshape(T, NH + NKV, head_dim)
    torch.testing.assert_close(got.norm(dim=-1), y.norm(dim=-1), rtol=1e-5, atol=1e-6)
    ident = torch.cat([torch.ones(50, head_dim // 2), torch.zeros(50, head_dim // 2)], dim=1)
    _, v2, gate2 = O.qkvg_epilogue(parts, pos, ident, s_gate, 0.9, NH, NKV, head_dim)
    assert torch.equal(v, v2) and torch.equal(gate, gate2)
