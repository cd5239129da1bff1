"""Cache rows outside the attended range never reach the output.

The kernel copies whole 16-row boxes, so the first and last chunk of a range (a sliding
window that starts inside a block, a sequence that ends inside one) carry rows the token
does not attend.  Those rows may hold anything in a real cache: here every row outside the
attended ranges is NaN, and the output must still match the oracle (which reads only the
attended positions, dory_decode_attention.py:131-133 masks) while the pool stays bit for bit
what it was except for the appended rows.  Head dims 64, 128 (zeroed in shared memory) and
256 (masked in the MMA operand), single-token, batched and shared-cache calls, windows that
start inside a block, split counts that put the edge chunks in different CTAs.
"""

from __future__ import annotations

import pytest
import torch

import dory_oracle as O
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows, run

pytestmark = pytest.mark.gpu

SHAPES = [(32, 8, 128), (16, 4, 256), (8, 1, 256), (32, 8, 64)]


def poison_outside(case: W.Case) -> W.Case:
    """Sets every cache row that no token of the case attends to NaN."""
    keep = torch.zeros(case.num_blocks, case.block_size, dtype=torch.bool)
    for t in range(case.tokens):
        first, last = O.attended(case.seq_lens[t], case.window)
        table = case.tables[case.table_rows[t]]
        for pos in range(first, last):
            keep[int(table[pos // case.block_size]), pos % case.block_size] = True
    nan = torch.tensor(float("nan"))
    case.key = torch.where(keep[:, :, None, None], case.key, nan)
    case.value = torch.where(keep[:, :, None, None], case.value, nan)
    return case


def check(case, layout="triton", **kw):
    out, d, before = run(case, layout, **kw)
    assert torch.isfinite(out).all()
    assert_close(out, oracle_out(case))
    exp = expected_raw(case, layout, before, oracle_rows(case))
    assert torch.equal(d["raw"].cpu().view(torch.int16), exp.view(torch.int16))


@pytest.mark.parametrize("splits", [1, 4, 16])
@pytest.mark.parametrize("window", [0, 200])
@pytest.mark.parametrize("shape", SHAPES)
def test_single_token(shape, window, splits):
    nh, nkv, hd = shape
    case = W.single(seed=800 + hd + window, context=333, pool_blocks=30, num_heads=nh,
                    num_kv_heads=nkv, head_dim=hd, window=window)
    check(poison_outside(case), splits=splits)


@pytest.mark.parametrize("shape", SHAPES)
def test_batched_with_padding(shape):
    nh, nkv, hd = shape
    case = W.batched(seed=810 + hd, lens=[0, 15, 16, 17, 333, 700, 1030, 2], num_heads=nh,
                     num_kv_heads=nkv, head_dim=hd, window=300)
    case.seq_lens[0] = 0
    check(poison_outside(case), splits=8)


@pytest.mark.parametrize("shape", SHAPES)
def test_shared_wavefront(shape):
    nh, nkv, hd = shape
    case = W.wavefront(seed=820 + hd, prompt=450, generated=5, tokens=4, num_heads=nh,
                       num_kv_heads=nkv, head_dim=hd, window=100)
    check(poison_outside(case), splits=4)


@pytest.mark.parametrize("layout", ["unbind", "bench"])
def test_other_layouts_256(layout):
    case = W.single(seed=830, context=519, pool_blocks=40, num_heads=16, num_kv_heads=4,
                    head_dim=256, window=301)
    check(poison_outside(case), layout=layout, splits=8)


@pytest.mark.parametrize("shape", [(32, 8, 128), (16, 4, 256)])
def test_out_of_range_block_is_reported(shape):
    nh, nkv, hd = shape
    case = W.single(seed=840, context=300, pool_blocks=30, num_heads=nh, num_kv_heads=nkv,
                    head_dim=hd)
    d = W.to_device(case, "triton", "cuda")
    bad = d["tables"].clone()
    bad[0, 3] = 10_000_000  # far outside the 30-block pool
    attn = DecodeAttention(nh, nkv, hd, torch.device("cuda"))
    attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                  d["key"], d["value"], bad[0], d["seq_lens"][0:1], 0, case.scale,
                  d["gate"][0], d["out"][0])
    torch.cuda.synchronize()
    assert attn.fetch_errors() & 1  # DORY_DEVERR_BLOCK_OOB
    assert attn.fetch_errors() == 0
