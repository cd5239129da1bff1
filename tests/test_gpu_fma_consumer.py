"""The CUDA-core consumer (DecodeAttention(consumer="fma"), DORY_FLAG_FMA_CONSUMER) against
the reference semantics, to the same bar as the tensor-core kernel.

The variant replaces only the score and P.V dot products of each 16-row chunk (FP32 FMAs and
a transposing butterfly instead of mma.sync tiles); the ring, the q/k normalisation, the
append, the split merge and the nibble-major output are the shared kernel's.  So the checks
are the tensor-core kernel's: the golden outputs of the reference's own eager code within
2e-2 abs / 1e-2 rel, the whole pool bit for bit after the append, NaN rows outside the
attended range, split layouts, windows, padding tokens, and agreement with the tensor-core
path on random cases at the configuration-1 shape (32q/8kv x 128).  Shapes the variant does
not cover (more than 4 query heads per KV head, 64/256-dim heads, shared-cache calls) are
refused before any launch.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import specs
import workloads as W
from dory_decode_attention import DecodeAttention
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows, run
from test_gpu_edge_rows import poison_outside

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = specs.specs()


def check_cache(case, layout, d, before):
    exp = expected_raw(case, layout, before, oracle_rows(case))
    got = d["raw"].cpu()
    assert torch.equal(got.view(torch.int16), exp.view(torch.int16)), \
        f"{int((got.view(torch.int16) != exp.view(torch.int16)).sum())} cache elements differ"


@pytest.mark.parametrize("layout", W.LAYOUTS)
@pytest.mark.parametrize("name", ["config1", "single_window", "batched"])
def test_golden(name, layout):
    case = CASES[name]()
    out, d, before = run(case, layout, consumer="fma")
    ref = torch.from_numpy(np.load(GOLDEN / f"{name}.npz")["out"])
    assert_close(out, ref)
    check_cache(case, layout, d, before)


@pytest.mark.parametrize("splits,min_bps", [(1, 1), (3, 1), (16, 1), (37, 1), (64, 1),
                                            (148, 1), (8, 4)])
def test_split_layouts(splits, min_bps):
    case = CASES["config1"]()
    out, d, before = run(case, "triton", splits=splits, min_blocks_per_split=min_bps,
                         consumer="fma")
    ref = torch.from_numpy(np.load(GOLDEN / "config1.npz")["out"])
    assert_close(out, ref)
    check_cache(case, "triton", d, before)


@pytest.mark.parametrize("shape", [(32, 8, 128), (8, 4, 128), (4, 4, 128), (6, 2, 128)])
@pytest.mark.parametrize("window", [0, 200])
@pytest.mark.parametrize("splits", [1, 4, 16])
def test_rows_outside_range_are_nan(shape, window, splits):
    nh, nkv, hd = shape
    case = W.single(seed=900 + nh + window, context=333, pool_blocks=30, num_heads=nh,
                    num_kv_heads=nkv, head_dim=hd, window=window)
    case = poison_outside(case)
    out, d, before = run(case, "triton", splits=splits, consumer="fma")
    assert torch.isfinite(out).all()
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_batched_with_padding():
    case = W.batched(seed=910, lens=[0, 15, 16, 17, 333, 700, 1030, 2], window=300)
    case.seq_lens[0] = 0
    case = poison_outside(case)
    out, d, before = run(case, "triton", splits=8, consumer="fma")
    assert torch.isfinite(out).all()
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


@pytest.mark.parametrize("seed", range(6))
def test_agrees_with_tensor_core_path(seed):
    g = torch.Generator().manual_seed(seed)
    context = int(torch.randint(1, 3000, (1,), generator=g))
    window = [0, 1024, 77][seed % 3]
    case = W.single(seed=950 + seed, context=context, pool_blocks=context // 16 + 20,
                    window=window)
    splits = [1, 8, 32][seed % 3]
    out_mma, _, _ = run(case, "triton", splits=splits)
    out_fma, d, before = run(case, "triton", splits=splits, consumer="fma")
    torch.testing.assert_close(out_fma, out_mma, atol=2e-2, rtol=1e-2)
    assert_close(out_fma, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_non_raw_call():
    case = CASES["config1"]()
    d = W.to_device(case, "triton", "cuda")
    dev = torch.device("cuda")
    outs = []
    for consumer in ("mma", "fma"):
        attn = DecodeAttention(32, 8, 128, dev, splits=16, consumer=consumer)
        q = d["qk"][0, :32 * 128].to(torch.bfloat16)
        out = torch.empty_like(d["out"][0])
        attn(q, d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], 0, case.scale,
             d["gate"][0], out)
        torch.cuda.synchronize()
        attn.check_errors()
        outs.append(out.cpu())
    torch.testing.assert_close(outs[1], outs[0], atol=2e-2, rtol=1e-2)


@pytest.mark.parametrize("shape", [(32, 4, 128), (16, 4, 256), (8, 2, 64)])
def test_unsupported_shapes_are_refused(shape):
    nh, nkv, hd = shape
    case = W.single(seed=960, context=100, pool_blocks=10, num_heads=nh, num_kv_heads=nkv,
                    head_dim=hd)
    with pytest.raises(NotImplementedError):
        run(case, "triton", consumer="fma")


def test_shared_cache_is_refused():
    case = W.wavefront(seed=961, prompt=100, generated=0, tokens=2)
    with pytest.raises(NotImplementedError):
        run(case, "triton", consumer="fma")
