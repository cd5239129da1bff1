"""Parity of the split merge at small split counts (2-16, the latency-bound range), with
splits left empty by the layout, edge lengths, padding requests, shared-cache wavefronts of
16 tokens, small batches, determinism and CUDA-graph replay with and without programmatic
dependent launch.  Outputs within the bf16 bar (2e-2 abs / 1e-2 rel) and caches bit for bit.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import specs
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows, run

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = specs.specs()


def golden(name):
    return torch.from_numpy(np.load(GOLDEN / f"{name}.npz")["out"])


def check_cache(case, layout, d, before):
    exp = expected_raw(case, layout, before, oracle_rows(case))
    got = d["raw"].cpu()
    assert torch.equal(got.view(torch.int16), exp.view(torch.int16))


@pytest.mark.parametrize("splits", [2, 5, 8, 9, 12, 16])
@pytest.mark.parametrize("name", ["config1", "single_window", "wavefront", "batched",
                                  "edge_17_w0", "edge_1025_w1024"])
def test_splits_split_counts(name, splits):
    case = CASES[name]()
    out, d, before = run(case, "triton", splits=splits)
    assert_close(out, golden(name))
    check_cache(case, "triton", d, before)


@pytest.mark.parametrize("layout", ["unbind", "bench"])
def test_splits_layouts(layout):
    case = CASES["config1"]()
    out, d, before = run(case, layout, splits=16)
    assert_close(out, golden("config1"))
    check_cache(case, layout, d, before)


def test_splits_small_batch_with_padding():
    case = W.batched(seed=90, lens=[0, 1, 15, 16, 17, 300, 1023, 1024, 1025, 2000, 31, 700,
                                    4000, 2, 64, 129])
    case.seq_lens[0] = 0
    case.seq_lens[9] = 0
    out, d, before = run(case, "triton", splits=4)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[9]) == 0
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_splits_shared_wavefront_16_tokens():
    case = W.wavefront(seed=91, prompt=1500, generated=20, tokens=16)
    out, d, before = run(case, "triton", splits=16)
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_splits_repeat_is_deterministic():
    case = CASES["config1"]()
    a, _, _ = run(case, "triton", splits=16)
    b, _, _ = run(case, "triton", splits=16)
    assert torch.equal(a, b)


@pytest.mark.parametrize("overlap", [False, True])
def test_splits_graph_replay(overlap):
    cases = [W.single(seed=95 + i, context=300 + 211 * i, pool_blocks=60, window=512 * (i % 2))
             for i in range(4)]
    ds = [W.to_device(c, "triton", "cuda") for c in cases]
    attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=16, overlap_launch=overlap)

    def chain():
        for c, d in zip(cases, ds):
            attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], c.sqk_factor, EPS, d["slots"][0:1],
                          d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], c.window,
                          c.scale, d["gate"][0], d["out"][0])

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = [d["out"].clone() for d in ds]
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain()
    for _ in range(3):
        for d in ds:
            d["out"].fill_(float("nan"))
        g.replay()
    torch.cuda.synchronize()
    attn.check_errors()
    for d, e, c in zip(ds, eager, cases):
        assert torch.equal(d["out"], e)
        assert_close(d["out"].cpu(), oracle_out(c))
