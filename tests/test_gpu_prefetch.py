"""The L2 prefetch distance (DecodeAttention(prefetch_chunks=...), DoryDecodeParams.
prefetch_chunks) changes when a CTA's K/V chunks start their DRAM reads, never the
arithmetic: outputs and the cache pool are the same to the bit for every setting, in plain
and in overlapped (programmatic dependent) launches, including a chain of overlapped calls
replayed from a CUDA graph, where the automatic setting prefetches each CTA's whole range."""

from __future__ import annotations

import pytest
import torch

import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close, oracle_out, run

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hd,nh,nkv", [(128, 32, 8), (256, 16, 4), (64, 16, 16)])
def test_prefetch_distance_changes_no_bits(hd, nh, nkv):
    case = W.single(seed=90 + hd, context=5000, pool_blocks=400, num_heads=nh, num_kv_heads=nkv,
                    head_dim=hd)
    outs = []
    for pf in (-1, 0, 1, 5, 1000):
        out, d, _ = run(case, "triton", splits=8, prefetch_chunks=pf)
        outs.append((out, d["raw"].cpu()))
    assert_close(outs[0][0], oracle_out(case))
    for out, raw in outs[1:]:
        assert torch.equal(out, outs[0][0])
        assert torch.equal(raw.view(torch.int16), outs[0][1].view(torch.int16))


@pytest.mark.parametrize("prefetch", [0, -1, 2])
def test_overlapped_chain_in_a_graph_matches_plain_launches(prefetch):
    """A chain of calls, each a programmatic dependent of the previous one (automatic
    prefetch: every chunk of a CTA's range before it waits), captured in a CUDA graph and
    replayed: the same bits as the same calls launched plainly."""
    cases = [W.single(seed=95 + i, context=700 + 900 * i, pool_blocks=250) for i in range(4)]
    results = {}
    for overlap in (False, True):
        devs = [W.to_device(c, "triton", "cuda") for c in cases]
        attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=12,
                               overlap_launch=overlap, prefetch_chunks=prefetch)

        def chain():
            for c, d in zip(cases, devs):
                attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], c.sqk_factor, EPS,
                              d["slots"][0:1], d["key"], d["value"], d["tables"][0],
                              d["seq_lens"][0:1], c.window, c.scale, d["gate"][0], d["out"][0])

        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            chain()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            chain()
        for d in devs:
            d["out"].zero_()
        g.replay()
        torch.cuda.synchronize()
        attn.check_errors()
        results[overlap] = [d["out"].cpu() for d in devs]
        del g
    for a, b, c in zip(results[False], results[True], cases):
        assert torch.equal(a, b)
        assert_close(a, oracle_out(c))
