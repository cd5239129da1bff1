"""Parity of large batched calls (64 sequences, thousands of (token, KV head, split) CTAs)
with the oracle, through DecodeAttention and the C ABI.

Outputs within the bf16 bar (2e-2 abs / 1e-2 rel) and a relative-L2 bound; the whole
cache pool bit for bit after the append.  Covers the three cache layouts, split counts and
minimum split sizes (many empty splits), windows, padding requests, edge lengths (1, 15-17,
block boundaries), cache offsets that are not whole blocks (copy path) mixed with whole-block
ones, repeat calls (the split counters reset themselves), CUDA-graph replay, overlapped
launches and the error word.
"""

from __future__ import annotations

import pytest
import torch

import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close, expected_raw, oracle_out, oracle_rows, run

pytestmark = pytest.mark.gpu

# Cached-context lengths with the edge values of the reference's tests among random ones.
EDGE = [0, 1, 14, 15, 16, 17, 31, 32, 33, 255, 256, 257, 1023, 1024, 1025, 1039, 2999]


def lens_for(seed: int, n: int = 64, hi: int = 1500) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    rnd = torch.randint(0, hi, (n - len(EDGE),), generator=g).tolist()
    return EDGE + rnd


def check_cache(case, layout, d, before):
    exp = expected_raw(case, layout, before, oracle_rows(case))
    got = d["raw"].cpu()
    assert torch.equal(got.view(torch.int16), exp.view(torch.int16)), \
        f"{int((got.view(torch.int16) != exp.view(torch.int16)).sum())} cache elements differ"


@pytest.mark.parametrize("layout", W.LAYOUTS)
@pytest.mark.parametrize("splits,min_bps", [(4, 1), (8, 64), (32, 1), (64, 8)])
def test_batch_batched_matches_oracle(layout, splits, min_bps):
    case = W.batched(seed=40 + splits, lens=lens_for(splits))
    out, d, before = run(case, layout, splits=splits, min_blocks_per_split=min_bps)
    assert_close(out, oracle_out(case))
    check_cache(case, layout, d, before)


@pytest.mark.parametrize("window", [1, 64, 1024])
def test_batch_windows(window):
    case = W.batched(seed=50 + window, lens=lens_for(window), window=window)
    out, d, before = run(case, "triton", splits=8)
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_batch_padding_requests():
    case = W.batched(seed=60, lens=lens_for(60))
    for t in (0, 5, 40, 63):
        case.seq_lens[t] = 0  # padding requests: zero output, nothing cached
    out, d, before = run(case, "triton", splits=8)
    for t in (0, 5, 40, 63):
        assert torch.count_nonzero(out[t]) == 0
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)


def test_batch_gqa8_and_head_dim_64():
    case = W.batched(seed=61, lens=lens_for(61, n=40), num_heads=64, num_kv_heads=8)
    out, d, before = run(case, "triton", splits=8)
    assert_close(out, oracle_out(case))
    check_cache(case, "triton", d, before)
    case = W.batched(seed=62, lens=lens_for(62), num_heads=32, num_kv_heads=8, head_dim=64)
    out, d, before = run(case, "unbind", splits=8)
    assert_close(out, oracle_out(case))
    check_cache(case, "unbind", d, before)


def test_batch_repeat_calls_are_identical():
    """The split counters reset themselves at the end of each launch."""
    case = W.batched(seed=63, lens=lens_for(63))
    d = W.to_device(case, "triton", "cuda")
    attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=8, max_tokens=case.tokens)
    outs = []
    for _ in range(4):
        attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS, d["cache_offsets"],
                            d["key"], d["value"], d["tables"], d["table_offsets"], d["seq_lens"],
                            case.window, case.scale, d["gate"], d["out"])
        outs.append(d["out"].clone())
    torch.cuda.synchronize()
    attn.check_errors()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert_close(outs[0].cpu(), oracle_out(case))


@pytest.mark.parametrize("overlap", [False, True])
def test_batch_graph_replay_and_overlap(overlap):
    """A chain of batched launches on distinct caches, captured in a CUDA graph (with and
    without programmatic dependent launch), matches eager calls bit for bit."""
    cases = [W.batched(seed=70 + i, lens=lens_for(70 + i, n=48), window=256 * (i % 2))
             for i in range(3)]
    results = []
    for use_graph in (False, True):
        ds = [W.to_device(c, "triton", "cuda") for c in cases]
        attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=8, max_tokens=48,
                               overlap_launch=overlap)

        def chain():
            for c, d in zip(cases, ds):
                attn.multi_from_raw(d["qk"], d["v"], d["sqk"], c.sqk_factor, EPS,
                                    d["cache_offsets"], d["key"], d["value"], d["tables"],
                                    d["table_offsets"], d["seq_lens"], c.window, c.scale,
                                    d["gate"], d["out"])

        if use_graph:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                chain()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            for d, c in zip(ds, cases):
                d["raw"].copy_(W.to_device(c, "triton", "cuda")["raw"])
                d["out"].fill_(float("nan"))
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                chain()
            g.replay()
        else:
            chain()
        torch.cuda.synchronize()
        attn.check_errors()
        results.append([(d["out"].cpu(), d["raw"].cpu()) for d in ds])
    for (o0, r0), (o1, r1) in zip(*results):
        assert torch.equal(o0, o1)
        assert torch.equal(r0.view(torch.int16), r1.view(torch.int16))
    for c, (o, _) in zip(cases, results[0]):
        assert_close(o, oracle_out(c))


def test_batch_cache_offsets_not_whole_blocks():
    """Per-token caches at element offsets that are not whole blocks (copy path) and at
    whole-block offsets (tensor path) in one call."""
    T, P = 64, 24
    cases = [W.single(seed=400 + t, context=(37 * t) % 360 + 1, pool_blocks=P) for t in range(T)]
    per = P * 8 * 16 * 256  # elements of one token's [P, 8, 16, 256] cache
    # odd tokens sit 8 elements past a block boundary
    offs = [t * (per + 32768) + (8 if t % 2 else 0) for t in range(T)]
    flat = torch.zeros(offs[-1] + per + 32768, dtype=torch.bfloat16, device="cuda")
    for t, c in enumerate(cases):
        raw_t = flat[offs[t]:offs[t] + per].view(P, 8, 16, 256)
        k, v = raw_t.transpose(1, 2).split(128, dim=-1)
        k.copy_(c.key.to(torch.bfloat16))
        v.copy_(c.value.to(torch.bfloat16))
    raw0 = flat[:per].view(P, 8, 16, 256)
    key, value = raw0.transpose(1, 2).split(128, dim=-1)
    cache_offsets = torch.tensor(offs, dtype=torch.int64, device="cuda")
    tables = torch.stack([c.tables[0] for c in cases]).cuda()
    table_offsets = torch.arange(T, dtype=torch.int64, device="cuda") * P
    qk = torch.stack([c.qk[0] for c in cases]).cuda()
    v_in = torch.stack([c.v[0] for c in cases]).cuda()
    gate = torch.stack([c.gate[0] for c in cases]).cuda()
    seq_lens = torch.tensor([c.seq_lens[0] for c in cases], dtype=torch.int32, device="cuda")
    sqk = cases[0].sqk.cuda()
    out = torch.full((T, 8, 512), float("nan"), device="cuda")
    before = [flat[offs[t]:offs[t] + per].view(P, 8, 16, 256).cpu() for t in range(T)]
    attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=4, max_tokens=T)
    attn.multi_from_raw(qk, v_in, sqk, 0.7, EPS, cache_offsets, key, value, tables,
                        table_offsets, seq_lens, 0, 128 ** -0.5, gate, out)
    torch.cuda.synchronize()
    attn.check_errors()
    for t, c in enumerate(cases):
        c.sqk = cases[0].sqk
        assert_close(out[t].cpu(), oracle_out(c)[0])
        exp = expected_raw(c, "triton", before[t], oracle_rows(c))
        got = flat[offs[t]:offs[t] + per].view(P, 8, 16, 256).cpu()
        assert torch.equal(got.view(torch.int16), exp.view(torch.int16)), t


def test_batch_out_of_range_block_is_reported_not_dereferenced():
    case = W.batched(seed=80, lens=lens_for(80))
    d = W.to_device(case, "triton", "cuda")
    bad = d["tables"].clone()
    bad[14, 2] = 50_000_000  # far outside the pool (sequence 14: 1025 cached rows)
    attn = DecodeAttention(32, 8, 128, torch.device("cuda"), splits=8, max_tokens=case.tokens)
    attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS, d["cache_offsets"],
                        d["key"], d["value"], bad, d["table_offsets"], d["seq_lens"],
                        case.window, case.scale, d["gate"], d["out"])
    torch.cuda.synchronize()
    assert attn.fetch_errors() & 1  # DORY_DEVERR_BLOCK_OOB
    # the other sequences are unaffected
    ref = oracle_out(case)
    keep = [t for t in range(case.tokens) if t != 14]
    assert_close(d["out"].cpu()[keep], ref[keep])
