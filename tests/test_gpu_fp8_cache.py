"""FP8 (e4m3) KV caches (DecodeAttention(kv_cache_dtype="fp8"), DORY_DTYPE_FP8_E4M3): the
kernel against the oracle's restatement of the format (oracle.e4m3_quantize /
e4m3_dequantize / *_fp8), which vLLM's fp8 kv_cache_dtype defines and the reference does not
have (parity unpinned: there is no reference output to compare with).

* Outputs within the bf16 bar (2e-2 abs / 1e-2 rel) of the oracle's FP32 attention over the
  dequantised cache, the new token's row included as the quantised values it appends.
* The caches bit for bit: only the appended slots change, and they hold e4m3(bf16(k) /
  k_scale) and e4m3(bf16(v) / v_scale) exactly.
* Layouts (K and V interleaved per row, or separate), 128- and 256-dim heads, 4 or 8 query
  heads per KV head, windows, split layouts, padding tokens, NaN bytes outside the attended
  ranges, scales other than 1, shared caches, the non-raw call; and agreement with the bf16
  path on a cache whose bf16 values are the dequantised ones (power-of-two scales keep them
  exact).
"""

from __future__ import annotations

import pytest
import torch

import dory_oracle as O
import specs
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close

pytestmark = pytest.mark.gpu

CASES = specs.specs()
DEV = torch.device("cuda")


def run_fp8(case: W.Case, layout="triton", splits=16, scales=(1.0, 1.0), window=None,
            min_blocks_per_split=1):
    """Raw-mode call(s) of `case` over e4m3 caches; returns (out [T, 8, Q/8], expected out,
    device key/value bytes [blocks, B, NKV, HD], expected bytes)."""
    ks, vs = scales
    dev = torch.device("cuda")
    d = W.to_device(case, layout, dev, kv8=scales)
    T = case.tokens
    attn = DecodeAttention(case.num_heads, case.num_kv_heads, case.head_dim, dev, splits=splits,
                           max_tokens=max(T, 1), kv_cache_dtype="fp8",
                           min_blocks_per_split=min_blocks_per_split)
    if T == 1:
        attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                      d["key"], d["value"], d["tables"][case.table_rows[0]], d["seq_lens"][0:1],
                      case.window, case.scale, d["gate"][0], d["out"][0], k_scale=ks,
                      v_scale=vs)
    else:
        attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS,
                            d["cache_offsets"], d["key"], d["value"], d["tables"],
                            d["table_offsets"], d["seq_lens"], case.window, case.scale,
                            d["gate"], d["out"], shared_cache=case.shared, k_scale=ks,
                            v_scale=vs)
    torch.cuda.synchronize()
    attn.check_errors()
    key8, value8 = W.e4m3_bytes(case.key, ks), W.e4m3_bytes(case.value, vs)
    if case.shared:  # write-all-first over one cache (oracle.multi_from_raw_fp8)
        width = case.tables.shape[1]
        want = O.multi_from_raw_fp8(
            case.qk, case.v, case.sqk, case.sqk_factor, EPS, torch.zeros(T, dtype=torch.int64),
            key8.view(-1), value8.view(-1), tuple(key8.shape), key8.stride(),
            case.tables.reshape(-1), torch.tensor([r * width for r in case.table_rows]),
            case.seq_lens, case.window, case.scale, case.gate, case.num_heads,
            case.num_kv_heads, ks, vs, shared_cache=True)
        return d["out"].cpu(), want, (d["key"].cpu(), d["value"].cpu()), (key8, value8)
    want = []
    for t in range(T):
        want.append(O.from_raw_fp8(case.qk[t], case.v[t], case.sqk, case.sqk_factor, EPS,
                                   case.slot(t) if case.seq_lens[t] > 0 else -1, key8, value8,
                                   case.tables[case.table_rows[t]], case.seq_lens[t],
                                   case.window, case.scale, case.gate[t], case.num_heads,
                                   case.num_kv_heads, ks, vs))
    return (d["out"].cpu(), torch.stack(want), (d["key"].cpu(), d["value"].cpu()),
            (key8, value8))


def check(case, **kw):
    out, want, (k, v), (k8, v8) = run_fp8(case, **kw)
    assert torch.isfinite(out).all()
    assert_close(out, want)
    assert torch.equal(k, k8), f"{int((k != k8).sum())} key bytes differ"
    assert torch.equal(v, v8), f"{int((v != v8).sum())} value bytes differ"


@pytest.mark.parametrize("scales", [(1.0, 1.0), (0.25, 0.5), (0.037, 1.7)])
@pytest.mark.parametrize("layout", W.LAYOUTS)
@pytest.mark.parametrize("name", ["config1", "single_window", "dory_shape", "gqa8"])
def test_raw_single_token(name, layout, scales):
    check(CASES[name](), layout=layout, scales=scales)


@pytest.mark.parametrize("splits,mbps", [(1, 1), (3, 1), (16, 1), (37, 1), (64, 1), (148, 1),
                                         (8, 4)])
def test_split_layouts(splits, mbps):
    check(CASES["config1"](), splits=splits, min_blocks_per_split=mbps, scales=(0.5, 0.5))


@pytest.mark.parametrize("hd", [128, 256])
def test_batched_with_padding_and_window(hd):
    nh, nkv = (32, 8) if hd == 128 else (16, 4)
    case = W.batched(seed=1200 + hd, lens=[0, 15, 16, 17, 333, 700, 1030, 2], num_heads=nh,
                     num_kv_heads=nkv, head_dim=hd, window=300)
    case.seq_lens[0] = 0
    check(case, splits=8, scales=(0.25, 0.25))


@pytest.mark.parametrize("hd", [128, 256])
def test_nan_bytes_outside_the_attended_rows(hd):
    nh, nkv = (32, 8) if hd == 128 else (16, 4)
    case = W.single(seed=1210 + hd, context=333, pool_blocks=30, num_heads=nh,
                    num_kv_heads=nkv, head_dim=hd, window=200)
    dev = torch.device("cuda")
    keep = torch.zeros(case.num_blocks, case.block_size, dtype=torch.bool)
    first, last = O.attended(case.seq_lens[0], case.window)
    for pos in range(first, last - 1):  # the new row is appended by the call
        keep[int(case.tables[0][pos // case.block_size]), pos % case.block_size] = True
    d = W.to_device(case, "triton", dev, kv8=(1.0, 1.0))
    nan = torch.tensor(0x7F, dtype=torch.uint8)  # e4m3 NaN
    k8 = torch.where(keep[:, :, None, None], W.e4m3_bytes(case.key, 1.0), nan)
    v8 = torch.where(keep[:, :, None, None], W.e4m3_bytes(case.value, 1.0), nan)
    d["key"].copy_(k8)
    d["value"].copy_(v8)
    attn = DecodeAttention(nh, nkv, hd, dev, splits=4, kv_cache_dtype="fp8")
    attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                  d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], case.window,
                  case.scale, d["gate"][0], d["out"][0])
    torch.cuda.synchronize()
    attn.check_errors()
    want = O.from_raw_fp8(case.qk[0], case.v[0], case.sqk, case.sqk_factor, EPS, case.slot(0),
                          k8.clone(), v8.clone(), case.tables[0], case.seq_lens[0], case.window,
                          case.scale, case.gate[0], nh, nkv, 1.0, 1.0)
    out = d["out"][0].cpu()
    assert torch.isfinite(out).all()
    assert_close(out, want)


def test_call_path_matches_bf16_path_on_the_same_values():
    """Non-raw calls: an e4m3 cache with power-of-two scales against a bf16 cache holding the
    dequantised values (exact in bf16); the kernels differ only in their MMA operand type."""
    case = CASES["config1"]()
    dev = torch.device("cuda")
    ks, vs = 0.25, 2.0
    d8 = W.to_device(case, "triton", dev, kv8=(ks, vs))
    d16 = W.to_device(case, "triton", dev)
    d16["key"].copy_(O.e4m3_dequantize(d8["key"].cpu().contiguous(), ks).to(torch.bfloat16))
    d16["value"].copy_(O.e4m3_dequantize(d8["value"].cpu().contiguous(), vs).to(torch.bfloat16))
    q = O.raw_qkv(case.qk[0], case.v[0], case.sqk, case.sqk_factor, EPS, 32, 8, 128)[0]
    q = q.reshape(-1).to(dev)
    outs = []
    for d, kind in ((d8, "fp8"), (d16, "auto")):
        attn = DecodeAttention(32, 8, 128, dev, splits=16, kv_cache_dtype=kind)
        attn(q, d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], 0, case.scale,
             d["gate"][0], d["out"][0], k_scale=ks, v_scale=vs)
        torch.cuda.synchronize()
        attn.check_errors()
        outs.append(d["out"][0].cpu())
    torch.testing.assert_close(outs[0], outs[1], atol=1e-5, rtol=1e-4)
    want = O.call_fp8(q.cpu(), d8["key"].cpu().contiguous(), d8["value"].cpu().contiguous(),
                      case.tables[0], case.seq_lens[0], 0, case.scale, case.gate[0], 32, ks, vs)
    assert_close(outs[0], want)


@pytest.mark.parametrize("shape", [(8, 2, 64), (32, 2, 128)])
def test_unsupported_shapes_are_refused(shape):
    nh, nkv, hd = shape
    case = W.single(seed=1220, context=100, pool_blocks=10, num_heads=nh, num_kv_heads=nkv,
                    head_dim=hd)
    with pytest.raises(NotImplementedError):
        run_fp8(case)


@pytest.mark.parametrize("hd", [128, 256])
@pytest.mark.parametrize("tokens", [2, 4, 6])
def test_shared_wavefront(tokens, hd):
    """Shared ("last_loop") caches: tokens at consecutive positions read each other's new
    rows as e4m3 bytes (write-all-first); groups of 8 / G tokens per CTA, more than four sub
    tokens, each CTA appending its own group's rows."""
    nh, nkv = (32, 8) if hd == 128 else (16, 4)
    case = W.wavefront(seed=1260 + tokens + hd, prompt=450, generated=3, tokens=tokens,
                       num_heads=nh, num_kv_heads=nkv, head_dim=hd)
    check(case, splits=8, scales=(0.5, 0.25))


def test_shared_wavefront_window_and_split_layouts():
    case = W.wavefront(seed=1270, prompt=700, tokens=4, window=300)
    for splits in (1, 16):
        check(case, splits=splits, scales=(1.0, 2.0))


def test_shared_with_distinct_tables_falls_back_per_token():
    """Tokens reading one pool through different table rows: processed per token, every new
    row still substituted where it aliases another token's block."""
    case = W.wavefront(seed=1271, prompt=300, tokens=4)
    case.tables = torch.cat([case.tables, case.tables])
    case.table_rows = [0, 0, 1, 1]
    check(case, splits=4, scales=(0.25, 0.5))


def test_bad_scale_and_dtype_are_refused():
    case = CASES["config1"]()
    with pytest.raises(ValueError):
        run_fp8(case, scales=(0.0, 1.0))
    with pytest.raises(ValueError):
        DecodeAttention(32, 8, 128, torch.device("cuda"), kv_cache_dtype="fp16")
    d = W.to_device(case, "triton", "cuda")  # bf16 caches given to an fp8 instance
    attn = DecodeAttention(32, 8, 128, torch.device("cuda"), kv_cache_dtype="fp8")
    with pytest.raises(ValueError):
        attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                      d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], 0, case.scale,
                      d["gate"][0], d["out"][0])


@pytest.mark.parametrize("shape", [(32, 8, 128), (16, 4, 256)])
def test_out_of_range_block_is_reported_and_left_out(shape):
    """A block id beyond the pool is reported (DORY_DEVERR_BLOCK_OOB), never dereferenced, and
    its 16 positions drop out of the softmax: the output equals the oracle's over the table
    without that entry (window 0, so the positions' order does not matter)."""
    nh, nkv, hd = shape
    case = W.single(seed=1230 + hd, context=300, pool_blocks=30, num_heads=nh,
                    num_kv_heads=nkv, head_dim=hd)
    dev = torch.device("cuda")
    ks, vs = 0.5, 0.25
    d = W.to_device(case, "triton", dev, kv8=(ks, vs))
    q = O.raw_qkv(case.qk[0], case.v[0], case.sqk, case.sqk_factor, EPS, nh, nkv, hd)[0]
    q = q.reshape(-1).to(dev)
    bad = d["tables"][0].clone()
    bad[3] = 10_000_000  # far outside the 30-block pool
    attn = DecodeAttention(nh, nkv, hd, dev, splits=4, kv_cache_dtype="fp8")
    attn(q, d["key"], d["value"], bad, d["seq_lens"][0:1], 0, case.scale, d["gate"][0],
         d["out"][0], k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    assert attn.fetch_errors() & 1  # DORY_DEVERR_BLOCK_OOB
    out = d["out"][0].cpu()
    assert torch.isfinite(out).all()
    table = case.tables[0]
    kept = torch.cat([table[:3], table[4:]])
    want = O.call_fp8(q.cpu(), d["key"].cpu().contiguous(), d["value"].cpu().contiguous(), kept,
                      case.seq_lens[0] - case.block_size, 0, case.scale, case.gate[0], nh, ks,
                      vs)
    assert_close(out, want)


@pytest.mark.parametrize("splits,sumsq", [(16, False), (16, True), (2, False), (2, True)])
def test_large_batch(splits, sumsq):
    """64 sequences x 8 KV heads: with 16 splits (8,192 CTAs) the 4-CTA-per-SM build of the
    128-dim FP8 kernel (grids of 2 or more waves), with 2 splits (1,024 CTAs) the 3-CTA build
    with the last-arriving split merging; with and without the output's sum of squares;
    padding, a window, outputs, statistic and cache bytes against the oracle."""
    case = W.batched(seed=1240, num_seqs=64, window=700)
    case.seq_lens[5] = 0
    ks, vs = 0.5, 0.25
    dev = torch.device("cuda")
    d = W.to_device(case, "triton", dev, kv8=(ks, vs))
    T = case.tokens
    attn = DecodeAttention(32, 8, 128, dev, splits=splits, max_tokens=T, kv_cache_dtype="fp8")
    ss = torch.full((T,), -1.0, device=dev) if sumsq else None
    attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS, d["cache_offsets"],
                        d["key"], d["value"], d["tables"], d["table_offsets"], d["seq_lens"],
                        case.window, case.scale, d["gate"], d["out"], out_sumsq=ss,
                        k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    attn.check_errors()
    key8, value8 = W.e4m3_bytes(case.key, ks), W.e4m3_bytes(case.value, vs)
    want = torch.stack([
        O.from_raw_fp8(case.qk[t], case.v[t], case.sqk, case.sqk_factor, EPS,
                       case.slot(t) if case.seq_lens[t] > 0 else -1, key8, value8,
                       case.tables[case.table_rows[t]], case.seq_lens[t], case.window,
                       case.scale, case.gate[t], 32, 8, ks, vs) for t in range(T)])
    out = d["out"].cpu()
    assert torch.isfinite(out).all()
    assert_close(out, want)
    assert torch.equal(d["key"].cpu(), key8)
    assert torch.equal(d["value"].cpu(), value8)
    if sumsq:
        torch.testing.assert_close(ss.cpu(), out.double().square().sum((1, 2)).float(),
                                   rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("hd", [128, 256])
def test_shared_wavefront_with_sumsq(hd):
    """The recurrent block's call: a shared-cache wavefront with the output's sum of squares
    (out_sumsq) over an e4m3 cache; outputs, statistic and bytes against the oracle."""
    nh, nkv = (32, 8) if hd == 128 else (16, 4)
    case = W.wavefront(seed=1280 + hd, prompt=900, generated=2, tokens=4, num_heads=nh,
                       num_kv_heads=nkv, head_dim=hd)
    ks, vs = 0.5, 0.5
    d = W.to_device(case, "triton", DEV, kv8=(ks, vs))
    attn = DecodeAttention(nh, nkv, hd, DEV, splits=8, max_tokens=4, kv_cache_dtype="fp8")
    ss = torch.full((4,), -1.0, device=DEV)
    attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS, d["cache_offsets"],
                        d["key"], d["value"], d["tables"], d["table_offsets"], d["seq_lens"],
                        case.window, case.scale, d["gate"], d["out"], shared_cache=True,
                        out_sumsq=ss, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    attn.check_errors()
    key8, value8 = W.e4m3_bytes(case.key, ks), W.e4m3_bytes(case.value, vs)
    want = O.multi_from_raw_fp8(
        case.qk, case.v, case.sqk, case.sqk_factor, EPS, torch.zeros(4, dtype=torch.int64),
        key8.view(-1), value8.view(-1), tuple(key8.shape), key8.stride(),
        case.tables.reshape(-1), torch.zeros(4, dtype=torch.int64), case.seq_lens,
        case.window, case.scale, case.gate, nh, nkv, ks, vs, shared_cache=True)
    out = d["out"].cpu()
    assert_close(out, want)
    assert torch.equal(d["key"].cpu(), key8)
    assert torch.equal(d["value"].cpu(), value8)
    torch.testing.assert_close(ss.cpu(), out.double().square().sum((1, 2)).float(),
                               rtol=1e-5, atol=1e-6)
