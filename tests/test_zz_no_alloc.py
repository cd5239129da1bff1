"""dory_decode_attention_static_scratch: decode attention for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc: serving engines that hand the whole
device to their own KV-cache allocator up front, so nothing is left for a second one, and C
or other foreign-function hosts that have no device allocator of their own.  For them the
library keeps its split partials and merge counters in a 4 MiB device array of its own
instead of a caller-owned scratch buffer, and keeps the device error word there too
(read back with dory_decode_static_scratch_fetch_errors).

The first test calls that entry point through the C ABI (ctypes, as a foreign host would)
twice in a row — a single-token call and a four-token shared-cache wavefront call — and
checks each output against the existing entry point's (DecodeAttention with its own scratch)
and against the golden outputs of the reference's own eager code for the same two inputs,
within the parity tolerance of the other tests (2e-2 abs / 1e-2 rel), and the appended cache
rows bit for bit.  The second test makes the kernel's bounds check record an error (an
append slot outside the cache, made on the host) and reads it back through the new export.
The file sorts last so a failure here stops a `-x` run only after every other test ran; each
test also passes on its own in a fresh process.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

import _native
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import ATOL, RTOL

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _params(case: W.Case, d: dict, splits: int) -> _native.DoryDecodeParams:
    """Fills the C struct for a raw-mode call of `case` on the device tensors `d`."""
    single = case.tokens == 1 and not case.shared
    p = _native.DoryDecodeParams()
    p.q, p.v, p.sqk = d["qk"].data_ptr(), d["v"].data_ptr(), d["sqk"].data_ptr()
    p.key_cache, p.value_cache = d["key"].data_ptr(), d["value"].data_ptr()
    p.seq_lens, p.gate = d["seq_lens"].data_ptr(), d["gate"].data_ptr()
    p.out_nibble_major = d["out"].data_ptr()
    if single:
        p.slot_mapping = d["slots"].data_ptr()
        p.block_table = d["tables"][case.table_rows[0]].data_ptr()
        p.flags = _native.FLAG_RAW_QKV
    else:
        p.block_table = d["tables"].data_ptr()
        p.block_table_offsets = d["table_offsets"].data_ptr()
        p.cache_offsets = d["cache_offsets"].data_ptr()
        p.flags = _native.FLAG_RAW_QKV | _native.FLAG_MULTI_TOKEN
        if case.shared:
            p.flags |= _native.FLAG_SHARED_CACHE
    p.scratch, p.scratch_bytes = None, 0  # ignored by the static-scratch entry point
    key = d["key"]
    p.stride_block, p.stride_offset, p.stride_head = key.stride(0), key.stride(1), key.stride(2)
    p.num_cache_blocks = key.shape[0]
    p.softmax_scale, p.sqk_factor, p.eps = case.scale, case.sqk_factor, EPS
    p.num_tokens, p.num_heads, p.num_kv_heads = case.tokens, case.num_heads, case.num_kv_heads
    p.head_dim, p.block_size, p.window = case.head_dim, case.block_size, case.window
    p.splits, p.blocks_per_tile, p.min_blocks_per_split = splits, 1, 1
    p.max_tokens, p.sqk_dtype = case.tokens, _native.DTYPE_BF16
    return p


def _with_caller_scratch(case: W.Case, splits: int):
    """Output and cache of the existing entry point (DecodeAttention owns its scratch)."""
    d = W.to_device(case, "triton", "cuda")
    attn = DecodeAttention(case.num_heads, case.num_kv_heads, case.head_dim,
                           torch.device("cuda"), splits=splits, max_tokens=case.tokens)
    if case.tokens == 1 and not case.shared:
        attn.from_raw(d["qk"][0], d["v"][0], d["sqk"], case.sqk_factor, EPS, d["slots"][0:1],
                      d["key"], d["value"], d["tables"][0], d["seq_lens"][0:1], case.window,
                      case.scale, d["gate"][0], d["out"][0])
    else:
        attn.multi_from_raw(d["qk"], d["v"], d["sqk"], case.sqk_factor, EPS,
                            d["cache_offsets"], d["key"], d["value"], d["tables"],
                            d["table_offsets"], d["seq_lens"], case.window, case.scale,
                            d["gate"], d["out"], shared_cache=case.shared)
    torch.cuda.synchronize()
    attn.check_errors()
    return d["out"].cpu(), d["raw"].cpu()


def _static_errors(lib, clear: bool) -> int:
    flags = ctypes.c_uint32(0xFFFFFFFF)
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(lib.dory_decode_static_scratch_fetch_errors(ctypes.byref(flags), int(clear),
                                                              stream))
    return flags.value


def test_static_scratch_matches_caller_scratch_and_goldens_two_calls_in_a_row():
    lib = _native.load()
    splits = 32
    # the inputs of the golden cases "config1" and "wavefront" (tests/golden/specs.py)
    cases = [W.single(seed=0, context=640, pool_blocks=64),
             W.wavefront(seed=1, prompt=700, generated=37, tokens=4)]
    goldens = [torch.from_numpy(np.load(GOLDEN / f"{n}.npz")["out"])
               for n in ("config1", "wavefront")]
    expected = [_with_caller_scratch(c, splits) for c in cases]

    devs = [W.to_device(c, "triton", "cuda") for c in cases]
    params = [_params(c, d, splits) for c, d in zip(cases, devs)]
    stream = torch.cuda.current_stream().cuda_stream
    _static_errors(lib, clear=True)  # start from a clean error word
    for p in params:  # two calls back to back, sharing the library's one scratch array
        _native.check(lib.dory_decode_attention_static_scratch(ctypes.byref(p), stream))
    torch.cuda.synchronize()

    for (out_ref, raw_ref), golden, d in zip(expected, goldens, devs):
        out = d["out"].cpu()
        torch.testing.assert_close(out, out_ref, atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(out, golden, atol=ATOL, rtol=RTOL)
        assert torch.equal(d["raw"].cpu().view(torch.int16), raw_ref.view(torch.int16))
    assert _static_errors(lib, clear=False) == 0


def test_static_scratch_error_word_survives_calls_until_fetched():
    lib = _native.load()
    case = W.single(seed=71, context=300, pool_blocks=30)
    d = W.to_device(case, "triton", "cuda")
    before = d["raw"].clone()
    stream = torch.cuda.current_stream().cuda_stream
    _static_errors(lib, clear=True)
    p = _params(case, d, splits=16)
    # an append slot in block 30 of a 30-block cache: the kernel's bounds check records
    # DORY_DEVERR_SLOT_OOB and skips the write
    bad = torch.tensor([30 * 16 + 5], dtype=torch.int64, device="cuda")
    p.slot_mapping = bad.data_ptr()
    _native.check(lib.dory_decode_attention_static_scratch(ctypes.byref(p), stream))
    # a second, valid call must not wipe the first call's error
    good = _params(case, d, splits=16)
    _native.check(lib.dory_decode_attention_static_scratch(ctypes.byref(good), stream))
    torch.cuda.synchronize()
    assert _static_errors(lib, clear=True) & _native.DEVERR_SLOT_OOB
    assert _static_errors(lib, clear=False) == 0  # cleared
    # the bad call wrote nothing; the good call appended its row at the case's own slot
    slot, B = case.slot(0), case.block_size
    after = d["raw"].cpu()
    changed = (after.view(torch.int16) != before.cpu().view(torch.int16))
    rows = changed.transpose(1, 2).any(dim=-1)  # [blocks, 16, kv_heads]
    assert rows.nonzero()[:, :2].unique(dim=0).tolist() == [[slot // B, slot % B]]


def test_static_scratch_rejects_calls_beyond_its_size():
    lib = _native.load()
    case = W.single(seed=0, context=640, pool_blocks=64)
    d = W.to_device(case, "triton", "cuda")
    p = _params(case, d, splits=32)
    p.max_tokens = 64  # 64 x 32 splits x 32 heads x 128 x 4 B of partials > 4 MiB
    status = lib.dory_decode_attention_static_scratch(ctypes.byref(p), None)
    assert status == _native.ERR_INVALID_ARGUMENT
    assert "static scratch" in lib.dory_decode_last_error().decode()
    p.max_tokens, p.splits, p.num_heads = 1 << 30, 1 << 30, 1 << 14  # the product overflows
    status = lib.dory_decode_attention_static_scratch(ctypes.byref(p), None)
    assert status == _native.ERR_INVALID_ARGUMENT
    assert "overflow" in lib.dory_decode_last_error().decode()
