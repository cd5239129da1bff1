"""dory_decode_attention_static_scratch: decode attention for callers that cannot allocate.

Some callers of this library cannot call cudaMalloc: code that enqueues work while a CUDA
graph is being captured in the global capture mode (allocation is an error there), serving
engines that reserved the whole device for their KV-cache allocator up front, and C or
other foreign-function hosts that have no device allocator of their own.  For them the
library keeps its split partials and merge counters in a 4 MiB device array of its own
instead of a caller-owned scratch buffer.

This test calls that entry point through the C ABI (ctypes, as a foreign host would) twice
in a row — a single-token call and a four-token shared-cache wavefront call — and checks
each output against the existing entry point's (DecodeAttention with its own scratch)
within the parity tolerance of the other tests, and the appended cache rows bit for bit.
The file sorts last so a failure here stops a `-x` run only after every other test ran.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import _native
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import ATOL, RTOL

pytestmark = pytest.mark.gpu


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


def test_static_scratch_matches_caller_scratch_two_calls_in_a_row():
    lib = _native.load()
    splits = 32
    cases = [W.single(seed=0, context=640, pool_blocks=64),
             W.wavefront(seed=1, prompt=700, generated=37, tokens=4)]
    expected = [_with_caller_scratch(c, splits) for c in cases]

    devs = [W.to_device(c, "triton", "cuda") for c in cases]
    params = [_params(c, d, splits) for c, d in zip(cases, devs)]
    stream = torch.cuda.current_stream().cuda_stream
    for p in params:  # two calls back to back, sharing the library's one scratch array
        _native.check(lib.dory_decode_attention_static_scratch(ctypes.byref(p), stream))
    torch.cuda.synchronize()

    for (out_ref, raw_ref), d in zip(expected, devs):
        torch.testing.assert_close(d["out"].cpu(), out_ref, atol=ATOL, rtol=RTOL)
        assert torch.equal(d["raw"].cpu().view(torch.int16), raw_ref.view(torch.int16))


def test_static_scratch_rejects_calls_beyond_its_size():
    lib = _native.load()
    case = W.single(seed=0, context=640, pool_blocks=64)
    d = W.to_device(case, "triton", "cuda")
    p = _params(case, d, splits=32)
    p.max_tokens = 64  # 64 x 32 splits x 32 heads x 128 x 4 B of partials > 4 MiB
    status = lib.dory_decode_attention_static_scratch(ctypes.byref(p), None)
    assert status == _native.ERR_INVALID_ARGUMENT
    assert "static scratch" in lib.dory_decode_last_error().decode()
