"""The C-ABI library: builds for sm_100a, loads without a GPU, exports every symbol the
header declares, and rejects bad arguments on the host before any CUDA call."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

import _native
import build_native

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "dory_decode.h"


@pytest.fixture(scope="module")
def lib():
    build_native.build()
    return _native.load()


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*[A-Za-z_][\w\s\*]*?\b(dory_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_binding_exports():
    assert declared_functions() == sorted(_native.EXPORTS)


def test_every_declared_symbol_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_abi_version_and_struct_layout(lib):
    assert lib.dory_decode_abi_version() == _native.ABI_VERSION
    assert lib.dory_decode_params_bytes() == ctypes.sizeof(_native.DoryDecodeParams)


def test_library_is_sm100a_only():
    # The build targets exactly compute_100a / sm_100a (no PTX for other arches).
    flags = " ".join(build_native.NVCC_FLAGS)
    assert "arch=compute_100a,code=sm_100a" in flags
    assert "sm_90" not in flags and "sm_89" not in flags


def test_scratch_bytes(lib):
    n = lib.dory_decode_scratch_bytes(4, 32, 32, 8, 128)
    # partial outputs alone: 4 tokens x 32 splits x 32 heads x 128 dims x 4 B
    assert n >= 4 * 32 * 32 * 128 * 4
    assert n % 256 == 0
    assert lib.dory_decode_scratch_bytes(0, 32, 32, 8, 128) == 0


def _params(**kw):
    p = _native.DoryDecodeParams()
    dummy = 0x1000  # never dereferenced: validation fails before any CUDA call
    for f in ("q", "v", "sqk", "slot_mapping", "key_cache", "value_cache", "block_table",
              "seq_lens", "gate", "out_nibble_major", "scratch"):
        setattr(p, f, dummy)
    p.scratch_bytes = 1 << 30
    p.stride_block, p.stride_offset, p.stride_head = 16 * 8 * 256, 256, 16 * 256
    p.num_tokens, p.num_heads, p.num_kv_heads, p.head_dim = 1, 32, 8, 128
    p.block_size, p.splits, p.blocks_per_tile, p.min_blocks_per_split = 16, 32, 1, 1
    p.max_tokens, p.flags = 1, _native.FLAG_RAW_QKV
    p.softmax_scale, p.eps, p.sqk_factor = 128 ** -0.5, 1e-6, 0.7
    for k, val in kw.items():
        setattr(p, k, val)
    return p


@pytest.mark.parametrize("kw,status,message", [
    (dict(num_heads=30, num_kv_heads=8), _native.ERR_INVALID_ARGUMENT, "multiple of KV heads"),
    (dict(num_tokens=2, max_tokens=1, flags=_native.FLAG_RAW_QKV | _native.FLAG_MULTI_TOKEN,
          cache_offsets=0x1000, block_table_offsets=0x1000),
     _native.ERR_INVALID_ARGUMENT, "too many tokens"),
    (dict(head_dim=96), _native.ERR_UNSUPPORTED, "head_dim"),
    (dict(block_size=8), _native.ERR_UNSUPPORTED, "block_size"),
    (dict(stride_offset=100), _native.ERR_ALIGNMENT, "16-byte"),
    (dict(key_cache=0x1004), _native.ERR_ALIGNMENT, "16-byte"),
    (dict(scratch_bytes=64), _native.ERR_INVALID_ARGUMENT, "scratch too small"),
    (dict(flags=_native.FLAG_MULTI_TOKEN | _native.FLAG_RAW_QKV), _native.ERR_INVALID_ARGUMENT,
     "offsets"),
    (dict(flags=_native.FLAG_SHARED_CACHE), _native.ERR_INVALID_ARGUMENT, "shared_cache"),
    (dict(window=-1), _native.ERR_INVALID_ARGUMENT, "window"),
])
def test_host_validation(lib, kw, status, message):
    p = _params(**kw)
    assert lib.dory_decode_attention(ctypes.byref(p), None) == status
    assert message in lib.dory_decode_last_error().decode()


def test_status_maps_to_reference_exceptions(lib):
    p = _params(num_heads=30)
    with pytest.raises(ValueError, match="multiple of KV heads"):
        _native.check(lib.dory_decode_attention(ctypes.byref(p), None))
    p = _params(head_dim=96)
    with pytest.raises(NotImplementedError):
        _native.check(lib.dory_decode_attention(ctypes.byref(p), None))


def test_qk_norm_struct_layout(lib):
    assert lib.dory_qk_norm_params_bytes() == ctypes.sizeof(_native.DoryQkNormParams)


def _qk_params(**kw):
    p = _native.DoryQkNormParams()
    for f in ("qk", "v", "sqk", "q_out", "key_cache", "value_cache", "slot_mapping"):
        setattr(p, f, 0x1000)  # never dereferenced: validation fails before any CUDA call
    p.num_tokens, p.num_heads, p.num_kv_heads, p.head_dim, p.block_size = 1, 32, 8, 128, 16
    p.flags, p.eps, p.sqk_factor = _native.QKNORM_WRITE_CACHE, 1e-6, 0.7
    for k, val in kw.items():
        setattr(p, k, val)
    return p


@pytest.mark.parametrize("kw,status,message", [
    (dict(head_dim=96), _native.ERR_UNSUPPORTED, "head_dim"),
    (dict(num_heads=0), _native.ERR_INVALID_ARGUMENT, "positive"),
    (dict(qk=None), _native.ERR_INVALID_ARGUMENT, "null tensor"),
    (dict(slot_mapping=None), _native.ERR_INVALID_ARGUMENT, "slot mapping"),
    (dict(flags=0), _native.ERR_INVALID_ARGUMENT, "k_out and v_out"),
    (dict(sqk_dtype=7), _native.ERR_INVALID_ARGUMENT, "sqk dtype"),
])
def test_qk_norm_host_validation(lib, kw, status, message):
    p = _qk_params(**kw)
    assert lib.dory_qk_norm_cache(ctypes.byref(p), None) == status
    assert message in lib.dory_decode_last_error().decode()


def _qkvg_params(**kw):
    p = _native.DoryQkvgParams()
    for f in ("partials", "positions", "cos_sin", "s_gate", "qk_out", "v_out", "gate_out"):
        setattr(p, f, 0x1000)  # never dereferenced: every case fails before any CUDA call
    p.num_tokens, p.num_heads, p.num_kv_heads, p.head_dim = 1, 4, 2, 64
    p.split_k, p.max_position, p.s_gate_factor = 2, 16, 0.9
    for k, val in kw.items():
        setattr(p, k, val)
    return p


@pytest.mark.parametrize("kw,status,message", [
    (dict(head_dim=96), _native.ERR_UNSUPPORTED, "head_dim"),
    (dict(num_heads=0), _native.ERR_INVALID_ARGUMENT, "positive"),
    (dict(split_k=0), _native.ERR_INVALID_ARGUMENT, "positive"),
    (dict(max_position=0), _native.ERR_INVALID_ARGUMENT, "positive"),
    (dict(positions_dtype=2), _native.ERR_INVALID_ARGUMENT, "dtype"),
    (dict(cos_sin_dtype=3), _native.ERR_INVALID_ARGUMENT, "dtype"),
    (dict(gate_out=None), _native.ERR_INVALID_ARGUMENT, "null tensor"),
    (dict(partials=0x1008), _native.ERR_ALIGNMENT, "16-byte"),
])
def test_qkvg_host_validation(lib, kw, status, message):
    assert lib.dory_qkvg_params_bytes() == ctypes.sizeof(_native.DoryQkvgParams)
    p = _qkvg_params(**kw)
    assert lib.dory_qkvg_epilogue(ctypes.byref(p), None) == status
    assert message in lib.dory_decode_last_error().decode()


def _residual_params(**kw):
    p = _native.DoryResidualParams()
    # distinct, 16-byte aligned, non-overlapping fake addresses (never dereferenced)
    p.partials, p.a, p.alpha, p.h_out, p.h_out_nibble_major = (
        0x10000, 0x20000, 0x30000, 0x40000, 0x50000)
    p.num_tokens, p.hidden, p.split_k = 1, 64, 1
    p.a_dtype, p.alpha_dtype = _native.DTYPE_BF16, _native.DTYPE_BF16
    p.alpha_scale, p.eps = 2.5, 1e-6
    for k, val in kw.items():
        setattr(p, k, val)
    return p


@pytest.mark.parametrize("kw,status,message", [
    (dict(hidden=12), _native.ERR_INVALID_ARGUMENT, "multiple of 8"),
    (dict(hidden=0), _native.ERR_INVALID_ARGUMENT, "multiple of 8"),
    (dict(hidden=16392), _native.ERR_UNSUPPORTED, "16384"),
    (dict(split_k=0), _native.ERR_INVALID_ARGUMENT, "split_k"),
    (dict(num_tokens=-1), _native.ERR_INVALID_ARGUMENT, "num_tokens"),
    (dict(a_dtype=5), _native.ERR_INVALID_ARGUMENT, "dtype"),
    (dict(x=0x60000, x_sumsq=0x70000, x_dim=16), _native.ERR_INVALID_ARGUMENT, "not both"),
    (dict(x=0x60000, x_dim=0), _native.ERR_INVALID_ARGUMENT, "x_dim"),
    (dict(alpha=None), _native.ERR_INVALID_ARGUMENT, "null tensor"),
    (dict(a=0x20002), _native.ERR_ALIGNMENT, "16-byte"),
    (dict(h_out=0x20000), _native.ERR_INVALID_ARGUMENT, "alias"),           # h_out == a
    (dict(h_out_nibble_major=0x10040), _native.ERR_INVALID_ARGUMENT, "alias"),  # inside partials
])
def test_residual_host_validation(lib, kw, status, message):
    assert lib.dory_residual_params_bytes() == ctypes.sizeof(_native.DoryResidualParams)
    p = _residual_params(**kw)
    assert lib.dory_residual_update(ctypes.byref(p), None) == status
    assert message in lib.dory_decode_last_error().decode()


def test_zero_token_calls_need_no_tensors(lib):
    """T = 0 returns OK before any pointer is looked at or any CUDA call is made."""
    p = _native.DoryResidualParams()
    p.num_tokens, p.hidden, p.split_k = 0, 64, 1
    assert lib.dory_residual_update(ctypes.byref(p), None) == _native.OK
