"""ctypes binding of libdory_decode.so (the C ABI declared in include/dory_decode.h).

There is no fallback: if the sm_100a library is missing or does not match this binding,
loading fails loudly.  The library is built in-tree by build_native.py.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "libdory_decode.so"

ABI_VERSION = 8

# DoryStatus
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_ALIGNMENT, ERR_CUDA = range(5)
# DoryDType
DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_FP8_E4M3 = range(4)
# DORY_FLAG_*
FLAG_RAW_QKV, FLAG_MULTI_TOKEN, FLAG_SHARED_CACHE, FLAG_OVERLAP_LAUNCH = 1, 2, 4, 8
FLAG_FMA_CONSUMER = 16
# DORY_QKNORM_*
QKNORM_WRITE_CACHE = 1
# DORY_DEVERR_*
DEVERR_BLOCK_OOB, DEVERR_SLOT_OOB, DEVERR_OFFSET_ALIGN, DEVERR_WAIT_TIMEOUT = 1, 2, 4, 8
DEVERR_POSITION_OOB = 16
DEVERR_NAMES = {DEVERR_BLOCK_OOB: "block id out of range", DEVERR_SLOT_OOB: "slot out of range",
                DEVERR_OFFSET_ALIGN: "cache offset not 16-byte aligned",
                DEVERR_WAIT_TIMEOUT: "pipeline wait timed out",
                DEVERR_POSITION_OOB: "rotary position outside the cos/sin table"}

# Every symbol include/dory_decode.h declares (checked by the CPU test suite).
EXPORTS = ("dory_decode_abi_version", "dory_decode_params_bytes", "dory_decode_scratch_bytes",
           "dory_decode_scratch_init", "dory_decode_attention", "dory_decode_fetch_errors",
           "dory_decode_last_error", "dory_decode_attention_static_scratch",
           "dory_decode_static_scratch_fetch_errors",
           "dory_qk_norm_params_bytes", "dory_qk_norm_cache", "dory_qkvg_params_bytes",
           "dory_qkvg_epilogue", "dory_residual_params_bytes", "dory_residual_update")

# Size of the library's static scratch array (DORY_DECODE_STATIC_SCRATCH_BYTES).
STATIC_SCRATCH_BYTES = 4 << 20

_vp, _i32, _i64, _f32, _u32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_uint32


class DoryDecodeParams(ctypes.Structure):
    """Mirror of DoryDecodeParams (include/dory_decode.h); field order is the ABI."""
    _fields_ = [
        ("q", _vp), ("v", _vp), ("sqk", _vp), ("slot_mapping", _vp),
        ("key_cache", _vp), ("value_cache", _vp), ("block_table", _vp),
        ("block_table_offsets", _vp), ("cache_offsets", _vp), ("seq_lens", _vp),
        ("gate", _vp), ("out_nibble_major", _vp), ("out_sumsq", _vp), ("scratch", _vp),
        ("scratch_bytes", _i64), ("stride_block", _i64), ("stride_offset", _i64),
        ("stride_head", _i64), ("num_cache_blocks", _i64),
        ("softmax_scale", _f32), ("sqk_factor", _f32), ("eps", _f32),
        ("num_tokens", _i32), ("num_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("block_size", _i32), ("window", _i32), ("splits", _i32), ("blocks_per_tile", _i32),
        ("min_blocks_per_split", _i32), ("max_tokens", _i32), ("sqk_dtype", _i32),
        ("flags", _u32), ("prefetch_chunks", _i32), ("kv_dtype", _i32),
        ("k_scale", _f32), ("v_scale", _f32),
    ]


class DoryQkNormParams(ctypes.Structure):
    """Mirror of DoryQkNormParams (include/dory_decode.h); field order is the ABI."""
    _fields_ = [
        ("qk", _vp), ("v", _vp), ("sqk", _vp), ("q_out", _vp), ("key_cache", _vp),
        ("value_cache", _vp), ("slot_mapping", _vp), ("k_out", _vp), ("v_out", _vp),
        ("error_word", _vp), ("stride_block", _i64), ("stride_offset", _i64),
        ("stride_head", _i64), ("num_cache_blocks", _i64), ("sqk_factor", _f32), ("eps", _f32),
        ("num_tokens", _i32), ("num_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("block_size", _i32), ("sqk_dtype", _i32), ("flags", _u32),
    ]


class DoryQkvgParams(ctypes.Structure):
    """Mirror of DoryQkvgParams (include/dory_decode.h); field order is the ABI."""
    _fields_ = [
        ("partials", _vp), ("positions", _vp), ("cos_sin", _vp), ("s_gate", _vp),
        ("qk_out", _vp), ("v_out", _vp), ("gate_out", _vp), ("error_word", _vp),
        ("s_gate_factor", _f32), ("num_tokens", _i32), ("num_heads", _i32),
        ("num_kv_heads", _i32), ("head_dim", _i32), ("split_k", _i32), ("max_position", _i32),
        ("positions_dtype", _i32), ("cos_sin_dtype", _i32), ("s_gate_dtype", _i32),
        ("flags", _u32),
    ]


class DoryResidualParams(ctypes.Structure):
    """Mirror of DoryResidualParams (include/dory_decode.h); field order is the ABI."""
    _fields_ = [
        ("partials", _vp), ("x", _vp), ("x_sumsq", _vp), ("a", _vp), ("alpha", _vp),
        ("h_out", _vp), ("h_out_nibble_major", _vp), ("alpha_scale", _f32), ("eps", _f32),
        ("num_tokens", _i32), ("hidden", _i32), ("x_dim", _i32), ("split_k", _i32),
        ("a_dtype", _i32), ("alpha_dtype", _i32), ("flags", _u32),
    ]


_lib = None


def load(path: os.PathLike | None = None) -> ctypes.CDLL:
    """Loads (once) and returns the library, checking its ABI version and struct size."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(path) if path is not None else LIBRARY
    if not path.exists():
        raise RuntimeError(
            f"{path} is missing: build the sm_100a library first (python {HERE / 'build_native.py'}"
            " or __graft_entry__.build()); there is no CPU or Triton fallback")
    lib = ctypes.CDLL(str(path))
    lib.dory_decode_abi_version.restype = _i32
    lib.dory_decode_abi_version.argtypes = []
    lib.dory_decode_params_bytes.restype = _i64
    lib.dory_decode_params_bytes.argtypes = []
    lib.dory_decode_scratch_bytes.restype = _i64
    lib.dory_decode_scratch_bytes.argtypes = [_i32, _i32, _i32, _i32, _i32]
    lib.dory_decode_scratch_init.restype = _i32
    lib.dory_decode_scratch_init.argtypes = [_vp, _i64, _vp]
    lib.dory_decode_attention.restype = _i32
    lib.dory_decode_attention.argtypes = [ctypes.POINTER(DoryDecodeParams), _vp]
    lib.dory_decode_fetch_errors.restype = _i32
    lib.dory_decode_fetch_errors.argtypes = [_vp, ctypes.POINTER(_u32), _i32, _vp]
    lib.dory_decode_last_error.restype = ctypes.c_char_p
    lib.dory_decode_last_error.argtypes = []
    lib.dory_decode_attention_static_scratch.restype = _i32
    lib.dory_decode_attention_static_scratch.argtypes = [ctypes.POINTER(DoryDecodeParams), _vp]
    lib.dory_decode_static_scratch_fetch_errors.restype = _i32
    lib.dory_decode_static_scratch_fetch_errors.argtypes = [ctypes.POINTER(_u32), _i32, _vp]
    lib.dory_qk_norm_params_bytes.restype = _i64
    lib.dory_qk_norm_params_bytes.argtypes = []
    lib.dory_qk_norm_cache.restype = _i32
    lib.dory_qk_norm_cache.argtypes = [ctypes.POINTER(DoryQkNormParams), _vp]
    lib.dory_qkvg_params_bytes.restype = _i64
    lib.dory_qkvg_params_bytes.argtypes = []
    lib.dory_qkvg_epilogue.restype = _i32
    lib.dory_qkvg_epilogue.argtypes = [ctypes.POINTER(DoryQkvgParams), _vp]
    lib.dory_residual_params_bytes.restype = _i64
    lib.dory_residual_params_bytes.argtypes = []
    lib.dory_residual_update.restype = _i32
    lib.dory_residual_update.argtypes = [ctypes.POINTER(DoryResidualParams), _vp]
    if lib.dory_decode_abi_version() != ABI_VERSION:
        raise RuntimeError(f"{path}: ABI version {lib.dory_decode_abi_version()} != {ABI_VERSION}")
    if lib.dory_decode_params_bytes() != ctypes.sizeof(DoryDecodeParams):
        raise RuntimeError(f"{path}: DoryDecodeParams is {lib.dory_decode_params_bytes()} bytes, "
                           f"the binding's is {ctypes.sizeof(DoryDecodeParams)}")
    if lib.dory_qk_norm_params_bytes() != ctypes.sizeof(DoryQkNormParams):
        raise RuntimeError(f"{path}: DoryQkNormParams is {lib.dory_qk_norm_params_bytes()} "
                           f"bytes, the binding's is {ctypes.sizeof(DoryQkNormParams)}")
    if lib.dory_qkvg_params_bytes() != ctypes.sizeof(DoryQkvgParams):
        raise RuntimeError(f"{path}: DoryQkvgParams is {lib.dory_qkvg_params_bytes()} "
                           f"bytes, the binding's is {ctypes.sizeof(DoryQkvgParams)}")
    if lib.dory_residual_params_bytes() != ctypes.sizeof(DoryResidualParams):
        raise RuntimeError(f"{path}: DoryResidualParams is {lib.dory_residual_params_bytes()} "
                           f"bytes, the binding's is {ctypes.sizeof(DoryResidualParams)}")
    _lib = lib
    return lib


def check_devices(device, *tensors) -> None:
    """ValueError unless every given tensor (None skipped) is on `device`, a CUDA device:
    the kernels dereference the raw pointers, so a host tensor or one on another GPU must
    be refused before the launch."""
    for t in tensors:
        if t is not None and t.device != device:
            raise ValueError(f"a tensor argument is on {t.device}; this call runs on {device}")


def check_device_index(index: int, *tensors) -> None:
    """check_devices by device index (Tensor.get_device(): -1 for host memory), the form the
    per-call launch paths use: comparing torch.device objects costs more than the launch."""
    for t in tensors:
        if t is not None and t.get_device() != index:
            raise ValueError(f"a tensor argument is on {t.device}; this call runs on cuda:{index}")


def check(status: int) -> None:
    """Maps a DoryStatus to the reference's exception types (ValueError for bad arguments)."""
    if status == OK:
        return
    message = load().dory_decode_last_error().decode(errors="replace")
    if status in (ERR_INVALID_ARGUMENT, ERR_ALIGNMENT):
        raise ValueError(message)
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(message)
    raise RuntimeError(message)
