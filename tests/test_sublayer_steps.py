"""Host-side checks of dory_sublayer_steps (no GPU).

* route_reference_kernels() replaces exactly the reference modules' kernel names that the
  sublayers launch (dory_attention._qk_norm_cache_kernel, dory_multi_token.
  _qkvg_epilogue_kernel and _residual_tokens_kernel, residual_update in dory_common,
  dory_attention and dory_mlp) and leaves the rest of those modules alone; stand-in modules
  play the reference here, which does not travel with the tests.
* This package does not shadow the reference's other kernel modules: with it first on
  sys.path, the only reference module name it defines is dory_decode_attention.
* The launch-form shims check their grids before touching the device.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

import pytest
import torch

import dory_sublayer_steps as S

PKG = Path(__file__).resolve().parent.parent / "dory-vllm-experiments_b200"
# kernels/*.py of the reference (module names only)
REFERENCE_MODULES = {
    "bench_attention", "bench_decode_attention", "bench_gemv", "bench_gemv_tokens",
    "bench_launch_cost", "bench_lm_head", "bench_mlp", "bench_multi_token", "bench_wavefront",
    "check_speculative_sampling", "dory_attention", "dory_common", "dory_decode_attention",
    "dory_fused_model", "dory_lm_head", "dory_mlp", "dory_multi_token", "dory_sampling",
    "dory_wavefront", "dory_wavefront_engine", "explore_gemv", "w4a16_gemv"}


def test_only_dory_decode_attention_is_shadowed():
    ours = {p.stem for p in PKG.glob("*.py")}
    assert ours & REFERENCE_MODULES == {"dory_decode_attention"}


def test_route_reference_kernels_replaces_only_the_kernels(monkeypatch):
    attention = types.ModuleType("dory_attention")
    attention._qk_norm_cache_kernel = "triton kernel"
    attention.FusedAttentionSublayer = object
    attention.residual_update = "reference function"
    multi = types.ModuleType("dory_multi_token")
    multi._qkvg_epilogue_kernel = "triton kernel"
    multi._residual_tokens_kernel = "triton kernel"
    multi.MultiTokenSublayers = object
    common = types.ModuleType("dory_common")
    common.residual_update = "reference function"
    common.EPS = 1e-6
    mlp = types.ModuleType("dory_mlp")
    mlp.residual_update = "reference function"
    for name, mod in (("dory_attention", attention), ("dory_multi_token", multi),
                      ("dory_common", common), ("dory_mlp", mlp)):
        monkeypatch.setitem(sys.modules, name, mod)
    routed = S.route_reference_kernels()
    assert routed == ["dory_attention._qk_norm_cache_kernel",
                      "dory_multi_token._qkvg_epilogue_kernel",
                      "dory_multi_token._residual_tokens_kernel",
                      "dory_common.residual_update", "dory_attention.residual_update",
                      "dory_mlp.residual_update"]
    assert attention._qk_norm_cache_kernel is S._qk_norm_cache_kernel
    assert multi._qkvg_epilogue_kernel is S._qkvg_epilogue_kernel
    assert multi._residual_tokens_kernel is S._residual_tokens_kernel
    for mod in (common, attention, mlp):
        assert mod.residual_update is S.residual_update
    assert attention.FusedAttentionSublayer is object and multi.MultiTokenSublayers is object
    assert common.EPS == 1e-6


def test_route_refuses_a_module_without_the_kernel(monkeypatch):
    monkeypatch.setitem(sys.modules, "dory_attention", types.ModuleType("dory_attention"))
    with pytest.raises(ImportError):
        S.route_reference_kernels()


def test_epilogue_shim_checks_grid():
    HD, Q, KV, T = 64, 128, 64, 1
    parts = torch.zeros(1, T, 2 * (Q + KV))
    with pytest.raises(ValueError):
        S._qkvg_epilogue_kernel[(5, T)](parts, torch.zeros(T, dtype=torch.int64),
                                        torch.zeros(8, HD), torch.ones(Q), torch.zeros(T, Q + KV),
                                        torch.zeros(T, KV), torch.zeros(T, Q), 1.0, Q_ROWS=Q,
                                        KV_ROWS=KV, HEAD_DIM=HD, SPLIT_K=1, T=T)


def test_epilogue_refuses_cpu_tensors():
    HD, NH, NKV, T = 64, 2, 1, 1
    Q, KV = NH * HD, NKV * HD
    with pytest.raises(RuntimeError):
        S.qkvg_epilogue(torch.zeros(1, T, 2 * (Q + KV)), torch.zeros(T, dtype=torch.int64),
                        torch.zeros(8, HD), torch.ones(Q), 1.0, torch.zeros(T, Q + KV),
                        torch.zeros(T, KV), torch.zeros(T, Q), NH, NKV, HD)


def test_residual_shim_checks_grid():
    T, H, K = 2, 64, 32
    with pytest.raises(ValueError):
        S._residual_tokens_kernel[(3,)](torch.zeros(1, T, H), torch.zeros(T, K),
                                        torch.zeros(T, H, dtype=torch.bfloat16), torch.zeros(H),
                                        torch.zeros(T, H, dtype=torch.bfloat16),
                                        torch.zeros(T, 8, H // 8), 1.0, 1e-6, H=H, K_IN=K,
                                        SPLIT_K=1, T=T, W_BLOCK=8, X_BLOCK=32, num_warps=8)


def test_residual_refuses_cpu_tensors_and_bad_arguments():
    T, H = 1, 64
    args = (torch.zeros(T, H, dtype=torch.bfloat16), torch.zeros(H), 1.0, 1e-6,
            torch.zeros(T, H, dtype=torch.bfloat16), torch.zeros(T, 8, H // 8))
    with pytest.raises(RuntimeError):
        S.residual_tokens(torch.zeros(1, T, H), torch.zeros(T, 16), *args)
    with pytest.raises(ValueError):  # partials not [split_k, T, H]
        S.residual_tokens(torch.zeros(T, H), None, *args)


def test_residual_update_refuses_aliasing():
    """The reference's residual_update raises when h_out aliases a (dory_common.py:74-75)."""
    a = torch.zeros(64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        S.residual_update(a, torch.zeros(64), torch.zeros(64), 1.0, a, torch.zeros(8, 8))
