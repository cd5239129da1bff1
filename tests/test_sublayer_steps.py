"""Host-side checks of dory_sublayer_steps (no GPU).

* route_reference_kernels() replaces exactly the reference modules' kernel names that the
  sublayers launch (dory_attention._qk_norm_cache_kernel, dory_multi_token.
  _qkvg_epilogue_kernel) and leaves the rest of those modules alone; stand-in modules play
  the reference here, which does not travel with the tests.
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
    multi = types.ModuleType("dory_multi_token")
    multi._qkvg_epilogue_kernel = "triton kernel"
    multi.MultiTokenSublayers = object
    monkeypatch.setitem(sys.modules, "dory_attention", attention)
    monkeypatch.setitem(sys.modules, "dory_multi_token", multi)
    routed = S.route_reference_kernels()
    assert routed == ["dory_attention._qk_norm_cache_kernel",
                      "dory_multi_token._qkvg_epilogue_kernel"]
    assert attention._qk_norm_cache_kernel is S._qk_norm_cache_kernel
    assert multi._qkvg_epilogue_kernel is S._qkvg_epilogue_kernel
    assert attention.FusedAttentionSublayer is object and multi.MultiTokenSublayers is object


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
