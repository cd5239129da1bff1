"""Golden-case specifications shared by make_golden.py (which evaluates them with the
reference's own eager functions) and the tests (which rebuild the same seeded inputs)."""

from __future__ import annotations

import hashlib

import numpy as np
import torch

import workloads as W

# Sequence lengths around block and window boundaries (the reference's edge-case list,
# EXPERIMENTS.md:325-327 — 0, 1, 15-17, 1023-1025, 1040, 3000 — with seq_len = context + 1).
EDGE_SEQ_LENS = (1, 15, 16, 17, 1023, 1024, 1025, 1040, 3000)


def specs() -> dict:
    """name -> zero-argument builder of a workloads.Case."""
    out = {
        # configuration 1: 32q/8kv x 128, block 16, 640 cached tokens, 64-block pool, seed 0
        "config1": lambda: W.single(seed=0, context=640, pool_blocks=64),
        "single_window": lambda: W.single(seed=10, context=1500, pool_blocks=100, window=1024),
        # the real model's attention shape: 16q/4kv x 256, sliding window 1024
        "dory_shape": lambda: W.single(seed=11, context=1100, pool_blocks=80, window=1024,
                                       num_heads=16, num_kv_heads=4, head_dim=256),
        "gqa8": lambda: W.single(seed=12, context=777, pool_blocks=60, num_heads=32,
                                 num_kv_heads=4, head_dim=128),
        # shared-KV wavefront (configuration 2 shape, short prompt for CPU speed)
        "wavefront": lambda: W.wavefront(seed=1, prompt=700, generated=37, tokens=4),
        "wavefront_window": lambda: W.wavefront(seed=13, prompt=1010, generated=5, tokens=4,
                                                window=1024),
        "wavefront_t2": lambda: W.wavefront(seed=14, prompt=333, generated=0, tokens=2),
        # batched independent sequences (configuration 3 shape, few sequences)
        "batched": lambda: W.batched(seed=2, lens=[128, 1152, 15, 640, 16, 300]),
    }
    for i, n in enumerate(EDGE_SEQ_LENS):
        for window in (0, 1024):
            out[f"edge_{n}_w{window}"] = (
                lambda n=n, window=window, i=i: W.single(
                    seed=100 + i, context=n - 1, pool_blocks=200, window=window, num_heads=8,
                    num_kv_heads=2, head_dim=64))
    return out


def digest(case: W.Case) -> str:
    """SHA-256 over every input tensor of a case (checks that regeneration matches)."""
    h = hashlib.sha256()
    for t in (case.qk, case.v, case.gate, case.sqk.float(), case.key, case.value, case.tables):
        h.update(np.ascontiguousarray(t.float().numpy() if t.dtype != torch.int32
                                      else t.numpy()).tobytes())
    h.update(np.asarray(case.seq_lens, dtype=np.int64).tobytes())
    h.update(np.asarray(case.table_rows, dtype=np.int64).tobytes())
    return h.hexdigest()


# ---- the multi-token q/k/v/gate epilogue (kernels/dory_multi_token.py:53-80) ----

class QkvgCase:
    """Seeded inputs of the epilogue: split-K partials FP32 [split_k, T, 2 * (Q + KV)],
    positions int64 [T], cos_sin [max_position, head_dim] (FP32 or BF16), s_gate BF16 [Q]."""

    def __init__(self, seed: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 split_k: int, tokens: int, cos_dtype=torch.float32, max_position: int = 4096,
                 s_gate_factor: float = 0.9):
        g = torch.Generator().manual_seed(seed)
        self.num_heads, self.num_kv_heads, self.head_dim = num_heads, num_kv_heads, head_dim
        Q, KV = num_heads * head_dim, num_kv_heads * head_dim
        self.partials = torch.randn(split_k, tokens, 2 * (Q + KV), generator=g)
        self.positions = torch.randint(0, max_position, (tokens,), generator=g)
        self.cos_sin = torch.randn(max_position, head_dim, generator=g).to(cos_dtype)
        self.s_gate = (torch.rand(Q, generator=g) + 0.5).to(torch.bfloat16)
        self.s_gate_factor = s_gate_factor

    @property
    def tokens(self) -> int:
        return self.partials.shape[1]


def qkvg_specs() -> dict:
    """name -> zero-argument builder of a QkvgCase."""
    return {
        "qkvg_128": lambda: QkvgCase(41, 4, 2, 128, 2, 3),
        "qkvg_256_bf16cos": lambda: QkvgCase(42, 2, 1, 256, 3, 2, cos_dtype=torch.bfloat16),
        "qkvg_64_t1": lambda: QkvgCase(43, 4, 4, 64, 1, 1),
        "qkvg_gqa8_split4": lambda: QkvgCase(44, 8, 1, 128, 4, 2, max_position=9000),
        # the real model's shape: 16q/4kv x 256, four wavefront rows
        "qkvg_dory": lambda: QkvgCase(45, 16, 4, 256, 2, 4, cos_dtype=torch.bfloat16,
                                      max_position=8300),
    }


def qkvg_digest(case: QkvgCase) -> str:
    h = hashlib.sha256()
    for t in (case.partials, case.positions, case.cos_sin.float(), case.s_gate.float()):
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


class ResidualCase:
    """Seeded inputs of the residual update: split-K partials FP32 [split_k, T, H] of the
    output GEMV, its input x FP32 [T, K] (None: the partials are b itself, residual_update),
    the sublayer input a [T, H] (unit rows, as the hidden state is) and alpha [H]."""

    def __init__(self, seed: int, tokens: int, hidden: int, x_dim: int | None, split_k: int,
                 dtype=torch.bfloat16, alpha_scale: float = 2.5):
        g = torch.Generator().manual_seed(seed)
        self.partials = torch.randn(split_k, tokens, hidden, generator=g) * 3.0
        self.x = None if x_dim is None else torch.randn(tokens, x_dim, generator=g)
        a = torch.randn(tokens, hidden, generator=g)
        self.a = (a / a.norm(dim=1, keepdim=True)).to(dtype)
        self.alpha = (torch.randn(hidden, generator=g) * 0.02).to(dtype)
        self.alpha_scale = alpha_scale

    @property
    def tokens(self) -> int:
        return self.partials.shape[1]

    @property
    def hidden(self) -> int:
        return self.partials.shape[2]


def residual_specs() -> dict:
    """name -> zero-argument builder of a ResidualCase.  The Dory shapes: hidden 2560, the
    attention output GEMV over 4096 inputs and the MLP down GEMV over 7168, both split-K 4
    (kernels/dory_multi_token.py:42, 44), four wavefront rows."""
    return {
        "residual_attn_dory": lambda: ResidualCase(51, 4, 2560, 4096, 4),
        "residual_mlp_dory": lambda: ResidualCase(52, 2, 2560, 7168, 4),
        # 37 groups of 8 (not a warp multiple), an input length not a multiple of 4, FP32 a
        "residual_ragged_f32": lambda: ResidualCase(53, 3, 296, 101, 3, dtype=torch.float32),
        # hidden 12288: two groups of 8 per thread
        "residual_wide": lambda: ResidualCase(54, 1, 12288, 4096, 2),
        # residual_update (kernels/dory_common.py:55-81): one token, b given
        "residual_update_dory": lambda: ResidualCase(55, 1, 2560, None, 1),
    }


def residual_digest(case: ResidualCase) -> str:
    h = hashlib.sha256()
    parts = [case.partials, case.a.float(), case.alpha.float()]
    if case.x is not None:
        parts.append(case.x)
    for t in parts:
        h.update(t.contiguous().numpy().tobytes())
    h.update(repr(case.alpha_scale).encode())
    return h.hexdigest()
