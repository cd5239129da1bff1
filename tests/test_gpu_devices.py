"""Every host wrapper refuses a tensor on another device before launching: the kernels
dereference raw pointers, so a host tensor must never reach them (it would fault the GPU).
Each case is checked to raise ValueError, and the instance's device error word stays clear.
"""

from __future__ import annotations

import pytest
import torch

import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from dory_sublayer_steps import qk_norm_cache, qkvg_epilogue, residual_tokens

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def test_decode_attention_refuses_host_tensors():
    case = W.single(seed=700, context=200, pool_blocks=20)
    d = W.to_device(case, "triton", DEV)
    attn = DecodeAttention(32, 8, 128, DEV)
    args = dict(qk=d["qk"][0], v=d["v"][0], sqk=d["sqk"], slot_mapping=d["slots"][0:1],
                block_table=d["tables"][0], seq_lens=d["seq_lens"][0:1], gate=d["gate"][0],
                out=d["out"][0])
    for name in args:
        bad = dict(args)
        bad[name] = args[name].cpu()
        with pytest.raises(ValueError):
            attn.from_raw(bad["qk"], bad["v"], bad["sqk"], case.sqk_factor, EPS,
                          bad["slot_mapping"], d["key"], d["value"], bad["block_table"],
                          bad["seq_lens"], 0, case.scale, bad["gate"], bad["out"])
    with pytest.raises(ValueError):
        attn.from_raw(args["qk"], args["v"], args["sqk"], case.sqk_factor, EPS,
                      args["slot_mapping"], d["key"], d["value"], args["block_table"],
                      args["seq_lens"], 0, case.scale, args["gate"], args["out"],
                      out_sumsq=torch.zeros(1))
    torch.cuda.synchronize()
    attn.check_errors()


def test_sublayer_steps_refuse_host_tensors():
    NH, NKV, HD, T = 4, 2, 64, 1
    Q, KV = NH * HD, NKV * HD
    with pytest.raises(ValueError):
        qkvg_epilogue(torch.zeros(1, T, 2 * (Q + KV), device=DEV),
                      torch.zeros(T, dtype=torch.int64), torch.zeros(8, HD, device=DEV),
                      torch.ones(Q, device=DEV), 1.0, torch.empty(T, Q + KV, device=DEV),
                      torch.empty(T, KV, device=DEV), torch.empty(T, Q, device=DEV),
                      NH, NKV, HD)
    with pytest.raises(ValueError):
        qk_norm_cache(torch.zeros(T, Q + KV, device=DEV), torch.zeros(T, KV, device=DEV),
                      torch.ones(Q), 1.0, EPS,
                      torch.empty(T, Q, dtype=torch.bfloat16, device=DEV), NH, HD,
                      k_out=torch.empty(T, KV, dtype=torch.bfloat16, device=DEV),
                      v_out=torch.empty(T, KV, dtype=torch.bfloat16, device=DEV))
    H = 64
    with pytest.raises(ValueError):
        residual_tokens(torch.zeros(1, T, H, device=DEV), None,
                        torch.zeros(T, H, dtype=torch.bfloat16, device=DEV), torch.zeros(H),
                        1.0, EPS, torch.zeros(T, H, dtype=torch.bfloat16, device=DEV),
                        torch.zeros(T, 8, H // 8, device=DEV))
    torch.cuda.synchronize()
