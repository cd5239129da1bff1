"""A whole wavefront step of the recurrent block's attention sublayers, as one CUDA graph,
against the oracle's chain (configuration 2's shape: 32q/8kv x 128, block size 16, four rows
at positions 2710..2713 at loop depths 3..0, 20 recurrent attention layers, each with one
"last_loop" cache that every loop writes and reads, one block table for all of them).

Per layer: the q/k/v/gate epilogue on seeded q/k/v/gate GEMV partials, multi_from_raw with
shared_cache and the output's sum of squares, and the residual update on seeded
output-GEMV partials fed that statistic (the NVFP4 GEMVs themselves are outside this
build; kernels/dory_multi_token.py:183-210, kernels/dory_wavefront_engine.py:405-432).
Checked: every layer's cache pool bit for bit (the four appended rows of each layer, no
other row touched), the last layer's attention output within the bf16 bar (2e-2 abs /
1e-2 rel), the block's output h (FP32 nibble-major) within 1e-5 relative of the oracle's,
and a graph replay giving the bits of the plain launch."""

from __future__ import annotations

import pytest
import torch

import dory_oracle as O
import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close
from wavefront_binding import AttentionSublayer, WavefrontLayer, WavefrontRecurrentBlock

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
NH, NKV, HD, B = 32, 8, 128, 16
LAYERS, ROWS, POSITION = 20, 4, 2710
HIDDEN = NH * HD


def build():
    g = torch.Generator().manual_seed(2026)
    need = -(-(POSITION + ROWS) // B)
    pool = need + 8
    table = torch.randperm(pool, generator=g)[:need].to(torch.int32)[None]
    caches_cpu, layers, subs = [], [], []
    Q, KV = NH * HD, NKV * HD
    cos_sin = torch.randn(POSITION + ROWS + 4, HD, generator=g)
    parts_q, parts_o = [], []
    for i in range(LAYERS):
        key = torch.randn(pool, B, NKV, HD, generator=g).to(torch.bfloat16)
        value = torch.randn(pool, B, NKV, HD, generator=g).to(torch.bfloat16)
        caches_cpu.append((key, value))
        kv = torch.empty(pool, NKV, B, 2 * HD, dtype=torch.bfloat16, device=DEV)  # vLLM Triton
        k_view, v_view = kv.transpose(1, 2).split(HD, dim=-1)
        k_view.copy_(key)
        v_view.copy_(value)
        layer = WavefrontLayer([kv] * ROWS, [0] * ROWS, table.shape[1], NKV, HD)
        sqk = (torch.rand(Q, generator=g) + 0.5).to(torch.bfloat16)
        s_gate = (torch.rand(Q, generator=g) + 0.5).to(torch.bfloat16)
        alpha = (torch.randn(HIDDEN, generator=g) * 0.02).to(torch.bfloat16)
        subs.append(dict(kv=kv, sqk=sqk, s_gate=s_gate, alpha=alpha))
        layers.append(AttentionSublayer(layer, sqk.to(DEV), s_gate.to(DEV), cos_sin.to(DEV),
                                        alpha.to(DEV), 0, HD ** -0.5))
        parts_q.append(torch.randn(2, ROWS, 2 * (Q + KV), generator=g) * 0.7)
        parts_o.append(torch.randn(4, ROWS, HIDDEN, generator=g))
    a = torch.randn(ROWS, HIDDEN, generator=g)
    h_in = (a / a.norm(dim=1, keepdim=True)).to(torch.bfloat16)
    return table, caches_cpu, layers, subs, cos_sin, parts_q, parts_o, h_in


def oracle_chain(table, caches_cpu, subs, cos_sin, parts_q, parts_o, h_in, positions, seq_lens):
    a = h_in
    out = None
    for i in range(LAYERS):
        qk, v, gate = O.qkvg_epilogue(parts_q[i], positions, cos_sin, subs[i]["s_gate"], 0.9, NH,
                                      NKV, HD)
        key, value = caches_cpu[i]
        out = O.multi_from_raw(qk, v, subs[i]["sqk"], W.SQK_FACTOR, EPS,
                               torch.zeros(ROWS, dtype=torch.int64), key.view(-1), value.view(-1),
                               tuple(key.shape), key.stride(), table.reshape(-1),
                               torch.zeros(ROWS, dtype=torch.int64), seq_lens, 0, HD ** -0.5, gate,
                               NH, NKV, shared_cache=True)
        natural = out.transpose(1, 2).reshape(ROWS, NH * HD)
        _, a, h_nm = O.residual_tokens(parts_o[i], natural, None, a, subs[i]["alpha"], 2.5)
    return out, h_nm


def test_recurrent_block_step_matches_oracle_chain_and_replays():
    table, caches_cpu, layers, subs, cos_sin, parts_q, parts_o, h_in = build()
    positions = list(range(POSITION, POSITION + ROWS))
    seq_lens = [p + 1 for p in positions]
    attn = DecodeAttention(NH, NKV, HD, DEV, splits=16, max_tokens=ROWS)
    block = WavefrontRecurrentBlock(attn, layers, table.to(DEV), HIDDEN, W.SQK_FACTOR, 0.9, 2.5,
                                    EPS, shared_cache=True)
    for i in range(LAYERS):
        block.qkvg_partials(i, ROWS).copy_(parts_q[i])
        block.out_partials(i, ROWS).copy_(parts_o[i])
    pos_d = torch.tensor(positions, dtype=torch.int64, device=DEV)
    len_d = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    h_in_d = h_in.to(DEV)
    h, h_nm = block.replay(ROWS, pos_d, len_d, h_in_d)  # plain launches, then captured
    torch.cuda.synchronize()
    attn.check_errors()
    first = (h.clone(), h_nm.clone(), block.attention_out[:ROWS].clone())

    out_ref, nm_ref = oracle_chain(table, caches_cpu, subs, cos_sin, parts_q, parts_o, h_in,
                                   torch.tensor(positions), seq_lens)
    for i in range(LAYERS):  # the oracle's chain appended into caches_cpu in place
        k_view, v_view = subs[i]["kv"].transpose(1, 2).split(HD, dim=-1)
        assert torch.equal(k_view.cpu().view(torch.int16), caches_cpu[i][0].view(torch.int16)), i
        assert torch.equal(v_view.cpu().view(torch.int16), caches_cpu[i][1].view(torch.int16)), i
    assert_close(first[2].cpu(), out_ref)
    torch.testing.assert_close(first[1].cpu(), nm_ref, rtol=1e-5, atol=1e-7)

    for _ in range(2):  # graph replays: the same bits
        h.fill_(0)
        h2, nm2 = block.replay(ROWS, pos_d, len_d, h_in_d)
        torch.cuda.synchronize()
        assert torch.equal(h2, first[0]) and torch.equal(nm2, first[1])
    attn.check_errors()
