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


def test_gemv_hooks_run_in_the_chain_and_the_graph():
    """The GEMVs between the steps given as hooks (matmul stand-ins over the nibble-major
    inputs, split-K along the input dimension, as the reference's GEMVs): each layer's
    q/k/v/gate GEMV reads the previous layer's h, so the chain is the real data flow.  The
    oracle's chain, fed the partials the hooks produced, gives the same cache bits and h
    within 1e-5; graph replays give the plain run's bits."""
    nh, nkv, hd, layers, rows, position = 8, 2, 64, 4, 3, 300
    Q, KV, H = nh * hd, nkv * hd, nh * hd
    g = torch.Generator().manual_seed(2028)
    need = -(-(position + rows) // B)
    table = torch.randperm(need + 4, generator=g)[:need].to(torch.int32)[None]
    cos_sin = torch.randn(position + rows + 4, hd, generator=g)
    subs, caches_cpu, kvs, w_q, w_o = [], [], [], [], []
    for i in range(layers):
        key = torch.randn(need + 4, B, nkv, hd, generator=g).to(torch.bfloat16)
        value = torch.randn(need + 4, B, nkv, hd, generator=g).to(torch.bfloat16)
        caches_cpu.append((key, value))
        kv = torch.empty(need + 4, nkv, B, 2 * hd, dtype=torch.bfloat16, device=DEV)
        k_view, v_view = kv.transpose(1, 2).split(hd, dim=-1)
        k_view.copy_(key)
        v_view.copy_(value)
        kvs.append(kv)
        sqk = (torch.rand(Q, generator=g) + 0.5).to(torch.bfloat16)
        s_gate = (torch.rand(Q, generator=g) + 0.5).to(torch.bfloat16)
        alpha = (torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)
        subs.append(dict(sqk=sqk, s_gate=s_gate, alpha=alpha))
        w_q.append((torch.randn(2 * (Q + KV), H, generator=g) / 16).to(DEV))
        w_o.append((torch.randn(H, Q, generator=g) / 16).to(DEV))
    layers_b = [AttentionSublayer(WavefrontLayer([kvs[i]] * rows, [0] * rows, table.shape[1],
                                                 nkv, hd),
                                  subs[i]["sqk"].to(DEV), subs[i]["s_gate"].to(DEV),
                                  cos_sin.to(DEV), subs[i]["alpha"].to(DEV), 0, hd ** -0.5)
                for i in range(layers)]

    def natural(nm):
        return nm.transpose(1, 2).reshape(nm.shape[0], -1)

    def qkvg_gemv(i, h_nm, partials):
        x = natural(h_nm)
        for s in range(partials.shape[0]):
            c = slice(s * H // partials.shape[0], (s + 1) * H // partials.shape[0])
            torch.matmul(x[:, c], w_q[i][:, c].t(), out=partials[s])

    def out_gemv(i, att_nm, partials):
        x = natural(att_nm)
        for s in range(partials.shape[0]):
            c = slice(s * Q // partials.shape[0], (s + 1) * Q // partials.shape[0])
            torch.matmul(x[:, c], w_o[i][:, c].t(), out=partials[s])

    attn = DecodeAttention(nh, nkv, hd, DEV, splits=8, max_tokens=rows)
    block = WavefrontRecurrentBlock(attn, layers_b, table.to(DEV), H, W.SQK_FACTOR, 0.9, 2.5, EPS,
                                    shared_cache=True, qkvg_gemv=qkvg_gemv, out_gemv=out_gemv)
    positions = list(range(position, position + rows))
    seq_lens = [p + 1 for p in positions]
    a0 = torch.randn(rows, H, generator=g)
    a0 = a0 / a0.norm(dim=1, keepdim=True)
    h_in = a0.to(torch.bfloat16)
    h_in_nm = a0.reshape(rows, H // 8, 8).transpose(1, 2).contiguous()
    pos_d = torch.tensor(positions, dtype=torch.int64, device=DEV)
    len_d = torch.tensor(seq_lens, dtype=torch.int32, device=DEV)
    h_d, h_nm_d = h_in.to(DEV), h_in_nm.to(DEV)
    h, h_nm = block.replay(rows, pos_d, len_d, h_d, h_nm_d)
    torch.cuda.synchronize()
    attn.check_errors()
    first = (h.clone(), h_nm.clone())
    parts_q = [block.qkvg_partials(i, rows).cpu() for i in range(layers)]
    parts_o = [block.out_partials(i, rows).cpu() for i in range(layers)]

    a = h_in
    nm_ref = None
    for i in range(layers):
        qk, v, gate = O.qkvg_epilogue(parts_q[i], torch.tensor(positions), cos_sin,
                                      subs[i]["s_gate"], 0.9, nh, nkv, hd)
        key, value = caches_cpu[i]
        out = O.multi_from_raw(qk, v, subs[i]["sqk"], W.SQK_FACTOR, EPS,
                               torch.zeros(rows, dtype=torch.int64), key.view(-1), value.view(-1),
                               tuple(key.shape), key.stride(), table.reshape(-1),
                               torch.zeros(rows, dtype=torch.int64), seq_lens, 0, hd ** -0.5, gate,
                               nh, nkv, shared_cache=True)
        _, a, nm_ref = O.residual_tokens(parts_o[i], natural(out), None, a, subs[i]["alpha"], 2.5)
    for i in range(layers):
        k_view, v_view = kvs[i].transpose(1, 2).split(hd, dim=-1)
        assert torch.equal(k_view.cpu().view(torch.int16), caches_cpu[i][0].view(torch.int16)), i
        assert torch.equal(v_view.cpu().view(torch.int16), caches_cpu[i][1].view(torch.int16)), i
    torch.testing.assert_close(first[1].cpu(), nm_ref, rtol=1e-5, atol=1e-7)
    for _ in range(2):
        h2, nm2 = block.replay(rows, pos_d, len_d, h_d, h_nm_d)
        torch.cuda.synchronize()
        assert torch.equal(h2, first[0]) and torch.equal(nm2, first[1])
    attn.check_errors()
