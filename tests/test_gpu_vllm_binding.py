"""vllm_binding against vLLM 0.22's own decode structures (the installed vllm package).

The KV cache is allocated in the shape vLLM's Triton backend asks for
(TritonAttentionBackend.get_kv_cache_shape: (blocks, 2, block_size, kv_heads, head_dim)) or in
the layout the reference's pinned vLLM uses ((blocks, kv_heads, block_size, 2 * head_dim)); the
metadata is a TritonAttentionMetadata of a decode batch (max_query_len 1) whose block_table
has a row stride wider than the rows in use and whose padded requests have seq_len 0 and
slot -1, as vLLM pads CUDA-graph decode batches.  Checked: outputs against the oracle, every
new k / v row at the slot vLLM's slot_mapping gives (block_table[t, pos // B] * B + pos % B)
and no other cache row touched; two layers with different tables through one binding.
"""

from __future__ import annotations

import pytest
import torch

import workloads as W
from dory_decode_attention import EPS, DecodeAttention
from gpu_helpers import assert_close, oracle_out, oracle_rows
from vllm_binding import VllmDecodeBinding, kv_cache_views

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def triton_backend():
    """vLLM's Triton attention backend module (imported only when a test runs)."""
    return pytest.importorskip("vllm.v1.attention.backends.triton_attn")


def vllm_batch(case: W.Case, layout: str, padded: int, extra_width: int = 3):
    """(kv_cache, metadata, slot_mapping list) of a decode batch in vLLM's structures."""
    triton_attn = triton_backend()
    NKV, HD, B = case.num_kv_heads, case.head_dim, case.block_size
    if layout == "vllm":
        shape = triton_attn.TritonAttentionBackend.get_kv_cache_shape(case.num_blocks, B, NKV, HD)
    else:
        shape = (case.num_blocks, NKV, B, 2 * HD)
    kv = torch.empty(shape, dtype=torch.bfloat16, device=DEV)
    key, value = kv_cache_views(kv, NKV, HD)
    key.copy_(case.key.to(torch.bfloat16))
    value.copy_(case.value.to(torch.bfloat16))
    T, width = case.tokens, case.tables.shape[1]
    R = T + padded
    table = torch.zeros(R, width + extra_width, dtype=torch.int32)
    for t in range(T):
        table[t, :width] = case.tables[case.table_rows[t]]
    seq_lens = torch.tensor(list(case.seq_lens) + [0] * padded, dtype=torch.int32)
    slots = []
    for t in range(R):
        n = int(seq_lens[t])
        slots.append(int(table[t, (n - 1) // B]) * B + (n - 1) % B if n > 0 else -1)
    meta = triton_attn.TritonAttentionMetadata(
        num_actual_tokens=T, max_query_len=1,
        query_start_loc=torch.arange(R + 1, dtype=torch.int32, device=DEV),
        max_seq_len=int(seq_lens.max()), seq_lens=seq_lens.to(DEV), block_table=table.to(DEV),
        slot_mapping=torch.tensor(slots, dtype=torch.int64, device=DEV), seq_threshold_3D=0,
        num_par_softmax_segments=0, softmax_segm_output=torch.empty(0, device=DEV),
        softmax_segm_max=torch.empty(0, device=DEV), softmax_segm_expsum=torch.empty(0, device=DEV),
        use_cascade=False, common_prefix_len=0, cu_prefix_query_lens=None, prefix_kv_lens=None,
        suffix_kv_lens=None)
    return kv, meta, slots


def run(binding, case, layout, padded):
    kv, meta, slots = vllm_batch(case, layout, padded)
    before = kv.clone()
    R, NH, NKV, HD = case.tokens + padded, case.num_heads, case.num_kv_heads, case.head_dim
    pad = lambda x, n: torch.cat([x, torch.zeros(padded, n)]) if padded else x  # noqa: E731
    qk = pad(case.qk, (NH + NKV) * HD).contiguous().to(DEV)
    v = pad(case.v, NKV * HD).contiguous().to(DEV)
    gate = pad(case.gate, NH * HD).contiguous().to(DEV)
    out = torch.full((R, 8, NH * HD // 8), float("nan"), device=DEV)
    binding.decode(meta, kv, qk, v, case.sqk.to(DEV), case.sqk_factor, EPS, case.window,
                   case.scale, gate, out)
    torch.cuda.synchronize()
    binding.attention.check_errors()
    return kv.cpu(), before.cpu(), out.cpu(), slots


def check(case, layout, padded, kv, before, out, slots):
    T = case.tokens
    assert_close(out[:T], oracle_out(case))
    assert torch.equal(out[T:], torch.zeros_like(out[T:]))
    key_b, val_b = kv_cache_views(before, case.num_kv_heads, case.head_dim)
    key_a, val_a = kv_cache_views(kv, case.num_kv_heads, case.head_dim)
    B = case.block_size
    changed = (key_a != key_b).any(-1).any(-1) | (val_a != val_b).any(-1).any(-1)  # [blocks, B]
    expect = torch.zeros_like(changed)
    rows = oracle_rows(case)
    for t in range(T):
        s = slots[t]
        expect[s // B, s % B] = True
        k_row, v_row = rows[t]
        assert torch.equal(key_a[s // B, s % B].view(torch.int16), k_row.view(torch.int16))
        assert torch.equal(val_a[s // B, s % B].view(torch.int16), v_row.view(torch.int16))
    # only the new tokens' slots changed (a slot may hold its old value by chance: subset)
    assert not (changed & ~expect).any()


@pytest.mark.parametrize("layout", ["vllm", "pinned"])
def test_decode_batch_with_padding(layout):
    case = W.batched(seed=960, lens=[15, 16, 640, 1025, 3, 300])
    attn = DecodeAttention(32, 8, 128, DEV, splits=8, max_tokens=8)
    kv, before, out, slots = run(VllmDecodeBinding(attn), case, layout, padded=2)
    check(case, layout, 2, kv, before, out, slots)


def test_two_layers_different_tables_and_shapes():
    attn = DecodeAttention(16, 4, 256, DEV, splits=16, max_tokens=4)
    binding = VllmDecodeBinding(attn)
    for seed, lens, window in ((961, [1200, 50], 1024), (962, [7, 2000, 640], 0)):
        case = W.batched(seed=seed, lens=lens, num_heads=16, num_kv_heads=4, head_dim=256,
                         window=window)
        kv, before, out, slots = run(binding, case, "vllm", padded=0)
        check(case, "vllm", 0, kv, before, out, slots)


def test_graph_capture_after_first_call():
    case = W.batched(seed=963, lens=[100, 900])
    attn = DecodeAttention(32, 8, 128, DEV, splits=8, max_tokens=2)
    binding = VllmDecodeBinding(attn)
    kv, meta, _ = vllm_batch(case, "vllm", padded=0)
    qk, v, gate = case.qk.to(DEV), case.v.to(DEV), case.gate.to(DEV)
    sqk = case.sqk.to(DEV)
    out = torch.zeros(2, 8, 512, device=DEV)

    def step():
        binding.decode(meta, kv, qk, v, sqk, case.sqk_factor, EPS, 0, case.scale, gate, out)

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    out.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    attn.check_errors()


def test_slot_mapping_decides_where_rows_go():
    """The metadata's slot_mapping, not the block table, says where each new row is cached:
    a request whose slot points into a block no table uses gets its row there, a request
    with slot -1 writes nothing, a padded row writes nothing.  Attention is unchanged (each
    token uses its new key and value at its own position either way)."""
    case = W.batched(seed=964, lens=[300, 40, 777], pool_factor=1.5)
    kv, meta, slots = vllm_batch(case, "vllm", padded=1)
    B, T = case.block_size, case.tokens
    used = set(case.tables.flatten().tolist())
    spare = next(b for b in range(case.num_blocks) if b not in used)
    custom = list(slots)
    custom[0] = spare * B + 5  # request 0: a row of an unused block
    custom[1] = -1             # request 1: not cached
    meta.slot_mapping = torch.tensor(custom, dtype=torch.int64, device=DEV)
    before = kv.clone()
    NH, NKV, HD = case.num_heads, case.num_kv_heads, case.head_dim
    pad = lambda x, n: torch.cat([x, torch.zeros(1, n)])  # noqa: E731
    qk = pad(case.qk, (NH + NKV) * HD).contiguous().to(DEV)
    v = pad(case.v, NKV * HD).contiguous().to(DEV)
    gate = pad(case.gate, NH * HD).contiguous().to(DEV)
    out = torch.full((T + 1, 8, NH * HD // 8), float("nan"), device=DEV)
    attn = DecodeAttention(NH, NKV, HD, DEV, splits=8, max_tokens=8)
    VllmDecodeBinding(attn).decode(meta, kv, qk, v, case.sqk.to(DEV), case.sqk_factor, EPS,
                                   case.window, case.scale, gate, out)
    torch.cuda.synchronize()
    attn.check_errors()
    assert_close(out[:T].cpu(), oracle_out(case))
    assert torch.equal(out[T:].cpu(), torch.zeros_like(out[T:].cpu()))
    key_b, val_b = kv_cache_views(before.cpu(), NKV, HD)
    key_a, val_a = kv_cache_views(kv.cpu(), NKV, HD)
    changed = (key_a != key_b).any(-1).any(-1) | (val_a != val_b).any(-1).any(-1)
    rows = oracle_rows(case)
    expect = torch.zeros_like(changed)
    for t in (0, 2):
        s = custom[t]
        expect[s // B, s % B] = True
        assert torch.equal(key_a[s // B, s % B].view(torch.int16), rows[t][0].view(torch.int16))
        assert torch.equal(val_a[s // B, s % B].view(torch.int16), rows[t][1].view(torch.int16))
    assert not (changed & ~expect).any()  # request 1's table slot and the padded row: untouched


def test_fp8_cache_in_vllm_shape():
    """vLLM's fp8 kv_cache_dtype: the cache tensor is uint8 e4m3 bytes in the backend's shape;
    outputs against the oracle's e4m3 restatement, the slots vLLM's slot_mapping gives hold the
    quantised rows, nothing else changes."""
    import dory_oracle as O
    triton_attn = triton_backend()
    case = W.batched(seed=1300, lens=[40, 700, 15, 333])
    NH, NKV, HD, B = case.num_heads, case.num_kv_heads, case.head_dim, case.block_size
    ks, vs = 0.5, 0.25
    shape = triton_attn.TritonAttentionBackend.get_kv_cache_shape(case.num_blocks, B, NKV, HD)
    kv = torch.empty(shape, dtype=torch.uint8, device=DEV)
    key, value = kv_cache_views(kv, NKV, HD)
    key.copy_(W.e4m3_bytes(case.key, ks))
    value.copy_(W.e4m3_bytes(case.value, vs))
    _, meta, slots = vllm_batch(case, "vllm", 0)
    attn = DecodeAttention(NH, NKV, HD, DEV, splits=8, max_tokens=case.tokens,
                           kv_cache_dtype="fp8")
    binding = VllmDecodeBinding(attn)
    out = torch.full((case.tokens, 8, NH * HD // 8), float("nan"), device=DEV)
    binding.decode(meta, kv, case.qk.to(DEV), case.v.to(DEV), case.sqk.to(DEV),
                   case.sqk_factor, EPS, 0, case.scale, case.gate.to(DEV), out, k_scale=ks,
                   v_scale=vs)
    torch.cuda.synchronize()
    attn.check_errors()
    key8, value8 = W.e4m3_bytes(case.key, ks), W.e4m3_bytes(case.value, vs)
    want = torch.stack([O.from_raw_fp8(case.qk[t], case.v[t], case.sqk, case.sqk_factor, EPS,
                                       slots[t], key8, value8, case.tables[case.table_rows[t]],
                                       case.seq_lens[t], 0, case.scale, case.gate[t], NH, NKV,
                                       ks, vs) for t in range(case.tokens)])
    assert_close(out.cpu(), want)
    k_dev, v_dev = kv_cache_views(kv, NKV, HD)
    assert torch.equal(k_dev.cpu(), key8) and torch.equal(v_dev.cpu(), value8)
