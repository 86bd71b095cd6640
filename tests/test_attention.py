"""The attention layer's plain KV-cache write and paged decode attention (nanovllm_b200.kernels.attention).

store_kvcache (nanovllm/layers/attention.py:11-41): bit-exact against the oracle's restatement of
store_kvcache_kernel (every written row equals the source row, every other row untouched), for strided k/v views
of a qkv buffer, slot -1, int32 and int64 slot maps, bf16/fp16/fp32, and rows whose addresses allow only narrow
accesses.

Decode attention (the flash_attn_with_kvcache call of attention.py:84-91): against the oracle (float64 softmax
attention over the paged cache, oracle/reference_math.py) within the bf16 tolerance rtol 1.6e-2 / atol 1e-2, and
against flash-attn's own flash_attn_with_kvcache on the same inputs where flash-attn takes them (pages of 256
tokens). Covers the decode-step shape (32 sequences x 1024 keys, Qwen3-0.6B heads), ragged and empty sequences,
grouped heads 1..8, 1..4 queries per sequence (causal bottom-right alignment), every split count, CUDA-graph
replay, and block-table entries / lengths out of range (skipped, flagged, never read).
"""
import pytest
import torch

from oracle import reference_math as om

RTOL, ATOL = 1.6e-2, 1e-2


# ---------------------------------------------------------------------------------------------------------------
# CPU: the oracle itself and the wrappers' host-side checks.

def test_oracle_paged_equals_contiguous():
    """The oracle's paged gather equals attention over the same keys laid out contiguously."""
    g = torch.Generator().manual_seed(0)
    B, n, hq, hkv, d, bs = 3, 2, 8, 2, 128, 16
    lens = [5, 40, 33]
    pages = 3
    kc = torch.randn(12, bs, hkv, d, generator=g).bfloat16()
    vc = torch.randn(12, bs, hkv, d, generator=g).bfloat16()
    table = torch.randperm(12, generator=g)[:B * pages].reshape(B, pages).int()
    q = torch.randn(B, n, hq, d, generator=g).bfloat16()
    sl = torch.tensor(lens, dtype=torch.int32)
    paged = om.paged_decode_attention(q, kc, vc, sl, table, 0.1, True)
    dense_k = kc[table.long()].reshape(B, pages * bs, hkv, d)
    dense_v = vc[table.long()].reshape(B, pages * bs, hkv, d)
    dense = om.paged_decode_attention(q, dense_k, dense_v, sl, None, 0.1, True)
    assert torch.equal(paged, dense)


def test_oracle_causal_alignment_and_empty_rows():
    """Query i of n sees keys [0, L - n + i]: with n = L + 1 the first query sees nothing (zeros) and the last one
    sees every key; softmax rows sum to one (a constant V row comes back unchanged)."""
    d, L, n = 128, 3, 4
    q = torch.randn(1, n, 1, d).bfloat16()
    kc = torch.randn(1, 8, 1, d).bfloat16()
    vc = torch.ones(1, 8, 1, d).bfloat16()
    out = om.paged_decode_attention(q, kc, vc, torch.tensor([L], dtype=torch.int32), None, 0.1, True)
    assert torch.equal(out[0, 0], torch.zeros(1, d))
    assert torch.allclose(out[0, 1:], torch.ones(n - 1, 1, d), atol=1e-6)


def test_store_kvcache_checks_mirror_the_reference():
    """The reference's assertions (attention.py:36-40) fire before anything touches a device."""
    from nanovllm_b200.kernels.attention import store_kvcache
    key = torch.zeros(4, 2, 8)
    cache = torch.zeros(2, 4, 2, 8)
    with pytest.raises(AssertionError):
        store_kvcache(key[..., ::2], key[..., ::2], cache, cache, torch.zeros(4, dtype=torch.int32))
    with pytest.raises(AssertionError):
        store_kvcache(key, key, cache, cache, torch.zeros(3, dtype=torch.int32))
    with pytest.raises(AssertionError):
        store_kvcache(key, key, cache.transpose(1, 2), cache, torch.zeros(4, dtype=torch.int32))


def test_auto_method_follows_the_measured_crossover(monkeypatch):
    """"auto" keeps the cluster kernel unless, at 1-2 rows per KV head, the (sequence, head) pairs overfill its
    resident CTAs (3 per SM) and leave the last wave less than 70 % full (148 SMs: 444 slots)."""
    from nanovllm_b200.kernels import attention as at
    monkeypatch.setitem(at._sm_counts, 0, 148)
    dev = torch.device("cuda", 0)
    assert at.choose_method(32, 8, 2, dev) == "cluster"      # decode step, 256 pairs: one partial wave
    assert at.choose_method(64, 8, 2, dev) == "streamk"      # 512 pairs: 1.15 waves
    assert at.choose_method(48, 8, 2, dev) == "cluster"      # 384 pairs fit
    assert at.choose_method(96, 8, 2, dev) == "cluster"      # 1.73 waves
    assert at.choose_method(128, 8, 2, dev) == "cluster"     # 2.31 waves
    assert at.choose_method(64, 8, 4, dev) == "cluster"      # more rows: not measured faster
    assert at.choose_method(100, 5, 1, dev) == "streamk"     # 500 pairs: 1.13 waves


# ---------------------------------------------------------------------------------------------------------------
# GPU: store_kvcache.

def _qkv_views(T, hq, hkv, d, dtype, device, pad=0, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    width = (hq + 2 * hkv) * d + pad
    qkv = torch.randn(T, width, generator=g).to(dtype).to(device)
    k = qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d) if pad == 0 else \
        torch.as_strided(qkv, (T, hkv, d), (width, d, 1), hq * d)
    v = torch.as_strided(qkv, (T, hkv, d), (width, d, 1), (hq + hkv) * d)
    return k, v


def _slots(T, num_slots, skip, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    s = torch.randperm(num_slots, generator=g)[:T].to(dtype)
    s[torch.randperm(T, generator=g)[:skip]] = -1
    return s


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("slot_dtype", [torch.int32, torch.int64])
@pytest.mark.parametrize("T,hkv,pad", [(1, 8, 0), (37, 8, 0), (2048, 8, 0), (300, 2, 1), (129, 1, 3)])
def test_store_kvcache_bitwise(cuda, dtype, slot_dtype, T, hkv, pad):
    from nanovllm_b200.kernels.attention import store_kvcache
    import nanovllm_b200
    d, hq, blocks, bs = 128, 2 * hkv, 16, 256
    k, v = _qkv_views(T, hq, hkv, d, dtype, cuda, pad=pad)
    slots = _slots(T, blocks * bs, T // 20, slot_dtype).to(cuda)
    base = torch.randn(blocks, bs, hkv, d).to(dtype).to(cuda)
    kc, vc = base.clone(), base.clone() + 1
    ek, ev = kc.clone(), vc.clone()
    nanovllm_b200.status(cuda, clear=True)
    store_kvcache(k, v, kc, vc, slots)
    om.store_kvcache(k, v, ek, ev, slots)
    torch.cuda.synchronize()
    assert torch.equal(kc, ek) and torch.equal(vc, ev)
    assert nanovllm_b200.status(cuda) == 0


@pytest.mark.gpu
def test_store_kvcache_empty_and_bad_slots(cuda):
    from nanovllm_b200.kernels.attention import store_kvcache
    import nanovllm_b200
    d, hkv, blocks, bs = 128, 8, 4, 16
    kc = torch.zeros(blocks, bs, hkv, d, dtype=torch.bfloat16, device=cuda)
    vc = torch.zeros_like(kc)
    k, v = _qkv_views(0, hkv, hkv, d, torch.bfloat16, cuda)
    store_kvcache(k, v, kc, vc, torch.zeros(0, dtype=torch.int32, device=cuda))  # no launch
    k, v = _qkv_views(4, hkv, hkv, d, torch.bfloat16, cuda)
    slots = torch.tensor([3, blocks * bs, -5, 7], dtype=torch.int32, device=cuda)
    nanovllm_b200.status(cuda, clear=True)
    store_kvcache(k, v, kc, vc, slots)
    assert nanovllm_b200.status(cuda, clear=True) == 2  # NVB200_STATUS_BAD_SLOT
    flat_k, flat_v = kc.view(-1, hkv * d), vc.view(-1, hkv * d)
    assert torch.equal(flat_k[3], k[0].reshape(-1)) and torch.equal(flat_v[7], v[3].reshape(-1))
    others = torch.ones(blocks * bs, dtype=torch.bool)
    others[[3, 7]] = False
    assert flat_k[others.to(cuda)].abs().sum() == 0 and flat_v[others.to(cuda)].abs().sum() == 0


# ---------------------------------------------------------------------------------------------------------------
# GPU: decode attention.

def _decode_inputs(B, n, hq, hkv, bs, lens, device, seed=0, extra_blocks=3):
    g = torch.Generator().manual_seed(seed)
    d = 128
    pages = max(1, max((L + bs - 1) // bs for L in lens))
    nb = B * pages + extra_blocks
    q = torch.randn(B, n, hq, d, generator=g).bfloat16().to(device)
    kc = torch.randn(nb, bs, hkv, d, generator=g).bfloat16().to(device)
    vc = torch.randn(nb, bs, hkv, d, generator=g).bfloat16().to(device)
    table = torch.randperm(nb, generator=g)[:B * pages].reshape(B, pages).int().to(device)
    sl = torch.tensor(lens, dtype=torch.int32, device=device)
    return q, kc, vc, sl, table


DECODE_CASES = [
    # B, n, hq, hkv, block_size, lens, causal, num_splits
    (32, 1, 16, 8, 256, [1024] * 32, True, 0),                  # the decode-step shape (Qwen3-0.6B, TP 1)
    (32, 1, 8, 4, 256, [1024] * 32, True, 0),                   # ... at TP 2
    (3, 1, 16, 8, 256, [1, 300, 1024], True, 0),
    (4, 1, 32, 8, 256, [513, 77, 1, 2000], True, 0),            # Qwen3-8B heads (group 4)
    (2, 2, 16, 8, 16, [40, 2], True, 0),                        # 2 queries per sequence, small pages
    (2, 4, 16, 4, 32, [100, 4], True, 2),                       # 16 rows per KV head
    (1, 1, 16, 8, 256, [4096], True, 8),
    (5, 1, 8, 1, 64, [0, 1, 65, 128, 700], False, 0),           # one KV head, an empty sequence
    (1, 3, 4, 2, 16, [2], True, 0),                             # more queries than keys
    (2, 1, 2, 2, 256, [257, 3000], True, 0),                    # group 1
]


@pytest.mark.gpu
@pytest.mark.parametrize("B,n,hq,hkv,bs,lens,causal,splits", DECODE_CASES)
def test_decode_attention_matches_oracle(cuda, B, n, hq, hkv, bs, lens, causal, splits):
    from nanovllm_b200.kernels.attention import flash_attn_with_kvcache
    import nanovllm_b200
    q, kc, vc, sl, table = _decode_inputs(B, n, hq, hkv, bs, lens, cuda)
    scale = 128 ** -0.5
    nanovllm_b200.status(cuda, clear=True)
    out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=table, softmax_scale=scale,
                                  causal=causal, num_splits=splits)
    ref = om.paged_decode_attention(q, kc, vc, sl, table, scale, causal)
    assert out.shape == (B, n, hq, 128) and out.dtype == torch.bfloat16
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
    assert nanovllm_b200.status(cuda) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("splits", [1, 2, 3, 4, 5, 6, 7, 8])
def test_decode_attention_every_split_count(cuda, splits):
    from nanovllm_b200.kernels.attention import flash_attn_with_kvcache
    q, kc, vc, sl, table = _decode_inputs(4, 1, 16, 8, 256, [1024, 700, 1, 2048], cuda, seed=splits)
    out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=table, softmax_scale=0.088,
                                  causal=True, num_splits=splits)
    ref = om.paged_decode_attention(q, kc, vc, sl, table, 0.088, True)
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)


@pytest.mark.gpu
@pytest.mark.parametrize("B,n,hq,hkv,lens", [(32, 1, 16, 8, [1024] * 32), (3, 2, 32, 8, [5, 600, 1500]),
                                             (2, 1, 16, 8, [256, 2049])])
def test_decode_attention_matches_flash_attn(cuda, B, n, hq, hkv, lens):
    """The same call through flash-attn's own kernel (the reference's decode path): both within the bf16 tolerance
    of each other and of the float64 oracle."""
    flash_attn = pytest.importorskip("flash_attn")
    from nanovllm_b200.kernels.attention import flash_attn_with_kvcache
    q, kc, vc, sl, table = _decode_inputs(B, n, hq, hkv, 256, lens, cuda, seed=7)
    kw = dict(cache_seqlens=sl, block_table=table, softmax_scale=128 ** -0.5, causal=True)
    ours = flash_attn_with_kvcache(q, kc, vc, **kw)
    theirs = flash_attn.flash_attn_with_kvcache(q, kc, vc, **kw)
    ref = om.paged_decode_attention(q, kc, vc, sl, table, 128 ** -0.5, True)
    torch.testing.assert_close(theirs.float(), ref, rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(ours.float(), theirs.float(), rtol=RTOL, atol=ATOL)
    err_ours = (ours.float() - ref).abs().max().item()
    err_theirs = (theirs.float() - ref).abs().max().item()
    assert err_ours <= 2 * err_theirs + 1e-3, (err_ours, err_theirs)


@pytest.mark.gpu
def test_decode_attention_without_block_table(cuda):
    from nanovllm_b200.kernels.attention import flash_attn_with_kvcache
    g = torch.Generator().manual_seed(3)
    q = torch.randn(3, 1, 8, 128, generator=g).bfloat16().to(cuda)
    kc = torch.randn(3, 300, 2, 128, generator=g).bfloat16().to(cuda)
    vc = torch.randn(3, 300, 2, 128, generator=g).bfloat16().to(cuda)
    sl = torch.tensor([300, 1, 129], dtype=torch.int32, device=cuda)
    out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, softmax_scale=0.1, causal=True)
    ref = om.paged_decode_attention(q, kc, vc, sl, None, 0.1, True)
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
    out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=7, softmax_scale=0.1, causal=False)
    ref = om.paged_decode_attention(q, kc, vc, torch.full((3,), 7), None, 0.1, False)
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)


@pytest.mark.gpu
def test_decode_attention_graph_replay(cuda):
    """Captured once, replayed on new cache contents and lengths: equal to eager calls bit for bit."""
    from nanovllm_b200.kernels.attention import flash_attn_with_kvcache
    q, kc, vc, sl, table = _decode_inputs(8, 1, 16, 8, 256, [900] * 8, cuda, seed=1)
    kw = dict(block_table=table, softmax_scale=0.088, causal=True)
    flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, **kw)  # first call outside the capture
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, **kw)
    for seed in range(3):
        g = torch.Generator().manual_seed(100 + seed)
        kc.copy_(torch.randn(kc.shape, generator=g).bfloat16())
        sl.copy_(torch.randint(1, 1024, (8,), generator=g, dtype=torch.int32))
        graph.replay()
        eager = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, **kw)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    del graph


@pytest.mark.gpu
def test_decode_attention_bad_table_and_length(cuda):
    """A block-table entry outside [0, num_blocks) and a length beyond the table are never followed: flagged in the
    status word; the other sequences are unaffected."""
    from nanovllm_b200.kernels.attention import flash_attn_with_kvcache
    import nanovllm_b200
    q, kc, vc, sl, table = _decode_inputs(3, 1, 16, 8, 256, [300, 300, 300], cuda, seed=2)
    good = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=sl, block_table=table, softmax_scale=0.1, causal=True)
    bad_table, bad_len = table.clone(), sl.clone()
    bad_table[0, 1] = kc.shape[0] + 5
    bad_len[1] = 10 ** 6
    nanovllm_b200.status(cuda, clear=True)
    out = flash_attn_with_kvcache(q, kc, vc, cache_seqlens=bad_len, block_table=bad_table, softmax_scale=0.1,
                                  causal=True)
    assert nanovllm_b200.status(cuda, clear=True) == 2
    assert torch.equal(out[2], good[2]) and out.isfinite().all()


# ---------------------------------------------------------------------------------------------------------------
# GPU: the stream-K decode kernel (nvb200_paged_decode_attention_streamk through decode_attention(method="streamk")).

STREAMK_CASES = DECODE_CASES + [
    # one sequence split over every resident CTA: hundreds of partial records merged by the last CTA to finish
    (1, 1, 8, 1, 256, [8192], True, 0),
    # many short sequences: ranges of many whole (sequence, head) segments, empty ones among them
    (300, 1, 16, 8, 16, [(i * 37) % 41 for i in range(300)], True, 0),
    # every sequence empty: no units at all, every output row zero
    (4, 1, 16, 8, 256, [0, 0, 0, 0], True, 0),
    # 16 query rows per KV head with long sequences (two CTAs per SM)
    (6, 4, 16, 4, 64, [3000, 17, 2048, 1, 999, 4096], True, 0),
    # 8 rows per KV head, non-causal, block size 16
    (9, 1, 64, 8, 16, [513] * 9, False, 0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("B,n,hq,hkv,bs,lens,causal,splits", STREAMK_CASES)
def test_decode_streamk_matches_oracle(cuda, B, n, hq, hkv, bs, lens, causal, splits):
    from nanovllm_b200.kernels.attention import decode_attention
    import nanovllm_b200
    q, kc, vc, sl, table = _decode_inputs(B, n, hq, hkv, bs, lens, cuda)
    scale = 128 ** -0.5
    nanovllm_b200.status(cuda, clear=True)
    out = decode_attention(q, kc, vc, sl, block_table=table, softmax_scale=scale, causal=causal, method="streamk")
    ref = om.paged_decode_attention(q, kc, vc, sl, table, scale, causal)
    assert out.shape == (B, n, hq, 128) and out.dtype == torch.bfloat16
    torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
    assert nanovllm_b200.status(cuda) == 0
    if all(L == 0 for L in lens):
        assert torch.equal(out, torch.zeros_like(out))


@pytest.mark.gpu
def test_decode_streamk_deterministic_and_close_to_cluster(cuda):
    """Repeated stream-K calls give identical bits (split pairs merge in CTA order, whichever CTA finishes last), and
    agree with the cluster kernel within the bf16 tolerance at the decode-step shape."""
    from nanovllm_b200.kernels.attention import decode_attention
    q, kc, vc, sl, table = _decode_inputs(32, 1, 16, 8, 256, [1024] * 31 + [777], cuda, seed=11)
    kw = dict(block_table=table, softmax_scale=128 ** -0.5, causal=True)
    first = decode_attention(q, kc, vc, sl, method="streamk", **kw)
    for _ in range(3):
        assert torch.equal(decode_attention(q, kc, vc, sl, method="streamk", **kw), first)
    cluster = decode_attention(q, kc, vc, sl, method="cluster", **kw)
    torch.testing.assert_close(first.float(), cluster.float(), rtol=RTOL, atol=ATOL)


@pytest.mark.gpu
def test_decode_streamk_graph_replay(cuda):
    """Captured once (after an eager call created the workspace), replayed on new cache contents and lengths: equal to
    eager stream-K calls bit for bit, so the workspace's counters are back at zero after every replay."""
    from nanovllm_b200.kernels.attention import decode_attention
    q, kc, vc, sl, table = _decode_inputs(8, 1, 16, 8, 256, [900] * 8, cuda, seed=1)
    kw = dict(block_table=table, softmax_scale=0.088, causal=True, method="streamk")
    decode_attention(q, kc, vc, sl, **kw)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = decode_attention(q, kc, vc, sl, **kw)
    for seed in range(3):
        g = torch.Generator().manual_seed(200 + seed)
        kc.copy_(torch.randn(kc.shape, generator=g).bfloat16())
        sl.copy_(torch.randint(0, 1024, (8,), generator=g, dtype=torch.int32))
        graph.replay()
        eager = decode_attention(q, kc, vc, sl, **kw)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
        ref = om.paged_decode_attention(q, kc, vc, sl, table, 0.088, True)
        torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
    del graph


@pytest.mark.gpu
def test_decode_streamk_bad_table_and_length(cuda):
    """As for the cluster kernel: out-of-range table entries and lengths are flagged, never followed, and the other
    sequences' rows are unaffected (within rounding: the clamped length changes how the batch's tiles are divided
    between CTAs, so a sequence may be merged from different pieces)."""
    from nanovllm_b200.kernels.attention import decode_attention
    import nanovllm_b200
    q, kc, vc, sl, table = _decode_inputs(3, 1, 16, 8, 256, [300, 300, 300], cuda, seed=2)
    kw = dict(softmax_scale=0.1, causal=True, method="streamk")
    good = decode_attention(q, kc, vc, sl, block_table=table, **kw)
    bad_table, bad_len = table.clone(), sl.clone()
    bad_table[0, 1] = kc.shape[0] + 5
    bad_len[1] = 10 ** 6
    nanovllm_b200.status(cuda, clear=True)
    out = decode_attention(q, kc, vc, bad_len, block_table=bad_table, **kw)
    assert nanovllm_b200.status(cuda, clear=True) == 2
    torch.testing.assert_close(out[2].float(), good[2].float(), rtol=RTOL, atol=ATOL)
    assert out.isfinite().all()


@pytest.mark.gpu
def test_decode_streamk_consecutive_shapes_share_the_workspace(cuda):
    """Calls whose batch sizes and row counts differ, one after another on the device's one workspace: each call's
    counters lie apart from every call's partial records, so no call reads another's leftovers."""
    from nanovllm_b200.kernels.attention import decode_attention
    shapes = [(2, 1, 16, 8, 256, [4096, 3000]), (300, 1, 16, 8, 16, [(i * 13) % 50 for i in range(300)]),
              (1, 4, 16, 4, 64, [5000]), (64, 1, 16, 8, 256, [700] * 64), (2, 1, 16, 8, 256, [4096, 1])]
    for i, (B, n, hq, hkv, bs, lens) in enumerate(shapes * 2):
        q, kc, vc, sl, table = _decode_inputs(B, n, hq, hkv, bs, lens, cuda, seed=50 + i)
        out = decode_attention(q, kc, vc, sl, block_table=table, softmax_scale=0.1, causal=True, method="streamk")
        ref = om.paged_decode_attention(q, kc, vc, sl, table, 0.1, True)
        torch.testing.assert_close(out.float(), ref, rtol=RTOL, atol=ATOL)
