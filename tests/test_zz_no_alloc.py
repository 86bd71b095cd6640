"""The allocation-free decode attention entry point, nvb200_paged_decode_attention_noalloc, called through the C ABI.

Some callers cannot allocate device memory when they call attention: an engine that reserved nearly all free HBM for
its KV cache at start-up (nano-vllm sizes the cache from gpu_memory_utilization), a decode loop that must not let
cudaMalloc or cudaFree synchronise the device, or a plugin host that passes a kernel only its input and output
pointers. This entry point serves them: it runs the stream-K decode kernel with its scratch in a fixed 4 MiB array
inside the library, and allocates nothing.

Checked here against the library's existing entry point (nvb200_paged_decode_attention) within the bf16 tolerance
used throughout the attention tests, over consecutive calls of different shapes: the array keeps what the previous
call left, so every call after the first also checks that leftovers do not leak into a result. The file is named
so that pytest collects it last; it builds its own inputs, so it passes alone in a fresh process as well.
"""
import ctypes

import pytest
import torch

RTOL, ATOL = 1.6e-2, 1e-2


def _inputs(B, n, hq, hkv, bs, lens, device, seed):
    g = torch.Generator().manual_seed(seed)
    d = 128
    pages = max(1, max((L + bs - 1) // bs for L in lens))
    nb = B * pages + 2
    q = torch.randn(B, n, hq, d, generator=g).bfloat16().to(device)
    kc = torch.randn(nb, bs, hkv, d, generator=g).bfloat16().to(device)
    vc = torch.randn(nb, bs, hkv, d, generator=g).bfloat16().to(device)
    table = torch.randperm(nb, generator=g)[:B * pages].reshape(B, pages).int().to(device)
    sl = torch.tensor(lens, dtype=torch.int32, device=device)
    return q, kc, vc, sl, table


def _args(out, q, kc, vc, sl, table, scale, causal):
    from nanovllm_b200 import _lib
    B, n, hq, d = q.shape
    nb, bs, hkv, _ = kc.shape
    a = _lib.PagedDecodeArgs()
    a.out, a.q = out.data_ptr(), q.data_ptr()
    a.q_batch_stride, a.q_token_stride, a.q_head_stride = q.stride(0), q.stride(1), q.stride(2)
    a.k_cache, a.v_cache = kc.data_ptr(), vc.data_ptr()
    a.cache_block_stride, a.cache_token_stride, a.cache_head_stride = kc.stride()[:3]
    a.num_blocks = nb
    a.block_table, a.block_table_stride, a.max_blocks_per_seq = table.data_ptr(), table.stride(0), table.shape[1]
    a.seqlens = sl.data_ptr()
    a.batch, a.queries_per_seq, a.num_q_heads, a.num_kv_heads, a.head_dim, a.block_size = B, n, hq, hkv, d, bs
    a.causal, a.num_splits, a.dtype = int(causal), 0, _lib.BF16
    a.softmax_scale = scale
    a.status = _lib.status_word(q.device).data_ptr()
    return a


# The grid of a call is the smaller of the CTAs the SMs hold at once, the CTAs whose partial records fit in the array
# (244 at 16 query rows per KV head) and U / 16, U = Hkv * sum_b ceil(L_b / 16) tiles (every CTA streams at least 16
# tiles). The 8 x 8192-key call at 16 rows (U = 16384, U / 16 = 1024) is the one whose grid the array cuts to 244;
# the others are cut by U / 16 or not at all.
CALLS = [
    # B, n, hq, hkv, block_size, lens, causal, seed
    (32, 1, 16, 8, 256, [1024] * 32, True, 0),                    # decode-step shape: pairs split between CTAs
    (6, 4, 16, 4, 64, [3000, 17, 2048, 1, 999, 4096], True, 1),   # 16 rows per KV head, ragged lengths (U / 16 = 159)
    (8, 4, 16, 4, 256, [8192] * 8, True, 5),                      # 16 rows per KV head, grid cut to what the array holds
    (32, 1, 16, 8, 256, [1024] * 31 + [5], True, 2),              # the first shape again, after larger calls' leftovers
    (1, 1, 8, 1, 256, [8192], False, 3),                          # one pair split over every CTA (U / 16 = 32)
]


@pytest.mark.gpu
def test_noalloc_matches_existing_entry_point_on_consecutive_calls(cuda):
    import nanovllm_b200
    from nanovllm_b200 import _lib
    lib = _lib.lib()
    nanovllm_b200.status(cuda, clear=True)
    for B, n, hq, hkv, bs, lens, causal, seed in CALLS:
        q, kc, vc, sl, table = _inputs(B, n, hq, hkv, bs, lens, cuda, seed)
        stream = _lib.stream_of(q)
        scale = 128 ** -0.5
        got = torch.full((B, n, hq, 128), float("nan"), dtype=torch.bfloat16, device=cuda)
        want = torch.empty_like(got)
        a_new = _args(got, q, kc, vc, sl, table, scale, causal)
        a_old = _args(want, q, kc, vc, sl, table, scale, causal)
        assert lib.nvb200_paged_decode_attention_noalloc(ctypes.byref(a_new), stream) == _lib.OK
        assert lib.nvb200_paged_decode_attention(ctypes.byref(a_old), stream) == _lib.OK
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), rtol=RTOL, atol=ATOL)
    assert nanovllm_b200.status(cuda) == 0


@pytest.mark.gpu
def test_noalloc_rejects_more_pairs_than_its_array_holds(cuda):
    """batch * num_kv_heads above NVB200_DECODE_NOALLOC_MAX_PAIRS (16384) is refused before any launch; the output
    is left as it was."""
    from nanovllm_b200 import _lib
    lib = _lib.lib()
    B, hkv = 16384 // 8 + 1, 8
    q, kc, vc, sl, table = _inputs(B, 1, 16, hkv, 16, [1] * B, cuda, seed=4)
    out = torch.zeros(B, 1, 16, 128, dtype=torch.bfloat16, device=cuda)
    a = _args(out, q, kc, vc, sl, table, 0.1, True)
    assert lib.nvb200_paged_decode_attention_noalloc(ctypes.byref(a), _lib.stream_of(q)) == _lib.ERR_UNSUPPORTED
    torch.cuda.synchronize()
    assert torch.equal(out, torch.zeros_like(out))


def test_noalloc_checks_arguments_without_a_gpu():
    """Argument checks come before any CUDA call: a null argument block is refused, an empty batch does nothing."""
    from nanovllm_b200 import _lib
    lib = _lib.lib()
    assert lib.nvb200_paged_decode_attention_noalloc(None, None) == _lib.ERR_ARG
    a = _lib.PagedDecodeArgs()
    a.batch, a.queries_per_seq, a.num_q_heads, a.num_kv_heads, a.head_dim = 0, 1, 16, 8, 128
    a.block_size, a.max_blocks_per_seq, a.dtype = 256, 1, _lib.BF16
    assert lib.nvb200_paged_decode_attention_noalloc(ctypes.byref(a), None) == _lib.OK
