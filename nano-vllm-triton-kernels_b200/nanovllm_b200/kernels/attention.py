"""The attention layer's cache write and decode attention on B200 (drop-ins for nanovllm/layers/attention.py).

* `store_kvcache(key, value, k_cache, v_cache, slot_mapping)`: the reference's plain KV-cache write
  (nanovllm/layers/attention.py:34-41, the route Attention.forward takes when q/k norm and RoPE ran before it,
  :75-76), with the same arguments and the same assertions. The copy runs in `nvb200_store_kvcache`.
* `flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=..., block_table=..., softmax_scale=..., causal=...)`:
  the decode attention of Attention.forward (:84-91), which calls flash-attn's function of that name with these
  keywords. Same keywords and result ([B, n, Hq, D] in q's dtype); the work runs in `nvb200_paged_decode_attention`,
  an sm_100a kernel that streams each sequence's K/V rows through the block table once. Options the decode branch
  never passes (new k/v to append, rotary, batch indices, left padding, sliding windows, softcap, ALiBi, the
  log-sum-exp output) raise NotImplementedError; `supports()` tells beforehand whether a call is covered.

Both launch on the current torch stream, allocate their outputs with torch (graph-capture safe) and never read
device data on the host. Out-of-range slots, block-table entries and sequence lengths are skipped (never read or
written) and flagged in the device status word (nanovllm_b200.status()).
"""
import ctypes
import math

import torch

from nanovllm_b200 import _lib

_SLOT_BYTES = {torch.int32: 4, torch.int64: 8}


def _require(cond: bool, msg: str = "") -> None:
    if not cond:
        raise AssertionError(msg)


def _max_rows(t: torch.Tensor, row: int) -> int:
    """Rows of `row` elements reachable from t's first element (the extent of t's strides), for bounds."""
    if t.numel() == 0:
        return 0
    extent = 1 + sum((s - 1) * st for s, st in zip(t.shape, t.stride()))
    return extent // row


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """key, value: [N, Hkv, D] with contiguous heads (any token stride). k_cache, v_cache: caches whose dim-1 stride
    is Hkv * D (a [blocks, block_size, Hkv, D] or [slots, Hkv * D] cache); row slot of the flattened cache receives
    token t when slot_mapping[t] = slot, and slot -1 stores nothing. In place."""
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    _require(key.stride(-1) == 1 and value.stride(-1) == 1)
    _require(key.stride(1) == head_dim and value.stride(1) == head_dim)
    _require(k_cache.stride(1) == D and v_cache.stride(1) == D)
    _require(slot_mapping.numel() == N)
    _require(value.shape == key.shape and key.dtype == value.dtype == k_cache.dtype == v_cache.dtype,
             "key, value and the caches must share shape [N, Hkv, D] and dtype")
    _require(key.dtype in _lib.DTYPE_CODE, "dtype must be bf16, fp16 or fp32")
    _require(slot_mapping.dtype in _SLOT_BYTES, "slot_mapping must be int32 or int64")
    _require(key.device.type == "cuda", "key must be a CUDA tensor")
    if N == 0:
        return
    slots = slot_mapping if slot_mapping.is_contiguous() else slot_mapping.contiguous()
    num_slots = min(_max_rows(k_cache, D), _max_rows(v_cache, D))
    _lib.check(_lib.lib().nvb200_store_kvcache(
        key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
        slots.data_ptr(), _SLOT_BYTES[slots.dtype], N, D, num_slots, _lib.DTYPE_CODE[key.dtype],
        _lib.status_word(key.device).data_ptr(), _lib.stream_of(key)), "store_kvcache")


def supports(q, k_cache, v_cache, k=None, v=None, rotary_cos=None, rotary_sin=None, cache_seqlens=None,
             cache_batch_idx=None, cache_leftpad=None, block_table=None, softmax_scale=None, causal=False,
             window_size=(-1, -1), softcap=0.0, rotary_interleaved=True, alibi_slopes=None, num_splits=0,
             return_softmax_lse=False) -> bool:
    """Whether flash_attn_with_kvcache below takes this call: the decode form (no new k/v, rotary, batch index,
    left padding, window, softcap, ALiBi or lse), bf16 with head_dim 128, at most 16 query rows per KV head
    (n * Hq / Hkv), a unit last stride everywhere and 16-byte aligned cache rows."""
    if any(x is not None for x in (k, v, rotary_cos, rotary_sin, cache_batch_idx, cache_leftpad, alibi_slopes)):
        return False
    if tuple(window_size) != (-1, -1) or softcap != 0.0 or return_softmax_lse or cache_seqlens is None:
        return False
    if q.dim() != 4 or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        return False
    B, n, hq, d = q.shape
    hkv = k_cache.shape[2]
    if not (q.dtype == k_cache.dtype == v_cache.dtype == torch.bfloat16) or d != 128 or k_cache.shape[3] != d:
        return False
    if hkv == 0 or hq % hkv or n * (hq // hkv) > 16:
        return False
    if q.stride(-1) != 1 or k_cache.stride(-1) != 1 or v_cache.stride() != k_cache.stride():
        return False
    if any(s % 8 for s in k_cache.stride()[:3]) or k_cache.data_ptr() % 16 or v_cache.data_ptr() % 16:
        return False
    if block_table is not None and (block_table.dtype != torch.int32 or block_table.dim() != 2
                                    or block_table.stride(-1) != 1):
        return False
    if block_table is None and k_cache.shape[0] < B:
        return False
    return True


# How flash_attn_with_kvcache runs when the caller leaves num_splits at 0: "cluster" (nvb200_paged_decode_attention:
# one CTA, or a thread-block cluster of CTAs, per (sequence, KV head)), "streamk" (nvb200_paged_decode_attention_streamk:
# a persistent grid with equal shares of all tiles, merging split pairs through a per-device workspace) or "auto".
DEFAULT_METHOD = "auto"

# "auto" picks stream-K only where it was measured faster on B200 (L2 flushed, median of 200): at 1-2 query rows per
# KV head, when the (sequence, head) pairs overfill the cluster kernel's resident CTAs (3 per SM at these row counts)
# and leave its last wave less than 70 % full. 64 x 2048 keys (512 pairs, 1.15 waves): 96 vs 115 us; 64 x 1024:
# 57 vs 63 us. Elsewhere the cluster kernel was as fast or faster (32 x 1024: 32.8 vs 36.9 us; 96 x 1024, 1.73 waves:
# 71.7 vs 77.8 us; 128 x 512: 59.4 vs 61.4 us).
_AUTO_MAX_ROWS = 2
_CLUSTER_CTAS_PER_SM = 3
_AUTO_LAST_WAVE_FILL = 0.7
_sm_counts = {}


def _sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _sm_counts.get(idx)
    if n is None:
        n = _sm_counts[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return n


def choose_method(batch: int, num_kv_heads: int, rows: int, device: torch.device) -> str:
    """The kernel "auto" runs for `batch` sequences of `rows` query rows per KV head (queries x group)."""
    if rows > _AUTO_MAX_ROWS:
        return "cluster"
    slots = _CLUSTER_CTAS_PER_SM * _sm_count(device)
    pairs = batch * num_kv_heads
    if pairs <= slots:
        return "cluster"
    waves = pairs / slots
    return "streamk" if waves / math.ceil(waves) < _AUTO_LAST_WAVE_FILL else "cluster"

# One workspace per device for the stream-K kernel: zeroed once at allocation (the kernel leaves its counters at
# zero), sized generously so that it rarely grows. Calls on one device share it, which is safe for calls ordered on
# one stream (nano-vllm runs one stream per rank); a workspace replaced by a larger one is kept alive, since a
# captured CUDA graph may still use it.
_MIN_WORKSPACE_BYTES = 8 << 20
_workspaces = {}
_retired = []


def _decode_workspace(device: torch.device, nbytes: int):
    """This device's stream-K workspace with at least nbytes, or None when it would have to be allocated while a
    CUDA graph is being captured (a buffer allocated there belongs to the graph's pool)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        if torch.cuda.is_current_stream_capturing():
            return None
        fresh = torch.zeros(max(nbytes, _MIN_WORKSPACE_BYTES), dtype=torch.uint8, device=torch.device("cuda", idx))
        if ws is not None:
            _retired.append(ws)
        _workspaces[idx] = ws = fresh
    return ws


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, rotary_cos=None, rotary_sin=None,
                            cache_seqlens=None, cache_batch_idx=None, cache_leftpad=None, block_table=None,
                            softmax_scale=None, causal=False, window_size=(-1, -1), softcap=0.0,
                            rotary_interleaved=True, alibi_slopes=None, num_splits=0, return_softmax_lse=False):
    """Decode attention over a paged KV cache. q: [B, n, Hq, D]; k_cache, v_cache: [num_blocks, block_size, Hkv, D]
    (with block_table [B, max_blocks] int32) or [B, max_len, Hkv, D] (without); cache_seqlens: [B] int32 or an int,
    the keys in the cache per sequence. softmax_scale defaults to D ** -0.5; causal aligns query i of n with key
    L - n + i. num_splits: CTAs of one thread-block cluster sharing one sequence (1-8, the cluster kernel); 0 = the
    module's DEFAULT_METHOD with its own split choice. Returns [B, n, Hq, D]."""
    if not supports(q, k_cache, v_cache, k, v, rotary_cos, rotary_sin, cache_seqlens, cache_batch_idx,
                    cache_leftpad, block_table, softmax_scale, causal, window_size, softcap, rotary_interleaved,
                    alibi_slopes, num_splits, return_softmax_lse):
        raise NotImplementedError("nanovllm_b200 flash_attn_with_kvcache: only the decode form (bf16, head_dim 128, "
                                  "n * Hq / Hkv <= 16, no new k/v, rotary, window, softcap, ALiBi or lse) is built")
    method = "cluster" if num_splits and num_splits > 0 else DEFAULT_METHOD
    return decode_attention(q, k_cache, v_cache, cache_seqlens, block_table=block_table, softmax_scale=softmax_scale,
                            causal=causal, num_splits=num_splits, method=method)


def decode_attention(q, k_cache, v_cache, cache_seqlens, block_table=None, softmax_scale=None, causal=False,
                     num_splits=0, method="cluster"):
    """flash_attn_with_kvcache's decode form with the kernel named: method "cluster" (num_splits CTAs per sequence,
    0 = automatic), "streamk" (num_splits ignored) or "auto" (choose_method). A stream-K call made while a CUDA graph
    is being captured, before this device's workspace exists, runs the cluster kernel (make one call before
    capturing)."""
    if method not in ("cluster", "streamk", "auto"):
        raise ValueError(f"decode_attention: unknown method {method!r}")
    if isinstance(cache_seqlens, int):
        cache_seqlens = torch.full((q.shape[0],), cache_seqlens, dtype=torch.int32, device=q.device)
    if not supports(q, k_cache, v_cache, cache_seqlens=cache_seqlens, block_table=block_table):
        raise NotImplementedError("nanovllm_b200 decode_attention: bf16, head_dim 128, n * Hq / Hkv <= 16")
    B, n, hq, d = q.shape
    nb, bs, hkv, _ = k_cache.shape
    _require(q.device.type == "cuda" and k_cache.device == q.device, "q and the caches must be on one CUDA device")
    _require(cache_seqlens.shape == (B,) and cache_seqlens.dtype == torch.int32, "cache_seqlens must be [B] int32")
    seqlens = cache_seqlens if cache_seqlens.is_contiguous() else cache_seqlens.contiguous()
    if block_table is not None:
        _require(block_table.shape[0] == B and block_table.shape[1] > 0, "block_table must be [B, max_blocks]")
    scale = d ** -0.5 if softmax_scale is None else float(softmax_scale)
    out = torch.empty(B, n, hq, d, dtype=q.dtype, device=q.device)
    if B == 0:
        return out
    a = _lib.PagedDecodeArgs()
    a.out, a.q = out.data_ptr(), q.data_ptr()
    a.q_batch_stride, a.q_token_stride, a.q_head_stride = q.stride(0), q.stride(1), q.stride(2)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    a.cache_block_stride, a.cache_token_stride, a.cache_head_stride = k_cache.stride()[:3]
    a.num_blocks = nb
    if block_table is not None:
        a.block_table, a.block_table_stride, a.max_blocks_per_seq = (block_table.data_ptr(), block_table.stride(0),
                                                                     block_table.shape[1])
    else:
        a.block_table, a.block_table_stride, a.max_blocks_per_seq = None, 0, 1
    a.seqlens = seqlens.data_ptr()
    a.batch, a.queries_per_seq, a.num_q_heads, a.num_kv_heads, a.head_dim, a.block_size = B, n, hq, hkv, d, bs
    a.causal, a.num_splits, a.dtype = int(bool(causal)), max(0, int(num_splits)), _lib.BF16
    a.softmax_scale = scale
    a.status = _lib.status_word(q.device).data_ptr()
    L = _lib.lib()
    if method == "auto":
        method = choose_method(B, hkv, n * (hq // hkv), q.device)
    if method == "streamk":
        need = L.nvb200_paged_decode_workspace_size(ctypes.byref(a))
        _require(need > 0, "decode_attention: no stream-K launch shape for these sizes")
        ws = _decode_workspace(q.device, need)
        if ws is not None:
            a.num_splits = 0
            _lib.check(L.nvb200_paged_decode_attention_streamk(ctypes.byref(a), ws.data_ptr(), ws.numel(),
                                                               _lib.stream_of(q)), "decode_attention (stream-K)")
            return out
    _lib.check(L.nvb200_paged_decode_attention(ctypes.byref(a), _lib.stream_of(q)), "flash_attn_with_kvcache")
    return out


def decode_splits(batch: int, num_kv_heads: int, max_blocks_per_seq: int, block_size: int, num_splits: int = 0) -> int:
    """The number of CTAs per (sequence, KV head) the kernel uses for these sizes."""
    return _lib.lib().nvb200_paged_decode_splits(batch, num_kv_heads, max_blocks_per_seq, block_size, num_splits)


__all__ = ["store_kvcache", "flash_attn_with_kvcache", "decode_attention", "choose_method", "supports",
           "decode_splits"]
