"""Fused q/k RMSNorm + neox RoPE + paged KV-cache write on B200 (drop-in for nanovllm/kernels/qk_norm_rope_kv.py).

Same call as the reference's `qk_norm_rope_kv` (nanovllm/kernels/qk_norm_rope_kv.py:92-125): the same arguments,
the same assertions on them (:106-114), the same freshly allocated outputs (:115-116) and no launch when T == 0
(:117). The work runs in `nvb200_qk_norm_rope_kv` (include/nvb200.h), a hand-written sm_100a kernel that stages each
token's q/k/v rows and cos/sin row in shared memory with bulk copies, normalises and rotates them, and bulk-stores
q_out, k_out and the k/v cache rows (slot -1 skipped).

Differences from the reference, all widening what it accepts:
  * kv_per_prog and num_warps are accepted and ignored (they tune the Triton launch). In particular the
    reference's `Hkv % kv_per_prog == 0` requirement (:107, kv_per_prog = 4) does not apply, so 1 or 2 kv heads
    per rank (tensor parallel 4/8 of Qwen3) work.
  * Out-of-range positions or slots never fault: they are skipped and flagged in the device status word
    (nanovllm_b200.status()).
"""
import ctypes

import torch

from nanovllm_b200 import _lib


def _require(cond: bool, msg: str = "") -> None:
    if not cond:
        raise AssertionError(msg)


def qk_norm_rope_kv(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
    q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float, cos_sin_cache: torch.Tensor,
    k_cache: torch.Tensor, v_cache: torch.Tensor, slot_mapping: torch.Tensor | None, write_k: bool,
    kv_per_prog: int | None = None, num_warps: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """q: [T, Hq, D], k, v: [T, Hkv, D] bf16, each with a contiguous head (any token stride: views of the qkv
    output work). positions: [T] int64. cos_sin_cache: [max_pos, 1, D] or [max_pos, D] fp32 (cos | sin).
    k_cache, v_cache: [blocks, block_size, Hkv, D] contiguous, or empty (then nothing is stored).
    slot_mapping: [T] int32, -1 = don't store. Returns (q_out [T, Hq, D], k_out [T, Hkv, D] or None)."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    _require(q.dtype == k.dtype == v.dtype == torch.bfloat16 and k.shape == v.shape == (T, Hkv, D),
             "q, k, v must be bf16 with k.shape == v.shape == (T, Hkv, D)")
    _require(Hq % Hkv == 0 and D % 2 == 0, "Hq must be a multiple of Hkv and D even")
    for x in (q, k, v):
        _require(x.stride(2) == 1 and x.stride(1) == D, "each head must be contiguous: stride(2) == 1, stride(1) == D")
    _require(positions.shape == (T,) and cos_sin_cache.dtype == torch.float32 and cos_sin_cache.shape[-1] == D,
             "positions must be [T] and cos_sin_cache fp32 [..., D]")
    _require(positions.dtype == torch.int64, "positions must be int64")
    _require(cos_sin_cache.stride(-1) == 1 and cos_sin_cache.numel() == cos_sin_cache.shape[0] * D,
             "cos_sin_cache must be [max_pos, D] or [max_pos, 1, D] rows with a unit last stride")
    _require(q_weight.dtype == k_weight.dtype == torch.bfloat16 and q_weight.shape == k_weight.shape == (D,)
             and q_weight.is_contiguous() and k_weight.is_contiguous(), "q/k weights must be contiguous bf16 [D]")
    store = k_cache.numel() > 0
    if store:
        _require(k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.shape[-2:] == (Hkv, D),
                 "k_cache, v_cache must be contiguous [..., Hkv, D]")
        _require(v_cache.shape == k_cache.shape and k_cache.dtype == v_cache.dtype == torch.bfloat16,
                 "v_cache must match k_cache (bf16)")
        _require(slot_mapping is not None and slot_mapping.shape == (T,), "slot_mapping must be [T]")
        _require(slot_mapping.dtype == torch.int32, "slot_mapping must be int32")
    dev = q.device
    _require(dev.type == "cuda", "q must be a CUDA tensor")
    q_out = torch.empty(T, Hq, D, dtype=q.dtype, device=dev)
    k_out = torch.empty(T, Hkv, D, dtype=k.dtype, device=dev) if write_k else None
    if T:
        a = _args(q_out, k_out, q, k, v, positions, q_weight, k_weight, eps, cos_sin_cache, k_cache, v_cache,
                  slot_mapping, store)
        _lib.check(_lib.lib().nvb200_qk_norm_rope_kv(ctypes.byref(a), _lib.stream_of(q)), "qk_norm_rope_kv")
    return q_out, k_out


def _args(q_out, k_out, q, k, v, positions, q_weight, k_weight, eps, cos_sin_cache, k_cache, v_cache, slot_mapping,
          store):
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    a = _lib.QkNormRopeKvArgs()
    a.q_out, a.k_out = q_out.data_ptr(), _lib.ptr(k_out)
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.q_token_stride, a.k_token_stride, a.v_token_stride = q.stride(0), k.stride(0), v.stride(0)
    a.positions = positions.data_ptr()
    a.slot_mapping = slot_mapping.data_ptr() if store else None
    a.q_weight, a.k_weight = q_weight.data_ptr(), k_weight.data_ptr()
    a.cos_sin, a.cos_sin_stride, a.num_positions = (cos_sin_cache.data_ptr(), cos_sin_cache.stride(0),
                                                    cos_sin_cache.shape[0])
    if store:
        a.k_cache, a.v_cache, a.num_slots = k_cache.data_ptr(), v_cache.data_ptr(), k_cache.numel() // (Hkv * D)
    a.num_tokens, a.num_q_heads, a.num_kv_heads, a.head_dim = T, Hq, Hkv, D
    a.eps = eps
    a.status = _lib.status_word(q.device).data_ptr()
    return a


def kernel_plan(q, k, v, positions, q_weight, k_weight, eps, cos_sin_cache, k_cache, v_cache, slot_mapping,
                write_k) -> tuple[str, int]:
    """Which kernel `qk_norm_rope_kv` with these arguments runs on their device, and the tokens one work unit covers:
    ("bulk" | "multi" | "direct" | "generic" | "none", tokens). Launches nothing (nvb200_qk_norm_rope_kv_plan)."""
    T, Hq, D = q.shape
    store = k_cache.numel() > 0
    # The plan query only checks the outputs' addresses (16-byte alignment, as a fresh torch allocation has), so one
    # small allocation stands in for q_out and k_out.
    stand_in = torch.empty(16, dtype=q.dtype, device=q.device)
    a = _args(stand_in, stand_in if write_k else None, q, k, v, positions, q_weight, k_weight, eps, cos_sin_cache,
              k_cache, v_cache, slot_mapping, store)
    kernel, tpu = ctypes.c_int32(-1), ctypes.c_int32(0)
    _lib.check(_lib.lib().nvb200_qk_norm_rope_kv_plan(ctypes.byref(a), ctypes.byref(kernel), ctypes.byref(tpu)),
               "qk_norm_rope_kv_plan")
    return _lib.QKNR_KERNELS[kernel.value], tpu.value


def linear_qkv_norm_rope_kv(x: torch.Tensor, qkv_weight: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                            positions: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float,
                            cos_sin_cache: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                            slot_mapping: torch.Tensor | None) -> torch.Tensor | None:
    """The decode qkv projection with this op as its epilogue (`nvb200_linear_qkv_norm_rope_kv`): the same result as
    qkv = x @ qkv_weight.t() (bf16) followed by qk_norm_rope_kv(q, k, v, ..., write_k=False) on its q | k | v parts,
    without writing qkv. qkv_weight: [(Hq + 2 Hkv) * 128, K] in nn.Linear layout, a model parameter (its loads may
    start while the preceding kernel finishes). Returns q_out [M, Hq, 128], or None when the kernel does not take the
    call (more than 32 rows, head_dim != 128, layouts), in which case the caller runs the two steps."""
    M, K = x.shape
    D = 128
    _require(x.dtype == qkv_weight.dtype == torch.bfloat16 and qkv_weight.shape == ((num_q_heads + 2 * num_kv_heads) * D, K),
             "x and qkv_weight must be bf16, qkv_weight [(Hq + 2 Hkv) * 128, K]")
    if (q_weight.shape != (D,) or x.stride(1) != 1 or qkv_weight.stride(1) != 1 or M > 32
            or num_q_heads % num_kv_heads or cos_sin_cache.shape[-1] != D):
        return None
    _require(positions.shape == (M,) and positions.dtype == torch.int64, "positions must be int64 [M]")
    _require(cos_sin_cache.dtype == torch.float32 and cos_sin_cache.stride(-1) == 1
             and cos_sin_cache.numel() == cos_sin_cache.shape[0] * D, "cos_sin_cache must be fp32 [max_pos, (1,) 128]")
    _require(q_weight.dtype == k_weight.dtype == torch.bfloat16 and k_weight.shape == (D,)
             and q_weight.is_contiguous() and k_weight.is_contiguous(), "q/k weights must be contiguous bf16 [128]")
    store = k_cache.numel() > 0
    if store:
        _require(k_cache.is_contiguous() and v_cache.is_contiguous() and k_cache.shape[-2:] == (num_kv_heads, D)
                 and v_cache.shape == k_cache.shape and k_cache.dtype == v_cache.dtype == torch.bfloat16,
                 "k_cache, v_cache must be contiguous bf16 [..., Hkv, 128]")
        _require(slot_mapping is not None and slot_mapping.shape == (M,) and slot_mapping.dtype == torch.int32,
                 "slot_mapping must be int32 [M]")
    q_out = torch.empty(M, num_q_heads, D, dtype=x.dtype, device=x.device)
    if M == 0:
        return q_out
    a = _lib.LinearQkvArgs()
    a.x, a.x_row_stride = x.data_ptr(), x.stride(0)
    a.qkv_weight, a.weight_row_stride, a.K = qkv_weight.data_ptr(), qkv_weight.stride(0), K
    g = a.qknr
    g.q_out, g.k_out = q_out.data_ptr(), None
    g.positions = positions.data_ptr()
    g.slot_mapping = slot_mapping.data_ptr() if store else None
    g.q_weight, g.k_weight = q_weight.data_ptr(), k_weight.data_ptr()
    g.cos_sin, g.cos_sin_stride, g.num_positions = (cos_sin_cache.data_ptr(), cos_sin_cache.stride(0),
                                                    cos_sin_cache.shape[0])
    if store:
        g.k_cache, g.v_cache, g.num_slots = k_cache.data_ptr(), v_cache.data_ptr(), k_cache.numel() // (num_kv_heads * D)
    g.num_tokens, g.num_q_heads, g.num_kv_heads, g.head_dim = M, num_q_heads, num_kv_heads, D
    g.eps = eps
    g.status = _lib.status_word(x.device).data_ptr()
    rc = _lib.lib().nvb200_linear_qkv_norm_rope_kv(ctypes.byref(a), _lib.stream_of(x))
    if rc == _lib.ERR_UNSUPPORTED:
        return None
    _lib.check(rc, "linear_qkv_norm_rope_kv")
    return q_out
