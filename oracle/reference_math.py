"""CPU restatement of the reference's torch implementation of the pre-attention hot path.

TEST INFRASTRUCTURE ONLY: the checker for nanovllm_b200 and the timed CPU baseline, never part of the product.

The reference (R3pere/nano-vllm-triton-kernels) computes these ops with torch code in nanovllm/layers/; its Triton
kernels reproduce that code's roundings. Each function below restates one piece of that torch code, op for op, so
that on the same inputs it rounds at the same points (the `.float()` upcasts, the `.to(dtype)` downcasts, and the
dtype multiplies). All functions are device-agnostic torch code: the parity tests run them on CPU tensors, and on
CUDA tensors for the largest sizes (the same eager torch ops the reference's own tests compare against).

Pinning: tests/golden/make_golden.py imports the reference itself (its layer modules, run eagerly on CPU), writes
its outputs on seeded inputs to tests/golden/golden.pt, and tests/test_oracle.py checks every function here against
those fixtures bit for bit.
"""
import math

import torch
import torch.nn.functional as F


def rms_forward(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm.rms_forward (nanovllm/layers/layernorm.py:20-30): fp32 mean of squares, x * rsqrt(var + eps) in fp32,
    rounded to x's dtype, then multiplied by the weight in that dtype."""
    orig = x.dtype
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    xf = xf * torch.rsqrt(var + eps)
    return xf.to(orig) * weight


def add_rms_forward(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                    eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """RMSNorm.add_rms_forward (nanovllm/layers/layernorm.py:32-44): s = x + residual in fp32; the new residual is
    s rounded to x's dtype; the normalised output uses the unrounded s."""
    orig = x.dtype
    s = x.float() + residual.float()
    new_residual = s.to(orig)
    var = s.pow(2).mean(dim=-1, keepdim=True)
    s = s * torch.rsqrt(var + eps)
    return s.to(orig) * weight, new_residual


def rope_cos_sin_cache(head_size: int, max_position: int, base: float) -> torch.Tensor:
    """RotaryEmbedding.__init__ (nanovllm/layers/rotary_embedding.py:17-35): [max_position, 1, head_size] fp32 rows
    of (cos | sin) of position * inv_freq, inv_freq = 1 / base^(2i / head_size)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, head_size, 2, dtype=torch.float) / head_size))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """apply_rotary_emb (nanovllm/layers/rotary_embedding.py:6-14): neox halves, fp32 products rounded separately,
    result rounded to x's dtype."""
    x1, x2 = torch.chunk(x.float(), 2, dim=-1)
    y1 = x1 * cos - x2 * sin
    y2 = x2 * cos + x1 * sin
    return torch.cat((y1, y2), dim=-1).to(x.dtype)


def rotary(positions: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
           cos_sin_cache: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """RotaryEmbedding.forward (nanovllm/layers/rotary_embedding.py:37-48) for q [T, Hq, D], k [T, Hkv, D]."""
    cos_sin = cos_sin_cache[positions]
    if cos_sin.dim() == 2:  # a [max_pos, D] table: add the head axis
        cos_sin = cos_sin.unsqueeze(1)
    cos, sin = cos_sin.chunk(2, dim=-1)
    return apply_rotary_emb(q, cos, sin), apply_rotary_emb(k, cos, sin)


def store_kvcache(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor) -> None:
    """store_kvcache_kernel (nanovllm/layers/attention.py:11-31): row t of k and v ([Hkv * D] elements) goes to row
    slot_mapping[t] of the flattened caches; slot -1 is skipped. In place."""
    T, hkv, d = k.shape
    keep = slot_mapping >= 0
    rows = slot_mapping[keep].long()
    k_cache.view(-1, hkv * d)[rows] = k.reshape(T, hkv * d)[keep]
    v_cache.view(-1, hkv * d)[rows] = v.reshape(T, hkv * d)[keep]


def qk_norm_rope_kv(q, k, v, positions, q_weight, k_weight, eps, cos_sin_cache, k_cache, v_cache, slot_mapping,
                    write_k):
    """The torch composition that nanovllm/kernels/qk_norm_rope_kv.py:92-125 replaces (q_norm, k_norm, rotary_emb,
    store_kvcache; nanovllm/models/qwen3.py:99-103 and layers/attention.py:64-76). Mutates the caches in place
    (unless they are empty) and returns (q_out, k_out or None)."""
    qn = rms_forward(q, q_weight, eps)
    kn = rms_forward(k, k_weight, eps)
    qr, kr = rotary(positions, qn, kn, cos_sin_cache)
    if k_cache.numel() > 0:
        store_kvcache(kr, v, k_cache, v_cache, slot_mapping)
    return qr.contiguous(), (kr.contiguous() if write_k else None)


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, cache_seqlens: torch.Tensor,
                           block_table: torch.Tensor | None, softmax_scale: float, causal: bool) -> torch.Tensor:
    """The decode branch of Attention.forward (nanovllm/layers/attention.py:84-91): flash_attn_with_kvcache(q,
    k_cache, v_cache, cache_seqlens=context_lens, block_table=block_tables, softmax_scale, causal=True) of the
    third-party flash-attn package (pip "flash-attn", unpinned in the reference's pyproject.toml:18; 2.8.3 in this
    image), restated from its documented semantics:
      * q [B, n, Hq, D]; caches [num_blocks, block_size, Hkv, D]; key j of sequence b is token j % block_size of
        block block_table[b, j // block_size] (no table: the cache is [B, max_len, Hkv, D] per sequence);
      * q head hq reads KV head hq // (Hq / Hkv) (grouped-query attention);
      * causal: query i of n sees keys [0, L - n + i], L = cache_seqlens[b] (the bottom-right alignment the
        reference's comment at attention.py:86-87 states); otherwise keys [0, L);
      * a query that sees no key gets zeros.
    Computed in float64 and returned as fp32 [B, n, Hq, D]."""
    B, n, hq, d = q.shape
    hkv = k_cache.shape[2]
    group = hq // hkv
    out = torch.zeros(B, n, hq, d, dtype=torch.float64, device=q.device)
    for b in range(B):
        L = int(cache_seqlens[b])
        if L <= 0:
            continue
        if block_table is None:
            keys, vals = k_cache[b, :L], v_cache[b, :L]
        else:
            bs = k_cache.shape[1]
            pages = block_table[b, :(L + bs - 1) // bs].long()
            keys = k_cache[pages].reshape(-1, hkv, d)[:L]
            vals = v_cache[pages].reshape(-1, hkv, d)[:L]
        kk = keys.double().repeat_interleave(group, dim=1)  # [L, Hq, D]
        vv = vals.double().repeat_interleave(group, dim=1)
        s = torch.einsum("ihd,jhd->hij", q[b].double(), kk) * softmax_scale  # [Hq, n, L]
        j = torch.arange(L, device=q.device)
        last = (L - n + torch.arange(n, device=q.device)) if causal else torch.full((n,), L - 1, device=q.device)
        s = s.masked_fill(j[None, None, :] > last[None, :, None], float("-inf"))
        seen = (last >= 0)[None, :, None]
        p = torch.softmax(s, dim=-1).nan_to_num(0.0) * seen
        out[b] = torch.einsum("hij,jhd->ihd", p, vv)
    return out.float()


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """SiluAndMul.silu_and_mul_compiled (nanovllm/layers/activation.py:15-18) run eagerly: silu of the gate half in
    fp32 rounded to x's dtype, times the up half in x's dtype."""
    n = x.shape[-1] // 2
    gate, up = x[..., :n], x[..., n:2 * n]
    return F.silu(gate) * up


def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """The reference's matmul oracle (tests/test_kernels_matmul.py:52): the float64 product of the inputs."""
    return a.double() @ b.double()


def tf32_round(x: torch.Tensor, mode: str = "rz") -> torch.Tensor:
    """x (fp32) reduced to tf32 (10 explicit mantissa bits): "rz" drops the low 13 bits (what the tensor core does
    with fp32 operands it reads as tf32), "rna" rounds to nearest, ties away from zero (cvt.rna.tf32.f32). Used to
    build the tf32 product reference a_tf32 @ b_tf32."""
    i = x.contiguous().view(torch.int32)
    if mode == "rna":
        i = i + 0x1000
    i = i & ~0x1FFF
    return i.view(torch.float32).reshape(x.shape)


# Byte / flop counts of the reference's microbenchmarks (scripts/bench_qk_rope_kv.py:50-52,
# scripts/bench_norm_act.py:3-5, scripts/bench_matmul.py:82).

def qk_norm_rope_kv_bytes(T: int, hq: int, hkv: int, d: int, write_k: bool = False) -> int:
    per_token = (hq + 2 * hkv) * d * 2 + 8 + 4 + d * 4 + (hq + 2 * hkv) * d * 2
    return T * (per_token + (hkv * d * 2 if write_k else 0)) + 2 * d * 2


def rms_norm_bytes(T: int, n: int) -> int:
    return (2 * T * n + n) * 2


def add_rms_norm_bytes(T: int, n: int) -> int:
    return (4 * T * n + n) * 2


def silu_and_mul_bytes(T: int, n: int) -> int:
    return 3 * T * n * 2


def store_kvcache_bytes(T: int, row_elems: int, elem_bytes: int = 2, kept: int | None = None) -> int:
    """store_kvcache: every token's slot is read (4 bytes); each kept token reads and writes its k and v rows."""
    kept = T if kept is None else kept
    return T * 4 + kept * 4 * row_elems * elem_bytes


def paged_decode_attention_bytes(seqlens, n: int, hq: int, hkv: int, d: int, block_size: int) -> int:
    """Decode attention reads every cached key and value row of its KV heads once (bf16), the queries and the
    block-table entries it follows, and writes the output: sum_b L_b * Hkv * D * 2 * 2 + 2 * B * n * Hq * D * 2 +
    4 * B + 4 * sum_b ceil(L_b / block_size)."""
    seqlens = [int(x) for x in seqlens]
    kv = sum(seqlens) * hkv * d * 2 * 2
    qo = 2 * len(seqlens) * n * hq * d * 2
    meta = 4 * len(seqlens) + 4 * sum((L + block_size - 1) // block_size for L in seqlens)
    return kv + qo + meta


def matmul_flops(m: int, n: int, k: int) -> int:
    return 2 * m * n * k


def bf16_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in bf16 steps between two bf16 tensors: bit patterns mapped to a monotonic integer line (the metric of
    tests/test_kernels_qk_rope_kv.py:46-51 in the reference)."""
    def line(t):
        i = t.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (line(a) - line(b)).abs()


def matmul_tolerance(dtype: str, prec: str, k: int) -> tuple[float, float]:
    """(rtol, atol) of tests/test_kernels_matmul.py:21-25: atol scales with sqrt(K)."""
    rtol, atol = {("fp32", "ieee"): (1e-4, 1e-4), ("fp32", "tf32"): (1e-2, 1e-2),
                  ("bf16", "ieee"): (1.6e-2, 1e-2)}[(dtype, prec)]
    return rtol, atol * math.sqrt(k)
