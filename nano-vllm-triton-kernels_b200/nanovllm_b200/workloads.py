"""Seeded synthetic inputs of the BASELINE configurations (shapes, sizes and value distributions only).

The reference measures on synthetic data too (scripts/bench_qk_rope_kv.py:55-76, scripts/bench_norm_act.py:207-227,
tests/test_kernels_*.py); these generators reproduce those shapes and distributions:
  * fused op: qkv_proj output [T, (Hq + 2 Hkv) * D] bf16 ~ N(0, 1) read through strided q/k/v views; q/k norm
    weights 1 + 0.1 N(0, 1); positions uniform in [0, max_pos); neox cos/sin table (theta); a paged KV cache
    [blocks, 256, Hkv, D]; slot_mapping = distinct random slots with a seeded 5 % set to -1;
  * norm/act: x, residual ~ N(0, 1) [T, hidden], weight 1 + 0.1 N(0, 1), gate_up [T, 2 * inter];
  * matmul: A [M, K], B = randn(N, K).t() (non-contiguous), both scaled by 1/sqrt(K).
Everything is created directly on the target device from a seeded torch.Generator.
"""
import math

import torch

BLOCK_SIZE = 256

# Attention shapes (Hq, Hkv, D) and norm/act sizes of the models in the BASELINE configurations.
QWEN3_06B = dict(hq=16, hkv=8, d=128, hidden=1024, inter=3072, max_pos=4096, theta=1e6)
QWEN3_8B = dict(hq=32, hkv=8, d=128, max_pos=32768, theta=1e6)


def rope_table(d: int, max_pos: int, theta: float, device) -> torch.Tensor:
    """The neox cos/sin table [max_pos, 1, d] fp32 that RotaryEmbedding builds (cos | sin of pos * theta^(-2i/d))."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float) / d))
    t = torch.arange(max_pos, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1).to(device)


def fused_inputs(T: int, hq: int, hkv: int, d: int = 128, max_pos: int = 4096, theta: float = 1e6,
                 num_blocks: int | None = None, skip_frac: float = 0.05, seed: int = 0, device="cuda",
                 cache_fill: str = "zeros", table: torch.Tensor | None = None) -> dict:
    """Inputs of one qk_norm_rope_kv call. num_blocks defaults to the smallest cache holding 2T slots."""
    g = torch.Generator(device=device).manual_seed(seed)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device=device, generator=g).to(torch.bfloat16)
    q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    q, k, v = q.view(T, hq, d), k.view(T, hkv, d), v.view(T, hkv, d)
    q_w = (1 + 0.1 * torch.randn(d, device=device, generator=g)).to(torch.bfloat16)
    k_w = (1 + 0.1 * torch.randn(d, device=device, generator=g)).to(torch.bfloat16)
    positions = torch.randint(0, max_pos, (T,), device=device, generator=g)
    if num_blocks is None:
        num_blocks = max(1, (2 * T + BLOCK_SIZE - 1) // BLOCK_SIZE)
    n_slots = num_blocks * BLOCK_SIZE
    assert n_slots >= T, "the cache must have a distinct slot for every token"
    slots = torch.randperm(n_slots, device=device, generator=g)[:T].to(torch.int32)
    n_skip = int(round(skip_frac * T))
    if n_skip:
        slots[torch.randperm(T, device=device, generator=g)[:n_skip]] = -1
    shape = (num_blocks, BLOCK_SIZE, hkv, d)
    if cache_fill == "zeros":
        k_cache = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        v_cache = torch.zeros(shape, dtype=torch.bfloat16, device=device)
    else:
        k_cache = torch.randn(shape, device=device, generator=g).to(torch.bfloat16)
        v_cache = torch.randn(shape, device=device, generator=g).to(torch.bfloat16)
    cos_sin = table if table is not None else rope_table(d, max_pos, theta, device)
    return dict(qkv=qkv, q=q, k=k, v=v, positions=positions, q_w=q_w, k_w=k_w, cos_sin=cos_sin,
                k_cache=k_cache, v_cache=v_cache, slots=slots, eps=1e-6)


def shard_kv_heads(x: dict, rank: int, world: int) -> dict:
    """Rank `rank`'s tensor-parallel shard of fused_inputs(): kv heads [rank*Hkv/world, (rank+1)*Hkv/world), the
    q heads that share them, and that slice of the cache (nano-vllm's QKVParallelLinear / KV-cache layout).
    positions, slot_mapping and the cos/sin table are replicated."""
    T, hq, d = x["q"].shape
    hkv = x["k"].shape[1]
    assert hkv % world == 0, "kv heads must divide evenly across ranks"
    gk, gq = hkv // world, hq // world
    q = x["q"][:, rank * gq:(rank + 1) * gq]
    k = x["k"][:, rank * gk:(rank + 1) * gk]
    v = x["v"][:, rank * gk:(rank + 1) * gk]
    kc = x["k_cache"][:, :, rank * gk:(rank + 1) * gk].contiguous()
    vc = x["v_cache"][:, :, rank * gk:(rank + 1) * gk].contiguous()
    return dict(x, q=q, k=k, v=v, k_cache=kc, v_cache=vc)


def norm_inputs(T: int, n: int, seed: int = 0, device="cuda", dtype=torch.bfloat16) -> dict:
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(T, n, device=device, generator=g).to(dtype)
    r = torch.randn(T, n, device=device, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(n, device=device, generator=g)).to(dtype)
    return dict(x=x, residual=r, w=w, eps=1e-6)


def silu_inputs(T: int, inter: int, seed: int = 0, device="cuda", dtype=torch.bfloat16) -> dict:
    g = torch.Generator(device=device).manual_seed(seed)
    return dict(x=torch.randn(T, 2 * inter, device=device, generator=g).to(dtype))


def matmul_inputs(M: int, N: int, K: int, dtype=torch.bfloat16, b_transposed: bool = True, seed: int = 0,
                  device="cuda") -> dict:
    g = torch.Generator(device=device).manual_seed(seed)
    s = 1.0 / math.sqrt(K)
    a = (torch.randn(M, K, device=device, generator=g) * s).to(dtype)
    if b_transposed:
        b = (torch.randn(N, K, device=device, generator=g) * s).to(dtype).t()
    else:
        b = (torch.randn(K, N, device=device, generator=g) * s).to(dtype)
    return dict(a=a, b=b)
