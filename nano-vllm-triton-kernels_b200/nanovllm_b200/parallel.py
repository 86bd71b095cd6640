"""Tensor-parallel layout of the hot path, as nano-vllm lays it out (one process per GPU).

* The fused q/k norm + RoPE + KV write and the norm/activation ops shard without a collective: rank r of `world`
  owns kv heads [r Hkv/world, (r+1) Hkv/world) and the q heads that share them (QKVParallelLinear,
  nanovllm/layers/linear.py:106-128) and that slice of every layer's KV cache (model_runner.py:253,262);
  positions, slot_mapping and the cos/sin table are replicated.
* Column-parallel matmul (qkv_proj, gate_up_proj) N-shards B: no collective.
* Row-parallel matmul (o_proj, down_proj) K-shards A's columns and B's rows and all-reduces the [M, N] partial
  products (nanovllm/layers/linear.py:131-156): the one exchange on this path, done with
  torch.distributed.all_reduce (NCCL over NVLink on B200; gloo on CPU in the tests).
"""
import torch
import torch.distributed as dist


def kv_head_range(num_kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    """[first, last) kv heads of `rank`; kv heads must divide evenly (nano-vllm asserts the same, qwen3.py:31-35)."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not divide across {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def q_head_range(num_q_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    """[first, last) q heads of `rank`: the q heads of its kv heads (GQA groups stay on one rank)."""
    first, last = kv_head_range(num_kv_heads, rank, world)
    group = num_q_heads // num_kv_heads
    return first * group, last * group


def shard_qkv_columns(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int, rank: int,
                      world: int) -> torch.Tensor:
    """This rank's columns of a full qkv_proj output [T, (Hq + 2 Hkv) D], laid out as the rank's own qkv_proj
    produces them: [q heads | k heads | v heads] of its shard, contiguous."""
    q0, q1 = q_head_range(num_q_heads, num_kv_heads, rank, world)
    k0, k1 = kv_head_range(num_kv_heads, rank, world)
    q = qkv[:, q0 * head_dim:q1 * head_dim]
    koff = num_q_heads * head_dim
    k = qkv[:, koff + k0 * head_dim:koff + k1 * head_dim]
    voff = koff + num_kv_heads * head_dim
    v = qkv[:, voff + k0 * head_dim:voff + k1 * head_dim]
    return torch.cat([q, k, v], dim=1)


def shard_kv_cache(cache: torch.Tensor, num_kv_heads: int, rank: int, world: int) -> torch.Tensor:
    """This rank's slice [blocks, block_size, Hkv/world, D] of a full cache [blocks, block_size, Hkv, D]."""
    k0, k1 = kv_head_range(num_kv_heads, rank, world)
    return cache[:, :, k0:k1].contiguous()


def column_shard(b: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Columns [r N/world, (r+1) N/world) of B [K, N] (a view; keeps B's strides)."""
    n = b.shape[1]
    if n % world:
        raise ValueError(f"N = {n} does not divide across {world} ranks")
    per = n // world
    return b[:, rank * per:(rank + 1) * per]


def row_shard(a: torch.Tensor, b: torch.Tensor, rank: int, world: int) -> tuple[torch.Tensor, torch.Tensor]:
    """A's columns and B's rows [r K/world, (r+1) K/world): the operands of one rank's row-parallel partial."""
    k = a.shape[1]
    if k % world:
        raise ValueError(f"K = {k} does not divide across {world} ranks")
    per = k // world
    return a[:, rank * per:(rank + 1) * per], b[rank * per:(rank + 1) * per]


def row_parallel_matmul(a_shard: torch.Tensor, b_shard: torch.Tensor, matmul=None,
                        group=None) -> torch.Tensor:
    """C = sum over ranks of A_r @ B_r: this rank's partial product (nanovllm_b200's matmul unless another
    implementation is passed) all-reduced in place across `group` (nanovllm/layers/linear.py:152-156)."""
    if matmul is None:
        from nanovllm_b200.kernels.matmul import matmul
    c = matmul(a_shard, b_shard)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(c, group=group)
    return c
