"""Tensor-parallel layout of the hot path, as nano-vllm lays it out (one process per GPU).

* The fused q/k norm + RoPE + KV write and the norm/activation ops shard without a collective: rank r of `world`
  owns kv heads [r Hkv/world, (r+1) Hkv/world) and the q heads that share them (QKVParallelLinear,
  nanovllm/layers/linear.py:106-128) and that slice of every layer's KV cache (model_runner.py:253,262);
  positions, slot_mapping and the cos/sin table are replicated.
* Column-parallel matmul (qkv_proj, gate_up_proj) N-shards B: no collective.
* Row-parallel matmul (o_proj, down_proj) K-shards A's columns and B's rows and all-reduces the [M, N] partial
  products (nanovllm/layers/linear.py:131-156): the one exchange on this path. row_parallel_matmul does it with
  torch.distributed.all_reduce (NCCL over NVLink; gloo on CPU in the tests); RowParallelAllReduce does the GEMM and
  the exchange in one kernel per rank over NVLink for decode-sized batches.
"""
import ctypes

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


class RowParallelAllReduce:
    """Row-parallel matmul fused with its all-reduce over NVLink (nvb200_matmul_allreduce): every rank calls it with
    its K shard A_r [M, K_r], B_r [K_r, N] and receives sum_r A_r @ B_r (bf16, summed in fp32 in rank order, so all
    ranks hold the same bits), in one kernel per rank that pushes its partial into every rank's exchange buffer and
    waits for theirs. Replaces F.linear followed by dist.all_reduce (nanovllm/layers/linear.py:131-156) for
    decode-sized batches (M <= 64); other shapes, and groups of one rank, run the matmul and an NCCL all-reduce.

    Construction is collective over `group` (the exchange buffers' CUDA IPC handles are all-gathered), and so is
    every call: all ranks make the same calls in the same order. The kernel keeps its call count in the buffers,
    so calls may be captured in a CUDA graph and replayed. Buffers live until close()."""

    def __init__(self, max_n: int, group=None, device=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.max_n = int(max_n)
        self.own = None
        self.peers = []
        if self.world < 2:
            return
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        from nanovllm_b200 import _lib
        lib = _lib.lib()
        with torch.cuda.device(self.device):
            buf, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
            _lib.check(lib.nvb200_allreduce_buffer_create(self.max_n, ctypes.byref(buf), handle), "allreduce buffer")
            self.own = buf.value
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.group_args = _lib.AllreduceGroup(world=self.world, rank=self.rank, max_n=self.max_n)
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.group_args.buffers[r] = self.own
                    continue
                peer = ctypes.c_void_p()
                _lib.check(lib.nvb200_allreduce_buffer_open((ctypes.c_char * 64).from_buffer_copy(h),
                                                            ctypes.byref(peer)), "allreduce buffer open")
                self.peers.append(peer.value)
                self.group_args.buffers[r] = peer.value

    def __call__(self, a_shard: torch.Tensor, b_shard: torch.Tensor) -> torch.Tensor:
        from nanovllm_b200 import _lib
        from nanovllm_b200.kernels.matmul import matmul
        if self.world < 2:
            return matmul(a_shard, b_shard)
        if not (a_shard.ndim == 2 and b_shard.ndim == 2 and a_shard.shape[1] == b_shard.shape[0]):
            raise AssertionError((a_shard.shape, b_shard.shape))
        M, K = a_shard.shape
        N = b_shard.shape[1]
        out = torch.empty((M, N), device=a_shard.device, dtype=a_shard.dtype)
        if a_shard.dtype == b_shard.dtype == torch.bfloat16 and M and N and K:
            rc = _lib.lib().nvb200_matmul_allreduce(
                out.data_ptr(), a_shard.data_ptr(), b_shard.data_ptr(), M, N, K, a_shard.stride(0), a_shard.stride(1),
                b_shard.stride(0), b_shard.stride(1), out.stride(0), ctypes.byref(self.group_args),
                _lib.status_word(a_shard.device).data_ptr(), _lib.stream_of(a_shard))
            if rc != _lib.ERR_UNSUPPORTED:  # (every rank takes the same branch: same shapes on every rank)
                _lib.check(rc, "matmul_allreduce")
                return out
        c = matmul(a_shard, b_shard)
        dist.all_reduce(c, group=self.group)
        return c

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after a device synchronisation)."""
        if self.own is None:
            return
        from nanovllm_b200 import _lib
        torch.cuda.synchronize(self.device)
        lib = _lib.lib()
        for p in self.peers:
            lib.nvb200_allreduce_buffer_close(p, 0)
        lib.nvb200_allreduce_buffer_close(self.own, 1)
        self.own, self.peers = None, []
