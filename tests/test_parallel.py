"""Tensor-parallel host logic on CPU: two gloo ranks (world_size 2) shard the fused op by kv head and the matmul by
column / row, compute with the oracle (CPU), exchange with torch.distributed, and must reproduce the single-rank
result exactly. No GPU: the kernels themselves are covered per shard by the GPU tests."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nanovllm_b200 import parallel
from oracle import reference_math as om

HQ, HKV, D, T = 16, 8, 128, 24


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(T, (HQ + 2 * HKV) * D, generator=g).to(torch.bfloat16)
    q_w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    k_w = (1 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    positions = torch.randint(0, 4096, (T,), generator=g)
    slots = torch.randperm(512, generator=g)[:T].to(torch.int32)
    slots[::5] = -1
    cache = torch.randn(2, 2, 256, HKV, D, generator=g).to(torch.bfloat16)
    table = om.rope_cos_sin_cache(D, 4096, 1e6)
    return qkv, q_w, k_w, positions, slots, cache, table


def _views(qkv, hq, hkv):
    q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
    return q.view(T, hq, D), k.view(T, hkv, D), v.view(T, hkv, D)


def _worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        qkv, q_w, k_w, positions, slots, cache, table = _inputs()
        # Fused op on this rank's heads and cache slice.
        mine = parallel.shard_qkv_columns(qkv, HQ, HKV, D, rank, world)
        q, k, v = _views(mine, HQ // world, HKV // world)
        kc = parallel.shard_kv_cache(cache[0], HKV, rank, world)
        vc = parallel.shard_kv_cache(cache[1], HKV, rank, world)
        q_out, _ = om.qk_norm_rope_kv(q, k, v, positions, q_w, k_w, 1e-6, table, kc, vc, slots, False)
        gathered = [torch.empty_like(q_out) for _ in range(world)]
        dist.all_gather(gathered, q_out)
        kcs = [torch.empty_like(kc) for _ in range(world)]
        dist.all_gather(kcs, kc)
        # Column- and row-parallel matmul (fp32 so the all-reduce sum is comparable).
        g = torch.Generator().manual_seed(9)
        a = torch.randn(16, 64, generator=g)
        b = torch.randn(48, 64, generator=g).t()
        col = parallel.column_shard(b, rank, world)
        cols = [torch.empty(16, 48 // world) for _ in range(world)]
        dist.all_gather(cols, (a @ col).contiguous())
        a_r, b_r = parallel.row_shard(a, b, rank, world)
        row = parallel.row_parallel_matmul(a_r, b_r, matmul=lambda x, y: x @ y)
        if rank == 0:
            torch.save(dict(q=torch.cat(gathered, dim=1), k_cache=torch.cat(kcs, dim=2), col=torch.cat(cols, dim=1),
                            row=row), os.path.join(result_dir, "out.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_shards_reassemble(tmp_path, world):
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    got = torch.load(tmp_path / "out.pt")
    qkv, q_w, k_w, positions, slots, cache, table = _inputs()
    q, k, v = _views(qkv, HQ, HKV)
    kc, vc = cache[0].clone(), cache[1].clone()
    q_out, _ = om.qk_norm_rope_kv(q, k, v, positions, q_w, k_w, 1e-6, table, kc, vc, slots, False)
    assert torch.equal(got["q"], q_out)  # heads are independent: sharding changes no bit
    assert torch.equal(got["k_cache"], kc)
    g = torch.Generator().manual_seed(9)
    a = torch.randn(16, 64, generator=g)
    b = torch.randn(48, 64, generator=g).t()
    assert torch.equal(got["col"], a @ b)
    torch.testing.assert_close(got["row"], a @ b, rtol=1e-5, atol=1e-5)


def test_head_ranges():
    assert parallel.kv_head_range(8, 3, 8) == (3, 4)
    assert parallel.q_head_range(32, 8, 1, 4) == (8, 16)
    with pytest.raises(ValueError):
        parallel.kv_head_range(8, 0, 3)
