"""Row-parallel matmul fused with its all-reduce over NVLink (nvb200_matmul_allreduce via
nanovllm_b200.parallel.RowParallelAllReduce) on two GPUs, one process each (NCCL group for the set-up): against
the fp64 product of the full operands within bf16 tolerance, against the reference's path (matmul, then an NCCL
all-reduce of the bf16 partials), and identical on both ranks; three calls per shape so both halves of the
exchange buffers and increasing epochs are used; and three replays of a CUDA graph that captured one call, with
new inputs each time; and a call that one rank skips, which must end on the other rank within its 1 s bound with
NVB200_STATUS_WAIT_TIMEOUT set. Needs two GPUs (skipped otherwise)."""
import datetime
import math
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2
# (M, N, K total): decode o_proj / down_proj of Qwen3-0.6B and -8B shards, M = 1 and odd M, ragged K shards. N a
# multiple of 8 with shards of at most 16 MB runs the weight-streaming kernel's all-reduce (K split over clusters of 1,
# 2 and 4 CTAs among these shapes); N = 1004 and the 8B down_proj shard (50 MB) the skinny kernel's.
SHAPES = [(32, 1024, 2048), (32, 1024, 6144), (1, 4096, 1024), (7, 1000, 512), (64, 2048, 1024), (32, 4096, 24576),
          (5, 1004, 512)]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=torch.device("cuda", rank))
    from nanovllm_b200 import _lib
    from nanovllm_b200.kernels.matmul import matmul
    from nanovllm_b200.parallel import RowParallelAllReduce
    results = []
    ar = RowParallelAllReduce(max_n=4096)
    try:
        for (M, N, K) in SHAPES:
            g = torch.Generator(device="cuda").manual_seed(M * 31 + N + K)
            a = (torch.randn(M, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
            w = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
            k0, k1 = rank * K // WORLD, (rank + 1) * K // WORLD
            a_r, b_r = a[:, k0:k1].contiguous(), w[:, k0:k1].t()
            for it in range(3):
                out = ar(a_r, b_r)
                ref_nccl = matmul(a_r, b_r)
                dist.all_reduce(ref_nccl)
                gathered = [torch.empty_like(out) for _ in range(WORLD)]
                dist.all_gather(gathered, out)
                results.append(dict(shape=(M, N, K), it=it, out=out.cpu(), nccl=ref_nccl.cpu(),
                                    same=all(torch.equal(gathered[0], x) for x in gathered),
                                    ref=(a.double() @ w.double().t()).cpu(), status=_lib.status(clear=True)))
        # Captured in a CUDA graph and replayed with new inputs: each replay is a new call (the kernel advances its
        # epoch in device memory), checked against the NCCL path.
        M, N, K = 32, 1024, 2048
        k0, k1 = rank * K // WORLD, (rank + 1) * K // WORLD
        a_in = torch.zeros(M, k1 - k0, device="cuda", dtype=torch.bfloat16)
        w_in = torch.zeros(N, k1 - k0, device="cuda", dtype=torch.bfloat16)
        ar(a_in, w_in.t())
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            g_out = ar(a_in, w_in.t())
        for it in range(3):
            g = torch.Generator(device="cuda").manual_seed(1000 + it)
            a = (torch.randn(M, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
            w = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
            a_in.copy_(a[:, k0:k1])
            w_in.copy_(w[:, k0:k1])
            graph.replay()
            ref_nccl = matmul(a_in, w_in.t())
            dist.all_reduce(ref_nccl)
            results.append(dict(shape=("graph", M, N, K), it=it, out=g_out.clone().cpu(), nccl=ref_nccl.cpu(),
                                same=True, ref=(a.double() @ w.double().t()).cpu(), status=_lib.status(clear=True)))
        torch.cuda.synchronize()
        del graph
    finally:
        ar.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        torch.save(results, os.path.join(out_dir, "out.pt"))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_row_parallel_allreduce(tmp_path):
    mp.start_processes(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, start_method="spawn")
    results = torch.load(tmp_path / "out.pt")
    assert len(results) == 3 * len(SHAPES) + 3
    for r in results:
        assert r["status"] == 0, r["shape"]
        assert r["same"], r["shape"]  # every rank holds the same bits
        scale = r["ref"].abs().max().item()
        torch.testing.assert_close(r["out"].double(), r["ref"], rtol=1.6e-2, atol=1e-2 * scale)
        torch.testing.assert_close(r["out"].double(), r["nccl"].double(), rtol=1.6e-2, atol=1e-2 * scale)


def _skip_worker(rank, port, out_dir):
    """Rank 1 skips the second of three calls. Rank 0's kernel then waits for a partial that never comes: its bounded
    wait (1 s) must run out, set NVB200_STATUS_WAIT_TIMEOUT and return, so the host sees the failure and the context
    stays usable. Both ranks then drop the exchange buffers (their epochs no longer agree) and set up new ones, and a
    normal call must give the right result again. No rank leaves while a kernel or collective of its own is in
    flight; NVLS is off (NCCL_NVLS_ENABLE=0) and the kernel exchanges data with plain peer stores and loads."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    from nanovllm_b200 import _lib
    from nanovllm_b200.parallel import RowParallelAllReduce
    M, N, K = 32, 1024, 2048
    k0, k1 = rank * K // WORLD, (rank + 1) * K // WORLD
    g = torch.Generator(device="cuda").manual_seed(5)
    a = (torch.randn(M, K, device="cuda", generator=g) / math.sqrt(K)).to(torch.bfloat16)
    w = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    a_r, b_r = a[:, k0:k1].contiguous(), w[:, k0:k1].t()
    ref = (a.double() @ w.double().t()).cpu()
    res = {}
    _lib.status(clear=True)
    ar = RowParallelAllReduce(max_n=N)
    try:
        out = ar(a_r, b_r)
        torch.cuda.synchronize()
        res["first"] = (out.cpu(), _lib.status(clear=True))
        dist.barrier()
        if rank == 0:
            t0 = time.perf_counter()
            out = ar(a_r, b_r)  # rank 1 never makes this call
            torch.cuda.synchronize()
            res["skipped"] = (_lib.status(clear=True), time.perf_counter() - t0)
        dist.barrier()
    finally:
        ar.close()
    dist.barrier()
    ar = RowParallelAllReduce(max_n=N)
    try:
        out = ar(a_r, b_r)
        torch.cuda.synchronize()
        res["after"] = (out.cpu(), _lib.status(clear=True))
    finally:
        ar.close()
        dist.barrier()
        dist.destroy_process_group()
    res["ref"] = ref
    torch.save(res, os.path.join(out_dir, f"skip{rank}.pt"))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_missing_peer_times_out_and_the_group_recovers(tmp_path):
    mp.start_processes(_skip_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, start_method="spawn")
    r0, r1 = (torch.load(tmp_path / f"skip{r}.pt") for r in range(WORLD))
    scale = r0["ref"].abs().max().item()
    for r in (r0, r1):
        assert r["first"][1] == 0 and r["after"][1] == 0
        torch.testing.assert_close(r["first"][0].double(), r["ref"], rtol=1.6e-2, atol=1e-2 * scale)
        torch.testing.assert_close(r["after"][0].double(), r["ref"], rtol=1.6e-2, atol=1e-2 * scale)
    status, seconds = r0["skipped"]
    assert status & 4, status  # NVB200_STATUS_WAIT_TIMEOUT
    assert 0.9 < seconds < 10, seconds  # the 1 s bound, then the call returned
