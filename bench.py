"""Benchmark of the B200 hot path; prints ONE JSON line (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
    (N > 1: launched as `python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...`)

Default workload (BASELINE config 3 at T = 8192, the headline "qk-norm+RoPE+KV-write GB/s at T=8192"): the fused
q/k RMSNorm + RoPE + paged KV write at the Qwen3-8B attention shape (32 q / 8 kv heads, head_dim 128, qkv bf16
[T, 6144] ~ N(0,1), cache [1024, 256, 8, 128], positions in [0, 32768), theta 1e6, 5 % of slots -1).
Multi-GPU: sharded by KV head as nano-vllm's tensor parallelism lays it out (rank r owns kv heads
[r*8/N, (r+1)*8/N) and the q heads sharing them, and that slice of the cache); no collective on the data path.
Weak scaling: the batch is 8192 * N tokens, so each rank moves the same bytes as the one-GPU run.

A step is one kernel launch over one batch. Between steps an L2 flush (a 256 MiB write, then a 256 MiB read of
another buffer so no dirty lines are left to write back) runs outside the timed events; `value` = all ranks' algorithmic bytes / max over ranks of the summed CUDA-event kernel times.
`e2e` = the same metric through the public Python API (nanovllm_b200.kernels.qk_norm_rope_kv) with the step's
inputs (qkv, positions, slots) copied from pinned host memory and q_out copied back inside the timed region.
`cpu_baseline` / `--impl reference`: the reference's torch implementation restated in oracle/ (bitwise equal to
it, tests/test_oracle.py), run on the host cores in bf16.

Other workloads (not the driver's headline): fused06b (config 1 shape at T = 8192), norm (config 2: rms_norm,
add_rms_norm, silu_and_mul at T = 8192), matmul (config 4, bf16 M = K = N = 4096), gateup (the gate_up GEMM with
the SiLU x Mul epilogue at the Qwen3-8B MLP shape, M = 4096), rowpar (decode-sized row-parallel GEMM fused with
its NVLink all-reduce, Qwen3-8B down_proj split over the ranks), attn (paged decode attention at the config-5
decode shape: 32 sequences x 1024 keys, Qwen3-0.6B heads, pages of 256; flash-attn's kernel timed beside it),
storekv (the plain KV-cache write at T = 8192, Qwen3-0.6B heads), decode (config 5: the reference's decode step per
backend).
"""
import argparse
import datetime
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "nano-vllm-triton-kernels_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

L2_FLUSH_BYTES = 256 << 20
E2E_CHUNK = 1024  # tokens per chunk of the fused op's end-to-end leg (copies of one chunk overlap another's kernel)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC_FUSED = "qk-norm+RoPE+KV-write GB/s (% HBM peak) at T=8192"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="fused8b",
                    choices=["fused8b", "fused06b", "norm", "rmsnorm", "addrmsnorm", "silu", "matmul", "gateup",
                             "rowpar", "attn", "storekv", "decode", "projections"])
    ap.add_argument("--proj-model", default="qwen3-0.6b", choices=sorted(PROJECTIONS),
                    help="--workload projections: which model's decode projections")
    ap.add_argument("--proj-rows", type=int, default=32, help="--workload projections: rows (decode batch)")
    ap.add_argument("--decode-worker", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--decode-backends", default="b200,compile,triton_fused")
    ap.add_argument("--decode-batch", type=int, default=32)
    ap.add_argument("--decode-ctx", type=int, default=1024)
    ap.add_argument("--decode-tp", type=int, default=1, help="tensor-parallel ranks of the decode step (one GPU each)")
    ap.add_argument("--decode-profile", action="store_true",
                    help="with --decode-worker: replay the decode graph once between cudaProfilerStart/Stop, untimed")
    ap.add_argument("--tokens", type=int, default=8192, help="tokens per step at N = 1")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak")
    ap.add_argument("--attn-shape", default="32,1024,16,8",
                    help="attn workload: sequences, keys per sequence, q heads, kv heads (default: the decode step)")
    ap.add_argument("--matmul-shape", default="4096,4096,4096", help="matmul workload: M, N, K (B = weight.t())")
    ap.add_argument("--cublas", action="store_true",
                    help="matmul / gateup workloads: time torch.matmul (cuBLAS) beside ours instead of the reference's "
                         "Triton kernel")
    ap.add_argument("--gateup-shape", default="4096,4096,12288",
                    help="gateup workload: M, K, intermediate size (default: Qwen3-8B MLP at M = 4096)")
    ap.add_argument("--attn-method", default="auto", choices=["auto", "cluster", "streamk"],
                    help="attn workload: the drop-in's automatic choice, or one decode kernel")
    ap.add_argument("--rank-shard-of", type=int, default=1,
                    help="fused workloads on one GPU: run the shard one rank of this many GPUs would run")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-copy-reference", action="store_true",
                    help="skip timing a torch copy of the same bytes beside an HBM-bound kernel")
    ap.add_argument("--no-decode-step", action="store_true",
                    help="skip the decode-step measurement the default (fused8b, one GPU) line carries")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return FALLBACK_PEAKS, "fallback"


def reference_kernel_module(name):
    """The reference's own Triton module nanovllm/kernels/<name>.py from its offline install (baseline/_ref), loaded
    by file so that the package's engine imports are not pulled in. Returns (module, None) or (None, why not)."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    path = os.path.join(ref, "nanovllm", "kernels", name + ".py")
    if not os.path.exists(path):
        return None, "the reference is not installed in baseline/_ref"
    if ref not in sys.path:  # some kernel modules import the package's own helpers
        sys.path.append(ref)
    try:
        spec = importlib.util.spec_from_file_location(f"_reference_kernels_{name}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod, None
    except Exception as e:  # e.g. triton missing on the box
        return None, f"importing the reference's {name}.py failed: {type(e).__name__}: {e}"[:300]


def load_traffic(key):
    """ncu DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) recorded under profiles/."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f).get(key)
    return None


# ---------------------------------------------------------------------------------------------------------------
# Distributed plumbing (one process per GPU, NCCL, 127.0.0.1 rendezvous).

def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus > 1 and world == 1:
        # Not launched by torchrun: relaunch ourselves under it.
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.gpus}",
               "--master-addr", "127.0.0.1", "--master-port", os.environ.get("MASTER_PORT", "29531"),
               *sys.argv]
        sys.exit(subprocess.call(cmd))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t)
    return float(t.item())


# ---------------------------------------------------------------------------------------------------------------
# Clocks during the timed region.

class ClockSampler:
    """nvidia-smi samples (every 20 ms) of the SM clock and throttle reasons; summary() keeps those taken between
    mark_start() and mark_end(), i.e. during the timed region."""
    QUERY = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def __enter__(self):
        # Started before the warm-up steps, so that nvidia-smi's start-up overlaps GPU work and nothing idles the
        # GPU between the warm-up and the timed steps.
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = datetime.datetime.now()

    def mark_end(self):
        self.t1 = datetime.datetime.now()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        rows = []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f")
                rows.append((ts, float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        inside = [r for r in rows if self.t0 and self.t1 and self.t0 <= r[0] <= self.t1]
        use = inside or rows
        if not use:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted({n for r in use for n, v in zip(names, r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[1] for r in use), "sm_max_mhz": max(r[2] for r in use),
                "reasons": reasons, "samples": len(use), "samples_in_timed_region": len(inside)}


def step_stats(per_step_ms):
    """Distribution of this rank's per-step event times (us): the line's value uses their sum; these show whether a
    few slow steps (e.g. the first after the warm-up) move it."""
    us = sorted(1e3 * x for x in per_step_ms)
    n = len(us)
    return {"mean": sum(us) / n, "min": us[0], "median": statistics.median(us), "p90": us[min(n - 1, (9 * n) // 10)],
            "max": us[-1], "first3": [round(1e3 * x, 2) for x in per_step_ms[:3]]}


# ---------------------------------------------------------------------------------------------------------------
# Workloads: each returns a dict with `launch()` (one step on device-resident inputs, on the current stream),
# `units` (algorithmic bytes or flops per step on this rank), `e2e()` (one step through the public API from pinned
# host buffers, returns (h2d_bytes, d2h_bytes)), `cpu()` (one step of the oracle on CPU) and metadata.

def fused_workload(args, rank, world, dev, hq_total, hkv_total, max_pos, num_blocks, label):
    from nanovllm_b200 import workloads
    from nanovllm_b200.kernels.qk_norm_rope_kv import qk_norm_rope_kv

    if args.rank_shard_of > 1:
        # One GPU runs the shard one rank of an N-GPU job would run (the weak-scaling batch of N x tokens, 8 / N kv
        # heads): the per-rank kernel of config 3 at N GPUs, measured where a multi-GPU box is not at hand.
        assert world == 1, "--rank-shard-of is a one-GPU option"
        world = args.rank_shard_of
    T = args.tokens * (world if args.scaling == "weak" else 1)
    assert hkv_total % world == 0, "kv heads must divide across the GPUs"
    hq, hkv, d = hq_total // world, hkv_total // world, 128
    # Each rank generates only its shard: its qkv_proj output [T, (hq + 2 hkv) * d] and cache slice.
    blocks = max(num_blocks, (T + 255) // 256 + 1)
    x = workloads.fused_inputs(T, hq, hkv, d, max_pos=max_pos, theta=1e6, num_blocks=blocks, seed=1234,
                               device=dev)
    # positions and slots are replicated across ranks: regenerate them from a rank-independent seed.
    g = torch.Generator(device=dev).manual_seed(99)
    x["positions"] = torch.randint(0, max_pos, (T,), device=dev, generator=g)
    slots = torch.randperm(blocks * 256, device=dev, generator=g)[:T].to(torch.int32)
    slots[torch.randperm(T, device=dev, generator=g)[:round(0.05 * T)]] = -1
    x["slots"] = slots
    bytes_per_step = T * ((hq + 2 * hkv) * d * 2 * 2 + 8 + 4 + d * 4) + 2 * d * 2

    def launch():
        qk_norm_rope_kv(x["q"], x["k"], x["v"], x["positions"], x["q_w"], x["k_w"], x["eps"], x["cos_sin"],
                        x["k_cache"], x["v_cache"], x["slots"], False)

    host = {}

    def e2e():
        """One step through the public API from pinned host memory, in chunks of E2E_CHUNK tokens on three streams:
        the host-to-device copy of chunk c + 1 and the device-to-host copy of chunk c - 1 run while chunk c computes
        (PCIe carries both directions at once, and the op is token-parallel). The streams start after, and the
        current stream waits for, all of a step's work, so steps do not overlap one another."""
        if not host:  # pinned host copies of the step's inputs, and the device buffers they are copied into
            host.update(qkv=x["qkv"].cpu().pin_memory(), positions=x["positions"].cpu().pin_memory(),
                        slots=x["slots"].cpu().pin_memory(),
                        q_out=torch.empty(T, hq, d, dtype=torch.bfloat16).pin_memory(),
                        dqkv=torch.empty_like(x["qkv"]), dpos=torch.empty_like(x["positions"]),
                        dslots=torch.empty_like(x["slots"]),
                        streams=[torch.cuda.Stream(dev) for _ in range(3)])
        dqkv, dpos, dslots = host["dqkv"], host["dpos"], host["dslots"]
        q, k, v = dqkv.split([hq * d, hkv * d, hkv * d], dim=-1)
        q, k, v = q.view(T, hq, d), k.view(T, hkv, d), v.view(T, hkv, d)
        s_in, s_cmp, s_out = host["streams"]
        main = torch.cuda.current_stream(dev)
        begin = torch.cuda.Event()
        begin.record(main)
        for s_ in (s_in, s_cmp, s_out):
            s_.wait_event(begin)
        for t0 in range(0, T, E2E_CHUNK):
            t1 = min(T, t0 + E2E_CHUNK)
            with torch.cuda.stream(s_in):
                dqkv[t0:t1].copy_(host["qkv"][t0:t1], non_blocking=True)
                dpos[t0:t1].copy_(host["positions"][t0:t1], non_blocking=True)
                dslots[t0:t1].copy_(host["slots"][t0:t1], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(s_in)
            s_cmp.wait_event(landed)
            with torch.cuda.stream(s_cmp):
                q_out, _ = qk_norm_rope_kv(q[t0:t1], k[t0:t1], v[t0:t1], dpos[t0:t1], x["q_w"], x["k_w"], x["eps"],
                                           x["cos_sin"], x["k_cache"], x["v_cache"], dslots[t0:t1], False)
                computed = torch.cuda.Event()
                computed.record(s_cmp)
            s_out.wait_event(computed)
            with torch.cuda.stream(s_out):
                host["q_out"][t0:t1].copy_(q_out, non_blocking=True)
                q_out.record_stream(s_out)
        for s_ in (s_in, s_cmp, s_out):
            done = torch.cuda.Event()
            done.record(s_)
            main.wait_event(done)
        h2d = host["qkv"].numel() * 2 + host["positions"].numel() * 8 + host["slots"].numel() * 4
        return h2d, host["q_out"].numel() * 2

    cpu_state = {}

    def cpu(tokens=T):
        """The oracle on the host over the first `tokens` tokens of the batch."""
        from oracle import reference_math as om
        if not cpu_state:
            cpu_state.update({k: (v.cpu() if torch.is_tensor(v) else v) for k, v in x.items()})
            c = cpu_state
            q, k, v = c["qkv"].split([hq * d, hkv * d, hkv * d], dim=-1)
            c["q"], c["k"], c["v"] = q.view(T, hq, d), k.view(T, hkv, d), v.view(T, hkv, d)
        c = cpu_state
        om.qk_norm_rope_kv(c["q"][:tokens], c["k"][:tokens], c["v"][:tokens], c["positions"][:tokens], c["q_w"],
                           c["k_w"], c["eps"], c["cos_sin"], c["k_cache"], c["v_cache"], c["slots"][:tokens], False)
        return tokens * ((hq + 2 * hkv) * d * 2 * 2 + 8 + 4 + d * 4) + 2 * d * 2

    # The reference's own Triton kernel on the same inputs (the same-box bar): it takes kv heads in groups of 4
    # (qk_norm_rope_kv.py:107), so shards of 1-2 kv heads (4/8 GPUs) have no reference kernel to time.
    library = None
    if hkv % 4 == 0:
        mod, why = reference_kernel_module("qk_norm_rope_kv")
        if mod is None:
            library = ("reference Triton qk_norm_rope_kv", why)
        else:
            def ref_launch():
                mod.qk_norm_rope_kv(x["q"], x["k"], x["v"], x["positions"], x["q_w"], x["k_w"], x["eps"],
                                    x["cos_sin"], x["k_cache"], x["v_cache"], x["slots"], False)
            library = ("reference Triton kernel nanovllm/kernels/qk_norm_rope_kv.py:92-125 (baseline/_ref, "
                       "JIT-compiled on this GPU)", ref_launch)
    else:
        library = ("reference Triton qk_norm_rope_kv", f"the reference kernel needs Hkv % 4 == 0; this shard has "
                                                       f"{hkv} kv heads")

    return dict(launch=launch, units=bytes_per_step, e2e=e2e, cpu=cpu, unit="GB/s", scale=1e9, bound="hbm",
                metric=METRIC_FUSED, dtype="bf16", launches_per_step=1, library=library,
                traffic_key=label,
                config={"workload": label, "tokens_per_step": T, "tokens_per_gpu_step_at_n1": args.tokens,
                        "q_heads": hq_total, "kv_heads": hkv_total, "head_dim": d,
                        "kv_heads_per_gpu": hkv, "cache_blocks": blocks, "block_size": 256,
                        "max_position": max_pos, "skip_fraction": 0.05, "write_k": False,
                        "parallelism": f"tp{world} (KV-head sharding, no collective)" if args.rank_shard_of <= 1
                        else f"one rank's shard of tp{world}, run alone on one GPU",
                        "l2": "flushed between timed steps (256 MiB write + 256 MiB read, outside the events)",
                        "bytes_formula": "T*((Hq+2Hkv)*D*2 read + 8 + 4 + D*4 + (Hq+2Hkv)*D*2 written) + 2*D*2"})


NORM_OPS = {"norm": ("rms_norm", "add_rms_norm", "silu_and_mul"), "rmsnorm": ("rms_norm",),
            "addrmsnorm": ("add_rms_norm",), "silu": ("silu_and_mul",)}


def norm_workload(args, rank, world, dev):
    """BASELINE config 2 at T = 8192 (hidden 1024, intermediate 3072): "norm" runs RMSNorm, Add+RMSNorm and SiLU x Mul
    as one step (three launches); "rmsnorm", "addrmsnorm" and "silu" run one of them alone."""
    from nanovllm_b200 import workloads
    from nanovllm_b200.kernels.rms_norm import fused_add_rms_norm, rms_norm
    from nanovllm_b200.kernels.swiglu import silu_and_mul
    ops = NORM_OPS[args.workload]
    T = args.tokens * (world if args.scaling == "weak" else 1)
    n, inter = 1024, 3072
    x = workloads.norm_inputs(T, n, seed=5, device=dev)
    gu = workloads.silu_inputs(T, inter, seed=6, device=dev)["x"]

    def op_bytes(tokens):
        b = {"rms_norm": (2 * tokens * n + n) * 2, "add_rms_norm": (4 * tokens * n + n) * 2,
             "silu_and_mul": 3 * tokens * inter * 2}
        return sum(b[o] for o in ops)

    calls = {"rms_norm": lambda: rms_norm(x["x"], x["w"], x["eps"]),
             "add_rms_norm": lambda: fused_add_rms_norm(x["x"], x["residual"], x["w"], x["eps"]),
             "silu_and_mul": lambda: silu_and_mul(gu)}

    def launch():
        for o in ops:
            calls[o]()

    xc = {}

    def cpu(tokens=T):
        from oracle import reference_math as om
        if not xc:
            xc.update({k: (v.cpu() if torch.is_tensor(v) else v) for k, v in x.items()}, gu=gu.cpu())
        if "rms_norm" in ops:
            om.rms_forward(xc["x"][:tokens], xc["w"], xc["eps"])
        if "add_rms_norm" in ops:
            om.add_rms_forward(xc["x"][:tokens], xc["residual"][:tokens], xc["w"], xc["eps"])
        if "silu_and_mul" in ops:
            om.silu_and_mul(xc["gu"][:tokens])
        return op_bytes(tokens)

    return dict(launch=launch, units=op_bytes(T), e2e=None, cpu=cpu, unit="GB/s", scale=1e9, bound="hbm",
                metric=" + ".join(ops) + " GB/s at T=8192", dtype="bf16", launches_per_step=len(ops),
                traffic_key=args.workload,
                config={"workload": args.workload, "ops": list(ops), "tokens_per_step": T, "hidden": n,
                        "intermediate": inter, "parallelism": f"replicas x{world}",
                        "l2": "flushed between timed steps",
                        "bytes_formula": "rms (2Tn+n)*2, add_rms (4Tn+n)*2, silu 3*T*inter*2 "
                                         "(scripts/bench_norm_act.py:3-5)"})


def matmul_workload(args, rank, world, dev):
    from nanovllm_b200 import workloads
    from nanovllm_b200.kernels.matmul import matmul
    M, N, K = (int(v) for v in args.matmul_shape.split(","))
    n_local = N // world if args.scaling == "strong" else N
    x = workloads.matmul_inputs(M, n_local, K, dtype=torch.bfloat16, seed=7, device=dev)
    units = 2 * M * n_local * K

    def launch():
        matmul(x["a"], x["b"])

    xc = {}

    def cpu(tokens=M):
        if not xc:
            xc.update(a=x["a"].cpu(), b=x["b"].cpu())
        xc["a"][:tokens] @ xc["b"]  # torch CPU bf16 matmul (fp32 accumulation) over the first `tokens` rows
        return 2 * tokens * n_local * K

    mod, why = reference_kernel_module("matmul")
    if args.cublas:
        library = ("cuBLAS (torch.matmul), the GEMM the reference's linear layers run", lambda: x["a"] @ x["b"])
    elif mod is None:
        library = ("reference Triton matmul", why)
    else:
        library = ("reference Triton kernel nanovllm/kernels/matmul.py:84-99 (baseline/_ref, autotuned and "
                   "JIT-compiled on this GPU)", lambda: mod.matmul(x["a"], x["b"]))

    return dict(launch=launch, units=units, e2e=None, cpu=cpu, unit="TFLOP/s", scale=1e12, bound="tensor",
                metric=f"matmul bf16 TFLOP/s at M={M}, N={N}, K={K}", dtype="bf16", launches_per_step=1,
                traffic_key="matmul",
                library=library,
                config={"workload": "matmul", "M": M, "N": n_local, "K": K, "b_layout": "weight.t() (K-major)",
                        "parallelism": f"column-parallel x{world}", "l2": "flushed between timed steps"})


def gateup_workload(args, rank, world, dev):
    """Qwen3-8B MLP gate_up projection with the SiLU x Mul epilogue: A [4096, 4096] @ [gate | up] weight.t()
    ([4096, 2 x 12288]) -> [4096, 12288], one kernel (nvb200_matmul_silu_and_mul). Column-parallel shards split the
    intermediate size (each rank its gate and up columns), as MergedColumnParallelLinear does."""
    from nanovllm_b200.kernels.matmul import matmul_silu_and_mul
    M, K, inter = (int(v) for v in args.gateup_shape.split(","))
    n_local = inter // world if args.scaling == "strong" else inter
    g = torch.Generator(device=dev).manual_seed(11)
    a = (torch.randn(M, K, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16)
    w = torch.randn(2 * n_local, K, device=dev, generator=g).to(torch.bfloat16)
    b = w.t()
    units = 2 * M * 2 * n_local * K

    def launch():
        matmul_silu_and_mul(a, b)

    # What the reference's Qwen3MLP runs (models/qwen3.py:133-137): the gate_up projection (F.linear: cuBLAS), then
    # SiluAndMul (its Triton kernel, nanovllm/kernels/swiglu.py, under the triton backends).
    mod, why = reference_kernel_module("swiglu")
    if mod is None:
        library = ("cuBLAS gate_up GEMM + reference Triton silu_and_mul", why)
    else:
        library = ("cuBLAS gate_up GEMM (torch.matmul) + reference Triton silu_and_mul (nanovllm/kernels/swiglu.py:"
                   "34-43, baseline/_ref)", lambda: mod.silu_and_mul(a @ b))

    xc = {}

    def cpu(tokens=M):
        if not xc:
            xc.update(a=a.cpu(), b=b.cpu())
        gu = xc["a"][:tokens] @ xc["b"]  # torch CPU bf16, then the reference's SiLU x Mul
        torch.nn.functional.silu(gu[:, :n_local]) * gu[:, n_local:]
        return 2 * tokens * 2 * n_local * K

    return dict(launch=launch, units=units, e2e=None, cpu=cpu, unit="TFLOP/s", scale=1e12, bound="tensor",
                metric=f"gate_up GEMM + SiLU x Mul bf16 TFLOP/s (M={M}, K={K}, intermediate {inter})", dtype="bf16",
                launches_per_step=1, traffic_key="gateup", library=library,
                config={"workload": "gateup", "M": M, "K": K, "intermediate": n_local,
                        "b_layout": "[gate | up] weight.t() (K-major)", "parallelism": f"column-parallel x{world}",
                        "l2": "flushed between timed steps"})


def rowpar_workload(args, rank, world, dev):
    """Decode-step row-parallel projection with its all-reduce: Qwen3-8B down_proj (K = 12288 split over the ranks,
    N = 4096) for a batch of 32 tokens, one fused GEMM + NVLink all-reduce per rank (RowParallelAllReduce; one GPU:
    the plain GEMM). Strong scaling: the layer is fixed, each rank holds K / N of it."""
    from nanovllm_b200.parallel import RowParallelAllReduce
    M, N, K = 32, 4096, 12288
    k_local = K // world
    g = torch.Generator(device=dev).manual_seed(13 + rank)
    a = (torch.randn(M, k_local, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16)
    w = torch.randn(N, k_local, device=dev, generator=g).to(torch.bfloat16)
    b = w.t()
    if world > 1:
        op = RowParallelAllReduce(max_n=N)  # collective set-up: every rank builds it
    else:
        from nanovllm_b200.kernels.matmul import matmul
        op = matmul

    def launch():
        op(a, b)

    xc = {}

    def cpu(tokens=M):
        if not xc:
            xc.update(a=a.cpu(), b=b.cpu())
        xc["a"][:tokens] @ xc["b"]  # this rank's partial on the host; the exchange is not timed on the CPU
        return 2 * tokens * N * k_local

    return dict(launch=launch, units=2 * M * N * k_local, e2e=None, cpu=cpu, unit="TFLOP/s", scale=1e12,
                bound="tensor", scaling="strong",
                metric="row-parallel down_proj GEMM + all-reduce bf16 TFLOP/s (Qwen3-8B, 32 tokens)", dtype="bf16",
                launches_per_step=1, traffic_key="rowpar",
                config={"workload": "rowpar", "M": M, "N": N, "K": K, "K_per_rank": k_local,
                        "parallelism": f"row-parallel x{world}, fused NVLink all-reduce",
                        "l2": "flushed between timed steps"})


def attn_workload(args, rank, world, dev):
    """Decode attention of the config-5 decode step (the flash_attn_with_kvcache call of the reference's
    Attention.forward): 32 sequences, one query each, 1024 keys per sequence in pages of 256 (randomly placed
    blocks), Qwen3-0.6B heads (16 q / 8 kv, head_dim 128), bf16 cache N(0,1). Sharded by KV head like the fused op
    (weak scaling multiplies the sequences by N). Four copies of the cache rotate between steps, so no step finds the
    previous one's keys in L2 even without the flush."""
    from nanovllm_b200.kernels.attention import flash_attn_with_kvcache
    from oracle import reference_math as om
    B0, ctx, hq0, hkv0 = (int(v) for v in args.attn_shape.split(","))
    B = B0 * (world if args.scaling == "weak" else 1)
    hq, hkv, d, bs = hq0 // world, hkv0 // world, 128, 256
    pages = (ctx + bs - 1) // bs
    nb = B * pages + 8
    g = torch.Generator(device=dev).manual_seed(17 + rank)
    copies = 4
    caches = [(torch.randn(nb, bs, hkv, d, device=dev, generator=g).to(torch.bfloat16),
               torch.randn(nb, bs, hkv, d, device=dev, generator=g).to(torch.bfloat16)) for _ in range(copies)]
    q = torch.randn(B, 1, hq, d, device=dev, generator=g).to(torch.bfloat16)
    table = torch.randperm(nb, device=dev, generator=g)[:B * pages].view(B, pages).to(torch.int32)
    seqlens = torch.full((B,), ctx, dtype=torch.int32, device=dev)
    scale = d ** -0.5
    units = om.paged_decode_attention_bytes([ctx] * B, 1, hq, hkv, d, bs)
    step = [0]

    from nanovllm_b200.kernels.attention import decode_attention

    def launch():
        kc, vc = caches[step[0] % copies]
        step[0] += 1
        if args.attn_method == "auto":  # the drop-in, as the reference's Attention.forward calls it
            flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seqlens, block_table=table, softmax_scale=scale,
                                    causal=True)
        else:
            decode_attention(q, kc, vc, seqlens, block_table=table, softmax_scale=scale, causal=True,
                             method=args.attn_method)

    def library():
        import flash_attn
        kc, vc = caches[step[0] % copies]
        step[0] += 1
        flash_attn.flash_attn_with_kvcache(q, kc, vc, cache_seqlens=seqlens, block_table=table, softmax_scale=scale,
                                           causal=True)

    host = {}

    def e2e():
        if not host:
            host.update(q=q.cpu().pin_memory(), lens=seqlens.cpu().pin_memory(), table=table.cpu().pin_memory(),
                        out=torch.empty(B, 1, hq, d, dtype=torch.bfloat16).pin_memory(), dq=torch.empty_like(q),
                        dlens=torch.empty_like(seqlens), dtable=torch.empty_like(table))
        host["dq"].copy_(host["q"], non_blocking=True)
        host["dlens"].copy_(host["lens"], non_blocking=True)
        host["dtable"].copy_(host["table"], non_blocking=True)
        kc, vc = caches[step[0] % copies]
        step[0] += 1
        out = flash_attn_with_kvcache(host["dq"], kc, vc, cache_seqlens=host["dlens"], block_table=host["dtable"],
                                      softmax_scale=scale, causal=True)
        host["out"].copy_(out, non_blocking=True)
        return q.numel() * 2 + seqlens.numel() * 4 + table.numel() * 4, out.numel() * 2

    xc = {}

    def cpu(tokens=B):
        if not xc:
            xc.update(q=q.cpu(), k=caches[0][0].cpu(), v=caches[0][1].cpu(), t=table.cpu(), l=seqlens.cpu())
        om.paged_decode_attention(xc["q"][:tokens], xc["k"], xc["v"], xc["l"][:tokens], xc["t"][:tokens], scale, True)
        return om.paged_decode_attention_bytes([ctx] * tokens, 1, hq, hkv, d, bs)

    return dict(launch=launch, units=units, e2e=e2e, cpu=cpu, unit="GB/s", scale=1e9, bound="hbm",
                metric=f"paged decode attention GB/s ({B0} seqs x {ctx} keys, {hq0}/{hkv0} heads)", dtype="bf16",
                launches_per_step=1, traffic_key="attn", library=("flash_attn.flash_attn_with_kvcache", library),
                e2e_path="nanovllm_b200.kernels.attention.flash_attn_with_kvcache (public API) with pinned host q, "
                         "lengths and block table",
                config={"workload": "attn", "tokens_per_step": B, "sequences": B, "keys_per_sequence": ctx,
                        "q_heads_per_gpu": hq, "kv_heads_per_gpu": hkv, "head_dim": d, "block_size": bs,
                        "queries_per_sequence": 1, "causal": True,
                        "parallelism": f"tp{world} (KV-head sharding, no collective)",
                        "l2": f"flushed between timed steps; {copies} cache copies rotate",
                        "bytes_formula": "sum_b L_b*Hkv*D*2*2 + 2*B*Hq*D*2 + 4*B + 4*sum_b ceil(L_b/256)"})


def storekv_workload(args, rank, world, dev):
    """The plain KV-cache write (store_kvcache, the attention layer's non-fused route) at T = 8192 tokens with the
    Qwen3-0.6B layout: k and v are strided views of the qkv projection output [T, 4096], the cache is
    [64, 256, 8, 128] per rank slice, 5 % of the slots are -1."""
    from nanovllm_b200.kernels.attention import store_kvcache
    from oracle import reference_math as om
    T = args.tokens * (world if args.scaling == "weak" else 1)
    hq, hkv, d = 16 // world, 8 // world, 128
    blocks = max(64, (T + 255) // 256 + 1)
    g = torch.Generator(device=dev).manual_seed(23 + rank)
    qkv = torch.randn(T, (hq + 2 * hkv) * d, device=dev, generator=g).to(torch.bfloat16)
    k = qkv[:, hq * d:(hq + hkv) * d].view(T, hkv, d)
    v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
    kc = torch.zeros(blocks, 256, hkv, d, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    g2 = torch.Generator(device=dev).manual_seed(99)
    slots = torch.randperm(blocks * 256, device=dev, generator=g2)[:T].to(torch.int32)
    slots[torch.randperm(T, device=dev, generator=g2)[:round(0.05 * T)]] = -1
    kept = T - round(0.05 * T)
    units = om.store_kvcache_bytes(T, hkv * d, 2, kept)

    def launch():
        store_kvcache(k, v, kc, vc, slots)

    xc = {}

    def cpu(tokens=T):
        if not xc:
            xc.update(k=k.cpu(), v=v.cpu(), kc=kc.cpu(), vc=vc.cpu(), s=slots.cpu())
        om.store_kvcache(xc["k"][:tokens], xc["v"][:tokens], xc["kc"], xc["vc"], xc["s"][:tokens])
        return om.store_kvcache_bytes(tokens, hkv * d, 2, int((xc["s"][:tokens] >= 0).sum()))

    return dict(launch=launch, units=units, e2e=None, cpu=cpu, unit="GB/s", scale=1e9, bound="hbm",
                metric="store_kvcache GB/s at T=8192 (Qwen3-0.6B heads)", dtype="bf16", launches_per_step=1,
                traffic_key="storekv",
                config={"workload": "storekv", "tokens_per_step": T, "kv_heads_per_gpu": hkv, "head_dim": d,
                        "cache_blocks": blocks, "block_size": 256, "skip_fraction": 0.05,
                        "parallelism": f"tp{world} (KV-head sharding, no collective)",
                        "l2": "flushed between timed steps",
                        "bytes_formula": "T*4 + kept*4*Hkv*D*2"})


def make_workload(args, rank, world, dev):
    if args.workload == "fused8b":
        return fused_workload(args, rank, world, dev, 32, 8, 32768, 1024, "fused8b")
    if args.workload == "fused06b":
        return fused_workload(args, rank, world, dev, 16, 8, 4096, 64, "fused06b")
    if args.workload in NORM_OPS:
        return norm_workload(args, rank, world, dev)
    if args.workload == "gateup":
        return gateup_workload(args, rank, world, dev)
    if args.workload == "rowpar":
        return rowpar_workload(args, rank, world, dev)
    if args.workload == "attn":
        return attn_workload(args, rank, world, dev)
    if args.workload == "storekv":
        return storekv_workload(args, rank, world, dev)
    return matmul_workload(args, rank, world, dev)


# ---------------------------------------------------------------------------------------------------------------

def time_cpu(fn, full, budget_s=10.0, max_reps=30):
    """Host-core timing of fn(rows) (which returns the units it processed): the full step when a run fits in a quarter
    of budget_s, else a prefix of rows sized to it (estimated from a 1/64 probe run after a first warm-up call).
    Median over runs after one warm-up,
    repeated until ~budget_s. Returns (units / second, runs, rows per run)."""
    probe = max(1, full // 64)
    fn(probe)  # one-time set-up (host copies of the inputs) outside the estimate
    t0 = time.perf_counter()
    fn(probe)
    est_full = (time.perf_counter() - t0) * full / probe
    rows = full if est_full <= budget_s / 4 else max(1, int(full * (budget_s / 4) / est_full))
    fn(rows)
    times, units = [], 0
    start = time.perf_counter()
    while len(times) < max_reps and (len(times) < 3 or time.perf_counter() - start < budget_s):
        t0 = time.perf_counter()
        units = fn(rows)
        times.append(time.perf_counter() - t0)
    return units / statistics.median(times), len(times), rows


def run_reference_arm(args, rank, world):
    """`--impl reference`: the reference's CPU implementation (the oracle port) on the host cores. Each step runs on
    a prefix of the one-GPU batch sized so that warm-up + steps take about two minutes."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    wargs = argparse.Namespace(**vars(args))
    wargs.scaling = "strong"  # one host: the one-GPU job
    dev = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
    wl = make_workload(wargs, 0, 1, dev)
    full = wl["config"].get("tokens_per_step", wl["config"].get("M"))
    with torch.inference_mode():
        t0 = time.perf_counter()
        wl["cpu"]()
        t_full = time.perf_counter() - t0
        per_step = 120.0 / (args.steps + args.warmup)
        tokens = max(1, min(full, int(full * per_step / max(t_full, 1e-9))))
        for _ in range(args.warmup):
            wl["cpu"](tokens)
        total, units = 0.0, 0
        for _ in range(args.steps):
            t0 = time.perf_counter()
            units += wl["cpu"](tokens)
            total += time.perf_counter() - t0
    value = units / total / wl["scale"]
    sample = (f"first {tokens} of the {full} rows/tokens of the one-GPU step ({wl['config']['workload']}) per step, "
              f"torch CPU bf16 eager restatement of the reference")
    line = {"metric": wl["metric"], "value": value, "unit": wl["unit"], "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
            "scaling": wl.get("scaling", args.scaling), "vs_baseline": None, "dtype": wl["dtype"], "data": "synthetic",
            "config": wl["config"], "impl": "reference",
            "cpu_baseline": {"value": value, "unit": wl["unit"], "cores": torch.get_num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": wl["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------------
# one decode step of a Qwen3-0.6B-architecture model (28 layers, hidden 1024, 16 q / 8 kv heads,
# head_dim 128, intermediate 3072, vocab 151936), random bf16 weights, batch 32 x 1024 tokens of context in the paged
# cache (N(0,1)), whole-step CUDA graph replay, timed as the reference's scripts/bench_decode.py:82-95 times it
# (CUDA events around 50 replays of graphs[("target", 1, bs)], median of 3). The reference's own ModelRunner builds
# and captures the model (offline install of the reference in baseline/_ref); kernel_backend "b200" runs it on
# nanovllm_b200 through nanovllm_b200.install(), "compile" / "triton_fused" are the reference's own backends.
# Each backend runs in its own process (ModelRunner takes most of the GPU memory for its KV cache).

QWEN3_06B = {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_size": 1024,
             "intermediate_size": 3072, "num_hidden_layers": 28, "num_attention_heads": 16, "num_key_value_heads": 8,
             "head_dim": 128, "vocab_size": 151936, "max_position_embeddings": 40960, "rms_norm_eps": 1e-6,
             "rope_theta": 1000000, "tie_word_embeddings": True, "torch_dtype": "bfloat16", "dtype": "bfloat16",
             "hidden_act": "silu", "attention_bias": False}


def decode_worker(backend: str, bs: int, ctx: int, tp: int = 1, profile_one: bool = False) -> dict:
    """One rank of the decode-step measurement (tp > 1: launched once per GPU by torch.distributed.run; the
    reference's ModelRunner then forms its own NCCL group, and every rank replays its graph in step with the others,
    as the reference's worker processes would)."""
    import tempfile
    ref = os.path.join(ROOT, "baseline", "_ref")
    sys.path.insert(0, ref)
    import nanovllm_b200
    nanovllm_b200.install()
    import nanovllm.engine.model_runner as mr
    from nanovllm.config import Config
    rank = int(os.environ.get("RANK", "0"))
    if tp > 1:
        import torch.distributed as tdist
        from multiprocessing.shared_memory import SharedMemory
        init = tdist.init_process_group

        def init_127(backend_name, init_method=None, **kw):
            # The runner's own rendezvous (tcp://localhost:2333) would wait forever under torch.distributed.run:
            # there, a tcp:// store connects to the launcher's store as a client, and nothing serves port 2333. Use
            # the launcher's rendezvous (env://, MASTER_ADDR = 127.0.0.1) instead.
            return init(backend_name, "env://", **kw)
        mr.dist.init_process_group = init_127
        mr.ModelRunner.loop = lambda self: None  # ranks > 0 return from __init__ instead of serving rank 0's calls
        if rank == 0:
            try:  # a segment left by an interrupted run would make the runner's create fail
                SharedMemory(name="nanovllm").unlink()
            except FileNotFoundError:
                pass

    def random_weights(model, path):  # no checkpoint: random-init every parameter (norm weights around 1)
        g = torch.Generator(device="cuda").manual_seed(0)
        with torch.no_grad():
            for name, p in model.named_parameters():
                if name.endswith("norm.weight"):
                    p.copy_(1 + 0.1 * torch.randn(p.shape, generator=g, device=p.device))
                else:
                    p.copy_(0.02 * torch.randn(p.shape, generator=g, device=p.device))
    mr.load_model = random_weights
    d = tempfile.mkdtemp()
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(QWEN3_06B, f)
    cfg = Config(d, kernel_backend=backend, max_num_seqs=bs, max_model_len=2048, max_num_batched_tokens=4096,
                 gpu_memory_utilization=0.5, tensor_parallel_size=tp)
    runner = mr.ModelRunner(cfg, rank, [])
    blocks_per_seq = (ctx + 1 + 255) // 256
    assert cfg.num_kvcache_blocks >= bs * blocks_per_seq
    with torch.inference_mode():  # the runner's graph buffers are inference tensors
        g = torch.Generator(device="cuda").manual_seed(1)
        runner.kv_caches["target"].normal_(generator=g)
        gv = runner.graph_vars
        gv["input_ids"][:bs] = torch.randint(0, QWEN3_06B["vocab_size"], (bs,), device="cuda", generator=g)
        gv["positions"][:bs] = ctx
        tables = torch.arange(bs * blocks_per_seq, dtype=torch.int32, device="cuda").view(bs, blocks_per_seq)
        gv["block_tables"].zero_()
        gv["block_tables"][:bs, :blocks_per_seq] = tables
        gv["slot_mapping"].fill_(-1)
        gv["slot_mapping"][:bs] = tables[:, ctx // 256] * 256 + ctx % 256
        gv["context_lens"].zero_()
        gv["context_lens"][:bs] = ctx + 1
        graph = runner.graphs[("target", 1, bs)]
        if profile_one:
            # One replay between cudaProfilerStart/Stop, for `ncu --profile-from-start off --graph-profiling node`:
            # the launch list of one decode step, kernel by kernel.
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStart()
            graph.replay()
            torch.cuda.synchronize()
            torch.cuda.cudart().cudaProfilerStop()
            return {"backend": backend, "profiled_replays": 1}
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if tp > 1:
            mr.dist.barrier()
        clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))).__enter__()
        for _ in range(10):
            graph.replay()
        per_run = []
        clocks.mark_start()
        for _ in range(3):
            if tp > 1:
                torch.cuda.synchronize()
                mr.dist.barrier()
            start.record()
            for _ in range(50):
                graph.replay()
            end.record()
            end.synchronize()
            t = start.elapsed_time(end) / 50
            if tp > 1:  # the slowest rank's time
                tt = torch.tensor([t], device="cuda")
                mr.dist.all_reduce(tt, op=mr.dist.ReduceOp.MAX)
                t = float(tt.item())
            per_run.append(t)
        clocks.mark_end()
        clocks.__exit__(None, None, None)
        out = gv["outputs"]["target"][:bs].float()
        res = {"backend": backend, "graph_replay_us": 1e3 * sorted(per_run)[1], "runs_us": [1e3 * x for x in per_run],
               "finite": bool(torch.isfinite(out).all()), "kv_blocks": cfg.num_kvcache_blocks, "tp": tp,
               "clocks": clocks.summary()}
    if tp > 1:
        torch.cuda.synchronize()
        del graph
        runner.graphs.clear()  # graphs holding NCCL calls go before the process group
        mr.dist.barrier()
        if rank == 0:
            runner.shm.close()
            runner.shm.unlink()
        else:
            runner.shm.close()
        mr.dist.destroy_process_group()
        return res if rank == 0 else None
    try:
        runner.exit()
    except Exception:
        pass
    return res


def decode_backends(args) -> dict:
    """Runs the decode-step worker once per backend, each in a fresh process (group), and returns their results."""
    results = {}
    for backend in args.decode_backends.split(","):
        cmd = [sys.executable, os.path.abspath(__file__), "--decode-worker", backend, "--decode-batch",
               str(args.decode_batch), "--decode-ctx", str(args.decode_ctx), "--decode-tp", str(args.decode_tp)]
        if args.decode_tp > 1:
            cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.decode_tp}",
                   "--master-addr", "127.0.0.1", "--master-port", "29581", *cmd[1:]]
        t0 = time.perf_counter()
        try:
            out = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        except subprocess.TimeoutExpired:
            results[backend] = {"backend": backend, "error": "worker did not finish within 900 s"}
            continue
        lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
        if out.returncode == 0 and lines:
            results[backend] = json.loads(lines[-1])
        else:
            results[backend] = {"backend": backend, "error": (out.stderr or out.stdout)[-800:]}
        results[backend]["worker_wall_s"] = round(time.perf_counter() - t0, 1)
    return results


def decode_summary(results: dict) -> dict:
    """The decode_step object of the headline line: each backend's median graph replay (us) and clocks."""
    out = {"metric": "decode-step graph replay us (Qwen3-0.6B arch, batch 32, ctx 1024, whole-step CUDA graph)",
           "method": "the reference's ModelRunner per backend in a fresh process; CUDA events around 50 replays, "
                     "median of 3 (scripts/bench_decode.py:82-95)", "higher_is_better": False}
    for name, r in results.items():
        key = name.replace("-", "_")
        out[f"{key}_us"] = r.get("graph_replay_us")
        out[f"{key}_detail"] = {k: v for k, v in r.items() if k not in ("backend", "graph_replay_us")}
    b, c = out.get("b200_us"), out.get("compile_us")
    out["b200_vs_compile"] = (c / b) if (b and c) else None
    return out


def run_decode(args) -> None:
    results = decode_backends(args)
    ours = results.get("b200", {})
    line = {"metric": "decode-step graph replay us (Qwen3-0.6B arch, batch 32, ctx 1024)",
            "value": ours.get("graph_replay_us"), "unit": "us", "n_gpus": args.decode_tp, "steps": 150, "warmup": 10,
            "ms_per_step": (ours.get("graph_replay_us") or 0) / 1e3, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, N(0,1) KV cache)",
            "config": {"workload": "decode", "model": "Qwen3-0.6B architecture", "batch": args.decode_batch,
                       "context": args.decode_ctx, "parallelism": f"tp{args.decode_tp}",
                       "graph": "whole-step CUDA graph"},
            "backends": results}
    print(json.dumps(line), flush=True)


# Decode projections (`--workload projections`): each projection of a Qwen3 decode layer preceded by this library's
# RMSNorm (as in the model, so that the projection kernel may start while the norm finishes), over enough distinct
# weights that they come from HBM (at least 28, at least 2.4x the L2 in all), captured in one CUDA graph and
# replayed; us per norm + projection, median of 5 x 10 replays. b200 runs the route install() takes for the layer
# (nanovllm_b200.kernels.matmul: linear_decode where decode_gemm_applies / fused_gate_up_applies admit it, else
# cuBLAS); cuBLAS is torch's F.linear (and the SiLU x Mul kernel for gate_up), what the reference's layers run.
PROJECTIONS = {"qwen3-0.6b": {"qkv_proj": (4096, 1024, False), "o_proj": (1024, 2048, False),
                              "gate_up_proj+silu": (3072, 1024, True), "down_proj": (1024, 3072, False)},
               "qwen3-8b": {"qkv_proj": (6144, 4096, False), "o_proj": (4096, 4096, False),
                            "gate_up_proj+silu": (12288, 4096, True), "down_proj": (4096, 12288, False)}}


def run_projections(args) -> None:
    import statistics
    import nanovllm_b200.kernels.matmul as mm
    from nanovllm_b200.kernels.rms_norm import rms_norm
    from nanovllm_b200.kernels.swiglu import silu_and_mul
    dev = torch.device("cuda", 0)
    rows = args.proj_rows
    res = {}

    def timed(fn, calls):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        out = []
        for _ in range(5):
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            for _ in range(10):
                graph.replay()
            e_.record()
            torch.cuda.synchronize()
            out.append(s_.elapsed_time(e_) * 1e3 / (10 * calls))
        del graph
        return statistics.median(out)

    g = torch.Generator(device=dev).manual_seed(17)
    with torch.inference_mode(), ClockSampler(0) as clocks:
        clocks.mark_start()
        for name, (n, k, swiglu) in PROJECTIONS[args.proj_model].items():
            w_rows = 2 * n if swiglu else n
            count = max(28, -(-int(2.4 * 126e6) // (w_rows * k * 2)))
            x = torch.randn(rows, k, device=dev, generator=g).to(torch.bfloat16)
            nw = (1 + 0.1 * torch.randn(k, device=dev, generator=g)).to(torch.bfloat16)
            ws = [torch.randn(w_rows, k, device=dev, generator=g).to(torch.bfloat16) for _ in range(count)]
            routed = (mm.fused_gate_up_applies(x, ws[0]) if swiglu else mm.decode_gemm_applies(x, ws[0]))

            def ours():
                for w in ws:
                    h = rms_norm(x, nw, 1e-6)
                    y = mm.linear_decode(h, w, swiglu=swiglu) if routed else None
                    if y is None:
                        y = h @ w.t()
                        if swiglu:
                            silu_and_mul(y)

            def cublas():
                for w in ws:
                    y = rms_norm(x, nw, 1e-6) @ w.t()
                    if swiglu:
                        silu_and_mul(y)

            def norm_only():
                for _ in ws:
                    rms_norm(x, nw, 1e-6)
            res[name] = {"shape": [rows, n, k], "weights": count, "routed_to_b200_kernel": routed,
                         "b200_us": timed(ours, count), "cublas_us": timed(cublas, count),
                         "norm_alone_us": timed(norm_only, count)}
            del ws
        clocks.mark_end()
    b = sum(r["b200_us"] for r in res.values())
    c = sum(r["cublas_us"] for r in res.values())
    line = {"metric": f"decode projections: us per layer for RMSNorm + projection, {args.proj_model} shapes, "
                      f"{rows} rows, CUDA graph", "value": b, "unit": "us", "n_gpus": 1, "steps": 50, "warmup": 4,
            "ms_per_step": b / 1e3, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded weights and rows)",
            "config": {"workload": "projections", "model": args.proj_model, "rows": rows,
                       "l2": "weights rotate over >= 2.4x the L2"},
            "cublas_us": c, "b200_vs_cublas": c / b, "projections": res, "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.decode_worker:
        res = decode_worker(args.decode_worker, args.decode_batch, args.decode_ctx, args.decode_tp,
                            args.decode_profile)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if args.workload == "decode":
        run_decode(args)
        return
    if args.workload == "projections":
        run_projections(args)
        return
    rank, world, local = setup_dist(args)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the kernels have no CPU path)")
    dev = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    peaks, peak_kind = load_peaks()
    wl = make_workload(args, rank, world, dev)
    flush_w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def flush_l2():
        # Write 256 MiB (evicts the step's lines), then read another 256 MiB so that the dirty lines of that
        # write are written back here, not during the timed kernel.
        flush_w.zero_()
        flush_r.max()

    with torch.inference_mode(), ClockSampler(local) as clocks:
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        for _ in range(args.warmup):
            flush_l2()
            wl["launch"]()
        barrier(world)
        clocks.mark_start()
        for i in range(args.steps):
            flush_l2()
            starts[i].record(stream)
            wl["launch"]()
            ends[i].record(stream)
        barrier(world)
        clocks.mark_end()
        per_step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        local_s = sum(per_step_ms) / 1e3
        total_s = max_over_ranks(local_s, world)
        all_units = sum_over_ranks(float(wl["units"]) * args.steps, world)
        value = all_units / total_s / wl["scale"]
        achieved = wl["units"] / (local_s / args.steps) / wl["scale"]  # this rank's kernel, per launch

        e2e = None
        if wl["e2e"] is not None and not args.no_e2e:
            for _ in range(max(2, args.warmup // 2)):
                wl["e2e"]()
            torch.cuda.synchronize()
            barrier(world)
            e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e_start.record(stream)
            for _ in range(args.steps):
                h2d, d2h = wl["e2e"]()
            e_end.record(stream)
            torch.cuda.synchronize()
            e_s = max_over_ranks(e_start.elapsed_time(e_end) / 1e3, world)
            e2e = {"value": all_units / e_s / wl["scale"], "unit": wl["unit"], "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h,
                   "path": wl.get("e2e_path", f"nanovllm_b200.kernels.qk_norm_rope_kv (public API) with pinned "
                                              f"host inputs/outputs, in chunks of {E2E_CHUNK} tokens whose copies "
                                              f"in both directions overlap the other chunks' kernels (three streams)")}

        library = None
        if wl.get("library") is not None:
            name, fn = wl["library"]
            if isinstance(fn, str):
                library = {"name": name, "unavailable": fn}
            else:
                # As many warm-up calls as our arm had, plus one for Triton's JIT/autotune on the first call; then
                # the same number of steps (at most 500), each after the same L2 flush, timed the same way.
                for _ in range(args.warmup + 1):
                    flush_l2()
                    fn()
                torch.cuda.synchronize()
                lib_steps = min(args.steps, 500)
                ls = [torch.cuda.Event(enable_timing=True) for _ in range(lib_steps)]
                le = [torch.cuda.Event(enable_timing=True) for _ in range(lib_steps)]
                for i in range(lib_steps):
                    flush_l2()
                    ls[i].record(stream)
                    fn()
                    le[i].record(stream)
                torch.cuda.synchronize()
                lib_ms = [a.elapsed_time(b) for a, b in zip(ls, le)]
                lib_s = sum(lib_ms) / 1e3 / lib_steps
                ours_s = local_s / args.steps
                library = {"name": name, "us_per_step": 1e6 * lib_s, "value": wl["units"] / lib_s / wl["scale"],
                           "unit": wl["unit"], "ours_us_per_step": 1e6 * ours_s, "speedup": lib_s / ours_s,
                           "step_us": step_stats(lib_ms),
                           "note": "the kernel the reference itself runs for this op, same inputs, same L2 flush and "
                                   "step timing, this rank"}

    if wl["bound"] == "hbm" and rank == 0 and not args.no_copy_reference:
        # The same bytes moved by torch's copy (half read, half written), flushed and timed the same way: what a plain
        # copy of this size achieves, launch and ramp-up included, beside the asymptotic copy peak of the roofline.
        half = max(16, int(wl["units"]) // 2 // 16 * 16)
        src = torch.empty(half, dtype=torch.uint8, device=dev).fill_(1)
        dst = torch.empty_like(src)
        cs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(50)]
        with torch.inference_mode():
            for _ in range(args.warmup):
                flush_l2()
                dst.copy_(src)
            for a_, b_ in cs:
                flush_l2()
                a_.record(stream)
                dst.copy_(src)
                b_.record(stream)
            torch.cuda.synchronize()
        copy_s = sum(a_.elapsed_time(b_) for a_, b_ in cs) / 1e3 / len(cs)
        ours_s = local_s / args.steps
        copy_ref = {"us": 1e6 * copy_s, "gbs": 2 * half / copy_s / 1e9, "ours_frac_of_copy_rate": copy_s / ours_s,
                    "note": "torch copy_ of the step's algorithmic bytes (half read, half written), same flush and "
                            "event timing"}
        del src, dst
    else:
        copy_ref = None
    if wl["bound"] == "hbm":
        peak = peaks["hbm_gbs"]
        roof_unit = "GB/s"
    else:
        peak = peaks["bf16_tflops"]
        roof_unit = "TFLOP/s"
    traffic = load_traffic(wl["traffic_key"])
    line = {"metric": wl["metric"], "value": value, "unit": wl["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * total_s / args.steps, "higher_is_better": True,
            "scaling": wl.get("scaling", args.scaling), "vs_baseline": None, "dtype": wl["dtype"],
            "data": "synthetic (seeded, BASELINE config shapes and distributions)", "config": wl["config"],
            "roofline": {"bound": wl["bound"], "achieved": achieved, "peak": peak, "unit": roof_unit,
                         "frac": achieved / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json)"
                         if peak_kind == "measured" else "fallback", "traffic": traffic,
                         "frac_of_nominal_8tbs": achieved / 8000.0 if wl["bound"] == "hbm" else None},
            "clocks": clocks.summary(), "gpu_launches": args.steps * wl["launches_per_step"],
            "gpu_launches_scope": "rank 0, timed region", "step_us": step_stats(per_step_ms)}
    if e2e is not None:
        line["e2e"] = e2e
    if library is not None:
        line["library_comparison"] = library
    if copy_ref is not None:
        line["roofline"]["same_size_copy"] = copy_ref
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(os.cpu_count() or 1)
        full = wl["config"].get("tokens_per_step", wl["config"].get("M"))
        with torch.inference_mode():
            rate, reps, rows = time_cpu(wl["cpu"], full)
        what = "the full step" if rows == full else f"the first {rows} of the step's {full} rows/tokens"
        line["cpu_baseline"] = {"value": rate / wl["scale"], "unit": wl["unit"],
                                "cores": torch.get_num_threads(), "kind": "port",
                                "sample": f"{what} on the host (torch CPU bf16 restatement of the reference), "
                                          f"median of {reps} runs"}
    if rank == 0 and world == 1 and args.workload == "fused8b" and not args.no_decode_step:
        # The headline metric's second half: the decode step per backend, same box, same run.
        # Each backend's worker is a fresh process; this process's tensors are released first.
        wl = None
        flush_w = flush_r = None
        torch.cuda.empty_cache()
        line["decode_step"] = decode_summary(decode_backends(args))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
