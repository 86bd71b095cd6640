"""Writes tests/golden/golden.pt: outputs of the reference's own torch code on small seeded inputs.

    python tests/golden/make_golden.py [--reference PATH]   (PATH: a checkout of R3pere/nano-vllm-triton-kernels)

It imports the reference's layer modules (nanovllm/layers/layernorm.py RMSNorm, rotary_embedding.py
RotaryEmbedding, activation.py SiluAndMul), runs them eagerly on CPU (torch.compiler.set_stance("force_eager"),
as the reference's tests do, tests/test_kernels_norm_act.py:69-71), and saves inputs and outputs. The reference is
only needed to regenerate the fixtures; tests read the saved file. Before writing, it checks the oracle
(oracle/reference_math.py) against the reference at the Qwen3-0.6B fused-op size of T = 2048 tokens and prints
the result.

The KV-cache write (store_kvcache_kernel, nanovllm/layers/attention.py:11-31) is a Triton kernel that cannot run on
CPU; its expected placement is pinned by the reference's own property tests instead (written rows equal the rotated
k / raw v, every other row untouched), which the GPU tests apply.
"""
import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import reference_math as om  # noqa: E402

EPS = 1e-6


def eager(fn, *args):
    with torch.compiler.set_stance("force_eager"):
        return fn(*args)


def make_norm(RMSNorm, n, g):
    norm = RMSNorm(n, eps=EPS).to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(n, generator=g))
    return norm


def randn(shape, g):
    return torch.randn(shape, generator=g).to(torch.bfloat16)


def qkv_views(qkv, hq, hkv, d):
    q, k, v = qkv.split([hq * d, hkv * d, hkv * d], dim=-1)
    return q.view(-1, hq, d), k.view(-1, hkv, d), v.view(-1, hkv, d)


def generate(ref_root: str) -> dict:
    sys.path.insert(0, ref_root)
    from nanovllm.layers.activation import SiluAndMul
    from nanovllm.layers.layernorm import RMSNorm
    from nanovllm.layers.rotary_embedding import RotaryEmbedding

    torch.set_grad_enabled(False)
    out = {"eps": EPS}
    g = torch.Generator().manual_seed(1234)

    # RMSNorm: [rows, n] for the q/k head size and the hidden size.
    for rows, n in ((7, 128), (5, 1024), (3, 200)):
        norm = make_norm(RMSNorm, n, g)
        x = randn((rows, n), g)
        out[f"rms_{rows}x{n}"] = dict(x=x, w=norm.weight.detach().clone(), y=eager(norm, x))

    # RMSNorm on the strided q view of a qkv_proj output (Qwen3-0.6B: 16 q, 8 kv heads of 128).
    norm = make_norm(RMSNorm, 128, g)
    qkv = randn((5, 32 * 128), g)
    q, _, _ = qkv_views(qkv, 16, 8, 128)
    out["rms_qview"] = dict(qkv=qkv, w=norm.weight.detach().clone(), y=eager(norm, q))

    # Add+RMSNorm: both outputs.
    for rows, n in ((7, 1024), (4, 128)):
        norm = make_norm(RMSNorm, n, g)
        x, r = randn((rows, n), g), randn((rows, n), g)
        y, s = eager(norm, x, r)
        out[f"add_rms_{rows}x{n}"] = dict(x=x, r=r, w=norm.weight.detach().clone(), y=y, s=s)

    # RoPE tables: rows at sampled positions (the full tables are large), for the two (max_pos, theta) in use.
    for max_pos in (4096, 40960):
        rope = RotaryEmbedding(128, 128, max_pos, 1e6)
        pos = torch.cat([torch.tensor([0, 1, max_pos - 1]), torch.randint(0, max_pos, (13,), generator=g)])
        out[f"rope_table_{max_pos}"] = dict(positions=pos, rows=rope.cos_sin_cache[pos].clone())

    # Fused composition (q_norm, k_norm, rotary) on strided views, Qwen3-0.6B and -8B head counts.
    for name, hq, hkv, T in (("fused_06b", 16, 8, 7), ("fused_8b", 32, 8, 5)):
        q_norm, k_norm = make_norm(RMSNorm, 128, g), make_norm(RMSNorm, 128, g)
        rope = RotaryEmbedding(128, 128, 4096, 1e6)
        qkv = randn((T, (hq + 2 * hkv) * 128), g)
        q, k, v = qkv_views(qkv, hq, hkv, 128)
        positions = torch.randint(0, 4096, (T,), generator=g)
        qr, kr = eager(rope, positions, eager(q_norm, q), eager(k_norm, k))
        out[name] = dict(hq=hq, hkv=hkv, qkv=qkv, positions=positions, q_w=q_norm.weight.detach().clone(),
                         k_w=k_norm.weight.detach().clone(), q_out=qr.contiguous(), k_out=kr.contiguous())

    # SiLU x Mul at the Qwen3-0.6B intermediate size.
    act = SiluAndMul()
    x = randn((3, 2 * 3072), g)
    out["silu_3x3072"] = dict(x=x, y=eager(act, x))
    return out


def check_oracle_full_size(ref_root: str) -> None:
    """Oracle vs the reference at BASELINE config 1 (T = 2048, Qwen3-0.6B attention shape): bitwise."""
    sys.path.insert(0, ref_root)
    from nanovllm.layers.layernorm import RMSNorm
    from nanovllm.layers.rotary_embedding import RotaryEmbedding

    torch.set_grad_enabled(False)
    g = torch.Generator().manual_seed(0)
    q_norm, k_norm = make_norm(RMSNorm, 128, g), make_norm(RMSNorm, 128, g)
    rope = RotaryEmbedding(128, 128, 4096, 1e6)
    qkv = torch.randn(2048, 4096, generator=g).to(torch.bfloat16)
    q, k, v = qkv_views(qkv, 16, 8, 128)
    positions = torch.randint(0, 4096, (2048,), generator=g)
    qr, kr = eager(rope, positions, eager(q_norm, q), eager(k_norm, k))
    table = om.rope_cos_sin_cache(128, 4096, 1e6)
    assert torch.equal(table, rope.cos_sin_cache), "rope table differs"
    kc = torch.zeros(64 * 256, 8, 128, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(16384, generator=g)[:2048].to(torch.int32)
    slots[torch.randperm(2048, generator=g)[:102]] = -1
    oq, ok = om.qk_norm_rope_kv(q, k, v, positions, q_norm.weight, k_norm.weight, EPS, table, kc, vc, slots, True)
    assert torch.equal(oq, qr) and torch.equal(ok, kr), "oracle differs from the reference at T=2048"
    print("oracle == reference (bitwise) at config 1: q_out", tuple(oq.shape), "k_out", tuple(ok.shape))


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    # The reference checkout: $NANOVLLM_REFERENCE, else a checkout named `reference` beside this repository.
    ap.add_argument("--reference",
                    default=os.environ.get("NANOVLLM_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference")))
    args = ap.parse_args()
    check_oracle_full_size(args.reference)
    data = generate(args.reference)
    path = os.path.join(HERE, "golden.pt")
    torch.save(data, path)
    print(f"wrote {path} ({os.path.getsize(path)} bytes, {len(data) - 1} cases)")
