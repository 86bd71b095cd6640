"""Parity of nanovllm_b200's fused q/k RMSNorm + RoPE + paged KV write (nvb200_qk_norm_rope_kv) with the oracle.

Mirrors the reference's tests/test_kernels_qk_rope_kv.py (same sizes, seeds style, slot pattern and checks):
  norm stage   kernel run with an identity rotation table (cos = 1, sin = 0, all positions 0): its outputs are its
               normed q and k; within MAX_ULP = 2 bf16 ulps of the oracle's RMSNorm (the sum-of-squares order
               differs from torch's; the reference's own bound).
  rope stage   the kernel's real output equals, bitwise, the oracle's rotary applied to the kernel's own normed q/k.
  KV write     cache rows at kept slots equal k_out / v bitwise; every other row is untouched (slot -1 skipped).
  end to end   within rtol 1.6e-2, atol 1e-2 of an all-fp32 computation (the north-star's bf16 tolerance).
The oracle runs on CPU for these sizes; the full-size (T = 8192, Qwen3-8B) cases check the same properties with
the oracle's torch ops run on the GPU.
"""
import pytest
import torch

from nanovllm_b200 import _lib, workloads
from nanovllm_b200.kernels.qk_norm_rope_kv import qk_norm_rope_kv
from oracle import reference_math as om

pytestmark = pytest.mark.gpu

MAX_ULP = 2
TOKENS = [1, 7, 128, 4097]
EPS = 1e-6
D, MAX_POS, THETA, BLOCK = 128, 40960, 1e6, 256
SHAPES = {"qwen3-0.6b": (16, 8), "qwen3-8b": (32, 8), "tp4-0.6b": (4, 2), "tp8-0.6b": (2, 1)}

_tables = {}


def table(dev, max_pos=MAX_POS):
    key = (dev, max_pos)
    if key not in _tables:
        _tables[key] = om.rope_cos_sin_cache(D, max_pos, THETA).to(dev)
    return _tables[key]


def make_inputs(dev, tokens, random_positions, hq=16, hkv=8, seed_extra=0):
    """The reference test's inputs (tests/test_kernels_qk_rope_kv.py:74-93): strided q/k/v views of a qkv output,
    random or arange positions, distinct random slots of a 2T-slot cache with every 5th token -1, random cache."""
    g = torch.Generator(device=dev).manual_seed(tokens * 2 + random_positions + 1000 * seed_extra)
    q_w = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).to(torch.bfloat16)
    k_w = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).to(torch.bfloat16)
    qkv = torch.randn(tokens, (hq + 2 * hkv) * D, device=dev, generator=g).to(torch.bfloat16)
    q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
    q, k, v = q.view(-1, hq, D), k.view(-1, hkv, D), v.view(-1, hkv, D)
    if random_positions:
        positions = torch.randint(0, MAX_POS, (tokens,), device=dev, generator=g)
    else:
        positions = torch.arange(tokens, device=dev)
    num_blocks = (2 * tokens + BLOCK - 1) // BLOCK
    slots = torch.randperm(num_blocks * BLOCK, device=dev, generator=g)[:tokens].to(torch.int32)
    slots[4::5] = -1
    cache = torch.randn(2, num_blocks, BLOCK, hkv, D, device=dev, generator=g).to(torch.bfloat16)
    return dict(q_w=q_w, k_w=k_w, q=q, k=k, v=v, positions=positions, slots=slots, cache=cache, hkv=hkv)


def identity_table(dev):
    return torch.cat([torch.ones(D // 2), torch.zeros(D // 2)]).view(1, 1, D).to(dev)


def run_fused(x, identity_rope=False, write_k=True):
    cache = x["cache"].clone()
    positions, cos_sin = x["positions"], table(x["q"].device)
    if identity_rope:
        positions = torch.zeros_like(positions)
        cos_sin = identity_table(x["q"].device)
    q_out, k_out = qk_norm_rope_kv(x["q"], x["k"], x["v"], positions, x["q_w"], x["k_w"], EPS, cos_sin, cache[0],
                                   cache[1], x["slots"], write_k=write_k)
    return dict(q=q_out, k_out=k_out, k_cache=cache[0], v_cache=cache[1])


def cpu(t):
    return t.detach().cpu()


CASES = [(t, rp) for t in TOKENS for rp in (True, False)]
IDS = [f"tokens={t}-{'random' if rp else 'arange'}" for t, rp in CASES]


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("tokens,random_positions", CASES, ids=IDS)
def test_norm_stage(cuda, shape, tokens, random_positions):
    hq, hkv = SHAPES[shape]
    x = make_inputs(cuda, tokens, random_positions, hq, hkv)
    normed = run_fused(x, identity_rope=True)
    for name, out, w, inp in (("q", normed["q"], x["q_w"], x["q"]), ("k", normed["k_out"], x["k_w"], x["k"])):
        ref = om.rms_forward(cpu(inp), cpu(w), EPS)
        worst = int(om.bf16_ulp_diff(cpu(out), ref).max())
        assert worst <= MAX_ULP, f"{name} norm: {worst} bf16 ulps from the oracle"


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("tokens,random_positions", CASES, ids=IDS)
def test_rope_stage_bitwise(cuda, shape, tokens, random_positions):
    hq, hkv = SHAPES[shape]
    x = make_inputs(cuda, tokens, random_positions, hq, hkv)
    normed, out = run_fused(x, identity_rope=True), run_fused(x)
    qr, kr = om.rotary(cpu(x["positions"]), cpu(normed["q"]), cpu(normed["k_out"]), cpu(table(cuda)))
    assert torch.equal(cpu(out["q"]), qr)
    assert torch.equal(cpu(out["k_out"]), kr)


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("tokens,random_positions", CASES, ids=IDS)
def test_kv_write(cuda, shape, tokens, random_positions):
    hq, hkv = SHAPES[shape]
    x = make_inputs(cuda, tokens, random_positions, hq, hkv)
    out = run_fused(x)
    check_kv_write(x, out, hkv)


def check_kv_write(x, out, hkv):
    slots = x["slots"]
    real = slots >= 0
    rows = slots[real].long()
    assert torch.equal(out["k_cache"].view(-1, hkv, D)[rows], out["k_out"][real])
    assert torch.equal(out["v_cache"].view(-1, hkv, D)[rows], x["v"][real])
    untouched = torch.ones(x["cache"].shape[1] * BLOCK, dtype=torch.bool, device=slots.device)
    untouched[rows] = False
    for i, name in enumerate(("k_cache", "v_cache")):
        before = x["cache"][i].view(-1, hkv, D)[untouched]
        assert torch.equal(out[name].view(-1, hkv, D)[untouched], before), name


def fp32_reference(x, positions, cos_sin):
    """Everything in fp32 (no intermediate bf16 rounding): the north-star's tolerance reference."""
    def norm(t, w):
        t = t.float()
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + EPS) * w.float()
    cs = cos_sin[positions].view(-1, 1, D)
    cos, sin = cs[..., :D // 2], cs[..., D // 2:]

    def rot(t):
        t1, t2 = t[..., :D // 2], t[..., D // 2:]
        return torch.cat((t1 * cos - t2 * sin, t2 * cos + t1 * sin), -1)
    return rot(norm(x["q"], x["q_w"])), rot(norm(x["k"], x["k_w"]))


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("tokens", [7, 4097])
def test_end_to_end_within_bf16_tolerance(cuda, shape, tokens):
    """Values within rtol 1.6e-2 / atol 1e-2 of the oracle (the reference's implementation), and no further from an
    all-fp32 computation than the oracle itself is. The reference rounds the normed head to bf16 before RoPE
    (layers/layernorm.py:29), which alone moves a near-cancelling RoPE output by up to ~0.02 from the all-fp32
    value; against fp32 the kernel must do as well as the oracle: no more elements outside the tolerance (x2 for
    rounding-boundary noise) and a largest deviation within 1.5x of the oracle's."""
    hq, hkv = SHAPES[shape]
    x = make_inputs(cuda, tokens, True, hq, hkv)
    out = run_fused(x)
    oq, ok = om.qk_norm_rope_kv(cpu(x["q"]), cpu(x["k"]), cpu(x["v"]), cpu(x["positions"]), cpu(x["q_w"]),
                                cpu(x["k_w"]), EPS, cpu(table(cuda)), torch.empty(0), torch.empty(0), None, True)
    torch.testing.assert_close(cpu(out["q"]).float(), oq.float(), rtol=1.6e-2, atol=1e-2)
    torch.testing.assert_close(cpu(out["k_out"]).float(), ok.float(), rtol=1.6e-2, atol=1e-2)
    rq, rk = fp32_reference(x, x["positions"], table(cuda))
    for got, ora, ref in ((out["q"], oq, rq), (out["k_out"], ok, rk)):
        got, ora, ref = cpu(got).float(), ora.float(), cpu(ref)
        bad_got = ((got - ref).abs() > 1e-2 + 1.6e-2 * ref.abs()).float().mean().item()
        bad_ora = ((ora - ref).abs() > 1e-2 + 1.6e-2 * ref.abs()).float().mean().item()
        assert bad_got <= 2 * bad_ora + 1e-5, (bad_got, bad_ora)
        assert (got - ref).abs().max() <= 1.5 * (ora - ref).abs().max() + 1e-3


@pytest.mark.parametrize("case", ["fused_06b", "fused_8b"])
def test_golden_fixture(cuda, case):
    """Kernel on the fixture inputs vs the reference's own outputs (tests/golden/golden.pt)."""
    import os
    g = torch.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.pt"))
    c = g[case]
    hq, hkv = c["hq"], c["hkv"]
    qkv = c["qkv"].to(cuda)
    q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
    q, k, v = q.view(-1, hq, D), k.view(-1, hkv, D), v.view(-1, hkv, D)
    empty = torch.empty(0, device=cuda, dtype=torch.bfloat16)
    q_out, k_out = qk_norm_rope_kv(q, k, v, c["positions"].to(cuda), c["q_w"].to(cuda), c["k_w"].to(cuda), g["eps"],
                                   table(cuda, 4096), empty, empty, None, True)
    for got, ref in ((q_out, c["q_out"]), (k_out, c["k_out"])):
        torch.testing.assert_close(cpu(got).float(), ref.float(), rtol=1.6e-2, atol=1e-2)
        assert (om.bf16_ulp_diff(cpu(got), ref) == 0).float().mean() > 0.9


# ---------------------------------------------------------------------------------------------------------------
# Variants of the call: no cache, no k_out, T = 0, other head sizes, layouts that take the generic kernel.

def test_empty_cache_stores_nothing(cuda):
    x = make_inputs(cuda, 33, True)
    empty = torch.empty(0, device=cuda, dtype=torch.bfloat16)
    q_out, k_out = qk_norm_rope_kv(x["q"], x["k"], x["v"], x["positions"], x["q_w"], x["k_w"], EPS, table(cuda),
                                   empty, empty, None, write_k=True)
    ref_q, ref_k = om.qk_norm_rope_kv(cpu(x["q"]), cpu(x["k"]), cpu(x["v"]), cpu(x["positions"]), cpu(x["q_w"]),
                                      cpu(x["k_w"]), EPS, cpu(table(cuda)), torch.empty(0), torch.empty(0), None,
                                      True)
    torch.testing.assert_close(cpu(q_out).float(), ref_q.float(), rtol=1.6e-2, atol=1e-2)
    torch.testing.assert_close(cpu(k_out).float(), ref_k.float(), rtol=1.6e-2, atol=1e-2)


def test_without_k_out(cuda):
    x = make_inputs(cuda, 64, True)
    a = run_fused(x, write_k=True)
    b = run_fused(x, write_k=False)
    assert b["k_out"] is None
    assert torch.equal(a["q"], b["q"]) and torch.equal(a["k_cache"], b["k_cache"])
    assert torch.equal(a["v_cache"], b["v_cache"])


def test_zero_tokens(cuda):
    x = make_inputs(cuda, 1, True)
    q = x["q"][:0]
    q_out, k_out = qk_norm_rope_kv(q, x["k"][:0], x["v"][:0], x["positions"][:0], x["q_w"], x["k_w"], EPS,
                                   table(cuda), x["cache"][0], x["cache"][1], x["slots"][:0], True)
    assert q_out.shape == (0, 16, D) and k_out.shape == (0, 8, D)


@pytest.mark.parametrize("head_dim", [64, 256, 96])
def test_other_head_dims(cuda, head_dim):
    """D = 64 and 256 take the bulk kernel with 4 / 16 lanes per head; D = 96 the generic kernel."""
    g = torch.Generator(device=cuda).manual_seed(head_dim)
    T, hq, hkv = 37, 8, 2
    qkv = torch.randn(T, (hq + 2 * hkv) * head_dim, device=cuda, generator=g).to(torch.bfloat16)
    q, k, v = qkv.split([hq * head_dim, hkv * head_dim, hkv * head_dim], dim=-1)
    q, k, v = q.view(T, hq, head_dim), k.view(T, hkv, head_dim), v.view(T, hkv, head_dim)
    w = (1 + 0.1 * torch.randn(2, head_dim, device=cuda, generator=g)).to(torch.bfloat16)
    tab = om.rope_cos_sin_cache(head_dim, 512, 1e4).to(cuda)
    pos = torch.randint(0, 512, (T,), device=cuda, generator=g)
    kc = torch.randn(1, 128, hkv, head_dim, device=cuda, generator=g).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    slots = torch.randperm(128, device=cuda, generator=g)[:T].to(torch.int32)
    slots[::3] = -1
    kc2, vc2 = kc.clone(), vc.clone()
    q_out, k_out = qk_norm_rope_kv(q, k, v, pos, w[0].contiguous(), w[1].contiguous(), EPS, tab, kc, vc, slots, True)
    rq, rk = om.qk_norm_rope_kv(cpu(q), cpu(k), cpu(v), cpu(pos), cpu(w[0]), cpu(w[1]), EPS, cpu(tab), kc2.cpu(),
                                vc2.cpu(), cpu(slots), True)
    torch.testing.assert_close(cpu(q_out).float(), rq.float(), rtol=1.6e-2, atol=1e-2)
    torch.testing.assert_close(cpu(k_out).float(), rk.float(), rtol=1.6e-2, atol=1e-2)
    keep = slots >= 0
    assert torch.equal(kc.view(-1, hkv, head_dim)[slots[keep].long()], k_out[keep])
    assert torch.equal(vc.view(-1, hkv, head_dim)[slots[keep].long()], v[keep])


def test_unaligned_token_stride_takes_generic_kernel(cuda):
    """A qkv buffer whose row stride is not a multiple of 8 elements cannot be moved by the bulk engine; the
    generic kernel must give the same bits as the bulk kernel's math allows (norm within 2 ulp, rope bitwise)."""
    T, hq, hkv = 50, 16, 8
    g = torch.Generator(device=cuda).manual_seed(7)
    wide = torch.randn(T, (hq + 2 * hkv) * D + 3, device=cuda, generator=g).to(torch.bfloat16)
    qkv = wide[:, 3:]
    q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
    x = make_inputs(cuda, T, True)
    x.update(q=q.view(T, hq, D), k=k.view(T, hkv, D), v=v.view(T, hkv, D))
    normed, out = run_fused(x, identity_rope=True), run_fused(x)
    for name, o, w, inp in (("q", normed["q"], x["q_w"], x["q"]), ("k", normed["k_out"], x["k_w"], x["k"])):
        assert int(om.bf16_ulp_diff(cpu(o), om.rms_forward(cpu(inp), cpu(w), EPS)).max()) <= MAX_ULP, name
    qr, kr = om.rotary(cpu(x["positions"]), cpu(normed["q"]), cpu(normed["k_out"]), cpu(table(cuda)))
    assert torch.equal(cpu(out["q"]), qr) and torch.equal(cpu(out["k_out"]), kr)
    check_kv_write(x, out, hkv)


def test_out_of_range_indices_are_flagged_not_written(cuda):
    """Slots past the cache and positions past the table are skipped (no fault) and reported in the status word."""
    x = make_inputs(cuda, 16, True)
    _lib.status(cuda, clear=True)
    n_slots = x["cache"].shape[1] * BLOCK
    bad = x["slots"].clone()
    bad[3] = n_slots + 5  # past the end: must not be written
    x2 = dict(x, slots=bad)
    out = run_fused(x2)
    assert _lib.status(cuda, clear=True) & _lib.STATUS_BAD_SLOT
    ref = run_fused(dict(x, slots=torch.where(torch.arange(16, device=cuda) == 3, -1, x["slots"])))
    assert torch.equal(out["k_cache"], ref["k_cache"]) and torch.equal(out["v_cache"], ref["v_cache"])
    pos = x["positions"].clone()
    pos[0] = MAX_POS + 1
    run_fused(dict(x, positions=pos))
    assert _lib.status(cuda, clear=True) & _lib.STATUS_BAD_POSITION
    run_fused(x)
    assert _lib.status(cuda) == 0


# ---------------------------------------------------------------------------------------------------------------
# Full size (BASELINE config 3 at T = 8192, Qwen3-8B: 32 q / 8 kv heads, cache [1024, 256, 8, 128]): properties.

@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_full_size_properties(cuda, world):
    x = workloads.fused_inputs(8192, 32, 8, max_pos=32768, num_blocks=1024, device=cuda, seed=3,
                               cache_fill="randn")
    xs = workloads.shard_kv_heads(x, world - 1, world)  # the last rank's shard
    hkv = xs["k"].shape[1]
    cache = torch.stack([xs["k_cache"], xs["v_cache"]])
    before = cache.clone()
    q_out, k_out = qk_norm_rope_kv(xs["q"], xs["k"], xs["v"], xs["positions"], xs["q_w"], xs["k_w"], xs["eps"],
                                   xs["cos_sin"], cache[0], cache[1], xs["slots"], True)
    ident = identity_table(cuda)
    nq, nk = qk_norm_rope_kv(xs["q"], xs["k"], xs["v"], torch.zeros_like(xs["positions"]), xs["q_w"], xs["k_w"],
                             xs["eps"], ident, torch.empty(0, device=cuda), torch.empty(0, device=cuda), None, True)
    # norm stage vs the oracle's RMSNorm (torch ops on the GPU at this size)
    assert int(om.bf16_ulp_diff(nq, om.rms_forward(xs["q"], xs["q_w"], xs["eps"])).max()) <= MAX_ULP
    assert int(om.bf16_ulp_diff(nk, om.rms_forward(xs["k"], xs["k_w"], xs["eps"])).max()) <= MAX_ULP
    # rope stage bitwise
    rq, rk = om.rotary(xs["positions"], nq, nk, xs["cos_sin"])
    assert torch.equal(q_out, rq) and torch.equal(k_out, rk)
    # exact slot placement and untouched slots
    check_kv_write(dict(xs, cache=before), dict(k_cache=cache[0], v_cache=cache[1], k_out=k_out), hkv)


# ---------------------------------------------------------------------------------------------------------------
# Tensor-parallel ranks' own qkv_proj outputs (BASELINE config 3 sharded by KV head at 4 and 8 GPUs). A rank's
# QKVParallelLinear writes [T, (Hq/w + 2 Hkv/w) D] with its q | k | v heads consecutive in each row
# (nanovllm/layers/linear.py:106-128): the layout that routes 1-2 kv heads per rank to the multi-token kernel
# (units of 4 or 8 consecutive tokens moved by one bulk copy). Same checks as the full-size test above, and the
# route itself is asserted through nvb200_qk_norm_rope_kv_plan.

from nanovllm_b200 import parallel  # noqa: E402
from nanovllm_b200.kernels.qk_norm_rope_kv import kernel_plan  # noqa: E402


def rank_inputs(dev, T, world, rank, seed=11):
    """Rank `rank`'s inputs at the Qwen3-8B shape: its own contiguous qkv_proj output (cut from a full one with the
    column split QKVParallelLinear makes), its cache slice [1024, 256, 8 / world, 128] (random), replicated
    positions (uniform in [0, 32768)) and slots (distinct, 5 % -1)."""
    hq, hkv = 32, 8
    g = torch.Generator(device=dev).manual_seed(seed + T)
    full = torch.randn(T, (hq + 2 * hkv) * D, device=dev, generator=g).to(torch.bfloat16)
    qkv = parallel.shard_qkv_columns(full, hq, hkv, D, rank, world)
    del full
    rq, rkv = hq // world, hkv // world
    q, k, v = qkv.split([rq * D, rkv * D, rkv * D], dim=-1)
    q, k, v = q.view(T, rq, D), k.view(T, rkv, D), v.view(T, rkv, D)
    q_w = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).to(torch.bfloat16)
    k_w = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).to(torch.bfloat16)
    positions = torch.randint(0, 32768, (T,), device=dev, generator=g)
    blocks = 1024
    slots = torch.randperm(blocks * BLOCK, device=dev, generator=g)[:T].to(torch.int32)
    slots[torch.randperm(T, device=dev, generator=g)[:round(0.05 * T)]] = -1
    cache = torch.randn(2, blocks, BLOCK, rkv, D, device=dev, generator=g).to(torch.bfloat16)
    return dict(q=q, k=k, v=v, q_w=q_w, k_w=k_w, positions=positions, slots=slots, cache=cache, eps=1e-6,
                cos_sin=table(dev, 32768), hkv=rkv)


# (world, T): the multi-token route needs ceil(T / B) >= 2 x SMs units (B = 4 at 4 ranks, 8 at 8 ranks); T = 1024
# is below that and runs a one-token-per-unit kernel (checked for parity all the same); 8193 leaves a last unit of
# one token, 8190 one of 2 (B = 4) / 6 (B = 8) tokens.
MULTI_CASES = [(w, t) for w in (4, 8) for t in (1024, 8192, 8193, 8190)]


@pytest.mark.parametrize("write_k", [True, False], ids=["k_out", "no_k_out"])
@pytest.mark.parametrize("store", [True, False], ids=["cache", "no_cache"])
@pytest.mark.parametrize("world,tokens", MULTI_CASES, ids=[f"tp{w}-T{t}" for w, t in MULTI_CASES])
def test_rank_qkv_layout_multi_token_kernel(cuda, world, tokens, store, write_k):
    x = rank_inputs(cuda, tokens, world, world - 1)
    hkv = x["hkv"]
    cache = x["cache"].clone()
    empty = torch.empty(0, device=cuda, dtype=torch.bfloat16)
    kc, vc = (cache[0], cache[1]) if store else (empty, empty)
    slots = x["slots"] if store else None
    args = (x["q"], x["k"], x["v"], x["positions"], x["q_w"], x["k_w"], x["eps"], x["cos_sin"], kc, vc, slots,
            write_k)
    route, tpu = kernel_plan(*args)
    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    B = 4 if world == 4 else 8
    if (tokens + B - 1) // B >= 2 * sms:
        assert (route, tpu) == ("multi", B), (route, tpu)
    else:  # the one-token-per-unit kernels: direct for batches of up to 40 MB of q/k/v rows, else bulk
        assert route in ("direct", "bulk"), route
    _lib.status(cuda, clear=True)
    q_out, k_out = qk_norm_rope_kv(*args)
    # The normed heads: the same layout through an identity rotation (cos 1, sin 0 at position 0), k_out on.
    ident = identity_table(cuda)
    nargs = (x["q"], x["k"], x["v"], torch.zeros_like(x["positions"]), x["q_w"], x["k_w"], x["eps"], ident, empty,
             empty, None, True)
    assert kernel_plan(*nargs)[0] == route
    nq, nk = qk_norm_rope_kv(*nargs)
    assert int(om.bf16_ulp_diff(nq, om.rms_forward(x["q"], x["q_w"], x["eps"])).max()) <= MAX_ULP
    assert int(om.bf16_ulp_diff(nk, om.rms_forward(x["k"], x["k_w"], x["eps"])).max()) <= MAX_ULP
    rq, rk = om.rotary(x["positions"], nq, nk, x["cos_sin"])
    assert torch.equal(q_out, rq)
    if write_k:
        assert torch.equal(k_out, rk)
    else:
        assert k_out is None
    if store:
        check_kv_write(dict(x, cache=x["cache"]), dict(k_cache=cache[0], v_cache=cache[1], k_out=rk), hkv)
    else:
        assert torch.equal(cache, x["cache"])
    assert _lib.status(cuda) == 0


# The decode qkv projection with this op as its epilogue (nvb200_linear_qkv_norm_rope_kv): against qkv = the fp64
# product rounded to bf16, then this op. The projection accumulates in fp32, so a few qkv elements round one bf16
# step away from the fp64 product's rounding, and the norm and rotation carry that on: within the bf16 tolerance, and
# bitwise on almost every element; cache rows outside the batch's slots (and slot -1 rows) untouched.
LINEAR_QKV = [(hq, hkv, M, K) for (hq, hkv) in SHAPES.values() for M, K in ((1, 1024), (7, 1024), (32, 1024))] + \
             [(32, 8, 32, 4096), (16, 8, 16, 2048), (4, 2, 32, 4096)]


@pytest.mark.parametrize("hq,hkv,M,K", LINEAR_QKV)
def test_linear_qkv_epilogue(cuda, hq, hkv, M, K):
    from nanovllm_b200.kernels.qk_norm_rope_kv import linear_qkv_norm_rope_kv
    x = make_inputs(cuda, M, True, hq=hq, hkv=hkv, seed_extra=K)
    g = torch.Generator(device=cuda).manual_seed(M * 31 + K + hq)
    a = (torch.randn(M, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    w = torch.randn((hq + 2 * hkv) * D, K, device=cuda, generator=g).to(torch.bfloat16)
    qkv = om.matmul(a, w.t()).to(torch.bfloat16)
    q, k, v = qkv.split([hq * D, hkv * D, hkv * D], dim=-1)
    cache_ref = x["cache"].clone()
    q_ref, _ = qk_norm_rope_kv(q.reshape(M, hq, D), k.reshape(M, hkv, D), v.reshape(M, hkv, D), x["positions"],
                               x["q_w"], x["k_w"], EPS, table(cuda), cache_ref[0], cache_ref[1], x["slots"],
                               write_k=False)
    cache = x["cache"].clone()
    _lib.status(cuda, clear=True)
    q_out = linear_qkv_norm_rope_kv(a, w, hq, hkv, x["positions"], x["q_w"], x["k_w"], EPS, table(cuda), cache[0],
                                    cache[1], x["slots"])
    assert q_out is not None and q_out.shape == (M, hq, D)
    assert _lib.status(cuda, clear=True) == 0
    for got, ref in ((q_out, q_ref), (cache[0], cache_ref[0]), (cache[1], cache_ref[1])):
        torch.testing.assert_close(cpu(got).float(), cpu(ref).float(), rtol=1.6e-2, atol=1e-2)
        assert (om.bf16_ulp_diff(cpu(got), cpu(ref)) == 0).float().mean() > 0.97
    # rows of the cache that no kept slot names are exactly as they were
    kept = x["slots"][x["slots"] >= 0].long()
    untouched = torch.ones(cache[0].numel() // (hkv * D), dtype=torch.bool, device=cuda)
    untouched[kept] = False
    for c, before in ((cache[0], x["cache"][0]), (cache[1], x["cache"][1])):
        assert torch.equal(c.view(-1, hkv, D)[untouched], before.view(-1, hkv, D)[untouched])


def test_linear_qkv_declines_what_it_does_not_take(cuda):
    from nanovllm_b200.kernels.qk_norm_rope_kv import linear_qkv_norm_rope_kv
    x = make_inputs(cuda, 33, True)
    a = torch.randn(33, 1024, device=cuda).to(torch.bfloat16)
    w = torch.randn(32 * D, 1024, device=cuda).to(torch.bfloat16)
    cache = x["cache"].clone()
    assert linear_qkv_norm_rope_kv(a, w, 16, 8, x["positions"], x["q_w"], x["k_w"], EPS, table(cuda), cache[0],
                                   cache[1], x["slots"]) is None  # more than 32 rows
    assert torch.equal(cache, x["cache"])
