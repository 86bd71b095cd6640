"""Parity of nanovllm_b200's rms_norm / fused_add_rms_norm / silu_and_mul with the oracle.

Mirrors the reference's tests/test_kernels_norm_act.py: rows 1/7/128/4097, n 128 (q/k norm) and 1024 (hidden), the
real strided q/k-norm view, both outputs of add_rms_norm, SiLU x Mul at 2 x 3072. Tolerance: within MAX_ULP = 2 bf16
ulps of the oracle (fp32 summation order differs); the new residual has no reduction and must be bitwise equal.
SiLU x Mul must be bitwise equal to the oracle's torch ops run on the GPU (the reference's check) and within 1 ulp
of the CPU oracle (CPU and GPU exp may differ in the last fp32 bit). Plus: fp16 / fp32, wide row strides, rows
longer than the register kernel holds (n = 4096, 8192), unaligned rows, and the BASELINE config-2 sizes.
"""
import pytest
import torch

from nanovllm_b200.kernels.rms_norm import fused_add_rms_norm, rms_norm
from nanovllm_b200.kernels.swiglu import silu_and_mul
from oracle import reference_math as om

pytestmark = pytest.mark.gpu

MAX_ULP = 2
ROWS = [1, 7, 128, 4097]
EPS = 1e-6


def cpu(t):
    return t.detach().cpu()


def ulps(a, b):
    return int(om.bf16_ulp_diff(cpu(a), cpu(b)).max()) if a.numel() else 0


def make(dev, shape, seed, dtype=torch.bfloat16):
    g = torch.Generator(device=dev).manual_seed(seed)
    return torch.randn(shape, device=dev, generator=g).to(dtype)


def weight(dev, n, seed, dtype=torch.bfloat16):
    g = torch.Generator(device=dev).manual_seed(seed + 99)
    return (1 + 0.1 * torch.randn(n, device=dev, generator=g)).to(dtype)


@pytest.mark.parametrize("n", [128, 1024])
@pytest.mark.parametrize("rows", ROWS)
def test_rms_norm(cuda, rows, n):
    x, w = make(cuda, (rows, n), rows * 7 + n), weight(cuda, n, rows)
    y = rms_norm(x, w, EPS)
    assert y.shape == x.shape and y.is_contiguous()
    assert ulps(y, om.rms_forward(cpu(x), cpu(w), EPS)) <= MAX_ULP


@pytest.mark.parametrize("tokens", ROWS)
def test_qk_norm_strided_view(cuda, tokens):
    qkv = make(cuda, (tokens, 32 * 128), tokens * 3 + 1)
    q, k, _ = qkv.split([16 * 128, 8 * 128, 8 * 128], dim=-1)
    w = weight(cuda, 128, tokens)
    for t in (q.view(-1, 16, 128), k.view(-1, 8, 128)):
        y = rms_norm(t, w, EPS)
        assert y.shape == t.shape and y.is_contiguous()
        assert ulps(y, om.rms_forward(cpu(t), cpu(w), EPS)) <= MAX_ULP


@pytest.mark.parametrize("n", [128, 1024])
@pytest.mark.parametrize("rows", ROWS)
def test_add_rms_norm(cuda, rows, n):
    x, r, w = make(cuda, (rows, n), rows * 5 + n), make(cuda, (rows, n), rows * 5 + n + 1), weight(cuda, n, rows)
    y, s = fused_add_rms_norm(x, r, w, EPS)
    ry, rs = om.add_rms_forward(cpu(x), cpu(r), cpu(w), EPS)
    assert ulps(y, ry) <= MAX_ULP
    assert torch.equal(cpu(s), rs)


@pytest.mark.parametrize("rows", ROWS)
def test_silu_and_mul(cuda, rows):
    x = make(cuda, (rows, 2 * 3072), rows)
    out = silu_and_mul(x)
    assert out.shape == (rows, 3072) and out.is_contiguous()
    assert torch.equal(out, om.silu_and_mul(x))  # oracle's torch ops on the GPU: bitwise
    assert ulps(out, om.silu_and_mul(cpu(x))) <= 1


def _same_bits(a, b):
    """Bit-for-bit equality of two bf16 tensors, any NaN matching any NaN."""
    return bool(((a.view(torch.int16) == b.view(torch.int16)) | (torch.isnan(a) & torch.isnan(b))).all())


def test_silu_every_bf16_gate(cuda):
    # silu(g) rounded to bf16 depends only on the 16-bit gate value, so running all 65,536 bit patterns (zeros,
    # subnormals, infinities and NaNs included) as gates covers every input the kernel can see. Up = 1 isolates the
    # rounded silu; the second pass multiplies by up values that include subnormals, signed zeros and non-finite
    # values.
    gate = torch.arange(-32768, 32768, dtype=torch.int32, device=cuda).to(torch.int16).view(torch.bfloat16)
    gate = gate.view(64, 1024)
    ones = torch.ones_like(gate)
    out = silu_and_mul(torch.cat([gate, ones], dim=1))
    assert _same_bits(out, om.silu_and_mul(torch.cat([gate, ones], dim=1)))
    g = torch.Generator(device=cuda).manual_seed(11)
    up = torch.randn(64, 1024, device=cuda, generator=g).to(torch.bfloat16)
    special = torch.tensor([0.0, -0.0, 1e-40, -1e-40, 9.2e-41, float("inf"), float("-inf"), float("nan"), 3e38,
                            -3e38, 1.2e-38, 65504.0], device=cuda).to(torch.bfloat16)
    up.view(-1)[: special.numel() * 512] = special.repeat(512)
    x = torch.cat([gate, up], dim=1)
    assert _same_bits(silu_and_mul(x), om.silu_and_mul(x))


# ---------------------------------------------------------------------------------------------------------------
# Large bf16 batches: long rows run the bulk-copy RMSNorm (units of one or more rows, a ragged last unit, dense or
# strided rows), the rest the register kernels; the same properties as above must hold for both.

@pytest.mark.parametrize("rows", [2048, 4099, 9001])
@pytest.mark.parametrize("n", [128, 1024, 4096, 6144])
@pytest.mark.parametrize("strided", [False, True])
def test_row_engine_norms(cuda, rows, n, strided):
    pad = 64 if strided else 0
    xw = make(cuda, (rows, n + pad), rows + n)
    rw = make(cuda, (rows, n + 2 * pad), rows + n + 1)
    x, r = xw[:, pad:pad + n], rw[:, :n]
    w = weight(cuda, n, rows)
    assert ulps(rms_norm(x, w, EPS), om.rms_forward(x, w, EPS)) <= MAX_ULP
    y, s = fused_add_rms_norm(x, r, w, EPS)
    ry, rs = om.add_rms_forward(x, r, w, EPS)
    assert ulps(y, ry) <= MAX_ULP and torch.equal(s, rs)
    assert om.bf16_ulp_diff(cpu(y), cpu(ry)).float().mean() < 0.05  # almost all elements bitwise
    assert _lib_status(cuda) == 0


@pytest.mark.parametrize("rows", [2048, 4099, 9001])
@pytest.mark.parametrize("n", [64, 1536, 3072, 8192])
@pytest.mark.parametrize("strided", [False, True])
def test_row_engine_silu(cuda, rows, n, strided):
    buf = make(cuda, (rows, 2 * n + (128 if strided else 0)), rows * 3 + n)
    x = buf[:, 64:64 + 2 * n] if strided else buf
    out = silu_and_mul(x)
    assert out.shape == (rows, n) and out.is_contiguous()
    assert torch.equal(out, om.silu_and_mul(x))
    assert _lib_status(cuda) == 0


def _lib_status(dev):
    from nanovllm_b200 import _lib
    return _lib.status(dev, clear=True)


# ---------------------------------------------------------------------------------------------------------------
# Config 2 (hidden 1024, gate_up [T, 6144] read as strided column views) at T in {1, 32, 2048, 8192}.

@pytest.mark.parametrize("T", [1, 32, 2048, 8192])
def test_config2_strided_views(cuda, T):
    wide = make(cuda, (T, 1024 + 256), T)
    x = wide[:, 128:128 + 1024]  # row stride 1280 > n: a column view
    res = make(cuda, (T, 1024), T + 1)
    w = weight(cuda, 1024, T)
    assert ulps(rms_norm(x, w, EPS), om.rms_forward(x, w, EPS)) <= MAX_ULP
    y, s = fused_add_rms_norm(x, res, w, EPS)
    ry, rs = om.add_rms_forward(x, res, w, EPS)
    assert ulps(y, ry) <= MAX_ULP and torch.equal(s, rs)
    buf = make(cuda, (T, 6144 + 512), T + 2)
    gate_up = buf[:, 256:256 + 6144]  # non-contiguous rows
    out = silu_and_mul(gate_up)
    assert torch.equal(out, om.silu_and_mul(gate_up))


# ---------------------------------------------------------------------------------------------------------------
# Other dtypes and shapes.

@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_other_dtypes(cuda, dtype):
    x, r, w = make(cuda, (333, 1024), 1, dtype), make(cuda, (333, 1024), 2, dtype), weight(cuda, 1024, 3, dtype)
    tol = dict(rtol=1e-2, atol=1e-2) if dtype == torch.float16 else dict(rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(rms_norm(x, w, EPS), om.rms_forward(x, w, EPS), **tol)
    y, s = fused_add_rms_norm(x, r, w, EPS)
    ry, rs = om.add_rms_forward(x, r, w, EPS)
    torch.testing.assert_close(y, ry, **tol)
    assert torch.equal(s, rs)
    g = make(cuda, (333, 2 * 1000), 4, dtype)
    torch.testing.assert_close(silu_and_mul(g), om.silu_and_mul(g), **tol)


@pytest.mark.parametrize("n", [4096, 8192, 100, 1000, 24])
def test_long_and_odd_rows(cuda, n):
    """n = 4096 / 8192 exceed the register kernel (one CTA per row); odd n disables the 16-byte vector path."""
    x, r, w = make(cuda, (65, n), n), make(cuda, (65, n), n + 1), weight(cuda, n, n)
    assert ulps(rms_norm(x, w, EPS), om.rms_forward(cpu(x), cpu(w), EPS)) <= MAX_ULP
    y, s = fused_add_rms_norm(x, r, w, EPS)
    ry, rs = om.add_rms_forward(cpu(x), cpu(r), cpu(w), EPS)
    assert ulps(y, ry) <= MAX_ULP and torch.equal(cpu(s), rs)
    g = make(cuda, (65, 2 * n), n + 2)
    assert torch.equal(silu_and_mul(g), om.silu_and_mul(g))


def test_unaligned_rows(cuda):
    base = make(cuda, (50, 1024 + 1), 9)
    x = base[:, 1:]  # 2-byte offset: scalar path
    w = weight(cuda, 1024, 9)
    assert ulps(rms_norm(x, w, EPS), om.rms_forward(cpu(x), cpu(w), EPS)) <= MAX_ULP
    g = make(cuda, (50, 2 * 512 + 1), 10)[:, 1:]
    assert torch.equal(silu_and_mul(g), om.silu_and_mul(g))


def test_reference_fallbacks(cuda):
    """Inputs the reference first copies to a contiguous [-1, n] (rms_norm.py:86-87, swiglu.py:37-38)."""
    x = make(cuda, (4, 6, 256), 11)
    w = weight(cuda, 256, 11)
    xt = x.transpose(0, 1)  # 3-D but non-unit... still unit last stride: read in place
    assert ulps(rms_norm(xt, w, EPS), om.rms_forward(cpu(xt), cpu(w), EPS)) <= MAX_ULP
    x4 = make(cuda, (2, 3, 4, 256), 12)
    y4 = rms_norm(x4, w, EPS)
    assert y4.shape == (24, 256)
    assert ulps(y4, om.rms_forward(cpu(x4).reshape(-1, 256), cpu(w), EPS)) <= MAX_ULP
    g3 = make(cuda, (3, 5, 64), 13)
    assert silu_and_mul(g3).shape == (15, 32)


def test_zero_rows(cuda):
    w = weight(cuda, 128, 0)
    assert rms_norm(torch.empty(0, 128, device=cuda, dtype=torch.bfloat16), w, EPS).shape == (0, 128)
    y, s = fused_add_rms_norm(torch.empty(0, 128, device=cuda, dtype=torch.bfloat16),
                              torch.empty(0, 128, device=cuda, dtype=torch.bfloat16), w, EPS)
    assert y.shape == s.shape == (0, 128)
    assert silu_and_mul(torch.empty(0, 256, device=cuda, dtype=torch.bfloat16)).shape == (0, 128)
