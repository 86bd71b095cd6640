"""Parity of nanovllm_b200's matmul (nvb200_matmul) with the oracle: the float64 product of the inputs.

Mirrors the reference's tests/test_kernels_matmul.py (same shapes, tolerances, seeds and the ieee != tf32 guard):
  fp32 "ieee": rtol 1e-4, atol 1e-4 * sqrt(K);  fp32 "tf32": rtol 1e-2, atol 1e-2 * sqrt(K);
  bf16:        rtol 1.6e-2, atol 1e-2 * sqrt(K).
Plus the north-star's rtol 1e-3 for fp32/tf32: tf32 against the float64 product of the tf32-rounded inputs (the
products the tensor cores form), and the BASELINE config-4 shapes (M in {32, 2048, 4096}, B = weight.t()).
"""
import math

import pytest
import torch

from nanovllm_b200.kernels.matmul import matmul
from oracle import reference_math as om

pytestmark = pytest.mark.gpu

DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16}
PRECISIONS = [("fp32", "ieee"), ("fp32", "tf32"), ("bf16", "ieee")]
SHAPES = [(1, 1024, 4096), (1, 3072, 1024), (7, 33, 65), (17, 129, 257), (100, 300, 70), (127, 255, 1000),
          (512, 512, 512), (1000, 1000, 1000), (3, 5, 2)]


def check(dev, M, N, K, dtype, prec, b_transposed):
    torch.manual_seed(0)
    a = torch.randn(M, K, device=dev, dtype=DTYPES[dtype])
    if b_transposed:  # nn.Linear layout: weight [N, K], matmul uses weight.t()
        b = torch.randn(N, K, device=dev, dtype=DTYPES[dtype]).t()
    else:
        b = torch.randn(K, N, device=dev, dtype=DTYPES[dtype])
    c = matmul(a, b, input_precision=prec)
    assert c.shape == (M, N) and c.dtype == a.dtype
    rtol, atol = om.matmul_tolerance(dtype, prec, K)
    torch.testing.assert_close(c.double(), om.matmul(a, b), rtol=rtol, atol=atol)
    return a, b, c


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("dtype,prec", PRECISIONS)
@pytest.mark.parametrize("b_transposed", [False, True])
def test_matmul(cuda, M, N, K, dtype, prec, b_transposed):
    check(cuda, M, N, K, dtype, prec, b_transposed)


def test_ieee_is_not_tf32(cuda):
    torch.manual_seed(0)
    a = torch.randn(256, 4096, device=cuda)
    b = torch.randn(4096, 256, device=cuda)
    ref = om.matmul(a, b)
    err_ieee = (matmul(a, b, "ieee").double() - ref).abs().max().item()
    err_tf32 = (matmul(a, b, "tf32").double() - ref).abs().max().item()
    assert err_ieee < 1e-2 < err_tf32, (err_ieee, err_tf32)


# A [M, K], B = randn(N, K).t() / sqrt(K)-scaled values.
CONFIG4 = [(M, K, N) for M in (32, 2048, 4096) for K, N in ((1024, 4096), (1024, 6144), (3072, 1024), (4096, 4096))]


@pytest.mark.parametrize("M,K,N", CONFIG4)
@pytest.mark.parametrize("dtype,prec", PRECISIONS)
def test_config4(cuda, M, K, N, dtype, prec):
    g = torch.Generator(device=cuda).manual_seed(M + K + N)
    s = 1 / math.sqrt(K)
    a = (torch.randn(M, K, device=cuda, generator=g) * s).to(DTYPES[dtype])
    b = (torch.randn(N, K, device=cuda, generator=g) * s).to(DTYPES[dtype]).t()
    c = matmul(a, b, prec)
    ref = om.matmul(a, b)
    scale = ref.abs().max().item()
    if dtype == "bf16":
        torch.testing.assert_close(c.double(), ref, rtol=1.6e-2, atol=1e-2 * scale)
    elif prec == "ieee":
        torch.testing.assert_close(c.double(), ref, rtol=1e-3, atol=1e-5 * scale)
    else:
        # tf32 products are exact in fp32 accumulation terms; compare with the fp64 product of tf32 operands
        ref_tf32 = om.matmul(om.tf32_round(a), om.tf32_round(b))
        torch.testing.assert_close(c.double(), ref_tf32, rtol=1e-3, atol=1e-4 * scale)


def test_zero_k(cuda):
    a = torch.randn(5, 0, device=cuda)
    b = torch.randn(0, 7, device=cuda)
    assert torch.equal(matmul(a, b), torch.zeros(5, 7, device=cuda))


def test_strided_operands(cuda):
    """Both operands non-contiguous in both dims (every other row/column of a bigger buffer)."""
    torch.manual_seed(1)
    A = torch.randn(130, 2 * 96, device=cuda, dtype=torch.bfloat16)
    B = torch.randn(2 * 96, 3 * 70, device=cuda, dtype=torch.bfloat16)
    a, b = A[::2, ::2], B[::2, ::3]
    c = matmul(a, b)
    rtol, atol = om.matmul_tolerance("bf16", "ieee", 96)
    torch.testing.assert_close(c.double(), om.matmul(a, b), rtol=rtol, atol=atol)


# Decode-sized rows (M <= 64) with A row-major and B = weight.t(): bf16 runs the weight-streaming kernel (column
# slices of 8-64 weight rows per CTA, 1-4 16-row tiles of A, 128-element K chunks with K tails and N tails); tf32
# runs the swap-AB kernel that splits K over a cluster of up to 8 CTAs and sums their partials through distributed
# shared memory (every M padding, K splits of 1-8 with ragged shares and K tails, N tails).
SKINNY = [(1, 4096, 1024), (7, 1000, 104), (16, 128, 64), (32, 4096, 1024), (32, 6144, 1024), (32, 1024, 3072),
          (33, 4096, 4096), (48, 3000, 1000), (64, 256, 8192), (64, 151936 // 16, 1024)]


@pytest.mark.parametrize("M,N,K", SKINNY)
@pytest.mark.parametrize("dtype,prec", [("bf16", "ieee"), ("fp32", "tf32")])
def test_skinny(cuda, M, N, K, dtype, prec):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + K)
    s = 1 / math.sqrt(K)
    a = (torch.randn(M, K, device=cuda, generator=g) * s).to(DTYPES[dtype])
    b = (torch.randn(N, K, device=cuda, generator=g) * s).to(DTYPES[dtype]).t()
    c = matmul(a, b, prec)
    assert c.shape == (M, N)
    ref = om.matmul(a, b) if dtype == "bf16" else om.matmul(om.tf32_round(a), om.tf32_round(b))
    scale = ref.abs().max().item()
    tol = dict(rtol=1.6e-2, atol=1e-2 * scale) if dtype == "bf16" else dict(rtol=1e-3, atol=1e-4 * scale)
    torch.testing.assert_close(c.double(), ref, **tol)
    from nanovllm_b200 import _lib
    assert _lib.status(cuda, clear=True) == 0


# Weight-streaming kernel: 16/32/64 padded rows, slices of 32-64 columns (odd tile counts included: 56 columns at
# 32 x 4096 x 4096), K splits over clusters of 1, 2, 4 and 8 CTAs, a K below one 64-element box (the chunk's second
# box entirely past K), a K tail inside each box, one column of output, N tails, more CTAs than SMs.
STREAM = [(1, 1, 64), (5, 300, 40), (16, 1184, 200), (17, 2368, 520), (31, 4736, 1000), (64, 7000, 136),
          (2, 9472, 1024), (40, 152, 2056), (64, 1024, 3072), (1, 151936, 1024), (32, 4096, 4096), (24, 900, 12288)]


@pytest.mark.parametrize("M,N,K", STREAM)
def test_stream(cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(M * 11 + N + K)
    a = (torch.randn(M, K, device=cuda, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    b = torch.randn(N, K, device=cuda, generator=g).to(torch.bfloat16).t()
    c = matmul(a, b)
    ref = om.matmul(a, b)
    scale = ref.abs().max().item()
    torch.testing.assert_close(c.double(), ref, rtol=1.6e-2, atol=1e-2 * scale)
    from nanovllm_b200 import _lib
    assert _lib.status(cuda, clear=True) == 0


# linear_decode: the weight-streaming kernel launched so that its weight loads overlap the preceding kernel (which
# lets it start early); its A rows are the preceding kernel's output and must be read only after that kernel ends.
# Every split of K over a cluster (1, 2, 4, 8 CTAs) and slice width the plan picks for these shapes, plain and
# gate_up forms, each call preceded by an RMSNorm that writes its input.
LINEAR_DECODE = [(32, 4096, 1024), (32, 1024, 2048), (32, 1024, 3072), (1, 4096, 1024), (64, 4096, 1024),
                 (64, 1024, 3072), (3, 40, 1024), (20, 56, 4096), (48, 100, 2000), (17, 2368, 520), (9, 24, 1024)]


@pytest.mark.parametrize("M,N,K", LINEAR_DECODE)
@pytest.mark.parametrize("swiglu", [False, True])
def test_linear_decode_after_the_kernel_that_writes_its_input(cuda, M, N, K, swiglu):
    from nanovllm_b200 import _lib
    from nanovllm_b200.kernels.matmul import linear_decode
    from nanovllm_b200.kernels.rms_norm import rms_norm
    g = torch.Generator(device=cuda).manual_seed(M + 3 * N + K)
    w = torch.randn(2 * N if swiglu else N, K, device=cuda, generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device=cuda, generator=g)).to(torch.bfloat16)
    xs = [torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16) for _ in range(4)]
    outs = []
    for x in xs:  # back to back on one stream: each norm's output feeds the next projection at once
        y = linear_decode(rms_norm(x, nw, 1e-6), w, swiglu=swiglu)
        assert y is not None and y.shape == (M, N)
        outs.append(y)
    for x, y in zip(xs, outs):
        xn = om.rms_forward(x, nw, 1e-6)
        ref = om.matmul(xn, w.t())
        if swiglu:
            ref = om.silu_and_mul(ref.to(torch.bfloat16)).double()
        scale = ref.abs().max().item()
        torch.testing.assert_close(y.double(), ref, rtol=1.6e-2, atol=1e-2 * scale)
    assert _lib.status(cuda, clear=True) == 0


def test_linear_decode_in_a_graph(cuda):
    """Captured as the decode step captures it (norm, projection, norm, projection ...), replayed with new inputs."""
    from nanovllm_b200.kernels.matmul import linear_decode
    from nanovllm_b200.kernels.rms_norm import rms_norm
    g = torch.Generator(device=cuda).manual_seed(21)
    M, K = 32, 1024
    ws = [torch.randn(n, K, device=cuda, generator=g).to(torch.bfloat16) for n in (4096, 2048, 6144, 1024)]
    nw = torch.ones(K, device=cuda, dtype=torch.bfloat16)
    x = torch.zeros(M, K, device=cuda, dtype=torch.bfloat16)
    swig = [False, False, True, False]

    def step():
        return [linear_decode(rms_norm(x, nw, 1e-6), w, swiglu=s) for w, s in zip(ws, swig)]
    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = step()
    for trial in range(3):
        x.copy_(torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        xn = om.rms_forward(x, nw, 1e-6)
        for w, s, y in zip(ws, swig, outs):
            ref = om.matmul(xn, w.t())
            if s:
                ref = om.silu_and_mul(ref.to(torch.bfloat16)).double()
            scale = ref.abs().max().item()
            torch.testing.assert_close(y.double(), ref, rtol=1.6e-2, atol=1e-2 * scale)


def test_linear_decode_declines_what_it_does_not_take(cuda):
    from nanovllm_b200.kernels.matmul import linear_decode
    w = torch.randn(256, 512, device=cuda).to(torch.bfloat16)
    assert linear_decode(torch.randn(65, 512, device=cuda).to(torch.bfloat16), w) is None  # more than 64 rows
    assert linear_decode(torch.randn(512, 8, device=cuda).to(torch.bfloat16).t(), w) is None  # A not K-major
    assert linear_decode(torch.randn(8, 512, device=cuda).to(torch.bfloat16), w[:255],
                         swiglu=True) is None  # an odd number of [gate; up] rows


def test_kernels_keep_their_own_shared_memory_limits(cuda):
    """Each kernel raises its own dynamic shared-memory limit: the large tiled kernels first, then the decode-sized
    kernels, in a fresh process (the limits are set once per process and kernel)."""
    import subprocess
    import sys
    code = """
import math, torch
from nanovllm_b200.kernels.matmul import matmul
from oracle import reference_math as om
dev = torch.device("cuda:0")
g = torch.Generator(device=dev).manual_seed(5)
for dtype, prec, M, N, K in [(torch.float32, "tf32", 4096, 4096, 4096), (torch.bfloat16, "ieee", 4096, 4096, 4096),
                             (torch.float32, "tf32", 32, 4096, 4096), (torch.bfloat16, "ieee", 32, 4096, 4096),
                             (torch.float32, "tf32", 64, 2048, 3072), (torch.bfloat16, "ieee", 64, 2048, 3072)]:
    a = (torch.randn(M, K, device=dev, generator=g) / math.sqrt(K)).to(dtype)
    b = torch.randn(N, K, device=dev, generator=g).to(dtype).t()
    c = matmul(a, b, prec)
    ref = om.matmul(om.tf32_round(a), om.tf32_round(b)) if dtype == torch.float32 else om.matmul(a, b)
    scale = ref.abs().max().item()
    torch.testing.assert_close(c.double(), ref, rtol=2e-2, atol=2e-2 * scale)
print("ok")
"""
    import os
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=600,
                         env={**os.environ, "PYTHONPATH": os.pathsep.join(
                             [root, os.path.join(root, "nano-vllm-triton-kernels_b200"),
                              os.environ.get("PYTHONPATH", "")])})
    assert out.returncode == 0 and out.stdout.strip().endswith("ok"), out.stdout[-2000:] + out.stderr[-2000:]


def test_skinny_row_view(cuda):
    """A as every other row of a wider buffer (row pitch > K) with M = 32."""
    g = torch.Generator(device=cuda).manual_seed(3)
    A = torch.randn(64, 1024 + 64, device=cuda, generator=g).to(torch.bfloat16)
    a = A[::2, 32:32 + 1024]
    b = torch.randn(2048, 1024, device=cuda, generator=g).to(torch.bfloat16).t()
    c = matmul(a, b)
    rtol, atol = om.matmul_tolerance("bf16", "ieee", 1024)
    torch.testing.assert_close(c.double(), om.matmul(a, b), rtol=rtol, atol=atol)


# gate_up GEMM with the SiLU x Mul epilogue: B = [gate | up] columns, out = silu(gate) * up without the [M, 2N]
# intermediate. Against the two-step form through this library (the same tensor-core accumulation, so bitwise
# where both run the tiled kernels, M > 64; the skinny kernel sums in another order) and against the oracle (fp64 product rounded to bf16, then the torch
# SiLU x Mul) within bf16 tolerance.
GATE_UP = [(100, 3072, 1024), (300, 1000, 104), (2048, 3072, 1024), (4096, 3072, 1024), (1000, 128, 256),
           (257, 200, 512), (32, 3072, 1024), (7, 384, 64),
           # decode-sized rows (the skinny kernel's gate_up form): one row, ragged N, K splits 1-8, 64 rows
           (1, 3072, 1024), (16, 200, 512), (33, 1000, 4096), (64, 1536, 1024), (32, 12288, 4096), (48, 96, 2048)]


@pytest.mark.parametrize("M,N,K", GATE_UP)
@pytest.mark.parametrize("b_transposed", [True, False])
def test_matmul_silu_and_mul(cuda, M, N, K, b_transposed):
    from nanovllm_b200.kernels.matmul import matmul_silu_and_mul
    from nanovllm_b200.kernels.swiglu import silu_and_mul
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    a = (torch.randn(M, K, device=cuda, generator=g) / math.sqrt(K)).to(torch.bfloat16)
    if b_transposed:
        b = torch.randn(2 * N, K, device=cuda, generator=g).to(torch.bfloat16).t()
    else:
        b = torch.randn(K, 2 * N, device=cuda, generator=g).to(torch.bfloat16)
    out = matmul_silu_and_mul(a, b)
    assert out.shape == (M, N) and out.dtype == torch.bfloat16
    two_step = silu_and_mul(matmul(a, b))
    ref = om.silu_and_mul(om.matmul(a, b).to(torch.bfloat16)).double()
    scale = ref.abs().max().item()
    if M > 64:
        assert torch.equal(out, two_step)
    else:  # the two-step GEMM is the skinny kernel here: another fp32 summation order
        torch.testing.assert_close(out.double(), two_step.double(), rtol=1.6e-2, atol=1e-2 * scale)
    torch.testing.assert_close(out.double(), ref, rtol=1.6e-2, atol=1e-2 * scale)
    from nanovllm_b200 import _lib
    assert _lib.status(cuda, clear=True) == 0
