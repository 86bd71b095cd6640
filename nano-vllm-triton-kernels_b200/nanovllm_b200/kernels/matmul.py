"""Tiled matmul C = A @ B on B200 (drop-in for nanovllm/kernels/matmul.py).

Same call as the reference's `matmul` (nanovllm/kernels/matmul.py:84-99): A [M, K] @ B [K, N] -> C [M, N] in A's
dtype, fp32 accumulation, B with any strides (e.g. an nn.Linear weight.t()), the same assertions. The work runs in
`nvb200_matmul` (include/nvb200.h): bf16 and tf32 on the tcgen05 tensor cores (TMA-fed shared-memory stages, TMEM
accumulators), fp32 "ieee" as exact fp32 FMA on the CUDA cores.
"""
import torch

from nanovllm_b200 import _lib


def matmul(a: torch.Tensor, b: torch.Tensor, input_precision: str = "ieee") -> torch.Tensor:
    """a [M, K] @ b [K, N] -> [M, N] in a's dtype. input_precision only matters for fp32 inputs:
    "ieee" = true fp32 FMA, "tf32" = tensor cores with tf32-rounded inputs."""
    if not (a.ndim == 2 and b.ndim == 2 and a.shape[1] == b.shape[0]):
        raise AssertionError((a.shape, b.shape))
    if not (a.dtype == b.dtype and a.dtype in (torch.float32, torch.bfloat16)):
        raise AssertionError((a.dtype, b.dtype))
    if input_precision not in ("ieee", "tf32"):
        raise AssertionError(input_precision)
    M, K = a.shape
    N = b.shape[1]
    c = torch.empty((M, N), device=a.device, dtype=a.dtype)
    if M and N:
        code = _lib.DTYPE_CODE[a.dtype]
        tf32 = int(a.dtype == torch.float32 and input_precision == "tf32")
        args = (M, N, K, a.stride(0), a.stride(1), b.stride(0), b.stride(1))
        ws_bytes = _lib.lib().nvb200_matmul_workspace_size(*args, code)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=a.device) if ws_bytes else None
        _lib.check(_lib.lib().nvb200_matmul(c.data_ptr(), a.data_ptr(), b.data_ptr(), *args, c.stride(0), c.stride(1),
                                            code, tf32, _lib.ptr(ws), ws_bytes,
                                            _lib.status_word(a.device).data_ptr(), _lib.stream_of(a)),
                   "matmul")
    return c


def matmul_silu_and_mul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """silu_and_mul(matmul(a, b)) for bf16 a [M, K] and b [K, 2 N] ([gate | up] columns, e.g. a merged gate_up
    weight.t()), -> [M, N] bf16, in one kernel (`nvb200_matmul_silu_and_mul`) that never writes the [M, 2 N]
    intermediate. Bitwise equal to the two-step form, which it runs instead for layouts the fused kernel does not
    take (and for K = 0)."""
    if not (a.ndim == 2 and b.ndim == 2 and a.shape[1] == b.shape[0] and b.shape[1] % 2 == 0):
        raise AssertionError((a.shape, b.shape))
    if not (a.dtype == b.dtype == torch.bfloat16):
        raise AssertionError((a.dtype, b.dtype))
    M, K = a.shape
    N = b.shape[1] // 2
    out = torch.empty((M, N), device=a.device, dtype=a.dtype)
    if M and N:
        rc = _lib.lib().nvb200_matmul_silu_and_mul(out.data_ptr(), a.data_ptr(), b.data_ptr(), M, N, K, a.stride(0),
                                                   a.stride(1), b.stride(0), b.stride(1), out.stride(0),
                                                   _lib.status_word(a.device).data_ptr(), _lib.stream_of(a))
        if rc == _lib.ERR_UNSUPPORTED:
            from nanovllm_b200.kernels.swiglu import silu_and_mul
            return silu_and_mul(matmul(a, b))
        _lib.check(rc, "matmul_silu_and_mul")
    return out


def linear_decode(x: torch.Tensor, weight: torch.Tensor, swiglu: bool = False) -> torch.Tensor | None:
    """x [M, K] @ weight[N, K].t() -> [M, N] bf16 for decode-sized batches (`nvb200_linear_decode`): the weight is a
    model parameter (no kernel in flight writes it), so its loads may overlap the preceding kernel. swiglu: weight
    holds [gate; up] rows (2 N) and the result is silu(x gate^T) * (x up^T), [M, N]. None when the kernel does not
    take the shape or layout (the caller then runs its own path)."""
    if not (x.dim() == 2 and weight.dim() == 2 and x.shape[1] == weight.shape[1]):
        raise AssertionError((x.shape, weight.shape))
    if not (x.dtype == weight.dtype == torch.bfloat16):
        raise AssertionError((x.dtype, weight.dtype))
    if x.stride(1) != 1 or weight.stride(1) != 1 or (swiglu and weight.shape[0] % 2):
        return None
    M, K = x.shape
    N = weight.shape[0] // 2 if swiglu else weight.shape[0]
    y = torch.empty((M, N), device=x.device, dtype=x.dtype)
    if M == 0 or N == 0:
        return y
    rc = _lib.lib().nvb200_linear_decode(y.data_ptr(), x.data_ptr(), weight.data_ptr(), M, N, K, x.stride(0),
                                         weight.stride(0), y.stride(0), int(swiglu),
                                         _lib.status_word(x.device).data_ptr(), _lib.stream_of(x))
    if rc == _lib.ERR_UNSUPPORTED:
        return None
    _lib.check(rc, "linear_decode")
    return y


# Which of a b200 model's linear layers run `linear_decode` (nanovllm_b200.install(), steps 7 and 8) instead of
# cuBLAS, as measured on B200 by `bench.py --workload projections` (each projection after this library's RMSNorm,
# weights rotating over more than the L2, one CUDA graph; us per norm + projection):
#   Qwen3-0.6B, 32 rows: o_proj 1024 x 2048      7.01 (cuBLAS  8.04)   down_proj 1024 x 3072    7.52 (cuBLAS  9.23)
#                        gate_up + SiLU x Mul    7.43 (cuBLAS + the SiLU x Mul kernel 9.28)
#                        qkv_proj 4096 x 1024    cuBLAS 6.15; the weight-streaming kernel measured slower at this shape
#   Qwen3-0.6B, 1 row:   o_proj 5.38 (9.91), down_proj 6.01 (11.87), gate_up + SiLU x Mul 6.32 (8.67)
#   Qwen3-8B, 32 rows:   o_proj 4096 x 4096 12.26 (11.73), down_proj 4096 x 12288 25.97 (25.23), gate_up 44.6 (42.6)
# so plain projections go through it when N <= K and the weight is at most 16 MB (the o and down projections of the
# small model), the gate_up projection with its SiLU x Mul when its weight is at most 32 MB; batches of at most 32
# rows (at 64 rows cuBLAS was as fast or faster).
DECODE_GEMM_MAX_ROWS = 32
DECODE_GEMM_MAX_WEIGHT_BYTES = 16 << 20
FUSED_GATE_UP_MAX_ROWS = 32
FUSED_GATE_UP_MAX_WEIGHT_BYTES = 32 << 20


def decode_gemm_applies(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether a linear layer of a b200 model runs x @ weight.t() through `linear_decode`."""
    return (x.dim() == 2 and 0 < x.shape[0] <= DECODE_GEMM_MAX_ROWS and weight.dim() == 2
            and x.dtype == weight.dtype == torch.bfloat16 and weight.shape[1] == x.shape[1]
            and weight.shape[0] <= weight.shape[1]
            and weight.numel() * weight.element_size() <= DECODE_GEMM_MAX_WEIGHT_BYTES)


def fused_gate_up_applies(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether Qwen3MLP under kernel_backend="b200" runs its gate_up projection and SiLU x Mul as
    linear_decode(x, weight, swiglu=True)."""
    return (x.dim() == 2 and 0 < x.shape[0] <= FUSED_GATE_UP_MAX_ROWS and x.dtype == weight.dtype == torch.bfloat16
            and weight.dim() == 2 and weight.shape[1] == x.shape[1] and weight.shape[0] % 2 == 0
            and weight.numel() * weight.element_size() <= FUSED_GATE_UP_MAX_WEIGHT_BYTES)
