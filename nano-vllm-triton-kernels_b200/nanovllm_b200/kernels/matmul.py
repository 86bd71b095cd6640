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


# Largest batch for which the model's MLP (nanovllm_b200.install(), step 7) runs matmul_silu_and_mul in place of the
# gate_up projection (cuBLAS) followed by the SiLU x Mul kernel. 0: never, as measured on B200 at the Qwen3-0.6B
# decode step (32 rows, weights streamed from HBM): the skinny kernel's gate_up form took 13.7 us per layer against
# 10.4 us for cuBLAS's projection and the SiLU x Mul kernel (ncu launch list), and the step rose from 1657 to 1780 us;
# at K = 1024 the projection alone also runs faster on cuBLAS than the fused tiled kernel for large batches.
FUSED_GATE_UP_MAX_ROWS = 0


def fused_gate_up_applies(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Whether Qwen3MLP under kernel_backend="b200" runs x through matmul_silu_and_mul(x, weight.t())."""
    return (x.dim() == 2 and 0 < x.shape[0] <= FUSED_GATE_UP_MAX_ROWS and x.dtype == weight.dtype == torch.bfloat16
            and weight.dim() == 2 and weight.shape[1] == x.shape[1] and weight.shape[0] % 2 == 0
            and x.stride(1) == 1 and weight.stride(1) == 1)
