"""RMSNorm and Add+RMSNorm on B200 (drop-in for nanovllm/kernels/rms_norm.py).

Same calls as the reference's `rms_norm` (nanovllm/kernels/rms_norm.py:83-98) and `fused_add_rms_norm` (:101-111):
same view handling (2-D [rows, n] or 3-D [T, H, n] strided views are read in place; anything else is first made a
contiguous [-1, n] copy, :86-87), same assertions, same contiguous outputs. The work runs in `nvb200_rms_norm` /
`nvb200_fused_add_rms_norm` (include/nvb200.h): rows held in registers, 16-byte vector loads, shuffle reductions.
Numerics as nanovllm/layers/layernorm.py:20-44: fp32 statistics, rounding to the dtype before the weight multiply,
and the add variant normalises the unrounded fp32 sum.
"""
import torch

from nanovllm_b200 import _lib


def _dtype_code(x: torch.Tensor, w: torch.Tensor) -> int:
    if x.dtype not in _lib.DTYPE_CODE:
        raise AssertionError(f"unsupported dtype {x.dtype}")
    if w.dtype != x.dtype or w.dim() != 1 or not w.is_contiguous():
        raise AssertionError("w must be a contiguous 1-D tensor of x's dtype")
    return _lib.DTYPE_CODE[x.dtype]


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dim. x: [rows, n] or [T, H, n] with a contiguous last dim (any other strides)."""
    n = x.shape[-1]
    if x.dim() != 3 and x.dim() != 2 or x.stride(-1) != 1:
        x = x.reshape(-1, n).contiguous()
    if x.dim() == 2:
        groups, rows_per_group, group_stride, row_stride = x.shape[0], 1, x.stride(0), 0
    else:
        groups, rows_per_group, group_stride, row_stride = x.shape[0], x.shape[1], x.stride(0), x.stride(1)
    code = _dtype_code(x, w)
    if w.shape[0] != n:
        raise AssertionError("w must have n elements")
    y = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if groups * rows_per_group:
        _lib.check(_lib.lib().nvb200_rms_norm(y.data_ptr(), x.data_ptr(), w.data_ptr(), groups, rows_per_group,
                                              group_stride, row_stride, n, eps, code,
                                              _lib.status_word(x.device).data_ptr(), _lib.stream_of(x)),
                   "rms_norm")
    return y


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor,
                       eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(RMSNorm(x + residual), x + residual), the sum in fp32. x, residual: [rows, n] with a contiguous last dim."""
    if not (x.shape == residual.shape and x.dim() == 2 and x.stride(-1) == 1 and residual.stride(-1) == 1):
        raise AssertionError("x and residual must be [rows, n] with a unit last stride")
    if residual.dtype != x.dtype:
        raise AssertionError("x and residual must have the same dtype")
    rows, n = x.shape
    code = _dtype_code(x, w)
    if w.shape[0] != n:
        raise AssertionError("w must have n elements")
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    s = torch.empty_like(x, memory_format=torch.contiguous_format)
    if rows:
        _lib.check(_lib.lib().nvb200_fused_add_rms_norm(y.data_ptr(), s.data_ptr(), x.data_ptr(), residual.data_ptr(),
                                                        w.data_ptr(), rows, n, x.stride(0), residual.stride(0), eps,
                                                        code, _lib.status_word(x.device).data_ptr(),
                                                        _lib.stream_of(x)),
                   "fused_add_rms_norm")
    return y, s
