"""SiLU-and-multiply on B200 (drop-in for nanovllm/kernels/swiglu.py).

Same call as the reference's `silu_and_mul` (nanovllm/kernels/swiglu.py:34-43): x [rows, 2n] holds [gate | up] in
the last dim and is read in place with any row stride; the output is contiguous [rows, n]. The work runs in
`nvb200_silu_and_mul` (include/nvb200.h) with 16-byte vectors. Numerics as nanovllm/layers/activation.py:15-18 run
eagerly: out = silu(gate.float()).to(dtype) * up.
"""
import torch

from nanovllm_b200 import _lib


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """silu(x[..., :n]) * x[..., n:] for x [..., 2 * n] with a contiguous last dim."""
    if x.dim() != 2 or x.stride(-1) != 1:
        x = x.reshape(-1, x.shape[-1]).contiguous()
    if x.dtype not in _lib.DTYPE_CODE:
        raise AssertionError(f"unsupported dtype {x.dtype}")
    rows, n = x.shape[0], x.shape[1] // 2
    out = torch.empty(rows, n, dtype=x.dtype, device=x.device)
    if rows and n:
        _lib.check(_lib.lib().nvb200_silu_and_mul(out.data_ptr(), x.data_ptr(), rows, n, x.stride(0),
                                                  _lib.DTYPE_CODE[x.dtype], _lib.status_word(x.device).data_ptr(),
                                                  _lib.stream_of(x)),
                   "silu_and_mul")
    return out
