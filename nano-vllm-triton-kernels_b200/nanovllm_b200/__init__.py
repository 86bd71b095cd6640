"""nanovllm_b200: B200 (sm_100a) kernels for nano-vllm-triton-kernels' pre-attention hot path.

`nanovllm_b200.kernels` mirrors the reference's `nanovllm.kernels` package (same module names, function names,
arguments and errors); every function runs a hand-written sm_100a kernel from libnvb200.so (include/nvb200.h)
through ctypes. `nanovllm_b200.install()` registers the backend as kernel_backend="b200" in an importable
reference nano-vllm.
"""
from nanovllm_b200._lib import status  # noqa: F401
from nanovllm_b200.install import install  # noqa: F401
from nanovllm_b200.kernels.qk_norm_rope_kv import qk_norm_rope_kv  # noqa: F401
from nanovllm_b200.kernels.rms_norm import fused_add_rms_norm, rms_norm  # noqa: F401
from nanovllm_b200.kernels.matmul import matmul  # noqa: F401
from nanovllm_b200.kernels.swiglu import silu_and_mul  # noqa: F401

__all__ = ["qk_norm_rope_kv", "rms_norm", "fused_add_rms_norm", "silu_and_mul", "matmul", "status", "install"]
