"""ctypes binding of libnvb200.so, the C ABI declared in include/nvb200.h.

The library is built in-tree (nano-vllm-triton-kernels_b200/build.py) and loaded from this package directory. There
is no fallback: if the library is missing or fails to load, every kernel call raises. A device status word per
CUDA device (int32, zeroed at creation) receives the kernels' NVB200_STATUS_* bits: see `status()`.
"""
import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnvb200.so")

# Return codes and dtype codes of nvb200.h.
OK, ERR_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_NO_DEVICE = 0, 1, 2, 3, 4
BF16, F16, F32 = 0, 1, 2
DTYPE_CODE = {torch.bfloat16: BF16, torch.float16: F16, torch.float32: F32}
STATUS_BAD_POSITION, STATUS_BAD_SLOT, STATUS_WAIT_TIMEOUT = 1, 2, 4
# NVB200_QKNR_KERNEL_* codes of nvb200_qk_norm_rope_kv_plan.
QKNR_KERNELS = {0: "none", 1: "generic", 2: "direct", 3: "multi", 4: "bulk"}

# Every extern "C" function of include/nvb200.h; tests check that the library exports each one.
EXPORTS = ("nvb200_status_string", "nvb200_qk_norm_rope_kv", "nvb200_qk_norm_rope_kv_plan", "nvb200_rms_norm",
           "nvb200_fused_add_rms_norm",
           "nvb200_silu_and_mul", "nvb200_matmul_workspace_size", "nvb200_matmul", "nvb200_matmul_silu_and_mul",
           "nvb200_linear_decode", "nvb200_linear_decode_plan", "nvb200_linear_qkv_norm_rope_kv",
           "nvb200_allreduce_buffer_bytes", "nvb200_allreduce_buffer_create", "nvb200_allreduce_buffer_open",
           "nvb200_allreduce_buffer_close", "nvb200_matmul_allreduce", "nvb200_store_kvcache",
           "nvb200_paged_decode_attention", "nvb200_paged_decode_splits", "nvb200_paged_decode_workspace_size",
           "nvb200_paged_decode_attention_streamk", "nvb200_paged_decode_attention_noalloc")

_vp, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float


class QkNormRopeKvArgs(ctypes.Structure):
    """nvb200_qk_norm_rope_kv_args (field order and types as in nvb200.h)."""
    _fields_ = [
        ("q_out", _vp), ("k_out", _vp), ("q", _vp), ("k", _vp), ("v", _vp),
        ("q_token_stride", _i64), ("k_token_stride", _i64), ("v_token_stride", _i64),
        ("positions", _vp), ("slot_mapping", _vp), ("q_weight", _vp), ("k_weight", _vp),
        ("cos_sin", _vp), ("cos_sin_stride", _i64), ("num_positions", _i64),
        ("k_cache", _vp), ("v_cache", _vp), ("num_slots", _i64),
        ("num_tokens", _i64), ("num_q_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("eps", _f32), ("status", _vp),
    ]


class LinearQkvArgs(ctypes.Structure):
    """nvb200_linear_qkv_args (field order and types as in nvb200.h)."""
    _fields_ = [
        ("x", _vp), ("x_row_stride", _i64), ("qkv_weight", _vp), ("weight_row_stride", _i64), ("K", _i64),
        ("qknr", QkNormRopeKvArgs),
    ]


class PagedDecodeArgs(ctypes.Structure):
    """nvb200_paged_decode_args (field order and types as in nvb200.h)."""
    _fields_ = [
        ("out", _vp), ("q", _vp), ("q_batch_stride", _i64), ("q_token_stride", _i64), ("q_head_stride", _i64),
        ("k_cache", _vp), ("v_cache", _vp), ("cache_block_stride", _i64), ("cache_token_stride", _i64),
        ("cache_head_stride", _i64), ("num_blocks", _i64), ("block_table", _vp), ("block_table_stride", _i64),
        ("seqlens", _vp), ("batch", _i32), ("queries_per_seq", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32),
        ("head_dim", _i32), ("block_size", _i32), ("max_blocks_per_seq", _i32), ("causal", _i32),
        ("num_splits", _i32), ("dtype", _i32), ("softmax_scale", _f32), ("status", _vp),
    ]


class AllreduceGroup(ctypes.Structure):
    """nvb200_allreduce_group (field order and types as in nvb200.h)."""
    _fields_ = [("world", ctypes.c_int), ("rank", ctypes.c_int), ("max_n", _i64), ("buffers", _vp * 8)]


class KernelError(RuntimeError):
    """A kernel entry point returned an error code."""


_lib = None
_lock = threading.Lock()


def _declare(lib):
    lib.nvb200_status_string.argtypes = [ctypes.c_int]
    lib.nvb200_status_string.restype = ctypes.c_char_p
    lib.nvb200_qk_norm_rope_kv.argtypes = [ctypes.POINTER(QkNormRopeKvArgs), _vp]
    lib.nvb200_qk_norm_rope_kv.restype = ctypes.c_int
    lib.nvb200_qk_norm_rope_kv_plan.argtypes = [ctypes.POINTER(QkNormRopeKvArgs), ctypes.POINTER(_i32),
                                                ctypes.POINTER(_i32)]
    lib.nvb200_qk_norm_rope_kv_plan.restype = ctypes.c_int
    lib.nvb200_rms_norm.argtypes = [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, ctypes.c_int, _vp, _vp]
    lib.nvb200_rms_norm.restype = ctypes.c_int
    lib.nvb200_fused_add_rms_norm.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, ctypes.c_int, _vp,
                                              _vp]
    lib.nvb200_fused_add_rms_norm.restype = ctypes.c_int
    lib.nvb200_silu_and_mul.argtypes = [_vp, _vp, _i64, _i64, _i64, ctypes.c_int, _vp, _vp]
    lib.nvb200_silu_and_mul.restype = ctypes.c_int
    lib.nvb200_matmul_workspace_size.argtypes = [_i64] * 7 + [ctypes.c_int]
    lib.nvb200_matmul_workspace_size.restype = _i64
    lib.nvb200_matmul.argtypes = [_vp, _vp, _vp] + [_i64] * 9 + [ctypes.c_int, ctypes.c_int, _vp, _i64, _vp, _vp]
    lib.nvb200_matmul.restype = ctypes.c_int
    lib.nvb200_matmul_silu_and_mul.argtypes = [_vp, _vp, _vp] + [_i64] * 8 + [_vp, _vp]
    lib.nvb200_matmul_silu_and_mul.restype = ctypes.c_int
    lib.nvb200_allreduce_buffer_bytes.argtypes = [_i64]
    lib.nvb200_allreduce_buffer_bytes.restype = _i64
    lib.nvb200_allreduce_buffer_create.argtypes = [_i64, ctypes.POINTER(_vp), _vp]
    lib.nvb200_allreduce_buffer_create.restype = ctypes.c_int
    lib.nvb200_allreduce_buffer_open.argtypes = [_vp, ctypes.POINTER(_vp)]
    lib.nvb200_allreduce_buffer_open.restype = ctypes.c_int
    lib.nvb200_allreduce_buffer_close.argtypes = [_vp, ctypes.c_int]
    lib.nvb200_allreduce_buffer_close.restype = ctypes.c_int
    lib.nvb200_matmul_allreduce.argtypes = [_vp, _vp, _vp] + [_i64] * 8 + [ctypes.POINTER(AllreduceGroup), _vp, _vp]
    lib.nvb200_matmul_allreduce.restype = ctypes.c_int
    lib.nvb200_linear_decode.argtypes = [_vp, _vp, _vp] + [_i64] * 6 + [ctypes.c_int, _vp, _vp]
    lib.nvb200_linear_decode.restype = ctypes.c_int
    lib.nvb200_linear_decode_plan.argtypes = [_i64, _i64, _i64, ctypes.c_int, _vp, _vp]
    lib.nvb200_linear_decode_plan.restype = ctypes.c_int
    lib.nvb200_linear_qkv_norm_rope_kv.argtypes = [ctypes.POINTER(LinearQkvArgs), _vp]
    lib.nvb200_linear_qkv_norm_rope_kv.restype = ctypes.c_int
    lib.nvb200_store_kvcache.argtypes = [_vp, _i64, _vp, _i64, _vp, _vp, _vp, ctypes.c_int, _i64, _i64, _i64,
                                         ctypes.c_int, _vp, _vp]
    lib.nvb200_store_kvcache.restype = ctypes.c_int
    lib.nvb200_paged_decode_attention.argtypes = [ctypes.POINTER(PagedDecodeArgs), _vp]
    lib.nvb200_paged_decode_attention.restype = ctypes.c_int
    lib.nvb200_paged_decode_splits.argtypes = [_i32] * 5
    lib.nvb200_paged_decode_splits.restype = ctypes.c_int
    lib.nvb200_paged_decode_workspace_size.argtypes = [ctypes.POINTER(PagedDecodeArgs)]
    lib.nvb200_paged_decode_workspace_size.restype = _i64
    lib.nvb200_paged_decode_attention_streamk.argtypes = [ctypes.POINTER(PagedDecodeArgs), _vp, _i64, _vp]
    lib.nvb200_paged_decode_attention_streamk.restype = ctypes.c_int
    lib.nvb200_paged_decode_attention_noalloc.argtypes = [ctypes.POINTER(PagedDecodeArgs), _vp]
    lib.nvb200_paged_decode_attention_noalloc.restype = ctypes.c_int


def lib():
    """The loaded library (loaded on first use). Raises if it is missing: there is no other implementation."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"{LIB_PATH} is missing: build it with "
                                      "`python nano-vllm-triton-kernels_b200/build.py`")
                handle = ctypes.CDLL(LIB_PATH)
                _declare(handle)
                _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != OK:
        msg = lib().nvb200_status_string(rc).decode()
        if rc == ERR_ARG:
            raise ValueError(f"{what}: {msg}")
        raise KernelError(f"{what}: {msg} (code {rc})")


def stream_of(t: torch.Tensor) -> int:
    """The current torch stream of t's device (kernels launch there, as Triton's do)."""
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t):
    return None if t is None else t.data_ptr()


_status = {}


def status_word(device: torch.device) -> torch.Tensor:
    """This device's int32 status word. Created (zeroed) on the first kernel call on the device, so make one call
    before capturing a CUDA graph."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _status.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = w
    return w


def status(device=None, clear: bool = False) -> int:
    """Reads (synchronising) the NVB200_STATUS_* bits the kernels set on `device`: 0 = every index was in range and
    every wait ended. clear=True zeroes the word afterwards."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = status_word(dev)
    v = int(w.item())
    if clear:
        w.zero_()
    return v
