"""The C ABI boundary without a GPU: libnvb200.so loads, exports every function include/nvb200.h declares, and the
ctypes mirror of nvb200_qk_norm_rope_kv_args has the C struct's layout (checked against gcc's offsetof)."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

from nanovllm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nvb200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NVB200_API\s+[\w\s\*]*?\b(nvb200_\w+)\s*\(", text)))


def test_header_declares_the_exports():
    assert declared_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing


def test_library_loads_through_the_package():
    lib = _lib.lib()
    assert lib.nvb200_status_string(0) == b"ok"
    assert b"argument" in lib.nvb200_status_string(1)


def test_no_gpu_means_error_not_crash():
    """Without a GPU the entry points return an error code (never touch memory)."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc = _lib.lib().nvb200_rms_norm(None, None, None, 1, 1, 8, 0, 8, 1e-6, _lib.BF16, None, None)
    assert rc == _lib.ERR_ARG  # null pointers are rejected before any CUDA call
    rc = _lib.lib().nvb200_rms_norm(8, 8, 8, 1, 1, 8, 0, 8, 1e-6, _lib.BF16, None, None)
    assert rc == _lib.ERR_NO_DEVICE


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
@pytest.mark.parametrize("ctype,cname", [(_lib.QkNormRopeKvArgs, "nvb200_qk_norm_rope_kv_args"),
                                         (_lib.PagedDecodeArgs, "nvb200_paged_decode_args"),
                                         (_lib.AllreduceGroup, "nvb200_allreduce_group"),
                                         (_lib.LinearQkvArgs, "nvb200_linear_qkv_args")])
def test_struct_layout_matches_header(tmp_path, ctype, cname):
    fields = [f[0] for f in ctype._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof({cname}, {f}));' for f in fields)
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "nvb200.h"\nint main(void) {\n' + body +
                   f'\n  printf("sizeof %zu\\n", sizeof({cname}));\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for f in fields:
        assert int(out[f]) == getattr(ctype, f).offset, f
    assert int(out["sizeof"]) == ctypes.sizeof(ctype)


def test_new_entry_points_reject_bad_arguments_without_a_gpu():
    """Argument checks run before any CUDA call (so they hold on a machine without a GPU too)."""
    lib = _lib.lib()
    # store_kvcache: negative sizes, bad slot width, null pointers with work to do.
    assert lib.nvb200_store_kvcache(8, 0, 8, 0, 8, 8, 8, 4, -1, 16, 4, _lib.BF16, None, None) == _lib.ERR_ARG
    assert lib.nvb200_store_kvcache(8, 0, 8, 0, 8, 8, 8, 2, 1, 16, 4, _lib.BF16, None, None) == _lib.ERR_ARG
    assert lib.nvb200_store_kvcache(None, 0, 8, 0, 8, 8, 8, 4, 1, 16, 4, _lib.BF16, None, None) == _lib.ERR_ARG
    assert lib.nvb200_store_kvcache(None, 0, None, 0, None, None, None, 4, 0, 16, 4, _lib.BF16, None, None) == _lib.OK
    # paged decode attention: a null args pointer, Hq not a multiple of Hkv, an empty batch (no launch).
    assert lib.nvb200_paged_decode_attention(None, None) == _lib.ERR_ARG
    a = _lib.PagedDecodeArgs()
    a.batch, a.queries_per_seq, a.num_q_heads, a.num_kv_heads, a.head_dim = 0, 1, 16, 8, 128
    a.block_size, a.max_blocks_per_seq, a.dtype = 256, 1, _lib.BF16
    assert lib.nvb200_paged_decode_attention(ctypes.byref(a), None) == _lib.OK
    a.num_q_heads = 12
    a.num_kv_heads = 8
    assert lib.nvb200_paged_decode_attention(ctypes.byref(a), None) == _lib.ERR_ARG
    # The split choice: one wave of two CTAs per SM (148 SMs when no GPU answers), at most 8, at least one tile per
    # warp of the longest sequence.
    assert lib.nvb200_paged_decode_splits(32, 8, 4, 256, 0) == 1
    assert lib.nvb200_paged_decode_splits(1, 8, 8, 256, 0) == 8
    assert lib.nvb200_paged_decode_splits(1, 1, 1, 64, 0) == 1
    assert lib.nvb200_paged_decode_splits(4, 4, 64, 256, 3) == 3
    # linear_decode: negative sizes, a swiglu flag other than 0/1, null pointers with work to do; nothing to do.
    assert lib.nvb200_linear_decode(8, 8, 8, -1, 16, 16, 16, 16, 16, 0, None, None) == _lib.ERR_ARG
    assert lib.nvb200_linear_decode(8, 8, 8, 1, 16, 16, 16, 16, 16, 2, None, None) == _lib.ERR_ARG
    assert lib.nvb200_linear_decode(None, 8, 8, 1, 16, 16, 16, 16, 16, 0, None, None) == _lib.ERR_ARG
    assert lib.nvb200_linear_decode(None, None, None, 0, 16, 16, 16, 16, 16, 0, None, None) == _lib.OK
    # linear_qkv_norm_rope_kv: a null args pointer, Hq not a multiple of Hkv, a cache without slots; no tokens.
    assert lib.nvb200_linear_qkv_norm_rope_kv(None, None) == _lib.ERR_ARG
    la = _lib.LinearQkvArgs()
    la.K, la.qknr.num_tokens, la.qknr.num_q_heads, la.qknr.num_kv_heads, la.qknr.head_dim = 1024, 4, 12, 8, 128
    la.qknr.num_positions = 4096
    assert lib.nvb200_linear_qkv_norm_rope_kv(ctypes.byref(la), None) == _lib.ERR_ARG
    la.qknr.num_q_heads, la.qknr.k_cache = 16, 8
    assert lib.nvb200_linear_qkv_norm_rope_kv(ctypes.byref(la), None) == _lib.ERR_ARG
    la.qknr.k_cache, la.qknr.num_tokens = None, 0
    assert lib.nvb200_linear_qkv_norm_rope_kv(ctypes.byref(la), None) == _lib.OK


def test_streamk_entry_points_check_arguments_without_a_gpu():
    """The stream-K decode entry point rejects what the plain one rejects before any CUDA call, takes an empty batch
    without a workspace (no launch), and without a GPU its workspace size is unknown (-1)."""
    import torch
    lib = _lib.lib()
    assert lib.nvb200_paged_decode_attention_streamk(None, None, 0, None) == _lib.ERR_ARG
    a = _lib.PagedDecodeArgs()
    a.batch, a.queries_per_seq, a.num_q_heads, a.num_kv_heads, a.head_dim = 0, 1, 16, 8, 128
    a.block_size, a.max_blocks_per_seq, a.dtype = 256, 1, _lib.BF16
    assert lib.nvb200_paged_decode_attention_streamk(ctypes.byref(a), None, 0, None) == _lib.OK
    a.num_q_heads = 12
    assert lib.nvb200_paged_decode_attention_streamk(ctypes.byref(a), None, 0, None) == _lib.ERR_ARG
    assert lib.nvb200_paged_decode_workspace_size(ctypes.byref(a)) == -1  # Hq not a multiple of Hkv
    if not torch.cuda.is_available():
        a.num_q_heads = 16
        assert lib.nvb200_paged_decode_workspace_size(ctypes.byref(a)) == -1


# The weight-streaming kernel's launch shape (tiles of 8 weight rows per CTA x CTAs splitting K), as calibrated by a
# sweep of every pair on B200 (148 SMs; this machine's library answers with 148 when no GPU is present).
PLANS = [((32, 1024, 2048, 0), (4, 4)),   # Qwen3-0.6B o_proj
         ((32, 1024, 3072, 0), (4, 4)),   # down_proj
         ((32, 3072, 1024, 1), (6, 1)),   # gate_up with SiLU x Mul
         ((32, 4096, 1024, 0), (4, 1)),   # qkv_proj
         ((32, 4096, 4096, 0), (7, 2)),   # Qwen3-8B o_proj
         ((32, 4096, 12288, 0), (7, 2)),  # Qwen3-8B down_proj
         ((1, 1024, 2048, 0), (4, 4)), ((64, 1024, 3072, 0), (4, 4))]


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="the SM count of this machine's GPU differs")
@pytest.mark.parametrize("shape,expected", PLANS)
def test_decode_projection_plan(shape, expected):
    lib = _lib.lib()
    tiles, split = ctypes.c_int32(0), ctypes.c_int32(0)
    assert lib.nvb200_linear_decode_plan(*shape, ctypes.byref(tiles), ctypes.byref(split)) == _lib.OK
    assert (tiles.value, split.value) == expected
    assert lib.nvb200_linear_decode_plan(65, 1024, 1024, 0, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.nvb200_linear_decode_plan(1, 1024, 1024, 2, None, None) == _lib.ERR_ARG
