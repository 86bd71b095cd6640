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
def test_struct_layout_matches_header(tmp_path):
    fields = [f[0] for f in _lib.QkNormRopeKvArgs._fields_]
    src = tmp_path / "layout.c"
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(nvb200_qk_norm_rope_kv_args, {f}));' for f in fields)
    src.write_text('#include <stddef.h>\n#include <stdio.h>\n#include "nvb200.h"\nint main(void) {\n' + body +
                   '\n  printf("sizeof %zu\\n", sizeof(nvb200_qk_norm_rope_kv_args));\n  return 0;\n}\n')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for f in fields:
        assert int(out[f]) == getattr(_lib.QkNormRopeKvArgs, f).offset, f
    assert int(out["sizeof"]) == ctypes.sizeof(_lib.QkNormRopeKvArgs)
