"""The C ABI library loads on a CPU-only host and exports every entry point
declared in include/xq4.h (no compute calls here)."""
import ctypes
import re
from pathlib import Path

import pytest

from xnpu_b200 import _lib, hal

HEADER = Path(__file__).resolve().parent.parent / "include" / "xq4.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(xq4_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("xq4_device_open", "xq4_buffer_create", "xq4_weight_import", "xq4_linear", "xq4_wait",
                 "xq4_linear_sharded", "xq4_dequant", "xq4_last_error_string"):
        assert must in names


def test_every_declared_symbol_is_exported():
    L = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_python_binding_covers_the_header():
    assert set(declared_functions()) == set(_lib.SIGNATURES)
    _lib.lib()  # binds every signature


def test_version_and_error_string():
    L = _lib.lib()
    assert b"sm_100a" in L.xq4_version()
    assert L.xq4_last_error_string() is not None


def test_layout_bytes():
    assert hal.gpu_layout_bytes(4096, 4096) == 256 * 64 * 576
    assert hal.gpu_layout_bytes(17, 96) == 2 * 2 * 576
    assert hal.gpu_layout_bytes(16, 33) == 0  # k must be a multiple of 32


def test_device_open_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(_lib.Xq4Error) as ei:
        hal.Device.open_default()
    assert ei.value.status == _lib.XQ4_ENODEV


@pytest.mark.parametrize("cname,pystruct", [("xq4_layout_desc", _lib.LayoutDesc),
                                            ("xq4_device_info", _lib.DeviceInfo),
                                            ("xq4_chain_op", _lib.ChainOp)])
def test_struct_layouts_match_the_header(tmp_path, cname, pystruct):
    """Every field of the ctypes mirror sits at the C compiler's offset, and
    the sizes agree (a C program built against include/xq4.h prints them)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f[0] for f in pystruct._fields_]
    src = tmp_path / "layout.c"
    body = "".join(f'    printf("{f} %zu\\n", offsetof({cname}, {f}));\n' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "xq4.h"\nint main(void) {{\n{body}'
                   f'    printf("sizeof %zu\\n", sizeof({cname}));\n    return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c11", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for f in fields:
        assert int(out[f]) == getattr(pystruct, f).offset, (cname, f)
    assert int(out["sizeof"]) == ctypes.sizeof(pystruct), cname


def test_null_arguments_are_rejected_without_a_device():
    """The entry points validate their arguments before touching CUDA: NULL
    handles give XQ4_EINVAL and a message, NULL destroys are no-ops."""
    L = _lib.lib()
    out = ctypes.c_void_p()
    seq = ctypes.c_uint64()
    op = _lib.ChainOp()
    for rc in (L.xq4_chain_create(None, ctypes.byref(op), 1, ctypes.byref(out)),
               L.xq4_chain_run(None, None),
               L.xq4_chain_submit(None, None, ctypes.byref(seq)),
               L.xq4_linear_raw(None, None, None, 1, 0, None),
               L.xq4_linear_sharded_fused(None, None, None, None, 1, 0, None),
               L.xq4_linear_sharded_noalloc(None, None, None, None, 1, 0, None)):
        assert rc == _lib.XQ4_EINVAL
        assert L.xq4_last_error_string()
    assert L.xq4_chain_destroy(None) == _lib.XQ4_OK
    assert L.xq4_weight_destroy(None) == _lib.XQ4_OK
    assert L.xq4_comm_destroy(None) == _lib.XQ4_OK
