"""The C-ABI library loads and exports every entry point include/galactus_b200.h
declares; host-only calls behave as documented without a GPU."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "galactus_b200.h"


def declared_in_header() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_in_header()
    assert len(names) >= 25
    for must in ["gx_remap_serve", "gx_mul_mat_id", "gx_moe_layer_forward", "gx_arena_create", "gx_swiglu_oai"]:
        assert must in names


def test_library_exports_every_declared_symbol(gxlib):
    lib = gxlib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(gxlib._lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (gx_\w+)", out))
    for name in declared_in_header():
        assert name in exported, name
        assert getattr(lib, name) is not None
    # and the Python binding knows a signature for each of them
    assert set(declared_in_header()) <= set(gxlib.declared_symbols())


def test_status_strings(gxlib):
    lib = gxlib.lib()
    for code in range(0, -13, -1):
        assert lib.gx_status_string(code)
    assert lib.gx_status_string(-4) == b"expert id outside [0, n_expert)"


def test_no_device_fails_loudly_without_gpu(gxlib):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    assert gxlib.lib().gx_device_init(0) == gxlib._lib.GX_ERR_CUDA


def test_argument_checks_before_any_device_work(gxlib):
    lib = gxlib.lib()
    # unsupported type, misaligned row length, null pointers: rejected on the host
    assert lib.gx_mul_mat_id(2, 16, 64, 8, 72, 4096, 4, 16, 1, 1, 256, 256, 16, 1, 1, 4, 16, None) == -2
    assert lib.gx_mul_mat_id(8, 16, 96, 8, 102, 4096, 4, 16, 1, 1, 384, 384, 16, 1, 1, 4, 16, None) == -3
    assert lib.gx_mul_mat_id(8, None, 64, 8, 68, 4096, 4, 16, 1, 1, 256, 256, 16, 1, 1, 4, 16, None) == -1
    assert lib.gx_quantize_rows(12, 16, 256, 1, 1024, 16, 292, None) == -2
    assert lib.gx_synth_weights(12, 16, 100, 1, 0, 0, 0.02, None) == -3
