"""CPU: the C-ABI library loads and exports every entry point declared in
include/quantr_cuda.h (no compute calls: this container has no GPU)."""
import ctypes
import os
import re

import quantr

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "quantr_cuda.h")

# Entry points that replace the reference's include/quant.h:84-92.
REFERENCE_SYMBOLS = ["quantize_row_q8_0", "dequantize_row", "vec_dot_q4K_q8_0", "vec_dot_q5K_q8_0",
                     "vec_dot_q6K_q8_0", "vec_dot_q8_0_q8_0", "matmul_q_fused"]


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][A-Za-z0-9_]*[A-Za-z0-9])\s*\(", src, flags=re.M)
    return sorted(set(n for n in names if not n.startswith("defined")))


def test_header_declares_reference_api():
    decl = declared_functions()
    for s in REFERENCE_SYMBOLS:
        assert s in decl


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(quantr.LIB_PATH)
    decl = declared_functions()
    assert len(decl) >= 20
    missing = [n for n in decl if not hasattr(L, n)]
    assert not missing, missing


def test_python_mirror_covers_every_declared_symbol():
    assert sorted(quantr.SIGNATURES) == declared_functions()


def test_error_strings_without_device():
    L = quantr.lib()
    assert L.quantr_gpu_error_string(0) == b"ok"
    assert b"unsupported" in L.quantr_gpu_error_string(4)
    assert L.quantr_gpu_last_error() == 0


def test_workspace_size_is_host_arithmetic():
    # 40 bytes per 32-element block, each region 256-byte aligned, plus the
    # engine's per-token padding allowance.
    assert quantr.workspace_bytes(2048, 1) == 2048 + 256 + 256 + 256 + 32
    assert quantr.workspace_bytes(4864, 16) >= 16 * 152 * 40


def test_row_bytes_floor_semantics():
    # src/quant.c:477-484: partial blocks at the end of a row are ignored.
    assert quantr.row_bytes(quantr.Q4_K, 896) == 3 * 144
    assert quantr.row_bytes(quantr.Q6_K, 1408) == 5 * 210
    assert quantr.row_bytes(quantr.Q8_0, 100) == 3 * 34
    assert quantr.row_bytes(quantr.Q5_K, 2048) == 8 * 176
