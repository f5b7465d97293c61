"""CPU checks of the drop-in boundary: the native libraries load without a GPU and
export every symbol that include/*.h declares (no compute calls here)."""
import ctypes
import os
import re
import subprocess

import pytest

from mojollama_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")

# which library exports the declarations of which header section
ENGINE_LIBS = ("combined_engine.so", "quant_kernels_omp.so", "cengine_batch_instr.so")


def _declared(header, start_marker=None, end_marker=None):
    text = open(os.path.join(INC, header)).read()
    if start_marker:
        text = text.split(start_marker, 1)[1]
    if end_marker and end_marker in text:
        text = text.split(end_marker, 1)[0]
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "for", "while")))


def _exports(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_core_library_exports_every_mlq_symbol():
    names = _declared("mojollama_b200.h")
    assert len(names) > 20
    missing = [n for n in names if n not in _exports(_lib.CORE)]
    assert not missing, missing


@pytest.mark.parametrize("lib", ENGINE_LIBS)
def test_engine_alias_exports_reference_symbols(lib):
    names = _declared("mojollama_b200_ref_abi.h", "engine set", "simd_ops.so set")
    assert "quant_matmul_omp" in names
    missing = [n for n in names if n not in _exports(_lib.lib_path(lib))]
    assert not missing, missing


def test_simd_and_gqa_alias_exports():
    text = open(os.path.join(INC, "mojollama_b200_ref_abi.h")).read()
    for section, lib, end in (("simd_ops.so set", "simd_ops.so", "#endif"),
                              ("gqa_attention.so set", "gqa_attention.so", "end of gqa_attention.so set")):
        names = _declared("mojollama_b200_ref_abi.h", section, end)
        assert names, section
        missing = [n for n in names if n not in _exports(_lib.lib_path(lib))]
        assert not missing, (lib, missing)


def test_libraries_load_without_a_gpu():
    so = _lib.core()
    assert so.mlq_block_bytes(12) == 144 and so.mlq_block_elems(12) == 256
    assert so.mlq_row_bytes(8, 2048) == 64 * 34
    assert so.mlq_row_bytes(12, 2880) == 0          # K-quants need K % 256 == 0
    for name in ENGINE_LIBS + ("simd_ops.so", "gqa_attention.so"):
        assert isinstance(_lib.load_alias(name), ctypes.CDLL)


def test_bad_arguments_are_reported_not_fatal():
    so = _lib.core()
    so.mlq_clear_error()
    rc = so.mlq_matmul(None, 8, None, None, 16, 64, 1)
    assert rc == 1 and so.mlq_last_error() == 1
    assert b"null" in so.mlq_last_error_message()
    rc = so.mlq_matmul(ctypes.c_void_p(1), 99, ctypes.c_void_p(1), ctypes.c_void_p(1), 16, 64, 1)
    assert rc == 2      # unsupported type, like the reference's silent `default:`
