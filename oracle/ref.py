"""ctypes loader for the reference C engine built from its own sources.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  ``oracle/Makefile`` compiles
the reference's quant_kernels_omp.c + cengine_batch_instr.c (the reference's
combined_engine.so), simd_ops.c and gqa_attention.c into ``oracle/_ref/``.  The
argtypes below restate the bindings of the reference's own Python engine
(src/mojollama/kernels/turbo_engine_v7_moe.py:240-423, turbo_engine_v77.py:93-121).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_cf = ctypes.POINTER(ctypes.c_float)
_cu = ctypes.POINTER(ctypes.c_uint8)
_ci = ctypes.c_int


def available() -> bool:
    return os.path.exists(os.path.join(REF_DIR, "libref_engine.so"))


def fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_cf)


def uptr(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(_cu)


def iptr(a: np.ndarray):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


class RefEngine:
    """The reference's combined_engine.so (+ simd_ops.so, gqa_attention.so)."""

    def __init__(self, ref_dir: str = REF_DIR):
        self.so = ctypes.CDLL(os.path.join(ref_dir, "libref_engine.so"))
        so = self.so
        so.quant_matmul_omp.argtypes = [_cu, _cf, _cf, _ci, _ci, _ci]
        so.f32_matmul_omp.argtypes = [_cf, _cf, _cf, _ci, _ci]
        for name in ("q4_0", "q4_1", "q5_0", "q8_0", "q4_k", "q5_k", "q6_k", "mxfp4"):
            getattr(so, f"{name}_matmul_omp").argtypes = [_cu, _cf, _cf, _ci, _ci]
        for name in ("q4_0", "q8_0", "q4_k", "q5_k", "q6_k", "mxfp4"):
            getattr(so, f"{name}_batch_matmul").argtypes = [_cu, _cf, _cf, _ci, _ci, _ci]
        for name in ("q4_k", "q5_k", "q6_k", "q8_0"):
            getattr(so, f"{name}_dequantize_row").argtypes = [_cu, _cf, _ci]
        so.quantize_row_q8_0.argtypes = [_cf, _cu, _ci]
        so.quantize_row_q8_0.restype = _ci
        so.q8_0_q8_0_matmul_omp.argtypes = [_cu, _cu, _cf, _ci, _ci, _ci]
        so.q4_k_row_dot_avx2.argtypes = [_cu, _cf, _ci, _ci]
        so.q4_k_row_dot_avx2.restype = ctypes.c_float
        so.q5_k_row_dot_avx2.argtypes = [_cu, _cf, _ci, _ci]
        so.q5_k_row_dot_avx2.restype = ctypes.c_float
        so.q6_k_row_dot_avx2.argtypes = [_cu, _cf, _ci, _ci]
        so.q6_k_row_dot_avx2.restype = ctypes.c_float
        so.batch_qkv_omp.argtypes = [_cu, _cu, _cu, _cf, _cf, _cf, _cf] + [_ci] * 7
        so.batch_gate_up_omp.argtypes = [_cu, _cu, _cf, _cf, _cf] + [_ci] * 5
        so.moe_forward_omp.argtypes = [ctypes.POINTER(_cu)] * 3 + [_cf, _ci, _ci, _ci, _ci, _ci,
                                                                  ctypes.POINTER(_ci), _cf, _ci,
                                                                  _cf, _cf, _cu]
        so.ssm_decode_step.argtypes = [_cf] * 9 + [_ci] * 7
        so.rope_init.argtypes = [_cf, _cf, _ci, _ci, _ci]
        # cengine_batch_instr.c:1233, 208, 591 (struct pointers passed as void*)
        so.batch_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _ci, ctypes.c_void_p]
        so.batch_forward.restype = None
        so.kv_init.argtypes = [ctypes.c_void_p, _ci, _ci, _ci]
        so.kv_init.restype = None
        so.moe_ffn.argtypes = [ctypes.c_void_p, _ci] + [ctypes.c_void_p] * 4 + [_ci]
        so.moe_ffn.restype = None
        so.set_num_threads.argtypes = [_ci]
        so.get_max_threads.restype = _ci
        so.silu.argtypes = [_cf, _ci]
        so.softmax.argtypes = [_cf, _ci]
        so.rms_norm.argtypes = [_cf, _cf, _cf, _ci]
        self.simd = None
        p = os.path.join(ref_dir, "libref_simd.so")
        if os.path.exists(p):
            self.simd = ctypes.CDLL(p)
            self.simd.rms_norm.argtypes = [_cf, _cf, _cf, _ci, ctypes.c_float]
            self.simd.silu.argtypes = [_cf, _cf, _ci]
            self.simd.residual_add.argtypes = [_cf, _cf, _cf, _ci]
            self.simd.apply_rope.argtypes = [_cf, _cf, _ci, _ci, _ci, _ci, ctypes.c_float]
        self.gqa = None
        p = os.path.join(ref_dir, "libref_gqa.so")
        if os.path.exists(p):
            self.gqa = ctypes.CDLL(p)
            self.gqa.gqa_attention_decode.argtypes = [_cf, _cf, _cf, _cf, _ci, _ci, _ci, _ci, _cf]

    # -- convenience wrappers (numpy in / numpy out) ------------------------------------
    def quant_matmul(self, w: np.ndarray, x: np.ndarray, n: int, k: int, qt: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        self.so.quant_matmul_omp(uptr(w), fptr(np.ascontiguousarray(x, np.float32)), fptr(out), n, k, qt)
        return out

    def batch_matmul(self, fmt: str, w: np.ndarray, x: np.ndarray, n: int, k: int, b: int) -> np.ndarray:
        out = np.zeros(b * n, np.float32)
        getattr(self.so, f"{fmt}_batch_matmul")(uptr(w), fptr(np.ascontiguousarray(x, np.float32)),
                                                fptr(out), n, k, b)
        return out.reshape(b, n)

    def dequantize_row(self, fmt: str, w: np.ndarray, n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        getattr(self.so, f"{fmt}_dequantize_row")(uptr(w), fptr(out), n)
        return out

    def quantize_row_q8_0(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(x.size // 32 * 34, np.uint8)
        self.so.quantize_row_q8_0(fptr(x), uptr(out), x.size)
        return out

    def set_num_threads(self, n: int) -> None:
        self.so.set_num_threads(n)
