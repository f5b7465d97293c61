"""The reference engine's ctypes bindings, restated against this build.

``load_kernels()`` returns the four handles the reference's engines keep
(``_kern``, ``_gqa_attn``, ``_cengine``, ``_simd``;
src/mojollama/kernels/turbo_engine_v7_moe.py:240-423 and turbo_engine_v77.py:93-121
of the reference) with the same argtypes, loaded from ``mojollama_b200/lib``.
A reference engine switches over by pointing its ``kernel_dir`` at that folder.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from ._lib import load_alias

cf = ctypes.POINTER(ctypes.c_float)
cu = ctypes.POINTER(ctypes.c_uint8)
ci = ctypes.c_int


@dataclass
class Kernels:
    kern: ctypes.CDLL       # combined_engine.so
    cengine: ctypes.CDLL    # cengine_batch_instr.so
    simd: ctypes.CDLL       # simd_ops.so
    gqa_attn: ctypes.CDLL   # gqa_attention.so


def _bind_engine(so: ctypes.CDLL) -> None:
    so.quant_matmul_omp.argtypes = [cu, cf, cf, ci, ci, ci]
    so.quant_matmul_omp.restype = None
    so.f32_matmul_omp.argtypes = [cf, cf, cf, ci, ci]
    so.f32_matmul_omp.restype = None
    for name in ("q4_0", "q4_1", "q5_0", "q8_0", "q4_k", "q5_k", "q6_k", "mxfp4"):
        fn = getattr(so, f"{name}_matmul_omp")
        fn.argtypes = [cu, cf, cf, ci, ci]
        fn.restype = None
    for name in ("q4_0", "q8_0", "q4_k", "q5_k", "q6_k", "mxfp4"):
        fn = getattr(so, f"{name}_batch_matmul")
        fn.argtypes = [cu, cf, cf, ci, ci, ci]
        fn.restype = None
    so.batch_qkv_omp.argtypes = [cu, cu, cu, cf, cf, cf, cf, ci, ci, ci, ci, ci, ci, ci]
    so.batch_qkv_omp.restype = None
    so.batch_gate_up_omp.argtypes = [cu, cu, cf, cf, cf, ci, ci, ci, ci, ci]
    so.batch_gate_up_omp.restype = None
    so.set_num_threads.argtypes = [ci]
    so.set_num_threads.restype = None
    for name in ("q6_k", "q4_k", "q5_k", "q8_0"):
        fn = getattr(so, f"{name}_dequantize_row")
        fn.argtypes = [cu, cf, ci]
        fn.restype = None
    so.quantize_row_q8_0.argtypes = [cf, cu, ci]
    so.quantize_row_q8_0.restype = ci
    so.q8_0_q8_0_matmul_omp.argtypes = [cu, cu, cf, ci, ci, ci]
    so.q8_0_q8_0_matmul_omp.restype = None
    # turbo_engine_v7_moe.py:338-353
    so.moe_forward_omp.argtypes = [ctypes.POINTER(cu), ctypes.POINTER(cu), ctypes.POINTER(cu), cf, ci, ci, ci, ci, ci,
                                   ctypes.POINTER(ctypes.c_int), cf, ci, cf, cf, cu]
    so.moe_forward_omp.restype = None
    # turbo_engine_v7_moe.py:396-410 (BC and KVBlock are passed by pointer)
    vp = ctypes.c_void_p
    so.batch_forward.argtypes = [vp, vp, ci, vp]
    so.batch_forward.restype = None
    so.moe_ffn.argtypes = [vp, ci, vp, vp, vp, vp, ci]
    so.moe_ffn.restype = None
    # turbo_engine_v7_moe.py:273-311 (cengine_batch_instr.c:859-899, 76 arguments)
    so.qwen36_batch_forward.argtypes = ([ci] * 10 + [ctypes.c_float] + [ci] * 7 + [vp, ci] + [vp] * 39 + [ci] * 3 +
                                        [vp] * 14)
    so.qwen36_batch_forward.restype = None


def load_kernels() -> Kernels:
    kern = load_alias("combined_engine.so")
    _bind_engine(kern)
    cengine = load_alias("cengine_batch_instr.so")
    _bind_engine(cengine)
    simd = load_alias("simd_ops.so")
    gqa = load_alias("gqa_attention.so")
    return Kernels(kern=kern, cengine=cengine, simd=simd, gqa_attn=gqa)
