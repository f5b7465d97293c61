"""ctypes loader for the in-tree native libraries.

Loading fails loudly when the libraries were not built: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
CORE = os.path.join(LIB_DIR, "libmojollama_b200.so")

_cf = ctypes.POINTER(ctypes.c_float)
_cu = ctypes.POINTER(ctypes.c_uint8)
_ci = ctypes.c_int
_vp = ctypes.c_void_p

_core = None


class NativeLibraryMissing(RuntimeError):
    pass


def lib_path(name: str) -> str:
    return os.path.join(LIB_DIR, name)


def core() -> ctypes.CDLL:
    """libmojollama_b200.so with argtypes for the mlq_* C-ABI (include/mojollama_b200.h)."""
    global _core
    if _core is not None:
        return _core
    if not os.path.exists(CORE):
        raise NativeLibraryMissing(
            f"{CORE} is missing: build it with `python -m mojollama_b200.build` "
            "(this package has no CPU fallback)")
    so = ctypes.CDLL(CORE, mode=ctypes.RTLD_GLOBAL)
    so.mlq_last_error.restype = _ci
    so.mlq_last_error_message.restype = ctypes.c_char_p
    so.mlq_init.argtypes = [_ci]
    so.mlq_set_device.argtypes = [_ci]
    so.mlq_get_stream.restype = _vp
    so.mlq_set_stream.argtypes = [_vp]
    so.mlq_use_own_stream.argtypes = []
    so.mlq_register_weights.argtypes = [_vp, ctypes.c_size_t]
    so.mlq_unregister_weights.argtypes = [_vp]
    so.mlq_cache_bytes.restype = ctypes.c_size_t
    so.mlq_launch_count.restype = ctypes.c_ulonglong
    so.mlq_set_ref_compat.argtypes = [_ci]
    so.mlq_block_elems.argtypes = [_ci]
    so.mlq_block_bytes.argtypes = [_ci]
    so.mlq_row_bytes.argtypes = [_ci, _ci]
    so.mlq_row_bytes.restype = ctypes.c_size_t
    so.mlq_matmul.argtypes = [_vp, _ci, _vp, _vp, _ci, _ci, _ci]
    so.mlq_gemv_fused.argtypes = [_ci, _ci, _vp, _vp, _vp, _vp, _ci, _vp, _ci, _ci]
    so.mlq_dequantize.argtypes = [_vp, _ci, _vp, ctypes.c_int64]
    so.mlq_quantize_q8_0.argtypes = [_vp, _vp, ctypes.c_int64]
    so.mlq_matmul_q8act.argtypes = [_vp, _ci, _vp, _vp, _ci, _ci, _ci]
    so.mlq_matmul_q8act_noalloc.argtypes = [_vp, _ci, _vp, _vp, _ci, _ci, _ci, _vp]
    so.mlq_noalloc_status.argtypes = [_vp]
    so.mlq_selftest_wait_timeout.argtypes = [_ci]
    so.mlq_moe_forward.argtypes = [_vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci, _vp, _vp, _ci, _vp]
    so.mlq_moe_router.argtypes = [_vp, _ci, _ci, _vp, _ci, _ci, _ci, _ci, _vp, _vp]
    so.mlq_ssm_decode_step.argtypes = [_vp] * 9 + [_ci] * 7
    so.mlq_ssm_layer_fused.argtypes = [_vp] * 10 + [_vp, _ci, _ci, _ci, _vp, _ci, _ci, _ci] + [_ci] * 7
    so.mlq_batch_forward.argtypes = [_vp, _vp, _ci, _vp]
    so.mlq_set_attention_windows.argtypes = [_vp, _vp, _ci]
    so.mlq_sample.argtypes = [_vp, _ci, _ci, ctypes.c_float, ctypes.c_ulonglong, ctypes.c_ulonglong, _vp]
    so.mlq_argmax.argtypes = [_vp, _ci, _ci, _vp]
    so.mlq_kv_snapshot.argtypes = [_vp, _ci, _vp]
    so.mlq_kv_restore.argtypes = [_vp, _ci, _vp]
    so.mlq_gguf_open.restype = _vp
    so.mlq_gguf_open.argtypes = [ctypes.c_char_p]
    for fn in ("mlq_gguf_close", "mlq_gguf_version"):
        getattr(so, fn).argtypes = [_vp]
    for fn in ("mlq_gguf_n_tensors", "mlq_gguf_n_kv"):
        getattr(so, fn).argtypes = [_vp]
        getattr(so, fn).restype = ctypes.c_int64
    for fn in ("mlq_gguf_alignment", "mlq_gguf_data_offset", "mlq_gguf_data_bytes"):
        getattr(so, fn).argtypes = [_vp]
        getattr(so, fn).restype = ctypes.c_uint64
    so.mlq_gguf_tensor.argtypes = [_vp, ctypes.c_int64, _vp]
    so.mlq_gguf_find.argtypes = [_vp, ctypes.c_char_p]
    so.mlq_gguf_find.restype = ctypes.c_int64
    so.mlq_gguf_kv_type.argtypes = [_vp, ctypes.c_char_p]
    so.mlq_gguf_kv_int.argtypes = [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]
    so.mlq_gguf_kv_float.argtypes = [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]
    so.mlq_gguf_kv_str.argtypes = [_vp, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
    so.mlq_gguf_kv_str.restype = ctypes.c_int64
    so.mlq_gguf_kv_array.argtypes = [_vp, ctypes.c_char_p, ctypes.POINTER(_ci)]
    so.mlq_gguf_kv_array.restype = ctypes.c_int64
    so.mlq_gguf_tensor_data.argtypes = [_vp, ctypes.c_int64]
    so.mlq_gguf_tensor_data.restype = _vp
    so.mlq_gguf_upload.argtypes = [_vp, _vp, ctypes.c_uint64]
    so.mlq_gguf_upload_tensor.argtypes = [_vp, ctypes.c_int64, _vp, ctypes.c_uint64]
    so.mlq_mamba2_step.argtypes = [_vp] * 12 + [_ci] * 6 + [ctypes.c_float, _ci]
    so.mlq_mamba2_layer.argtypes = [_vp, _ci, _ci, _vp, _ci, _vp, _ci] + [_vp] * 9 + [_ci] * 5 + [ctypes.c_float, _ci]
    so.mlq_batch_forward_sample.argtypes = [_vp, _vp, _ci, _vp, ctypes.c_float, ctypes.c_ulonglong,
                                            ctypes.c_ulonglong, _vp]
    so.mlq_moe_ffn.argtypes = [_vp, _ci, _vp, _vp, _ci]
    so.mlq_forget_model_plans.restype = None
    so.mlq_sizeof_bc.restype = ctypes.c_size_t
    so.mlq_ep_dispatch.argtypes = [_vp, _ci, _ci, _ci, _ci, _vp, _ci, _vp, _vp, _vp, _vp]
    so.mlq_moe_rows.argtypes = [_ci, _ci, _ci, _vp, _vp, _vp, ctypes.c_longlong, ctypes.c_longlong,
                                ctypes.c_longlong, _ci, _vp, _ci, _ci, _ci, _vp, _vp]
    so.mlq_ep_dispatch_packed.argtypes = [_vp, _ci, _ci, _ci, _ci, _ci, _vp, _ci, _vp, _vp]
    so.mlq_moe_rows_packed.argtypes = [_ci, _ci, _ci, _vp, _vp, _vp, ctypes.c_longlong, ctypes.c_longlong,
                                       ctypes.c_longlong, _ci, _vp, _ci, _ci, _ci, _vp]
    so.mlq_ep_combine.argtypes = [_vp, _vp, _vp, _ci, _ci, _ci, _vp, _vp]
    so.mlq_attn_decode_flat.argtypes = [_vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci]
    so.mlq_attn_decode_paged.argtypes = [_vp, _vp, _vp, _vp, _ci, _ci, _ci, _vp, _ci, _ci, _ci, _ci, _ci, _vp]
    so.mlq_page_table_init.argtypes = [_vp, _ci, _ci, _ci, _ci, _ci]
    so.mlq_page_table_alloc.argtypes = [_vp]
    so.mlq_page_table_free.argtypes = [_vp, _ci]
    so.mlq_page_table_free.restype = None
    so.mlq_map_page.argtypes = [_vp, _ci, _ci]
    so.mlq_map_page.restype = None
    so.mlq_page_table_destroy.argtypes = [_vp]
    so.mlq_page_table_destroy.restype = None
    so.mlq_kv_init.argtypes = [_vp, _ci, _ci, _ci]
    so.mlq_kv_alloc.argtypes = [_vp]
    so.mlq_kv_free.argtypes = [_vp]
    so.mlq_kv_free.restype = None
    so.mlq_sizeof_page_table.restype = ctypes.c_size_t
    so.mlq_sizeof_kv_block.restype = ctypes.c_size_t
    so.mlq_kv_cache_update.argtypes = [_vp, _vp, _vp, _vp, _ci, _ci, _ci, _ci, _ci]
    _ll = ctypes.c_longlong
    so.mlq_rms_norm.argtypes = [_vp, _vp, _vp, _ci, _ci, ctypes.c_float, _ci, _vp]
    so.mlq_silu.argtypes = [_vp, _vp, _ll, _ci]
    so.mlq_swiglu.argtypes = [_vp, _vp, _vp, _ll]
    so.mlq_add.argtypes = [_vp, _vp, _vp, _ll]
    so.mlq_softmax.argtypes = [_vp, _ci, _ci]
    so.mlq_rope_interleaved.argtypes = [_vp, _vp, _ci, _ci, _ci, _ci, ctypes.c_float]
    so.mlq_rope_init.argtypes = [_vp, _vp, _ci, _ci, _ci, ctypes.c_double]
    so.mlq_rope_neox.argtypes = [_vp, _ci, _ci, _ci, _ci, _vp, _ci, _vp, _vp, _ci, _ci]
    _core = so
    return so


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = core().mlq_last_error_message().decode(errors="replace")
        raise RuntimeError(f"{what or 'mojollama_b200'} failed ({rc}): {msg}")


def load_alias(name: str) -> ctypes.CDLL:
    """One of the reference-named alias libraries (combined_engine.so, ...)."""
    core()   # load the core first (RTLD_GLOBAL) so the alias resolves against this build
    p = lib_path(name)
    if not os.path.exists(p):
        raise NativeLibraryMissing(f"{p} is missing: run `python -m mojollama_b200.build`")
    return ctypes.CDLL(p)
