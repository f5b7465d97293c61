"""ctypes mirrors of the reference batch engine's structs and a small BC builder.

The reference drives ``batch_forward`` / ``moe_ffn`` with a ``BC`` struct that its Python
fills through ctypes (src/mojollama/kernels/forward/zaya_bc.py:4-130,
src/mojollama/q4k_compare.py:60-90); the C definition is cengine_batch_instr.c:536-589,
the KV structs cengine_batch_instr.c:160-207.  The classes here have the same field
order and types, so the same struct bytes drive this library's ``batch_forward``
(include/mojollama_b200_ref_abi.h).

KV blocks for this library come from ``kv_init`` of this library (``KVCache`` below):
their page pools and k/v arrays live in device memory; the page table, free list and
``seq_len`` stay in the host struct as in the reference.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import core

_vp = ctypes.c_void_p
_pvp = ctypes.POINTER(ctypes.c_void_p)
_pi = ctypes.POINTER(ctypes.c_int)
_pf = ctypes.POINTER(ctypes.c_float)
_ci = ctypes.c_int

MAX_BLOCKS = 1024   # cengine_batch_instr.c:23
BLOCK_SIZE = 64     # cengine_batch_instr.c:22
SSM_GROUPS, SSM_STATE, SSM_DT_RANK = 32, 128, 32   # cengine_batch_instr.c:1253
SHEXP_FF = 512      # cengine_batch_instr.c:1444


class PageTable(ctypes.Structure):
    _fields_ = [("page_size", _ci), ("n_pages", _ci), ("pages", _pf), ("table", _pi), ("free_pages", _pi),
                ("free_count", _ci), ("_nkh", _ci), ("_hd", _ci), ("_n_layers", _ci)]


class KVBlock(ctypes.Structure):
    _fields_ = [("k", _pf), ("v", _pf), ("n_blocks", _ci), ("seq_len", _ci * 64),
                ("block_map", (_ci * 1024) * 64), ("pt", PageTable)]


def _arr(name):
    return (name, _pvp)


class BC(ctypes.Structure):
    _fields_ = [
        ("L", _ci), ("N", _ci), ("NH", _ci), ("NKH", _ci), ("HD", _ci), ("FF", _ci), ("V", _ci),
        ("eps", ctypes.c_float),
        _arr("wQ"), _arr("wK"), _arr("wV"), _arr("wO"), _arr("wG"), _arr("wU"), _arr("wD"),
        _arr("wAN"), _arr("wFN"),
        ("nQ", _pi), ("nK", _pi), ("nV", _pi), ("nO", _pi), ("nG", _pi), ("nU", _pi), ("nD", _pi),
        ("nc", _ci),
        ("emb", _vp), ("onw", _vp), ("wOut", _vp),
        ("outNR", _ci), ("outNC", _ci), ("outQuant", _ci),
        ("kv_array", _pvp), ("logits", _pf),
        ("n_experts", _ci), ("n_experts_per_tok", _ci), ("moe_intermediate", _ci),
        _arr("w_gate_inp"), _arr("w_gate_exps"), _arr("w_up_exps"), _arr("w_down_exps"),
        ("gate_exp_quant", _ci), ("up_exp_quant", _ci), ("down_exp_quant", _ci),
        ("q_quant", _pi), ("k_quant", _pi), ("v_quant", _pi), ("o_quant", _pi),
        ("g_quant", _pi), ("u_quant", _pi), ("d_quant", _pi),
        ("emb_quant", _ci),
        _arr("wQK"), ("qk_quant", _pi),
        ("cos_table", _pf), ("sin_table", _pf), ("max_ctx", _ci),
        ("workspace", _pf), ("ws_size", _ci),
        ("rope_dim", _ci), ("full_attn_interval", _ci),
        _arr("wQKV"), ("qkv_quant", _pi),
        _arr("wAttnG"), ("attnG_quant", _pi),
        _arr("ssm_conv1d"), _arr("ssm_a"), _arr("ssm_dt_bias"), _arr("ssm_alpha"), _arr("ssm_beta"),
        _arr("ssm_norm"),
        _arr("wSsmOut"), ("ssm_out_quant", _pi),
        ("ssm_state", _pf),
        _arr("wSHexpG"), _arr("wSHexpU"), _arr("wSHexpD"),
        ("shexp_g_quant", _pi), ("shexp_u_quant", _pi), ("shexp_d_quant", _pi),
        _arr("wShexpRouter"),
        ("layer_types", _pi), ("n_layers_actual", _ci),
        _arr("w_zaya_ffn_gate_inp"), _arr("w_zaya_ffn_gate"), _arr("w_zaya_mlp2"), _arr("w_zaya_mlp4"),
        _arr("w_zaya_router_bias"), _arr("w_zaya_ffn_norm"),
        _arr("w_zaya_res_hs_w"), _arr("w_zaya_res_hs_b"), _arr("w_zaya_res_res_w"), _arr("w_zaya_res_res_b"),
        ("zaya_ffn_gate_inp_quant", _ci), ("zaya_ffn_gate_quant", _ci), ("zaya_mlp2_quant", _ci),
        ("zaya_mlp4_quant", _ci),
        ("has_moe_layer", _pi), ("zaya_expert_n", _ci), ("zaya_moe_intermediate", _ci),
        _arr("w_cca_v1"), _arr("w_cca_v2"), _arr("w_ssm_conv1d"),
        ("cca_v1_quant", _ci), ("cca_v2_quant", _ci),
    ]


def _addr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, int):
        return a
    return a.ctypes.data


class BCBuilder:
    """Fills a BC from numpy arrays and keeps every array it points at alive.

    ``layers(name, items)`` sets a per-layer pointer array (items: numpy arrays, raw
    addresses or None); ``ints(name, values)`` a per-layer int array; ``ptr(name, a)`` a
    plain pointer member; scalars are set on ``.bc`` directly."""

    def __init__(self):
        self.bc = BC()
        self._keep = []

    def keep(self, *objs):
        self._keep.extend(objs)

    def layers(self, name, items):
        arr = (_vp * len(items))(*[_addr(x) for x in items])
        self._keep.append((arr, list(items)))
        setattr(self.bc, name, ctypes.cast(arr, _pvp))

    def ints(self, name, values):
        arr = (_ci * len(values))(*[int(v) for v in values])
        self._keep.append(arr)
        setattr(self.bc, name, ctypes.cast(arr, _pi))

    def ptr(self, name, a):
        if a is None:
            return
        self._keep.append(a)
        ftype = dict(BC._fields_)[name]
        setattr(self.bc, name, ctypes.cast(_vp(_addr(a)), ftype))

    def kv_array(self, blocks):
        arr = (_vp * len(blocks))(*[ctypes.addressof(b) for b in blocks])
        self._keep.append((arr, list(blocks)))
        self.bc.kv_array = ctypes.cast(arr, _pvp)


class KVCache:
    """One sequence's KVBlock made by this library's kv_init (device page pool)."""

    def __init__(self, n_layers: int, nkh: int, hd: int, page_size: int | None = None, n_pages: int | None = None):
        self._lib = core()
        self.block = KVBlock()
        rc = self._lib.mlq_kv_init(ctypes.byref(self.block), n_layers, nkh, hd)
        if rc != 0:
            raise RuntimeError(f"kv_init failed: {self._lib.mlq_last_error_message()}")
        if page_size is not None:
            # re-initialise the embedded page table with another page geometry
            self._lib.mlq_page_table_destroy(ctypes.byref(self.block.pt))
            rc = self._lib.mlq_page_table_init(ctypes.byref(self.block.pt), n_pages or MAX_BLOCKS, page_size, nkh, hd,
                                               n_layers)
            if rc != 0:
                raise RuntimeError(f"page_table_init failed: {self._lib.mlq_last_error_message()}")

    @property
    def seq_len(self) -> int:
        return self.block.seq_len[0]

    def free(self):
        if self.block.k or self.block.pt.pages:
            self._lib.mlq_kv_free(ctypes.byref(self.block))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def batch_forward(bc: BC, tokens, ws: np.ndarray | None = None) -> None:
    """batch_forward(const BC*, tokens, B, ws) of this library; raises on error."""
    lib = core()
    tok = np.ascontiguousarray(tokens, dtype=np.int32)
    wsp = None if ws is None else ws.ctypes.data
    rc = lib.mlq_batch_forward(ctypes.byref(bc), tok.ctypes.data, len(tok), wsp)
    if rc != 0:
        raise RuntimeError(f"batch_forward failed ({rc}): {lib.mlq_last_error_message()}")
