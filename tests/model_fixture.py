"""Small seeded models in the reference batch engine's layout, for the batch_forward tests.

``make_model`` returns the oracle's model dict (oracle/model.py); ``fill_bc`` points a
``BC`` (mojollama_b200.bc) at the same arrays, so the oracle, this library and the
reference build all read identical bytes."""
from __future__ import annotations

import ctypes

import numpy as np

from oracle import formats as F
from oracle import model as OM
from oracle import ops as O


def _w(rng, qt, rows, cols, scale=0.06):
    x = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
    if qt == F.F32:
        return (x.reshape(-1).view(np.uint8).copy(), qt)
    return (F.quantize(qt, x.reshape(-1)), qt)


def make_model(kind: str, seed: int = 0, **kw):
    """kind: 'dense' (attention layers with separate, QK-fused and optionally QKV-fused
    projections; dense SwiGLU FFN) or 'hybrid' (SSM layer + attention layer; MoE FFN with
    a shared expert).  Sizes are small enough for the oracle to finish in seconds."""
    rng = np.random.default_rng(seed)
    if kind == "dense":
        m = dict(L=3, N=256, NH=4, NKH=2, HD=64, FF=512, V=384, eps=1e-5, rope_dim=64, max_ctx=256)
    elif kind == "hybrid":
        m = dict(L=2, N=256, NH=4, NKH=1, HD=64, FF=512, V=320, eps=1e-6, rope_dim=32, max_ctx=256)
    elif kind == "qkv8192":     # the reference's fused-QKV split is hard-wired to 8192 rows
        m = dict(L=1, N=2048, NH=32, NKH=2, HD=128, FF=256, V=256, eps=1e-5, rope_dim=128, max_ctx=128)
    else:
        raise ValueError(kind)
    m.update(kw)
    L, N, NH, NKH, HD = m["L"], m["N"], m["NH"], m["NKH"], m["HD"]
    inner, kvrow = NH * HD, NKH * HD
    m["emb"] = (rng.standard_normal((m["V"], N)) * 0.5).astype(np.float32)
    m["onw"] = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    m["wout"] = _w(rng, F.Q8_0, m["V"], N)
    m["cos"], m["sin"] = O.rope_tables(m["max_ctx"], HD, m["rope_dim"])
    m["moe"] = None
    layers = []
    attn_modes = kw.get("attn_modes") or {"dense": ["sep", "qk", "qkv"], "hybrid": [None, "sep"],
                                          "qkv8192": ["qkv"]}[kind]
    for l in range(L):
        ly = {"an": (1 + 0.1 * rng.standard_normal(N)).astype(np.float32),
              "fn": (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)}
        mode = attn_modes[l]
        if mode is None:
            ly["type"] = "ssm"
            ly["conv"] = (rng.standard_normal(2 * inner) * 0.5).astype(np.float32)
            ly["a"] = (-0.5 * rng.random(OM.SSM_GROUPS)).astype(np.float32)
            ly["dt_bias"] = (0.1 * rng.standard_normal(OM.SSM_GROUPS)).astype(np.float32)
            ly["alpha"] = (0.1 * rng.standard_normal(OM.SSM_GROUPS * OM.SSM_DT_RANK)).astype(np.float32)
            ly["beta"] = (0.1 * rng.standard_normal(OM.SSM_GROUPS * OM.SSM_DT_RANK)).astype(np.float32)
            ly["norm"] = np.ones(inner, np.float32)
            ly["attn_gate"] = _w(rng, F.Q8_0, inner, N)
            ly["ssm_out"] = _w(rng, F.Q4_0, N, inner)
        else:
            ly["type"] = "attn"
            if mode == "qkv":
                ly["qkv"] = _w(rng, F.Q8_0, inner + 2 * N, N)
            elif mode == "qk":
                ly["qk"] = _w(rng, F.Q4_0, inner + kvrow, N)
                ly["v"] = _w(rng, F.Q8_0, kvrow, N)
            else:
                ly["q"] = _w(rng, F.Q8_0, inner, N)
                ly["k"] = _w(rng, F.Q4_1, kvrow, N)
                ly["v"] = _w(rng, F.Q5_K, kvrow, N)
            ly["o"] = _w(rng, F.Q8_0, N, inner)
        if kind == "hybrid":
            pass
        else:
            ly["gate"] = _w(rng, F.Q5_K, m["FF"], N)
            ly["up"] = _w(rng, F.Q8_0, m["FF"], N)
            ly["down"] = _w(rng, F.Q4_0, N, m["FF"])
        layers.append(ly)
    if kind == "hybrid":
        E, k, M = 8, 2, 256
        m["moe"] = dict(E=E, k=k, M=M, gq=F.Q5_K, uq=F.Q5_K, dq=F.Q5_K)
        for ly in layers:
            ly["router"] = (rng.standard_normal((E, N)) * 0.2).astype(np.float32)
            for name, rows, cols in (("gate_exps", M, N), ("up_exps", M, N), ("down_exps", N, M)):
                ly[name] = {e: _w(rng, F.Q5_K, rows, cols)[0] for e in range(E)}
            ly["shexp"] = {"g": _w(rng, F.Q8_0, OM.SHEXP_FF, N), "u": _w(rng, F.Q8_0, OM.SHEXP_FF, N),
                           "d": _w(rng, F.Q8_0, N, OM.SHEXP_FF),
                           "router": (rng.standard_normal(N) * 0.1).astype(np.float32)}
    m["layers"] = layers
    return m


def _cat_experts(d):
    return np.ascontiguousarray(np.concatenate([d[e] for e in sorted(d)]))


def fill_bc(m, builder, kv_blocks, logits, ssm_state=None, workspace=None):
    """Point builder.bc at model m.  kv_blocks: ctypes KVBlock objects (one per sequence)."""
    from mojollama_b200 import bc as BCm
    b = builder
    c = b.bc
    L, N, NH, NKH, HD = m["L"], m["N"], m["NH"], m["NKH"], m["HD"]
    inner, kvrow = NH * HD, NKH * HD
    c.L, c.N, c.NH, c.NKH, c.HD, c.FF, c.V = L, N, NH, NKH, HD, m["FF"], m["V"]
    c.eps, c.nc, c.rope_dim, c.max_ctx = m["eps"], N, m["rope_dim"], m["max_ctx"]
    ly = m["layers"]

    def W(name):
        return [x[name][0] if x.get(name) else None for x in ly]

    def Q(name, dflt=8):
        return [x[name][1] if x.get(name) else dflt for x in ly]

    for f, key in (("wQ", "q"), ("wK", "k"), ("wV", "v"), ("wO", "o"), ("wG", "gate"), ("wU", "up"),
                   ("wD", "down"), ("wQK", "qk"), ("wQKV", "qkv"), ("wAttnG", "attn_gate"),
                   ("wSsmOut", "ssm_out")):
        b.layers(f, W(key))
    for f, key in (("q_quant", "q"), ("k_quant", "k"), ("v_quant", "v"), ("o_quant", "o"), ("g_quant", "gate"),
                   ("u_quant", "up"), ("d_quant", "down"), ("qk_quant", "qk"), ("qkv_quant", "qkv"),
                   ("attnG_quant", "attn_gate"), ("ssm_out_quant", "ssm_out")):
        b.ints(f, Q(key))
    for f, v in (("nQ", inner), ("nK", kvrow), ("nV", kvrow), ("nO", N), ("nG", m["FF"]), ("nU", m["FF"]),
                 ("nD", N)):
        b.ints(f, [v] * L)
    b.layers("wAN", [x["an"] for x in ly])
    b.layers("wFN", [x["fn"] for x in ly])
    b.ints("layer_types", [1 if x["type"] == "ssm" else 0 for x in ly])
    for f, key in (("ssm_conv1d", "conv"), ("ssm_a", "a"), ("ssm_dt_bias", "dt_bias"), ("ssm_alpha", "alpha"),
                   ("ssm_beta", "beta"), ("ssm_norm", "norm")):
        b.layers(f, [x.get(key) for x in ly])
    b.ptr("emb", m["emb"])
    b.ptr("onw", m["onw"])
    b.ptr("wOut", m["wout"][0])
    c.outNR, c.outNC, c.outQuant, c.emb_quant = m["V"], N, m["wout"][1], 0
    b.ptr("cos_table", m["cos"])
    b.ptr("sin_table", m["sin"])
    moe = m["moe"]
    if moe:
        c.n_experts, c.n_experts_per_tok, c.moe_intermediate = moe["E"], moe["k"], moe["M"]
        c.gate_exp_quant, c.up_exp_quant, c.down_exp_quant = moe["gq"], moe["uq"], moe["dq"]
        if "_cat" not in m:
            m["_cat"] = [{k: _cat_experts(x[k]) for k in ("gate_exps", "up_exps", "down_exps")} for x in ly]
        b.layers("w_gate_inp", [x["router"] for x in ly])
        for f in ("gate_exps", "up_exps", "down_exps"):
            b.layers("w_" + f, [cat[f] for cat in m["_cat"]])
        sh = [x.get("shexp") for x in ly]
        b.layers("wSHexpG", [s["g"][0] if s else None for s in sh])
        b.layers("wSHexpU", [s["u"][0] if s else None for s in sh])
        b.layers("wSHexpD", [s["d"][0] if s else None for s in sh])
        b.ints("shexp_g_quant", [s["g"][1] if s else 8 for s in sh])
        b.ints("shexp_u_quant", [s["u"][1] if s else 8 for s in sh])
        b.ints("shexp_d_quant", [s["d"][1] if s else 8 for s in sh])
        b.layers("wShexpRouter", [s["router"] if s else None for s in sh])
    b.kv_array(kv_blocks)
    b.ptr("logits", logits)
    if ssm_state is not None:
        b.ptr("ssm_state", ssm_state)
    if workspace is not None:
        b.ptr("workspace", workspace)
        c.ws_size = int(workspace.size)
    c.n_layers_actual = L
    return c


def ws_stride(m, B):
    """S of batch_forward (cengine_batch_instr.c:1236-1239): the workspace's xn region
    starts at B*S floats."""
    N, inner, kvrow = m["N"], m["NH"] * m["HD"], m["NKH"] * m["HD"]
    S = max(N, inner, m["FF"], kvrow, inner + kvrow, 8192)
    return S


# ------------------------------------------------------------------ qwen36_batch_forward
def make_qwen36_model(seed=0, qkv_layout="std", L=4, layer_pattern=(1, 1, 1, 0), N=256, experts=(8, 2, 256),
                      expert_fmt=F.Q4_0, shexp_fmt=F.Q8_0):
    """Hybrid model in qwen36_batch_forward's layout: SSM layers (layer_types 1) and
    attention layers with a fused QKV projection; MoE (experts = (E, top-k, n_ff) of
    expert_fmt, F32 router) with a 512-wide shared expert of shexp_fmt.  qkv_layout 'std': rows
    NH*HD + 2*n_kv (Q|K|V); 'ref': NH*HD + 2N (Q|K|V with N-wide K and V sections, the layout
    the reference's split assumes)."""
    rng = np.random.default_rng(seed)
    m = dict(L=L, N=N, NH=4, NKH=2, HD=64, FF=512, V=320, eps=1e-6, rope_dim=32, max_ctx=64,
             ssm_inner=256, ssm_groups=32, ssm_state=128, ssm_dt_rank=32)
    N, inner, n_kv = m["N"], m["NH"] * m["HD"], m["NKH"] * m["HD"]
    m["emb"] = (rng.standard_normal((m["V"], N)) * 0.5).astype(np.float32)
    m["onw"] = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    m["wout"] = _w(rng, F.Q8_0, m["V"], N)
    m["cos"], m["sin"] = O.rope_tables(m["max_ctx"], m["HD"], m["rope_dim"])
    E, k, M = experts
    m["moe"] = dict(E=E, k=k, M=M, gq=expert_fmt, uq=expert_fmt, dq=expert_fmt)
    layers = []
    for l in range(L):
        ly = {"an": (1 + 0.1 * rng.standard_normal(N)).astype(np.float32),
              "fn": (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)}
        if layer_pattern[l % len(layer_pattern)] == 1:
            IN = m["ssm_inner"]
            ly["type"] = "ssm"
            ly["conv"] = (rng.standard_normal(2 * IN) * 0.5).astype(np.float32)
            ly["a"] = (-0.5 * rng.random(32)).astype(np.float32)
            ly["dt_bias"] = (0.1 * rng.standard_normal(32)).astype(np.float32)
            ly["alpha"] = (0.1 * rng.standard_normal(32 * 32)).astype(np.float32)
            ly["beta"] = (0.1 * rng.standard_normal(32 * 32)).astype(np.float32)
            ly["norm"] = np.ones(IN, np.float32)
            ly["attn_gate"] = _w(rng, F.Q8_0, IN, N)
            ly["ssm_out"] = _w(rng, F.Q4_0, N, IN)
        else:
            ly["type"] = "attn"
            ly["qkv_rows"] = inner + 2 * (n_kv if qkv_layout == "std" else N)
            ly["qkv"] = _w(rng, F.Q8_0, ly["qkv_rows"], N)
            ly["o"] = _w(rng, F.Q4_0, N, inner)
        ly["router"] = (rng.standard_normal((E, N)) * 0.2).astype(np.float32)
        for name, rows, cols in (("gate_exps", M, N), ("up_exps", M, N), ("down_exps", N, M)):
            ly[name] = {e: _w(rng, expert_fmt, rows, cols)[0] for e in range(E)}
        ly["shexp"] = {"si": 512, "g": _w(rng, shexp_fmt, 512, N), "u": _w(rng, shexp_fmt, 512, N),
                       "d": _w(rng, shexp_fmt, N, 512), "router": (rng.standard_normal(N) * 0.1).astype(np.float32)}
        layers.append(ly)
    m["layers"] = layers
    return m


# cengine_batch_instr.c:859-899: 76 arguments
QWEN36_ARGTYPES = ([ctypes.c_int] * 10 + [ctypes.c_float] + [ctypes.c_int] * 7 + [ctypes.c_void_p, ctypes.c_int] +
                   [ctypes.c_void_p] * 39 + [ctypes.c_int] * 3 + [ctypes.c_void_p] * 14)


class Qwen36Call:
    """Builds qwen36_batch_forward's 73 arguments for model m (keeps the arrays alive)."""

    def __init__(self, m, kv_k, kv_v, kv_lens, ssm_state):
        self.m, self.keep = m, []
        L, N = m["L"], m["N"]
        ly = m["layers"]
        if "_cat" not in m:
            m["_cat"] = [{k: _cat_experts(x[k]) for k in ("gate_exps", "up_exps", "down_exps")} for x in ly]

        def P(items):
            arr = (ctypes.c_void_p * L)(*[None if x is None else (x if isinstance(x, int) else x.ctypes.data)
                                          for x in items])
            self.keep.append((arr, items))
            return ctypes.cast(arr, ctypes.c_void_p).value

        def I(vals):
            arr = np.ascontiguousarray(vals, dtype=np.int32)
            self.keep.append(arr)
            return arr.ctypes.data

        def W(key, sub=0):
            return [x[key][sub] if x.get(key) is not None and x["type"] in (("ssm",) if key in ("attn_gate", "ssm_out")
                                                                           else ("attn",)) else None for x in ly]

        inner = m["NH"] * m["HD"]
        self.fields = dict(
            attn_norm_w=P([x["an"] for x in ly]), ffn_norm_w=P([x["fn"] for x in ly]),
            attn_qkv_raw=P(W("qkv")), qkv_nr=I([x.get("qkv_rows", 0) for x in ly]), qkv_nc=I([N] * L),
            qkv_qt=I([x["qkv"][1] if x["type"] == "attn" else 8 for x in ly]),
            attn_gate_raw=P(W("attn_gate")), gate_nr=I([m["ssm_inner"]] * L), gate_nc=I([N] * L),
            gate_qt=I([x["attn_gate"][1] if x["type"] == "ssm" else 8 for x in ly]),
            ssm_out_raw=P(W("ssm_out")), ssm_out_nr=I([N] * L), ssm_out_nc=I([m["ssm_inner"]] * L),
            ssm_out_qt=I([x["ssm_out"][1] if x["type"] == "ssm" else 8 for x in ly]),
            attn_out_raw=P(W("o")), out_nr=I([N] * L), out_nc=I([inner] * L),
            out_qt=I([x["o"][1] if x["type"] == "attn" else 8 for x in ly]),
            gate_exp_raw=P([c["gate_exps"] for c in m["_cat"]]), gate_exp_qt=I([m["moe"]["gq"]] * L),
            up_exp_raw=P([c["up_exps"] for c in m["_cat"]]), up_exp_qt=I([m["moe"]["uq"]] * L),
            down_exp_raw=P([c["down_exps"] for c in m["_cat"]]), down_exp_qt=I([m["moe"]["dq"]] * L),
            shexp_gate_raw=P([x["shexp"]["g"][0] for x in ly]), shexp_up_raw=P([x["shexp"]["u"][0] for x in ly]),
            shexp_down_raw=P([x["shexp"]["d"][0] for x in ly]), shexp_router=P([x["shexp"]["router"] for x in ly]),
            shexp_int=I([x["shexp"]["si"] for x in ly]),
            moe_router_raw=P([x["router"] for x in ly]), moe_router_qt=I([0] * L),
            shexp_gate_qt=I([x["shexp"]["g"][1] for x in ly]), shexp_up_qt=I([x["shexp"]["u"][1] for x in ly]),
            shexp_down_qt=I([x["shexp"]["d"][1] for x in ly]),
            ssm_conv1d=P([x.get("conv") for x in ly]), ssm_a=P([x.get("a") for x in ly]),
            ssm_dt_bias=P([x.get("dt_bias") for x in ly]), ssm_alpha=P([x.get("alpha") for x in ly]),
            ssm_beta=P([x.get("beta") for x in ly]), ssm_norm=P([x.get("norm") for x in ly]),
            layer_types=I([1 if x["type"] == "ssm" else 0 for x in ly]))
        self.kv_k, self.kv_v, self.kv_lens, self.ssm_state = kv_k, kv_v, kv_lens, ssm_state

    def ws_size(self, B):
        m = self.m
        inner, n_kv = m["NH"] * m["HD"], m["NKH"] * m["HD"]
        S = max(m["N"], inner, m["FF"], n_kv, inner + 2 * n_kv, m["moe"]["M"], 512, 8192)
        return 12 * B * S, S

    def __call__(self, fn, tokens, logits, ws, q8_ws=None):
        m, f = self.m, self.fields
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        self.keep.append(tok)
        addr = lambda a: None if a is None else (a if isinstance(a, int) else a.ctypes.data)
        fn.argtypes = QWEN36_ARGTYPES
        fn.restype = None
        fn(len(tok), m["L"], m["N"], m["NH"], m["NKH"], m["HD"], m["FF"], m["moe"]["E"], m["moe"]["k"], m["moe"]["M"],
           m["eps"], m["rope_dim"], m["max_ctx"], m["ssm_inner"], m["ssm_groups"], m["ssm_state"], 4,
           m["ssm_dt_rank"], m["emb"].ctypes.data, 0, f["layer_types"], tok.ctypes.data, logits.ctypes.data,
           f["attn_norm_w"], f["ffn_norm_w"], f["attn_qkv_raw"], f["qkv_nr"], f["qkv_nc"], f["qkv_qt"],
           f["attn_gate_raw"], f["gate_nr"], f["gate_nc"], f["gate_qt"], f["ssm_out_raw"], f["ssm_out_nr"],
           f["ssm_out_nc"], f["ssm_out_qt"], f["attn_out_raw"], f["out_nr"], f["out_nc"], f["out_qt"],
           f["gate_exp_raw"], f["gate_exp_qt"], f["up_exp_raw"], f["up_exp_qt"], f["down_exp_raw"],
           f["down_exp_qt"], f["shexp_gate_raw"], f["shexp_up_raw"], f["shexp_down_raw"], f["shexp_router"],
           f["shexp_int"], f["moe_router_raw"], f["moe_router_qt"], f["shexp_gate_qt"], f["shexp_up_qt"],
           f["shexp_down_qt"], m["onw"].ctypes.data, m["wout"][0].ctypes.data, m["V"], m["N"], m["wout"][1],
           f["ssm_conv1d"], f["ssm_a"], f["ssm_dt_bias"], f["ssm_alpha"], f["ssm_beta"], f["ssm_norm"],
           addr(self.ssm_state), addr(self.kv_k), addr(self.kv_v), addr(self.kv_lens), m["cos"].ctypes.data,
           m["sin"].ctypes.data, ws.ctypes.data, None if q8_ws is None else q8_ws.ctypes.data)
