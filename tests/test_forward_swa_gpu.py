"""batch_forward with per-layer sliding-window attention (mlq_set_attention_windows) and a
GPT-OSS-shaped small model: d_model 2880, bf16 attention projections, MXFP4 routed experts
(top-4 of 8, renormalisation off as in the batch engine's moe_ffn rule), layers alternating
full and windowed attention, 16-slot KV pages.  Checked against the oracle's forward_step
(oracle/model.py, with the window of each layer applied to oracle.ops.gqa_decode) on every
step, on the direct launches and on the graph-replayed step."""
import ctypes

import numpy as np
import pytest

from mojollama_b200 import bc as BCm
from oracle import formats as F
from oracle import model as OM
from oracle import ops as O

from model_fixture import _w, fill_bc, make_model

pytestmark = pytest.mark.gpu
MODEL_TOL = 3e-3


def _greedy_ok(got, ref):
    for g, r in zip(np.atleast_2d(got), np.atleast_2d(ref)):
        top = np.argsort(r)[::-1]
        if r[top[0]] - r[top[1]] > 1e-2:
            assert int(np.argmax(g)) == int(top[0])


def _gptoss_like(seed=0, L=2, window=4):
    rng = np.random.default_rng(seed)
    m = dict(L=L, N=2880, NH=8, NKH=2, HD=64, FF=0, V=384, eps=1e-5, rope_dim=64, max_ctx=64)
    N, inner, kvrow = m["N"], m["NH"] * m["HD"], m["NKH"] * m["HD"]
    m["emb"] = (rng.standard_normal((m["V"], N)) * 0.5).astype(np.float32)
    m["onw"] = (1 + 0.1 * rng.standard_normal(N)).astype(np.float32)
    m["wout"] = _w(rng, F.BF16, m["V"], N, scale=0.03)
    m["cos"], m["sin"] = O.rope_tables(m["max_ctx"], m["HD"], m["rope_dim"])
    E, k, M = 8, 4, 256
    m["moe"] = dict(E=E, k=k, M=M, gq=F.MXFP4, uq=F.MXFP4, dq=F.MXFP4)
    layers = []
    for l in range(L):
        ly = {"type": "attn", "an": (1 + 0.1 * rng.standard_normal(N)).astype(np.float32),
              "fn": (1 + 0.1 * rng.standard_normal(N)).astype(np.float32),
              "q": _w(rng, F.BF16, inner, N, 0.03), "k": _w(rng, F.BF16, kvrow, N, 0.03),
              "v": _w(rng, F.BF16, kvrow, N, 0.03), "o": _w(rng, F.BF16, N, inner, 0.03),
              "window": window if l % 2 else 0,
              "router": (rng.standard_normal((E, N)) * 0.05).astype(np.float32)}
        for name, rows, cols in (("gate_exps", M, N), ("up_exps", M, N), ("down_exps", N, M)):
            ly[name] = {e: _w(rng, F.MXFP4, rows, cols, 0.03)[0] for e in range(E)}
        layers.append(ly)
    m["layers"] = layers
    return m


def _run(lib, m, B, steps, page_size, graph):
    import torch
    stream = torch.cuda.Stream() if graph else None
    if graph:
        assert lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream)) == 0
    try:
        caches = [BCm.KVCache(m["L"], m["NKH"], m["HD"], page_size=page_size, n_pages=16) for _ in range(B)]
        logits = torch.zeros(B * m["V"], device="cuda")
        bld = BCm.BCBuilder()
        fill_bc(m, bld, [c.block for c in caches], np.zeros(1, np.float32))
        bld.bc.logits = ctypes.cast(ctypes.c_void_p(logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        win = np.array([ly.get("window", 0) for ly in m["layers"]], np.int32)
        assert lib.mlq_set_attention_windows(ctypes.byref(bld.bc), win.ctypes.data, m["L"]) == 0
        st = OM.new_state(m, B)
        rng = np.random.default_rng(B + steps)
        d_tok = torch.zeros(B, dtype=torch.int32, device="cuda")
        for step in range(steps):
            toks = rng.integers(0, m["V"], B).astype(np.int32)
            d_tok.copy_(torch.from_numpy(toks))
            torch.cuda.synchronize()
            rc = lib.mlq_batch_forward(ctypes.byref(bld.bc), ctypes.c_void_p(d_tok.data_ptr()), B, None)
            assert rc == 0, lib.mlq_last_error_message()
            torch.cuda.synchronize()
            got = logits.cpu().numpy().reshape(B, m["V"])
            want, _ = OM.forward_step(m, st, list(range(B)), list(toks))
            assert O.rel_l2(got, want) < MODEL_TOL, (step, O.rel_l2(got, want))
            _greedy_ok(got, want)
        lib.mlq_set_attention_windows(ctypes.byref(bld.bc), None, 0)
    finally:
        if graph:
            lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("graph", [False, True])
def test_sliding_window_layers_match_oracle(cuda_device, graph):
    m = make_model("dense", seed=51, attn_modes=["sep", "sep", "sep"])
    for l, ly in enumerate(m["layers"]):
        ly["window"] = [0, 3, 5][l]
    _run(cuda_device, m, B=2, steps=9, page_size=4, graph=graph)


def test_gptoss_shaped_model_matches_oracle(cuda_device):
    _run(cuda_device, _gptoss_like(), B=3, steps=7, page_size=16, graph=True)


def test_windows_argument_checks(cuda_device):
    lib = cuda_device
    bld = BCm.BCBuilder()
    bad = np.array([0, -1], np.int32)
    assert lib.mlq_set_attention_windows(ctypes.byref(bld.bc), bad.ctypes.data, 2) == 1
    assert lib.mlq_set_attention_windows(None, bad.ctypes.data, 2) == 1
