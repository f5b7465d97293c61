"""CPU pin of the whole-model oracle (oracle/model.py) against the reference's own
batch_forward (cengine_batch_instr.c:1233-1493, built from its sources into oracle/_ref).

The reference projects its workspace's never-written xn region; the oracle's
compatibility mode follows that data flow, so the two must agree on every step's logits,
final hidden state (left in ws[0:B*N]), SSM state and sequence lengths.  The oracle's
default mode differs from it only in which buffer feeds the projections."""
import ctypes

import numpy as np
import pytest

from mojollama_b200.bc import BCBuilder, KVBlock
from oracle import model as OM
from oracle import ops as O
from oracle import ref as R

from model_fixture import fill_bc, make_model, ws_stride

needs_ref = pytest.mark.skipif(not R.available(), reason="reference build (oracle/_ref) not present")


@pytest.mark.parametrize("kind,kw,B,steps", [
    ("dense", dict(attn_modes=["sep", "qk", "sep"]), 2, 3),
    ("hybrid", {}, 3, 2),
    ("qkv8192", {}, 2, 2),
], ids=["dense", "hybrid_ssm_moe", "fused_qkv"])
@needs_ref
def test_oracle_compat_step_matches_reference_build(kind, kw, B, steps):
    ref = R.RefEngine()
    m = make_model(kind, seed=21, **kw)
    L, V, N = m["L"], m["V"], m["N"]
    kvrow = m["NKH"] * m["HD"]
    S = ws_stride(m, B)
    kvs = [KVBlock() for _ in range(B)]
    for kv in kvs:
        ref.so.kv_init(ctypes.byref(kv), L, m["NKH"], m["HD"])
    logits = np.zeros(B * V, np.float32)
    ssm = np.zeros(L * OM.SSM_GROUPS * OM.SSM_STATE, np.float32)
    work = np.zeros(m["max_ctx"] * kvrow * 2 + 4096, np.float32)
    b = BCBuilder()
    fill_bc(m, b, kvs, logits, ssm_state=ssm, workspace=work)
    st = OM.new_state(m, B)
    rng = np.random.default_rng(22)
    xn = (rng.standard_normal((B, N)) * 0.7).astype(np.float32)
    for step in range(steps):
        toks = rng.integers(0, V, B).astype(np.int32)
        ws = np.zeros(12 * B * S, np.float32)
        ws[B * S:B * S + B * N] = xn.reshape(-1)
        ref.so.batch_forward(ctypes.byref(b.bc), toks.ctypes.data, B, ws.ctypes.data)
        want, h = OM.forward_step(m, st, list(range(B)), toks, compat_xn=xn)
        assert O.rel_l2(logits.reshape(B, V), want) < 1e-5
        assert O.rel_l2(ws[:B * N].reshape(B, N), h) < 1e-5
        if m["moe"]:
            assert O.rel_l2(ssm, st["ssm"].reshape(-1)) < 1e-5
        assert all(kv.seq_len[0] == step + 1 for kv in kvs)


@pytest.mark.parametrize("B", [1, 2])
@needs_ref
def test_oracle_qwen36_step_matches_reference_build(B):
    """qwen36_batch_forward (cengine_batch_instr.c:859-1231) on a 3 SSM + 1 attention layer
    MoE model whose fused QKV uses the layout the reference's split reads (N-wide K and V
    sections), Q4_0 experts (which moe_forward_omp computes exactly), three steps with the
    caller advancing kv_lens as the reference's Python does (turbo_engine_v7_moe.py:1889)."""
    from model_fixture import Qwen36Call, make_qwen36_model
    ref = R.RefEngine()
    m = make_qwen36_model(seed=31, qkv_layout="ref")
    L, N, V = m["L"], m["N"], m["V"]
    n_kv = m["NKH"] * m["HD"]
    kv_k = np.zeros((L, m["max_ctx"], n_kv), np.float32)
    kv_v = np.zeros_like(kv_k)
    kv_lens = np.zeros(L, np.int32)
    ssm = np.zeros(L * 32 * 128, np.float32)
    call = Qwen36Call(m, kv_k, kv_v, kv_lens, ssm)
    st = OM.qwen36_new_state(m)
    rng = np.random.default_rng(32)
    for step in range(3):
        toks = rng.integers(0, V, B).astype(np.int32)
        logits = np.zeros(B * V, np.float32)
        wsn, S = call.ws_size(B)
        ws = np.zeros(wsn, np.float32)
        q8 = np.zeros(64 * 1024, np.uint8)
        call(ref.so.qwen36_batch_forward, toks, logits, ws, q8)
        want, x = OM.qwen36_step(m, st, toks)
        assert O.rel_l2(logits.reshape(B, V), want) < 1e-5
        assert O.rel_l2(ws[:B * N].reshape(B, N), x) < 1e-5
        assert O.rel_l2(ssm, st["ssm"].reshape(-1)) < 1e-5
        assert O.rel_l2(kv_k[:, :step + 1], st["kv_k"][:, :step + 1]) < 1e-5
        assert O.rel_l2(kv_v[:, :step + 1], st["kv_v"][:, :step + 1]) < 1e-5
        kv_lens += 1
        st["kv_lens"] += 1


@pytest.mark.parametrize("modes", [["sep", "qk", "qkv"], ["sep", "sep", "sep"]])
def test_forward_sequence_equals_stepwise_forward(modes):
    """The teacher-forced layer-outer restatement (used at full model size, where one
    decode per position would take minutes) computes the same logits as P consecutive
    forward_step calls."""
    m = make_model("dense", seed=3, attn_modes=modes)
    P, B = 5, 3
    tok = np.random.default_rng(4).integers(0, m["V"], (P, B))
    seq = OM.forward_sequence(m, tok)
    st = OM.new_state(m, B)
    for p in range(P):
        lg, _ = OM.forward_step(m, st, list(range(B)), list(tok[p]))
        assert O.rel_l2(seq[p], lg) < 1e-6, p
