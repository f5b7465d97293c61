"""Whole-model decode step of the reference batch engine, restated in numpy (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  ``forward_step`` computes one
``batch_forward`` step (cengine_batch_instr.c:1233-1493) for B sequences the way that
function is laid out, with the normalised activations feeding the projections.

With ``compat_xn`` ([B][N]) it follows the reference's own data flow instead: every
projection, the SSM step, the router and the experts read the workspace's ``xn`` region
(which the reference never writes, cengine_batch_instr.c:1241), the normalised activations
overwrite x, a layer without FFN keeps them, and the fused QKV / QK projections hand
sequence b the Q slice at b*NH*HD of the flat projection buffer (:1330-1357).  That mode
is pinned against the reference build (tests/test_model_oracle.py); both modes share
every other line.  Per-op pieces are the pinned restatements of oracle/ops.py.

Model description (plain dict; weights are (raw GGUF bytes, type) pairs):
  L N NH NKH HD FF V eps rope_dim max_ctx; emb f32 [V][N]; onw f32 [N];
  wout (raw, qt) [V][N]; cos, sin f32 [max_ctx][rope_dim/2];
  layers[l]: type 'attn' | 'ssm'; an, fn f32 [N];
    attn: 'qkv' (rows NH*HD + 2N: Q, K at NH*HD, V at NH*HD + N) | 'qk' + 'v' | 'q','k','v';
          'o' [N][NH*HD] or 'attn_gate' [N][NH*HD] (used instead of 'o' when present)
    ssm:  conv f32 [2*inner], a, dt_bias f32 [32], alpha, beta f32 [32*32],
          'attn_gate' [inner][N] or None, 'ssm_out' [N][inner] or None
    dense FFN: 'gate', 'up' [FF][N], 'down' [N][FF] (or none of them: no FFN)
    MoE (model['moe'] set): 'router' f32 [E][N], 'gate_exps', 'up_exps' {e: raw [M][N]},
          'down_exps' {e: raw [N][M]}, optional 'shexp' {'g','u' [512][N], 'd' [N][512],
          'router' f32 [N]}
  moe: None or {'E', 'k', 'M', 'gq', 'uq', 'dq'}
State: {'kv': [per sequence: [per layer: (list of K rows, list of V rows)]],
        'ssm': f32 [L][32][128] (shared by the batch, as the reference keeps it)}.
"""
from __future__ import annotations

import numpy as np

from . import ops as O

SSM_GROUPS, SSM_STATE, SSM_DT_RANK = 32, 128, 32   # cengine_batch_instr.c:1253
SHEXP_FF = 512                                    # cengine_batch_instr.c:1444


def new_state(model, n_seq):
    L = model["L"]
    return {"kv": [[([], []) for _ in range(L)] for _ in range(n_seq)],
            "ssm": np.zeros((L, SSM_GROUPS, SSM_STATE), np.float32)}


def _mv(w, x, rows, cols):
    raw, qt = w
    return O.gemv(raw, qt, np.asarray(x, np.float32), rows, cols)


def forward_step(model, state, seqs, tokens, compat_xn=None):
    """One decode step: sequences ``seqs`` (indices into state['kv']) take ``tokens``.
    Returns (logits [B][V], final normalised hidden state [B][N])."""
    compat = compat_xn is not None
    L, N, NH, NKH, HD = model["L"], model["N"], model["NH"], model["NKH"], model["HD"]
    inner, kvrow = NH * HD, NKH * HD
    eps = model["eps"]
    rope_dim = model.get("rope_dim") or HD
    B = len(tokens)
    x = np.stack([model["emb"][t] for t in tokens]).astype(np.float32)
    for l in range(L):
        ly = model["layers"][l]
        xn, res = O.rms_norm(x, ly["an"], eps, sanitize=True)        # :1258-1279
        if compat:
            x, xn = xn, np.asarray(compat_xn, np.float32)
        if ly["type"] == "ssm":                                        # :1284-1320
            interm, st = O.ssm_decode_step(xn, ly["conv"], ly["a"], ly["dt_bias"], ly["alpha"], ly["beta"],
                                           state["ssm"][l], B, N, inner, SSM_GROUPS, SSM_STATE, SSM_DT_RANK)
            state["ssm"][l] = st
            gate = _mv(ly["attn_gate"], xn, inner, N) if ly.get("attn_gate") else np.zeros((B, inner))
            att = (interm.astype(np.float64) * gate).astype(np.float32)
            o = _mv(ly["ssm_out"], att, N, inner) if ly.get("ssm_out") else np.zeros((B, N))
            x = (res + o).astype(np.float32)
        else:                                                          # :1322-1400
            if ly.get("qkv"):
                qkv = _mv(ly["qkv"], xn, inner + 2 * N, N)
                q, k, v = qkv[:, :inner], qkv[:, inner:inner + kvrow], qkv[:, inner + N:inner + N + kvrow]
                if compat:
                    q = qkv.reshape(-1)[:B * inner].reshape(B, inner)
            elif ly.get("qk"):
                qk = _mv(ly["qk"], xn, inner + kvrow, N)
                q, k = qk[:, :inner], qk[:, inner:]
                if compat:
                    q = qk.reshape(-1)[:B * inner].reshape(B, inner)
                v = _mv(ly["v"], xn, kvrow, N)
            else:
                q, k, v = _mv(ly["q"], xn, inner, N), _mv(ly["k"], xn, kvrow, N), _mv(ly["v"], xn, kvrow, N)
            att = np.zeros((B, inner), np.float32)
            for b, sq in enumerate(seqs):
                ks, vs = state["kv"][sq][l]
                pos = len(ks)
                qb = O.rope_neox(q[b], NH, HD, pos, model["cos"], model["sin"], rope_dim)
                kb = O.rope_neox(k[b], NKH, HD, pos, model["cos"], model["sin"], rope_dim)
                ks.append(kb)
                vs.append(np.asarray(v[b], np.float32))
                att[b] = O.gqa_decode(qb, np.stack(ks), np.stack(vs), NH, NKH, HD, ly.get("window", 0))
            wo = ly["attn_gate"] if ly.get("attn_gate") else ly["o"]
            x = (res + _mv(wo, att, N, inner)).astype(np.float32)
        xn, res = O.rms_norm(x, ly["fn"], eps, sanitize=True)        # :1408-1427
        if compat:
            x, xn = xn, np.asarray(compat_xn, np.float32)
        moe = model.get("moe")
        if moe:                                                        # :1430-1457
            ffn = np.zeros((B, N))
            for b in range(B):
                lg = (ly["router"].astype(np.float64) @ xn[b].astype(np.float64))
                idx, w = O.router_topk(lg, moe["k"], renorm=False)
                ffn[b] = O.moe_forward(ly["gate_exps"], ly["up_exps"], ly["down_exps"],
                                       (moe["gq"], moe["uq"], moe["dq"]), xn[b], moe["M"], N, idx, w, clamp=False)
                sh = ly.get("shexp")
                if sh:
                    score = float(xn[b].astype(np.float64) @ sh["router"].astype(np.float64))
                    if score > 0:
                        g = _mv(sh["g"], xn[b], SHEXP_FF, N)[0].astype(np.float64)
                        u = _mv(sh["u"], xn[b], SHEXP_FF, N)[0].astype(np.float64)
                        h = (u / (1 + np.exp(-u))) * g
                        ffn[b] += score * _mv(sh["d"], h, N, SHEXP_FF)[0]
            x = (res + ffn).astype(np.float32)
        elif ly.get("gate"):                                           # :1458-1466
            FF = model["FF"]
            g = _mv(ly["gate"], xn, FF, N).astype(np.float64)
            u = _mv(ly["up"], xn, FF, N).astype(np.float64)
            h = (g / (1 + np.exp(-g))) * u
            x = (res + _mv(ly["down"], h, N, FF)).astype(np.float32)
        elif not compat:
            x = res
    h, _ = O.rms_norm(x, model["onw"], eps, sanitize=True)           # :1469-1489
    return _mv(model["wout"], h, model["V"], N), h


def forward_sequence(model, tokens):
    """Teacher-forced decode of a dense-attention model: ``tokens`` [P][B] are fed one
    position at a time from an empty cache, exactly as P consecutive ``forward_step``
    calls (cengine_batch_instr.c:1233-1493, default data flow) would; returns the logits
    of every position [P][B][V].  Each layer is computed for all P*B rows at once
    (position p attends to positions 0..p of its own sequence), so every weight matrix is
    decoded once per call instead of once per position.  Attention layers with
    separate / QK-fused / QKV-fused projections and dense SwiGLU FFNs only (no SSM, no
    MoE).  Checked against forward_step in tests/test_model_oracle.py."""
    L, N, NH, NKH, HD = model["L"], model["N"], model["NH"], model["NKH"], model["HD"]
    inner, kvrow = NH * HD, NKH * HD
    eps = model["eps"]
    rope_dim = model.get("rope_dim") or HD
    tok = np.asarray(tokens, np.int64)
    P, B = tok.shape
    R = P * B                                                  # row r = p * B + b
    x = model["emb"][tok.reshape(-1)].astype(np.float32)
    if model.get("moe"):
        raise ValueError("forward_sequence: dense models only")
    for l in range(L):
        ly = model["layers"][l]
        if ly["type"] != "attn":
            raise ValueError("forward_sequence: attention layers only")
        xn, res = O.rms_norm(x, ly["an"], eps, sanitize=True)
        if ly.get("qkv"):
            qkv = _mv(ly["qkv"], xn, inner + 2 * N, N)
            q, k, v = qkv[:, :inner], qkv[:, inner:inner + kvrow], qkv[:, inner + N:inner + N + kvrow]
        elif ly.get("qk"):
            qk = _mv(ly["qk"], xn, inner + kvrow, N)
            q, k = qk[:, :inner], qk[:, inner:]
            v = _mv(ly["v"], xn, kvrow, N)
        else:
            q, k, v = _mv(ly["q"], xn, inner, N), _mv(ly["k"], xn, kvrow, N), _mv(ly["v"], xn, kvrow, N)
        qr = np.empty((R, inner), np.float32)
        kr = np.empty((R, kvrow), np.float32)
        for r in range(R):
            pos = r // B
            qr[r] = O.rope_neox(q[r], NH, HD, pos, model["cos"], model["sin"], rope_dim)
            kr[r] = O.rope_neox(k[r], NKH, HD, pos, model["cos"], model["sin"], rope_dim)
        vr = np.asarray(v, np.float32)
        att = np.zeros((R, inner), np.float32)
        for b in range(B):
            ks, vs = kr[b::B], vr[b::B]                        # positions 0..P-1 of sequence b
            for p in range(P):
                att[p * B + b] = O.gqa_decode(qr[p * B + b], ks[:p + 1], vs[:p + 1], NH, NKH, HD)
        wo = ly["attn_gate"] if ly.get("attn_gate") else ly["o"]
        x = (res + _mv(wo, att, N, inner)).astype(np.float32)
        xn, res = O.rms_norm(x, ly["fn"], eps, sanitize=True)
        if ly.get("gate"):
            FF = model["FF"]
            g = _mv(ly["gate"], xn, FF, N).astype(np.float64)
            u = _mv(ly["up"], xn, FF, N).astype(np.float64)
            h = (g / (1 + np.exp(-g))) * u
            x = (res + _mv(ly["down"], h, N, FF)).astype(np.float32)
        else:
            x = res
    h, _ = O.rms_norm(x, model["onw"], eps, sanitize=True)
    return _mv(model["wout"], h, model["V"], N).reshape(P, B, model["V"])


# ------------------------------------------------------------------ qwen36_batch_forward
def qwen36_new_state(model):
    L, n_kv = model["L"], model["NKH"] * model["HD"]
    return {"kv_k": np.zeros((L, model["max_ctx"], n_kv), np.float32),
            "kv_v": np.zeros((L, model["max_ctx"], n_kv), np.float32),
            "kv_lens": np.zeros(L, np.int32),
            "ssm": np.zeros((L, model["ssm_groups"], model["ssm_state"]), np.float32)}


def qwen36_step(model, state, tokens):
    """One qwen36_batch_forward call (cengine_batch_instr.c:859-1231) for tokens [B].

    x stays the residual (the norm clamps only its own output, :996-1002); attention layers
    read Q at 0, K at NH*HD and V half-way through the non-Q part of the projection; every
    token writes its K/V to slot kv_lens[l] of the shared flat cache (the last token's row
    stays) and attends over slots 0..pos-1 plus its own row (:1055-1079); MoE: router,
    softmax, insertion top-k, renormalised weights (:1113-1152), moe_forward_omp with the
    +-80 SiLU clamp (:1169), shared expert silu(clamp(gate)) * up scaled by its positive
    router score (:1178-1207); final norm and logits (:1222-1227).  kv_lens is not advanced
    (the caller does that).  Returns (logits [B][V], x before the final norm [B][N])."""
    L, N, NH, NKH, HD = model["L"], model["N"], model["NH"], model["NKH"], model["HD"]
    inner, n_kv = NH * HD, NKH * HD
    eps = model["eps"]
    rope_dim = model.get("rope_dim") or HD
    B = len(tokens)
    x = np.stack([model["emb"][t] for t in tokens]).astype(np.float32)
    for l in range(L):
        ly = model["layers"][l]
        xn, _ = O.rms_norm(x, ly["an"], eps, sanitize=True)
        if ly["type"] == "ssm":
            IN = model["ssm_inner"]
            interm, st = O.ssm_decode_step(xn, ly["conv"], ly["a"], ly["dt_bias"], ly["alpha"], ly["beta"],
                                           state["ssm"][l], B, N, IN, model["ssm_groups"], model["ssm_state"],
                                           model["ssm_dt_rank"])
            state["ssm"][l] = st
            att = (interm.astype(np.float64) * _mv(ly["attn_gate"], xn, IN, N)).astype(np.float32)
            x = (x + _mv(ly["ssm_out"], att, N, IN)).astype(np.float32)
        else:
            nq = ly["qkv_rows"]
            qkv = _mv(ly["qkv"], xn, nq, N)
            voff = inner + (nq - inner) // 2
            pos = int(state["kv_lens"][l])
            att = np.zeros((B, inner), np.float32)
            for b in range(B):
                qb = O.rope_neox(qkv[b, :inner], NH, HD, pos, model["cos"], model["sin"], rope_dim)
                kb = O.rope_neox(qkv[b, inner:inner + n_kv], NKH, HD, pos, model["cos"], model["sin"], rope_dim)
                vb = qkv[b, voff:voff + n_kv]
                ks = np.concatenate([state["kv_k"][l, :pos], kb[None]])
                vs = np.concatenate([state["kv_v"][l, :pos], vb[None]])
                att[b] = O.gqa_decode(qb, ks, vs, NH, NKH, HD)
                state["kv_k"][l, pos], state["kv_v"][l, pos] = kb, vb
            x = (x + _mv(ly["o"], att, N, inner)).astype(np.float32)
        xn, _ = O.rms_norm(x, ly["fn"], eps, sanitize=True)
        moe = model.get("moe")
        if moe and ly.get("router") is not None:
            ffn = np.zeros((B, N))
            for b in range(B):
                lg = ly["router"].astype(np.float64) @ xn[b].astype(np.float64)
                idx, w = O.router_topk(lg, moe["k"], renorm=True)
                ffn[b] = O.moe_forward(ly["gate_exps"], ly["up_exps"], ly["down_exps"],
                                       (moe["gq"], moe["uq"], moe["dq"]), xn[b], moe["M"], N, idx, w, clamp=True)
                sh = ly.get("shexp")
                if sh:
                    score = float(xn[b].astype(np.float64) @ sh["router"].astype(np.float64))
                    if score > 0:
                        si = sh["si"]
                        g = _mv(sh["g"], xn[b], si, N)[0].astype(np.float64)
                        u = _mv(sh["u"], xn[b], si, N)[0].astype(np.float64)
                        ffn[b] += score * _mv(sh["d"], O.silu_clamped(g) * u, N, si)[0]
            x = (x + ffn).astype(np.float32)
    h, _ = O.rms_norm(x, model["onw"], eps, sanitize=True)
    return _mv(model["wout"], h, model["V"], N), x
