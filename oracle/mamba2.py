"""Mamba-2 decode step (selective state-space update), restated in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  The reference has no real Mamba-2:
its ``ssm_decode_step`` (cengine_batch_instr.c:736-797) is a toy that the library keeps
byte-compatible under its own name.  This is the published Mamba-2 recurrence (Dao & Gu,
"Transformers are SSMs", 2024) as the hybrid model of config 5 needs it, one token per
sequence:

  proj = W_in u                                    -> z [d_inner] | xBC [conv_dim] | dt [H]
  conv: window = last d_conv inputs of xBC (newest last); a = silu(b + sum_k w[:, k] window[:, k])
  a -> x [H][P] | B [G][S] | C [G][S]           (head h reads group h // (H / G))
  dt_h = softplus(dt_h + dt_bias_h), clamped to dt_limit; A_h = -exp(A_log_h)
  state[h] = exp(dt_h A_h) state[h] + dt_h x[h] B[g]^T          ([P][S])
  y[h] = state[h] C[g] + D_h x[h]
  out = W_out (norm_w * rmsnorm(y * silu(z)))     (RMS over groups of norm_group elements)

Pinned against an independent implementation: the plain-torch Mamba2Mixer of Hugging Face
transformers 5.5.0 run in float64 (tests/golden/gen_mamba2.py writes tests/golden/
mamba2.npz: its first token goes through transformers' chunked SSD path, later tokens
through its recurrent decode path; tests/test_mamba2.py checks this file against both).
Shapes: conv_state [B][conv_dim][d_conv], ssm_state [B][H][P][S]."""
from __future__ import annotations

import numpy as np


def softplus(x):
    x = np.asarray(x, np.float64)
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def silu(x):
    x = np.asarray(x, np.float64)
    return x / (1.0 + np.exp(-x))


def mamba2_step(xbc, z, dt, conv_state, conv_w, conv_b, A_log, dt_bias, D, norm_w, ssm_state, H, P, S, G,
                eps=1e-5, norm_group=None, dt_limit=(0.0, np.inf)):
    """One token per sequence.  xbc [B][conv_dim], z [B][H*P] or None, dt [B][H].
    conv_state [B][conv_dim][d_conv] and ssm_state [B][H][P][S] are updated in place (float32
    arrays, as the device keeps them).  norm_w None: no norm (y * silu(z) when z is given).
    Returns y [B][H*P] (float32)."""
    xbc = np.asarray(xbc, np.float64)
    Bn, conv_dim = xbc.shape
    d_inner = H * P
    conv_state[:, :, :-1] = conv_state[:, :, 1:]
    conv_state[:, :, -1] = xbc
    acc = (conv_state.astype(np.float64) * np.asarray(conv_w, np.float64)[None]).sum(-1)
    if conv_b is not None:
        acc = acc + np.asarray(conv_b, np.float64)
    a = silu(acc)
    x = a[:, :d_inner].reshape(Bn, H, P)
    Bm = a[:, d_inner:d_inner + G * S].reshape(Bn, G, S)
    Cm = a[:, d_inner + G * S:d_inner + 2 * G * S].reshape(Bn, G, S)
    dtv = np.clip(softplus(np.asarray(dt, np.float64) + np.asarray(dt_bias, np.float64)), dt_limit[0], dt_limit[1])
    A = -np.exp(np.asarray(A_log, np.float64))
    rep = H // G
    y = np.zeros((Bn, H, P))
    for b in range(Bn):
        for h in range(H):
            g = h // rep
            st = ssm_state[b, h].astype(np.float64) * np.exp(dtv[b, h] * A[h]) + dtv[b, h] * np.outer(x[b, h], Bm[b, g])
            ssm_state[b, h] = st
            y[b, h] = st @ Cm[b, g] + (0.0 if D is None else float(D[h])) * x[b, h]
    y = y.reshape(Bn, d_inner)
    if z is not None:
        y = y * silu(z)
    if norm_w is not None:
        gs = norm_group or d_inner
        yg = y.reshape(Bn, d_inner // gs, gs)
        yg = yg / np.sqrt((yg ** 2).mean(-1, keepdims=True) + eps)
        y = yg.reshape(Bn, d_inner) * np.asarray(norm_w, np.float64)
    return y.astype(np.float32)


def mamba2_layer_step(u, W_in, W_out, conv_state, ssm_state, p, eps=1e-5, norm_group=None):
    """The mixer for one token per sequence: u [B][hidden] -> out [B][hidden], with W_in
    [d_inner + conv_dim + H][hidden] (rows z | xBC | dt) and W_out [hidden][d_inner] as
    float arrays, p = dict(H, P, S, G, conv_w, conv_b, A_log, dt_bias, D, norm_w)."""
    H, P, S, G = p["H"], p["P"], p["S"], p["G"]
    d_inner, conv_dim = H * P, H * P + 2 * G * S
    proj = np.asarray(u, np.float64) @ np.asarray(W_in, np.float64).T
    z, xbc, dt = proj[:, :d_inner], proj[:, d_inner:d_inner + conv_dim], proj[:, d_inner + conv_dim:]
    y = mamba2_step(xbc, z, dt, conv_state, p["conv_w"], p["conv_b"], p["A_log"], p["dt_bias"], p["D"],
                    p["norm_w"], ssm_state, H, P, S, G, eps=eps, norm_group=norm_group)
    return (y.astype(np.float64) @ np.asarray(W_out, np.float64).T).astype(np.float32)
