"""Per-op CPU restatements of the reference C engine's math (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Each function names the
reference code it restates.  Dot products are accumulated in float64 so the
oracle is at least as accurate as the reference's fp32 accumulation; the parity
bar for fp32-accumulated GPU outputs is relative L2 <= 1e-3.
"""
from __future__ import annotations

import numpy as np

from . import formats as F


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def gemv(w_raw: np.ndarray, qt: int, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """out[b][r] = sum_k W[r][k] * x[b][k] with W decoded exactly (float64 accumulate).

    The math every *_matmul_omp / *_batch_matmul of the reference computes where it is
    correct (quant_kernels_omp.c:135-734, cengine_batch_instr.c:68-534): x [B][K],
    out [B][N] (cengine_batch_instr.c:251)."""
    w = F.dequantize(qt, w_raw, n_rows * n_cols).reshape(n_rows, n_cols).astype(np.float64)
    xb = np.asarray(x, np.float64).reshape(-1, n_cols)
    return (xb @ w.T).astype(np.float32)


def rms_norm(x, w, eps, sanitize=False):
    """simd_ops.c:35 / quant_kernels_omp.c:956 (eps 1e-5); sanitize = the batch engine's
    RMS_NORM_SIMD (cengine_batch_instr.c:1258-1279): NaN -> 0, clamp +-1000 first.
    Returns (out, clamped input)."""
    x = np.asarray(x, np.float32).copy()
    if sanitize:
        x = np.where(np.isnan(x), np.float32(0), x)
        x = np.clip(x, -1000, 1000).astype(np.float32)
    ss = (x.astype(np.float64) ** 2).sum(axis=-1, keepdims=True)
    inv = 1.0 / np.sqrt(ss / x.shape[-1] + eps)
    out = (x * inv) * (np.ones(x.shape[-1]) if w is None else np.asarray(w, np.float64))
    return out.astype(np.float32), x


def silu(x, mode=0):
    """mode 0: x/(1+exp(-x)) (quant_kernels_omp.c:981); mode 1: simd_ops.c:56 -- Pade
    tanh on the first n - n%8 elements, exact on the tail."""
    x = np.asarray(x, np.float64)
    exact = x / (1.0 + np.exp(-x))
    if mode == 0:
        return exact.astype(np.float32)
    n = x.size
    body = n - n % 8
    h = x[:body] * 0.5
    v2 = h * h
    t = h * (27 + v2) / (27 + 9 * v2)
    out = exact.copy()
    out[:body] = x[:body] * (0.5 + 0.5 * t)
    return out.astype(np.float32)


def swiglu(g, u):
    """quant_kernels_omp.c:2157-2164: silu(clamp(g, -80, 80)) * u."""
    g = np.clip(np.asarray(g, np.float64), -80, 80)
    return (g / (1 + np.exp(-g)) * np.asarray(u, np.float64)).astype(np.float32)


def softmax(x):
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def rope_interleaved(q, k, n_heads, n_kv, hd, pos, base):
    """simd_ops.c:122 apply_rope: pairs (d, d+1), freq = 1/base^((d/2)/(hd/2))."""
    def rot(v, nh):
        v = np.asarray(v, np.float64).reshape(nh, hd).copy()
        d = np.arange(0, hd, 2)
        ang = pos * (1.0 / np.power(base, (d // 2) / (hd // 2)))
        c, s = np.cos(ang), np.sin(ang)
        a0, a1 = v[:, 0::2].copy(), v[:, 1::2].copy()
        v[:, 0::2] = a0 * c - a1 * s
        v[:, 1::2] = a0 * s + a1 * c
        return v.reshape(-1).astype(np.float32)
    return rot(q, n_heads), rot(k, n_kv)


def rope_tables(max_ctx, hd, rope_dim, base=10000.0):
    """cengine_batch_instr.c:674 rope_init: theta = pos / base^(2j/hd), j < rope_dim/2."""
    j = np.arange(rope_dim // 2)
    pos = np.arange(max_ctx)[:, None]
    theta = pos / np.power(base, 2.0 * j / hd)
    return np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)


def rope_neox(buf, n_heads, hd, pos, cos_t, sin_t, rope_dim):
    """cengine_batch_instr.c:686 rope_apply: rotate (x[j], x[j + rope_dim/2]) of each head."""
    b = np.asarray(buf, np.float64).reshape(n_heads, hd).copy()
    hd2 = rope_dim // 2
    c, s = cos_t[pos, :hd2].astype(np.float64), sin_t[pos, :hd2].astype(np.float64)
    a0, a1 = b[:, :hd2].copy(), b[:, hd2:2 * hd2].copy()
    b[:, :hd2] = a0 * c - a1 * s
    b[:, hd2:2 * hd2] = a1 * c + a0 * s
    return b.reshape(-1).astype(np.float32)


def gqa_decode(q, k, v, n_head, n_kv, hd, window=0):
    """Decode attention of one query per head over a flat KV [seq][n_kv*hd]
    (gqa_attention.c:93-135, cengine_batch_instr.c:141-158): head h uses KV head
    h // (n_head // n_kv); scores scaled by 1/sqrt(hd); softmax; P.V.  window > 0
    keeps the last `window` positions."""
    q = np.asarray(q, np.float64).reshape(n_head, hd)
    k = np.asarray(k, np.float64).reshape(-1, n_kv, hd)
    v = np.asarray(v, np.float64).reshape(-1, n_kv, hd)
    sl = k.shape[0]
    lo = sl - window if (window and sl > window) else 0
    rep = n_head // n_kv
    out = np.zeros((n_head, hd))
    for h in range(n_head):
        g = h // rep
        s = k[lo:, g, :] @ q[h] / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h] = p @ v[lo:, g, :]
    return out.reshape(-1).astype(np.float32)


class PagedKV:
    """The reference's page table semantics (cengine_batch_instr.c:173-202): LIFO free
    list starting at page 0, logical -> physical table, pages [n_pages][page_size][row]."""

    def __init__(self, n_pages, page_size, row):
        self.page_size, self.row = page_size, row
        self.k = np.zeros((n_pages, page_size, row), np.float32)
        self.v = np.zeros_like(self.k)
        self.free = list(range(n_pages - 1, -1, -1))
        self.tables = {}

    def alloc(self):
        return self.free.pop() if self.free else -1

    def write(self, seq, pos, krow, vrow):
        t = self.tables.setdefault(seq, {})
        blk, off = divmod(pos, self.page_size)
        if blk not in t:
            t[blk] = self.alloc()
        self.k[t[blk], off] = krow
        self.v[t[blk], off] = vrow

    def gather(self, seq, length):
        t = self.tables[seq]
        ks = np.stack([self.k[t[p // self.page_size], p % self.page_size] for p in range(length)])
        vs = np.stack([self.v[t[p // self.page_size], p % self.page_size] for p in range(length)])
        return ks, vs


def _exp_ps_simd_ref(x):
    """The reference's exp_ps_simd (gqa_attention.c:32-48) as it computes: n = rint(x*log2e
    + 0.5), f = x*log2e - n, then a Horner chain that starts at 1 and adds the Taylor
    coefficients of 2^f in reverse order (0.693, 0.240, 0.0555, 0.00962, 0.00133), times
    2^n.  It is not exp(x) (p(0) = 0.00133); this models the reference, not the math."""
    x = np.asarray(x, np.float32)
    t = (x * np.float32(1.4426950408889634)).astype(np.float32)
    n = np.rint((t + np.float32(0.5)).astype(np.float32)).astype(np.int32)
    f = (t - n.astype(np.float32)).astype(np.float32)
    p = np.ones_like(f)
    for c in (0.6931471805599453, 0.2402265069591007, 0.0555041086648216, 0.0096181291076285,
              0.0013333558146428):
        p = (p * f + np.float32(c)).astype(np.float32)
    biased = np.clip(n + 127, 0, 255).astype(np.uint32)
    return (p * (biased << np.uint32(23)).view(np.float32)).astype(np.float32)


def gqa_decode_reference_quirk(q, k, v, n_head, n_kv, hd):
    """gqa_attention_decode exactly as the reference computes it single-threaded
    (gqa_attention.c:50-135): fp32 scores, softmax_simd with exp_ps_simd on the first
    seq_len - seq_len%8 scores (clamped to [-80, 80] after the max shift), expf on the
    tail, 1/(sum + 1e-10).  Used only to show the deviation is understood."""
    q = np.asarray(q, np.float32).reshape(n_head, hd)
    k = np.asarray(k, np.float32).reshape(-1, n_kv, hd)
    v = np.asarray(v, np.float32).reshape(-1, n_kv, hd)
    sl = k.shape[0]
    rep = n_head // n_kv
    body = sl - sl % 8
    out = np.zeros((n_head, hd), np.float64)
    for h in range(n_head):
        g = h // rep
        s = ((k[:, g, :].astype(np.float64) @ q[h].astype(np.float64)).astype(np.float32)
             * np.float32(1.0 / np.sqrt(np.float32(hd)))).astype(np.float32)
        m = s.max()
        e = np.empty(sl, np.float32)
        e[:body] = _exp_ps_simd_ref(np.clip(s[:body] - m, -80, 80))
        e[body:] = np.minimum(np.exp((s[body:] - m).astype(np.float64)), 1e38).astype(np.float32)
        p = e / (e.astype(np.float64).sum() + 1e-10)
        out[h] = p @ v[:, g, :].astype(np.float64)
    return out.reshape(-1).astype(np.float32)


def silu_clamped(g):
    g = np.clip(np.asarray(g, np.float64), -80, 80)
    return g / (1 + np.exp(-g))


def moe_forward(gate, up, down, qts, x, n_ff, n_embd, idx, w, clamp=True):
    """moe_forward_omp (quant_kernels_omp.c:2066-2250) where it is W.x: for each selected
    expert e = idx[i]: h = silu(clamp(gate_e x, +-80)) * (up_e x); combined += w[i] * down_e h.
    clamp=False: the batch engine's moe_ffn (cengine_batch_instr.c:648-663), no clamp.
    gate/up/down: dict expert -> raw bytes; fp64 accumulation."""
    qg, qu, qd = qts
    x = np.asarray(x, np.float64)
    out = np.zeros(n_embd)
    for i, e in enumerate(idx):
        g = gemv(gate[e], qg, x, n_ff, n_embd)[0].astype(np.float64)
        u = gemv(up[e], qu, x, n_ff, n_embd)[0].astype(np.float64)
        h = (silu_clamped(g) if clamp else g / (1 + np.exp(-g))) * u
        out += float(w[i]) * gemv(down[e], qd, h, n_embd, n_ff)[0].astype(np.float64)
    return out.astype(np.float32)


def router_topk(logits, k, renorm):
    """cengine_batch_instr.c:1116-1152 / gptoss_batch_forward.c:53-93: softmax with
    1/(sum + 1e-10), insertion top-k (strictly greater wins: ties keep the lower index),
    optional renormalisation with 1/(sum + 1e-10)."""
    lg = np.asarray(logits, np.float64)
    p = np.exp(lg - lg.max())
    p = p / (p.sum() + 1e-10)
    order = sorted(range(len(p)), key=lambda e: (-p[e], e))[:k]
    w = p[order]
    if renorm:
        w = w / (w.sum() + 1e-10)
    return np.array(order, np.int32), w.astype(np.float32)


def ssm_decode_step(x, conv_w, a, dt_bias, alpha, beta, state, B, N, inner, groups, state_size, dt_rank):
    """cengine_batch_instr.c:736-797 as the reference computes it (see its docstring in
    mojollama_b200/csrc/ssm.cu): returns (interm [B][inner], new state)."""
    x = np.asarray(x, np.float64).reshape(B, N)
    st = np.asarray(state, np.float64).reshape(groups, state_size).copy()
    interm = np.zeros((B, inner))
    for b in range(B):
        conv = np.array([x[b, i % N] * conv_w[i] for i in range(2 * inner)])
        g = conv[:inner]
        interm[b] = g / (1 + np.exp(-g)) * conv[inner:]
        xi = np.array([x[b, j % N] for j in range(dt_rank)])
        for grp in range(groups):
            dt = dt_bias[grp] + np.dot(alpha[grp * dt_rank:(grp + 1) * dt_rank], xi)
            dt = dt if dt > 20 else np.log1p(np.exp(dt))
            bx = np.dot(beta[grp * dt_rank:(grp + 1) * dt_rank], xi) * dt
            st[grp] *= np.exp(a[grp] * dt)
            st[grp, 0] += bx
    return interm.astype(np.float32), st.astype(np.float32)
