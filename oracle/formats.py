"""GGUF block formats the reference C engine decodes -- numpy restatement (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the product never imports this.

Each decoder follows the reference's own scalar decode and gguf-py 0.19.0 in the
same float32 operation order, so the outputs are bit-identical:

  Q8_0   34 B / 32   d:f16, qs:i8[32]            v = qs*d
         quant_kernels_omp.c:868-879 (q8_0_dequantize_row)
  Q4_0   18 B / 32   d:f16, qs:u8[16]            v = (nib-8)*d, lo nib -> j, hi -> j+16
         quant_kernels_omp.c:77-93 (decode_q4_0), cengine_batch_instr.c:125-138 (q4d)
  Q4_1   20 B / 32   d:f16, m:f16, qs:u8[16]     v = nib*d + m
         quant_kernels_omp.c:95-113 (decode_q4_1)
  Q5_0   22 B / 32   d:f16, qh:u32, qs:u8[16]    v = ((nib | hbit<<4) - 16)*d   (GGUF order:
         lo nib -> j, hi nib -> j+16; the reference's q5_0_row_dot,
         quant_kernels_omp.c:1244-1256, interleaves nibbles instead -- a deviation)
  Q4_K  144 B / 256  d,dmin:f16, scales:u8[12], qs:u8[128]
         v = (d*sc)*nib - (dmin*m); quant_kernels_omp.c:62-70 (get_scale_min_k4), 804-828
  Q5_K  176 B / 256  d,dmin:f16, scales:u8[12], qh:u8[32], qs:u8[128]
         quant_kernels_omp.c:830-866 (q5_k_dequantize_row)
  Q6_K  210 B / 256  ql:u8[128], qh:u8[64], sc:i8[16], d:f16 (at byte 208)
         v = (d*sc[i/16])*(q6-32); quant_kernels_omp.c:762-798 (q6_k_dequantize_row)
  MXFP4  17 B / 32   e:u8 (byte 0), qs:u8[16]    v = kval[nib] * 2^(e-128),
         kval = doubled E2M1 {0,1,2,3,4,6,8,12,-0,-1,...}, lo nib -> j, hi -> j+16
         (GGUF / gguf-py MXFP4, type 39)
  MXFP4_REF 17 B / 32  qs:u8[16], e:u8 (byte 16)  v = sext4(nib) * 2^(e-127),
         element 2i = lo nib of byte i, 2i+1 = hi nib -- the layout the reference's
         C decoder actually reads for type 39 (quant_kernels_omp.c:486-573).
  F32, F16, BF16     plain arrays (BF16/F16 are not in the reference's dispatcher,
         quant_kernels_omp.c:1355-1388; they are added for the bf16 attention weights).
"""
from __future__ import annotations

import numpy as np

# ggml / GGUF type codes (quant_kernels_omp.c:6-14); MXFP4_REF is a private code for
# the reference's own 17-byte MXFP4 layout so that both layouts can be addressed.
F32, F16, Q4_0, Q4_1, Q5_0, Q8_0 = 0, 1, 2, 3, 6, 8
Q4_K, Q5_K, Q6_K, BF16, MXFP4 = 12, 13, 14, 30, 39
MXFP4_REF = 1039

# (elements per block, bytes per block)
BLOCK = {
    F32: (1, 4), F16: (1, 2), BF16: (1, 2),
    Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q8_0: (32, 34),
    Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
    MXFP4: (32, 17), MXFP4_REF: (32, 17),
}
NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0",
         Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", MXFP4: "MXFP4",
         MXFP4_REF: "MXFP4_REF"}
BY_NAME = {v: k for k, v in NAMES.items()}

MXFP4_KVALUES = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], np.int8)


def row_bytes(qt: int, k: int) -> int:
    be, bb = BLOCK[qt]
    if k % be:
        raise ValueError(f"{NAMES[qt]} needs K % {be} == 0, got K={k}")
    return (k // be) * bb


def _f16(u8pair: np.ndarray) -> np.ndarray:
    """(..., 2) little-endian bytes -> float32 via IEEE half (exact)."""
    return np.ascontiguousarray(u8pair).view(np.float16)[..., 0].astype(np.float32)


def _blocks(raw: np.ndarray, n: int, qt: int) -> np.ndarray:
    be, bb = BLOCK[qt]
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    nb = n // be
    if raw.size < nb * bb:
        raise ValueError("buffer too small")
    return raw[: nb * bb].reshape(nb, bb)


def scale_min_k4(scales: np.ndarray):
    """6-bit (scale, min) pairs of a K-quant super-block.

    Follows get_scale_min_k4 (quant_kernels_omp.c:62-70): pairs 0..3 are the low
    6 bits of bytes 0..3 / 4..7; pairs 4..7 take a low nibble from bytes 8..11 and
    the top two bits of bytes 0..3 / 4..7.  scales: (nb, 12) uint8 -> two (nb, 8).
    """
    q = scales.astype(np.uint8)
    sc = np.empty(q.shape[:-1] + (8,), np.uint8)
    mn = np.empty_like(sc)
    for j in range(4):
        sc[..., j] = q[..., j] & 63
        mn[..., j] = q[..., j + 4] & 63
    for j in range(4, 8):
        sc[..., j] = (q[..., j + 4] & 0xF) | ((q[..., j - 4] >> 6) << 4)
        mn[..., j] = (q[..., j + 4] >> 4) | ((q[..., j] >> 6) << 4)
    return sc, mn


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of scale_min_k4 for values in [0, 63]."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    q = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    for j in range(4):
        q[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        q[..., j + 4] = (mn[..., j] & 63) | ((mn[..., j + 4] >> 4) << 6)
        q[..., j + 8] = (sc[..., j + 4] & 0xF) | ((mn[..., j + 4] & 0xF) << 4)
    return q


def mxfp4_half_scale(e: np.ndarray) -> np.ndarray:
    """2^(e-128) as float32, exact for every byte e (denormal for e < 2)."""
    e = e.astype(np.uint32)
    bits = np.where(e < 2, np.uint32(0x00200000) << e, (e - 1) << np.uint32(23)).astype(np.uint32)
    return bits.view(np.float32)


# ----------------------------------------------------------------------------- dequantize

def dequantize(qt: int, raw, n: int) -> np.ndarray:
    """Decode n elements of type qt from raw bytes into float32 (bit-exact)."""
    raw = np.asarray(raw)
    if qt == F32:
        return np.ascontiguousarray(raw).view(np.uint8).reshape(-1)[: 4 * n].view(np.float32).copy()
    if qt == F16:
        return np.ascontiguousarray(raw).view(np.uint8).reshape(-1)[: 2 * n].view(np.float16).astype(np.float32)
    if qt == BF16:
        u16 = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)[: 2 * n].view(np.uint16)
        return (u16.astype(np.uint32) << 16).view(np.float32)
    b = _blocks(raw, n, qt)
    nb = b.shape[0]
    if qt == Q8_0:
        d = _f16(b[:, 0:2])[:, None]
        q = b[:, 2:34].view(np.int8).astype(np.float32)
        return (q * d).reshape(-1)
    if qt in (Q4_0, Q4_1, Q5_0):
        hdr = {Q4_0: 2, Q4_1: 4, Q5_0: 6}[qt]
        qs = b[:, hdr:hdr + 16]
        nib = np.concatenate([qs & 0xF, qs >> 4], axis=1).astype(np.int32)   # j, j+16
        d = _f16(b[:, 0:2])[:, None]
        if qt == Q4_0:
            return ((nib - 8).astype(np.float32) * d).reshape(-1)
        if qt == Q4_1:
            m = _f16(b[:, 2:4])[:, None]
            return (nib.astype(np.float32) * d + m).reshape(-1)
        qh = np.ascontiguousarray(b[:, 2:6]).view(np.uint32)[:, 0]
        hb = ((qh[:, None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.int32)
        return (((nib | (hb << 4)) - 16).astype(np.float32) * d).reshape(-1)
    if qt in (Q4_K, Q5_K):
        d = _f16(b[:, 0:2])[:, None]
        dmin = _f16(b[:, 2:4])[:, None]
        sc, mn = scale_min_k4(b[:, 4:16])
        ds = d * sc.astype(np.float32)        # (nb, 8)   d1 = d * sc
        dm = dmin * mn.astype(np.float32)     #           m1 = min * m
        qs = b[:, 16:144] if qt == Q4_K else b[:, 48:176]
        qs = qs.reshape(nb, 4, 32)
        q = np.empty((nb, 8, 32), np.int32)
        q[:, 0::2] = qs & 0xF
        q[:, 1::2] = qs >> 4
        if qt == Q5_K:
            qh = b[:, 16:48]
            for g in range(4):
                q[:, 2 * g] += ((qh >> (2 * g)) & 1).astype(np.int32) << 4
                q[:, 2 * g + 1] += ((qh >> (2 * g + 1)) & 1).astype(np.int32) << 4
        return (ds[:, :, None] * q.astype(np.float32) - dm[:, :, None]).reshape(-1)
    if qt == Q6_K:
        ql = b[:, 0:128].reshape(nb, 2, 64)
        qh = b[:, 128:192].reshape(nb, 2, 32)
        sc = b[:, 192:208].view(np.int8).astype(np.float32)
        d = _f16(b[:, 208:210])[:, None]
        q = np.empty((nb, 2, 4, 32), np.int32)
        q[:, :, 0] = (ql[:, :, 0:32] & 0xF) | ((qh & 3) << 4)
        q[:, :, 1] = (ql[:, :, 32:64] & 0xF) | (((qh >> 2) & 3) << 4)
        q[:, :, 2] = (ql[:, :, 0:32] >> 4) | (((qh >> 4) & 3) << 4)
        q[:, :, 3] = (ql[:, :, 32:64] >> 4) | (((qh >> 6) & 3) << 4)
        q = (q - 32).reshape(nb, 16, 16).astype(np.float32)
        ds = (d * sc)[:, :, None]
        return (ds * q).reshape(-1)
    if qt == MXFP4:
        s = mxfp4_half_scale(b[:, 0])[:, None]
        qs = b[:, 1:17]
        nib = np.concatenate([qs & 0xF, qs >> 4], axis=1)
        return (MXFP4_KVALUES[nib].astype(np.float32) * s).reshape(-1)
    if qt == MXFP4_REF:
        qs = b[:, 0:16]
        s = (b[:, 16].astype(np.uint32) << np.uint32(23)).view(np.float32)[:, None]
        nib = np.empty((nb, 32), np.int32)
        nib[:, 0::2] = qs & 0xF
        nib[:, 1::2] = qs >> 4
        v = np.where(nib > 7, nib - 16, nib).astype(np.float32)
        return (v * s).reshape(-1)
    raise ValueError(f"unsupported type {qt}")


# ----------------------------------------------------------------------------- quantize

def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """The reference's Q8_0 activation quantizer (quantize_row_q8_0,
    quant_kernels_omp.c:1406-1455): d = amax/127 (1 if 0), id = 1/d,
    q = round-half-even(clamp(x*id, -127, 127)), d stored as f16 (RNE)."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    d = np.where(d == 0, np.float32(1.0), d).astype(np.float32)
    idv = (np.float32(1.0) / d).astype(np.float32)
    v = np.clip(x * idv[:, None], np.float32(-127), np.float32(127))
    q = np.rint(v).astype(np.int8)
    out = np.empty((x.shape[0], 34), np.uint8)
    out[:, 0:2] = d.astype(np.float16)[:, None].view(np.uint8)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """GGUF Q4_0 rule (gguf-py Q4_0.quantize_blocks): d = x[argmax|x|] / -8,
    q = trunc(x/d + 8.5) clipped to [0, 15]."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    imax = np.abs(x).argmax(axis=1)[:, None]
    mx = np.take_along_axis(x, imax, axis=1)
    d = (mx / np.float32(-8)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    q = np.trunc(x * idv + np.float32(8.5)).astype(np.int32).clip(0, 15).astype(np.uint8)
    out = np.empty((x.shape[0], 18), np.uint8)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def quantize_q4_1(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32).reshape(-1, 32)
    lo = x.min(axis=1)
    hi = x.max(axis=1)
    d = ((hi - lo) / 15).astype(np.float16)
    m = lo.astype(np.float16)
    df = d.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(df > 0, np.rint((x - m.astype(np.float32)[:, None]) / df), 0)
    q = q.clip(0, 15).astype(np.uint8)
    out = np.empty((x.shape[0], 20), np.uint8)
    out[:, 0:2] = d[:, None].view(np.uint8)
    out[:, 2:4] = m[:, None].view(np.uint8)
    out[:, 4:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def quantize_q5_0(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / 15).astype(np.float16)
    df = d.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(df > 0, np.rint(x / df), 0)
    q = (q.clip(-16, 15) + 16).astype(np.uint32)
    qh = np.zeros(x.shape[0], np.uint32)
    for j in range(32):
        qh |= ((q[:, j] >> 4) & 1) << np.uint32(j)
    nib = (q & 0xF).astype(np.uint8)
    out = np.empty((x.shape[0], 22), np.uint8)
    out[:, 0:2] = d[:, None].view(np.uint8)
    out[:, 2:6] = qh[:, None].view(np.uint8)
    out[:, 6:] = nib[:, :16] | (nib[:, 16:] << 4)
    return out.reshape(-1)


def quantize_mxfp4(x: np.ndarray) -> np.ndarray:
    """GGUF MXFP4 rule (gguf-py MXFP4.quantize_blocks): e = floor(log2 amax) - 2 + 127,
    nearest doubled-E2M1 code (first index on ties)."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    with np.errstate(divide="ignore"):
        e = np.where(amax > 0, np.floor(np.log2(amax)) - 2 + 127, 0).astype(np.uint8)
    s = mxfp4_half_scale(e)
    err = np.abs(s[:, None, None] * MXFP4_KVALUES.astype(np.float32)[None, None, :] - x[:, :, None])
    best = err.argmin(axis=-1).astype(np.uint8)
    out = np.empty((x.shape[0], 17), np.uint8)
    out[:, 0] = e
    out[:, 1:] = best[:, :16] | (best[:, 16:] << 4)
    return out.reshape(-1)


def mxfp4_to_ref_layout(raw: np.ndarray) -> np.ndarray:
    """Re-encode GGUF MXFP4 blocks into the reference's 17-byte layout with the
    nearest sign-extended int4 mantissa (exact where the E2M1 value is an integer
    multiple of the scale, i.e. |kval| <= 8 after rescaling).  Used only to feed the
    reference's C MXFP4 kernels comparable inputs for timing and compat tests."""
    n = raw.size // 17 * 32
    v = dequantize(MXFP4, raw, n).reshape(-1, 32)
    amax = np.abs(v).max(axis=1)
    with np.errstate(divide="ignore"):
        e = np.where(amax > 0, np.ceil(np.log2(np.maximum(amax, 1e-38) / 7)) + 127, 0)
    e = np.clip(e, 1, 254).astype(np.uint32)
    s = (e << np.uint32(23)).view(np.float32)
    q = np.clip(np.rint(v / s[:, None]), -8, 7).astype(np.int32) & 0xF
    out = np.empty((v.shape[0], 17), np.uint8)
    out[:, 0:16] = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    out[:, 16] = e.astype(np.uint8)
    return out.reshape(-1)


def _kquant_scales(x, nlev, nsub):
    """Own K-quant scale search: per sub-block range [min(0, lo), hi] -> (scale, -min)."""
    lo = np.minimum(x.min(axis=-1), 0)
    hi = x.max(axis=-1)
    scale = (hi - lo) / nlev
    mins = -lo
    d = (scale.max(axis=-1) / 63).astype(np.float16)
    dmin = (mins.max(axis=-1) / 63).astype(np.float16)
    df = d.astype(np.float32)[:, None]
    dmf = dmin.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df > 0, np.rint(scale / df), 0).clip(0, 63).astype(np.uint8)
        mn = np.where(dmf > 0, np.rint(mins / dmf), 0).clip(0, 63).astype(np.uint8)
    ds = df * sc.astype(np.float32)
    dm = dmf * mn.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(ds[..., None] > 0, np.rint((x + dm[..., None]) / ds[..., None]), 0)
    q = q.clip(0, nlev).astype(np.uint8)
    return d, dmin, sc, mn, q


def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    """Own Q4_K encoder (any valid encoding; parity is on the decode)."""
    x = np.asarray(x, np.float32).reshape(-1, 8, 32)
    nb = x.shape[0]
    d, dmin, sc, mn, q = _kquant_scales(x, 15, 8)
    out = np.empty((nb, 144), np.uint8)
    out[:, 0:2] = d[:, None].view(np.uint8)
    out[:, 2:4] = dmin[:, None].view(np.uint8)
    out[:, 4:16] = pack_scale_min_k4(sc, mn)
    qs = q[:, 0::2] | (q[:, 1::2] << 4)          # (nb, 4, 32)
    out[:, 16:] = qs.reshape(nb, 128)
    return out.reshape(-1)


def quantize_q5_k(x: np.ndarray) -> np.ndarray:
    """Own Q5_K encoder."""
    x = np.asarray(x, np.float32).reshape(-1, 8, 32)
    nb = x.shape[0]
    d, dmin, sc, mn, q = _kquant_scales(x, 31, 8)
    out = np.empty((nb, 176), np.uint8)
    out[:, 0:2] = d[:, None].view(np.uint8)
    out[:, 2:4] = dmin[:, None].view(np.uint8)
    out[:, 4:16] = pack_scale_min_k4(sc, mn)
    qh = np.zeros((nb, 32), np.uint8)
    for s in range(8):
        qh |= ((q[:, s] >> 4) & 1).astype(np.uint8) << s
    out[:, 16:48] = qh
    lo = q & 0xF
    out[:, 48:] = (lo[:, 0::2] | (lo[:, 1::2] << 4)).reshape(nb, 128)
    return out.reshape(-1)


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    """Own Q6_K encoder: int8 scale per 16 elements, q6 in [0, 63] stored as q+32."""
    x = np.asarray(x, np.float32).reshape(-1, 16, 16)
    nb = x.shape[0]
    amax = np.abs(x).max(axis=-1)
    scale = amax / 31
    d = (scale.max(axis=-1) / 127).astype(np.float16)
    df = d.astype(np.float32)[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df > 0, np.rint(scale / df), 0).clip(-128, 127).astype(np.int8)
    ds = df * sc.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(ds[..., None] != 0, np.rint(x / ds[..., None]), 0)
    q = (q.clip(-32, 31) + 32).astype(np.uint8).reshape(nb, 2, 4, 32)   # half, quadrant, l
    ql = np.empty((nb, 2, 64), np.uint8)
    ql[:, :, 0:32] = (q[:, :, 0] & 0xF) | ((q[:, :, 2] & 0xF) << 4)
    ql[:, :, 32:64] = (q[:, :, 1] & 0xF) | ((q[:, :, 3] & 0xF) << 4)
    qh = ((q[:, :, 0] >> 4) | ((q[:, :, 1] >> 4) << 2) | ((q[:, :, 2] >> 4) << 4)
          | ((q[:, :, 3] >> 4) << 6)).astype(np.uint8)
    out = np.empty((nb, 210), np.uint8)
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.view(np.uint8)
    out[:, 208:210] = d[:, None].view(np.uint8)
    return out.reshape(-1)


def quantize(qt: int, x) -> np.ndarray:
    """Encode float32 values into type qt (returns the raw bytes)."""
    x = np.asarray(x, np.float32).reshape(-1)
    if qt == F32:
        return x.view(np.uint8).copy()
    if qt == F16:
        return x.astype(np.float16).view(np.uint8).copy()
    if qt == BF16:
        u = x.view(np.uint32)
        r = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)   # RNE
        return r.view(np.uint8).copy()
    enc = {Q8_0: quantize_q8_0, Q4_0: quantize_q4_0, Q4_1: quantize_q4_1, Q5_0: quantize_q5_0,
           Q4_K: quantize_q4_k, Q5_K: quantize_q5_k, Q6_K: quantize_q6_k, MXFP4: quantize_mxfp4}
    if qt == MXFP4_REF:
        return mxfp4_to_ref_layout(quantize_mxfp4(x))
    return enc[qt](x)


def random_blocks(qt: int, n: int, rng: np.random.Generator) -> np.ndarray:
    """Random raw bytes for n elements of type qt with finite, moderate scales
    (random bit patterns everywhere else) -- decode fixtures, not realistic weights."""
    be, bb = BLOCK[qt]
    nb = n // be
    b = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)

    def f16s(lo, hi, size):
        return rng.uniform(lo, hi, size=size).astype(np.float16).view(np.uint8).reshape(size[0], 2)

    if qt in (Q8_0, Q4_0, Q5_0):
        b[:, 0:2] = f16s(-0.05, 0.05, (nb, 1))
    elif qt == Q4_1:
        b[:, 0:2] = f16s(0.0, 0.05, (nb, 1))
        b[:, 2:4] = f16s(-0.5, 0.5, (nb, 1))
    elif qt in (Q4_K, Q5_K):
        b[:, 0:2] = f16s(0.0, 0.01, (nb, 1))
        b[:, 2:4] = f16s(0.0, 0.01, (nb, 1))
    elif qt == Q6_K:
        b[:, 208:210] = f16s(-0.01, 0.01, (nb, 1))
    elif qt == MXFP4:
        b[:, 0] = rng.integers(100, 140, size=nb, dtype=np.uint8)
    elif qt == MXFP4_REF:
        b[:, 16] = rng.integers(100, 140, size=nb, dtype=np.uint8)
    elif qt in (F32, F16, BF16):
        return quantize(qt, rng.standard_normal(n).astype(np.float32))
    return b.reshape(-1)
