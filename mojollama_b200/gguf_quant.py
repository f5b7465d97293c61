"""Host-side GGUF block encoders (numpy), for building synthetic models and for
requantizing weights at load (the reference requantizes K-quant output heads to
Q8_0: src/mojollama/kernels/turbo_engine_v7_moe.py:515-518, 620-666).

Q8_0 follows the reference's activation quantizer (quant_kernels_omp.c:1406-1455);
Q4_0 and MXFP4 follow the GGUF rules (byte-identical to gguf-py 0.19.0); the
K-quant, Q4_1 and Q5_0 encoders are our own (any valid encoding decodes exactly).
Device-side Q8_0 quantization is mlq_quantize_q8_0 in the native library.
"""
from __future__ import annotations

import numpy as np

F32, F16, Q4_0, Q4_1, Q5_0, Q8_0 = 0, 1, 2, 3, 6, 8
Q4_K, Q5_K, Q6_K, BF16, MXFP4 = 12, 13, 14, 30, 39
MXFP4_REF = 1039
BLOCK = {
    F32: (1, 4), F16: (1, 2), BF16: (1, 2),
    Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q8_0: (32, 34),
    Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
    MXFP4: (32, 17), MXFP4_REF: (32, 17),
}
MXFP4_KVALUES = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], np.int8)


def row_bytes(qt: int, k: int) -> int:
    be, bb = BLOCK[qt]
    if k % be:
        raise ValueError(f"type {qt} needs K % {be} == 0, got K={k}")
    return (k // be) * bb


def mxfp4_half_scale(e: np.ndarray) -> np.ndarray:
    e = e.astype(np.uint32)
    bits = np.where(e < 2, np.uint32(0x00200000) << e, (e - 1) << np.uint32(23)).astype(np.uint32)
    return bits.view(np.float32)


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Pack eight 6-bit (scale, min) pairs into the 12 K-quant scale bytes."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    q = np.zeros(sc.shape[:-1] + (12,), np.uint8)
    for j in range(4):
        q[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        q[..., j + 4] = (mn[..., j] & 63) | ((mn[..., j + 4] >> 4) << 6)
        q[..., j + 8] = (sc[..., j + 4] & 0xF) | ((mn[..., j + 4] & 0xF) << 4)
    return q



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


def quantize_mxfp4_ref(x: np.ndarray) -> np.ndarray:
    """The reference C decoder's own 17-byte MXFP4 layout {qs[16], e}: element 2i is the
    low nibble of byte i, 2i+1 the high nibble, value = sext4(nibble) * 2^(e-127)
    (quant_kernels_omp.c:486-573).  Nearest int4 mantissa for the block amax."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    with np.errstate(divide="ignore"):
        e = np.where(amax > 0, np.ceil(np.log2(np.maximum(amax, 1e-38) / 7)) + 127, 0)
    e = np.clip(e, 1, 254).astype(np.uint32)
    s = (e << np.uint32(23)).view(np.float32)
    q = np.clip(np.rint(x / s[:, None]), -8, 7).astype(np.int32) & 0xF
    out = np.empty((x.shape[0], 17), np.uint8)
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
        return quantize_mxfp4_ref(x)
    return enc[qt](x)
