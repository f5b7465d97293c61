"""Next-token selection, restated in numpy (TEST INFRASTRUCTURE ONLY, see oracle/__init__.py).

The reference chooses each next token on the host with np.argmax over the step's logits
(src/mojollama/kernels/turbo_engine_v7_moe.py:2101-2114 of the reference): ``argmax`` is
that call.  Temperature sampling has no counterpart in the reference's C or Python engine;
``sample`` is the published Gumbel-max construction (Gumbel 1954; e.g. Maddison, Tarlow &
Minka 2014): token = argmax_i (logit_i / T + g_i), g_i = -log(-log u_i), a draw from
softmax(logit / T).  u_i comes from the SplitMix64 finaliser (Steele, Lea & Flood 2014)
used as a counter-based generator keyed by (seed, step, row, index): the same bits the
library's kernel (mojollama_b200/csrc/sampling.cu) draws, here in float64."""
from __future__ import annotations

import numpy as np

_M1, _M2, _GOLD = np.uint64(0xBF58476D1CE4E5B9), np.uint64(0x94D049BB133111EB), np.uint64(0x9E3779B97F4A7C15)


def mix64(z):
    """SplitMix64 finaliser on uint64 arrays (wrapping arithmetic)."""
    z = np.asarray(z, np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def uniforms(seed: int, step: int, row: int, n: int) -> np.ndarray:
    """u_i in (0, 1), 23 random bits each (exactly representable in fp32, below 1), i < n."""
    key = mix64(np.uint64(seed) ^ mix64((np.uint64(step) << np.uint64(20)) ^ np.uint64(row)))
    with np.errstate(over="ignore"):
        h = mix64(key + _GOLD * (np.arange(n, dtype=np.uint64) + np.uint64(1)))
    return ((h >> np.uint64(41)).astype(np.float64) + 0.5) * 2.0 ** -23


def argmax(logits) -> np.ndarray:
    """np.argmax per row: the first maximum, a NaN counting as the maximum."""
    return np.argmax(np.asarray(logits, np.float32), axis=-1).astype(np.int32)


def gumbel_scores(logits, temperature: float, seed: int, step: int) -> np.ndarray:
    """logit / T - log(-log u) per element, float64, rows [B][V]."""
    lg = np.atleast_2d(np.asarray(logits, np.float64))
    out = np.empty_like(lg)
    for b in range(lg.shape[0]):
        u = uniforms(seed, step, b, lg.shape[1])
        out[b] = lg[b] / temperature - np.log(-np.log(u))
    return out


def sample(logits, temperature: float, seed: int, step: int) -> np.ndarray:
    if not temperature > 0:
        return argmax(logits)
    return np.argmax(gumbel_scores(logits, temperature, seed, step), axis=-1).astype(np.int32)
