"""GPU parity of the grouped expert path (mlq_moe_rows: planner, packed activation rows,
grouped gate/up and down GEMV) against the oracle: y[r] = down_e(silu(clamp(gate_e x_r,
+-80)) * up_e x_r), e = eid[r] (the expert FFN of cengine_batch_instr.c:591-665 and
quant_kernels_omp.c:2157-2164 for one routed row).  Covers one-row and many-row experts
(chunks of 8 rows and a ragged rest), unused experts, mixed gate/up types (separate
launches), short rows (a lane group per weight row), rows whose length is not a multiple of
128 bytes, and ids outside [0, E) (row left unwritten).  Tolerance: relative L2 <= 1e-3
per row."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import formats as F
from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _experts(qt, E, rows, cols, rng):
    raw = F.random_blocks(qt, E * rows * cols, rng)
    mats = F.dequantize(qt, raw, E * rows * cols).astype(np.float64).reshape(E, rows, cols)
    return raw, mats


def _run(lib, qts, E, N, FF, eid, seed):
    qg, qu, qd = qts
    rng = np.random.default_rng(seed)
    graw, G = _experts(qg, E, FF, N, rng)
    uraw, U = _experts(qu, E, FF, N, rng)
    draw, D = _experts(qd, E, N, FF, rng)
    R = len(eid)
    x = rng.standard_normal((R, N)).astype(np.float32)
    dev = {k: torch.from_numpy(v).cuda() for k, v in (("g", graw), ("u", uraw), ("d", draw))}
    dx = torch.from_numpy(x).cuda()
    de = torch.from_numpy(np.asarray(eid, np.int32)).cuda()
    y = torch.full((R, N), float("nan"), device="cuda")
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    rc = lib.mlq_moe_rows(qg, qu, qd, vp(dev["g"]), vp(dev["u"]), vp(dev["d"]), F.row_bytes(qg, N) * FF,
                          F.row_bytes(qu, N) * FF, F.row_bytes(qd, FF) * N, E, vp(de), R, FF, N, vp(dx), vp(y))
    assert rc == 0, lib.mlq_last_error_message()
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for r, e in enumerate(eid):
        if not 0 <= e < E:
            assert np.isnan(got[r]).all(), f"row {r} (id {e}) was written"
            continue
        xr = x[r].astype(np.float64)
        h = O.silu_clamped(G[e] @ xr) * (U[e] @ xr)
        want = D[e] @ h
        assert O.rel_l2(got[r], want) < TOL, (r, e, O.rel_l2(got[r], want))


def _skewed(rng, E, R):
    """one expert takes 20 rows (chunks 8 + 8 + 4), the rest spread, some experts unused"""
    eid = [3] * 20 + list(rng.integers(0, E, R - 20))
    rng.shuffle(eid)
    return eid


@pytest.mark.parametrize("qts,E,N,FF", [
    ((F.Q4_K, F.Q4_K, F.Q6_K), 16, 512, 256),       # config-3 formats; down rows of 4 units
    ((F.Q4_K, F.Q4_K, F.Q6_K), 8, 2048, 768),       # config-3 shapes
    ((F.Q8_0, F.Q4_0, F.Q5_0), 8, 96, 160),         # mixed gate/up; 96-byte rows (partial swizzle group)
    ((F.MXFP4, F.MXFP4, F.MXFP4), 4, 2880, 64),     # gpt-oss width, not a multiple of 128
    ((F.Q5_K, F.Q5_K, F.Q4_1), 6, 256, 512),
])
def test_moe_rows_matches_oracle(cuda_device, qts, E, N, FF):
    rng = np.random.default_rng(E * 1000 + N)
    _run(cuda_device, qts, E, N, FF, _skewed(rng, E, 40), seed=N + FF)


def test_moe_rows_single_rows(cuda_device):
    """decode shape: every active expert sees one row"""
    rng = np.random.default_rng(5)
    eid = list(rng.permutation(32)[:24])
    _run(cuda_device, (F.Q4_K, F.Q4_K, F.Q6_K), 32, 512, 256, eid, seed=11)


def test_moe_rows_ids_out_of_range(cuda_device):
    eid = [2, -1, 0, 5, 2, 9, 1, 2]      # E = 6: -1 and 9 stay unwritten
    _run(cuda_device, (F.Q8_0, F.Q8_0, F.Q8_0), 6, 128, 64, eid, seed=3)
