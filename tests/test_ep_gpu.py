"""Expert-parallel MoE on the GPU: the dispatch / expert-row / combine kernels behind
mojollama_b200/ep.py's CudaBackend against the oracle backend of tests/test_ep_cpu.py
(dispatch bit-exact; outputs relative L2 <= 1e-3), one rank; and two NCCL ranks on two
GPUs when the box has them (expert slices exchanged over NVLink)."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import formats as F
from oracle import ops as O

from test_ep_cpu import E, FF, K_TOP, N, OracleBackend, _model, _want

pytestmark = pytest.mark.gpu
TOL = 1e-3


class _L:   # the fields the oracle dispatch reads
    def __init__(self, world, e_local, k):
        self.world, self.e_local, self.k = world, e_local, k


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_ep_dispatch_matches_oracle(cuda_device, world):
    """fixed-capacity dispatch: positions, in-band expert ids (-1 for unused rows) and the
    used rows' data bit for bit"""
    from mojollama_b200.ep import CudaBackend
    rng = np.random.default_rng(world)
    T, k, e_local, n = 300, 8, 16, 128
    idx = np.stack([rng.choice(e_local * world, k, replace=False) for _ in range(T)]).astype(np.int32)
    x = rng.standard_normal((T, n)).astype(np.float32)
    lay = _L(world, e_local, k)
    lay.N = n
    lay.cap = T * min(k, e_local)
    pos, send = CudaBackend().dispatch(lay, torch.from_numpy(idx).cuda(), torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    wp, ws = OracleBackend().dispatch(lay, torch.from_numpy(idx), torch.from_numpy(x))
    got, want = send.cpu().numpy(), ws.numpy()
    assert np.array_equal(pos.cpu().numpy(), wp.numpy())
    gid = np.ascontiguousarray(got[:, n]).view(np.int32)
    wid = np.ascontiguousarray(want[:, n]).view(np.int32)
    assert np.array_equal(gid, wid)
    used = wid >= 0
    assert used.sum() == T * k
    assert np.array_equal(got[used, :n], want[used, :n])


@pytest.mark.parametrize("renorm", [True, False])
def test_ep_layer_one_rank_matches_oracle(cuda_device, renorm):
    from mojollama_b200.ep import EPMoELayer
    mats, router = _model()
    d = {n: torch.from_numpy(m).cuda() for n, m in mats.items()}
    layer = EPMoELayer(0, 1, E, K_TOP, N, FF, F.Q8_0, F.Q8_0, F.Q8_0, d["gate"], d["up"], d["down"],
                       torch.from_numpy(router).cuda(), renorm=renorm, max_tokens=16)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((9, N)).astype(np.float32)
    res = rng.standard_normal((9, N)).astype(np.float32)
    got = layer.forward(torch.from_numpy(x).cuda(), torch.from_numpy(res).cuda()).cpu().numpy()
    assert O.rel_l2(got, _want(mats, router, x, res, renorm)) < TOL


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nccl_rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    from mojollama_b200 import core
    from mojollama_b200.ep import EPMoELayer, expert_slice
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        lib = core()
        assert lib.mlq_init(rank) == 0
        lib.mlq_set_stream(torch.cuda.current_stream().cuda_stream)
        mats, router = _model()
        sl = {n: expert_slice(torch.from_numpy(m), rank, world, E).cuda() for n, m in mats.items()}
        layer = EPMoELayer(rank, world, E, K_TOP, N, FF, F.Q8_0, F.Q8_0, F.Q8_0, sl["gate"], sl["up"], sl["down"],
                           torch.from_numpy(router).cuda(), renorm=True, max_tokens=8)
        rng = np.random.default_rng(200 + rank)
        x = rng.standard_normal((6 + rank, N)).astype(np.float32)
        res = rng.standard_normal((6 + rank, N)).astype(np.float32)
        got = layer.forward(torch.from_numpy(x).cuda(), torch.from_numpy(res).cuda()).cpu().numpy()
        q.put((rank, float(O.rel_l2(got, _want(mats, router, x, res, True)))))
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_nccl(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert all(v < TOL for v in res.values()), res
