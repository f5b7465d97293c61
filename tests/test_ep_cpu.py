"""Expert parallelism on CPU ranks (gloo, world size 2 and 4): the collective logic of
mojollama_b200/ep.py -- the fixed-capacity blocks, the two equal-split all-to-all exchanges,
the return path and the ordered combine -- driven by an oracle backend (numpy, fp64), against
the single-rank MoE FFN of the oracle over all experts (moe_forward,
cengine_batch_instr.c:1113-1207 math).

The device kernels behind the product backend are checked against the same oracle in
tests/test_ep_gpu.py."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import formats as F
from oracle import ops as O

E, K_TOP, N, FF, T = 8, 2, 64, 64, 5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class OracleBackend:
    """The product backend's four device steps, restated with numpy on CPU tensors."""

    def route(self, layer, x):
        lg = x.double().numpy() @ layer.router.double().numpy().T
        idx, w = zip(*[O.router_topk(r, layer.k, layer.renorm) for r in lg])
        return torch.from_numpy(np.array(idx, np.int32)), torch.from_numpy(np.array(w, np.float32))

    def dispatch(self, layer, idx, x):
        """fixed-capacity layout: destination d's rows at d * cap + j in slot order, the
        destination-local expert id in-band at column N (int bits), -1 for unused rows"""
        flat = idx.reshape(-1).numpy()
        dest = flat // layer.e_local
        cap, n = layer.cap, layer.N
        send = np.zeros((layer.world * cap, n + 4), np.float32)
        ids = send[:, n].view(np.int32)
        ids[:] = -1
        pos = np.empty(len(flat), np.int32)
        fill = np.zeros(layer.world, np.int64)
        xs = x.numpy()
        for s_, d in enumerate(dest):
            p = d * cap + fill[d]
            fill[d] += 1
            pos[s_] = p
            send[p, :n] = xs[s_ // layer.k]
            ids[p] = flat[s_] - d * layer.e_local
        return torch.from_numpy(pos), torch.from_numpy(send)

    def experts(self, layer, recv):
        rv = recv.numpy()
        n = layer.N
        eids = np.ascontiguousarray(rv[:, n]).view(np.int32)
        y = np.zeros((rv.shape[0], n), np.float32)
        g_all, u_all, d_all = layer.gate.numpy(), layer.up.numpy(), layer.down.numpy()
        for r, (xr, e) in enumerate(zip(rv[:, :n], eids)):
            if not 0 <= e < layer.e_local:
                continue
            g = O.gemv(g_all[e * layer.gstride:(e + 1) * layer.gstride], layer.gq, xr, layer.n_ff, layer.N)[0]
            u = O.gemv(u_all[e * layer.ustride:(e + 1) * layer.ustride], layer.uq, xr, layer.n_ff, layer.N)[0]
            h = O.silu_clamped(g) * u
            y[r] = O.gemv(d_all[e * layer.dstride:(e + 1) * layer.dstride], layer.dq, h, layer.N, layer.n_ff)[0]
        return torch.from_numpy(y)

    def combine(self, layer, recv_y, pos, w, residual):
        ry, p, ww = recv_y.numpy().astype(np.float64), pos.numpy(), w.numpy()
        out = residual.numpy().astype(np.float64).copy() if residual is not None else np.zeros((ww.shape[0], layer.N))
        for t in range(ww.shape[0]):
            for i in range(layer.k):
                out[t] += ww[t, i] * ry[p[t * layer.k + i]]
        return torch.from_numpy(out.astype(np.float32))


def _model(seed=0):
    rng = np.random.default_rng(seed)
    mats = {name: np.concatenate([F.quantize(F.Q8_0, (rng.standard_normal(r * c) * 0.05).astype(np.float32))
                                  for _ in range(E)])
            for name, r, c in (("gate", FF, N), ("up", FF, N), ("down", N, FF))}
    router = (rng.standard_normal((E, N)) * 0.5).astype(np.float32)
    return mats, router


def _want(mats, router, x, res, renorm):
    per = {n: len(m) // E for n, m in mats.items()}
    split = {n: {e: m[e * per[n]:(e + 1) * per[n]] for e in range(E)} for n, m in mats.items()}
    out = []
    for t in range(x.shape[0]):
        idx, w = O.router_topk(router.astype(np.float64) @ x[t].astype(np.float64), K_TOP, renorm)
        out.append(res[t] + O.moe_forward(split["gate"], split["up"], split["down"], (F.Q8_0,) * 3, x[t], FF, N,
                                          idx, w))
    return np.stack(out)


def _rank(rank, world, port, renorm, q):
    from mojollama_b200.ep import EPMoELayer, expert_slice
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mats, router = _model()
        sl = {n: expert_slice(torch.from_numpy(m), rank, world, E) for n, m in mats.items()}
        layer = EPMoELayer(rank, world, E, K_TOP, N, FF, F.Q8_0, F.Q8_0, F.Q8_0, sl["gate"], sl["up"], sl["down"],
                           torch.from_numpy(router), renorm=renorm, backend=OracleBackend(), max_tokens=T + world)
        rng = np.random.default_rng(100 + rank)
        x = rng.standard_normal((T + rank, N)).astype(np.float32)   # ranks hold different token counts
        res = rng.standard_normal((T + rank, N)).astype(np.float32)
        got = layer.forward(torch.from_numpy(x), torch.from_numpy(res)).numpy()
        want = _want(mats, router, x, res, renorm)
        q.put((rank, float(O.rel_l2(got, want))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,renorm", [(2, True), (4, False)])
def test_ep_moe_matches_single_rank_oracle(world, renorm):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, PORTS[world], renorm, q))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=5) for _ in range(world))
    for p in procs:
        assert p.exitcode == 0
    assert all(v < 1e-6 for v in results.values()), results


PORTS = {2: _free_port(), 4: _free_port()}


def test_ep_rejects_uneven_expert_split():
    from mojollama_b200.ep import EPMoELayer
    with pytest.raises(ValueError):
        EPMoELayer(0, 3, E, K_TOP, N, FF, F.Q8_0, F.Q8_0, F.Q8_0, None, None, None, None, backend=OracleBackend())
