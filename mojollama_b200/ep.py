"""Expert-parallel MoE layer: the experts of one MoE FFN split over ranks.

The math is the batch engine's routed-expert FFN (cengine_batch_instr.c:591-665 moe_ffn,
:1113-1207 in qwen36_batch_forward): router GEMV, softmax, insertion top-k (optionally
renormalised), per expert silu(clamp(gate x, +-80)) * (up x) -> down, weighted sum added
to the residual.  Here the E experts are split into contiguous slices of E / world per
rank; attention, the router and the shared expert stay replicated.

One forward, per rank (T local tokens, at most ``max_tokens``):
  1. route:    idx, w = top-k(softmax(W_r x))                          (device)
  2. dispatch: every destination rank d gets a fixed block of cap = max_tokens * min(k, E/world)
               rows [d * cap, (d + 1) * cap), slot order kept, the destination-local expert id
               carried in-band in each row (-1 marks an unused row)       (device)
  3. exchange: one all-to-all with equal splits (NCCL over NVLink on GPUs); no counts
               travel to the host, so nothing in a forward waits for the host
  4. experts:  every received row through its one local expert, unused rows skipped (device)
  5. exchange: the expert outputs go back, equal splits again
  6. combine:  out[t] = residual[t] + sum_i w[t][i] * y[t, i], i in order (device)
Every step is deterministic: positions are stable, the combine adds slots in order.  The
fixed blocks move more bytes than a variable split when routing is uneven (the blocks are
sized for the worst case), and in exchange the layer issues no host synchronisation, so a
stack of layers is enqueued as fast as the host can launch and can be captured whole.

The device work goes through a backend object.  `CudaBackend` is the product path (the
kernels of libmojollama_b200; there is no other implementation).  The collective logic is
backend-independent, so tests drive it on CPU ranks (gloo) with a backend of their own.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._lib import core

_BLOCK = {0: (1, 4), 2: (32, 18), 3: (32, 20), 6: (32, 22), 8: (32, 34), 12: (256, 144), 13: (256, 176),
          14: (256, 210), 39: (32, 17), 1039: (32, 17)}


def row_bytes(qt: int, cols: int) -> int:
    be, bb = _BLOCK[qt]
    return cols // be * bb


def _vp(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class CudaBackend:
    """Routing, dispatch, expert and combine kernels of libmojollama_b200 on the current
    CUDA device and the library stream."""

    def __init__(self):
        self.lib = core()

    def _ok(self, rc: int, what: str):
        if rc != 0:
            raise RuntimeError(f"{what} failed ({rc}): {self.lib.mlq_last_error_message()}")

    def route(self, layer: "EPMoELayer", x: torch.Tensor):
        T = x.shape[0]
        idx = torch.empty((T, layer.k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, layer.k), dtype=torch.float32, device=x.device)
        self._ok(self.lib.mlq_moe_router(_vp(x), T, layer.N, _vp(layer.router), layer.router_qt, layer.E, layer.k,
                                         int(layer.renorm), _vp(idx), _vp(w)), "mlq_moe_router")
        return idx, w

    def dispatch(self, layer: "EPMoELayer", idx: torch.Tensor, x: torch.Tensor):
        """pos [T*k] and the packed send rows [world * cap][N + 4] (ids in-band at column N)"""
        T, k = idx.shape
        cap = layer.cap
        pos = torch.empty(T * k, dtype=torch.int32, device=x.device)
        send = torch.empty((layer.world * cap, layer.N + 4), dtype=torch.float32, device=x.device)
        self._ok(self.lib.mlq_ep_dispatch_packed(_vp(idx), T, k, layer.e_local, layer.world, cap, _vp(x), layer.N,
                                                 _vp(pos), _vp(send)), "mlq_ep_dispatch_packed")
        return pos, send

    def experts(self, layer: "EPMoELayer", recv: torch.Tensor):
        """y [R][N] for the packed received rows (rows with id -1 are left unwritten)"""
        R = recv.shape[0]
        y = torch.empty((R, layer.N), dtype=torch.float32, device=recv.device)
        if R:
            self._ok(self.lib.mlq_moe_rows_packed(layer.gq, layer.uq, layer.dq, _vp(layer.gate), _vp(layer.up),
                                                  _vp(layer.down), layer.gstride, layer.ustride, layer.dstride,
                                                  layer.e_local, _vp(recv), R, layer.n_ff, layer.N, _vp(y)),
                     "mlq_moe_rows_packed")
        return y

    def combine(self, layer: "EPMoELayer", recv_y: torch.Tensor, pos: torch.Tensor, w: torch.Tensor,
                residual: torch.Tensor | None):
        T, k = w.shape
        out = torch.empty((T, layer.N), dtype=torch.float32, device=recv_y.device)
        self._ok(self.lib.mlq_ep_combine(_vp(recv_y), _vp(pos), _vp(w), T, k, layer.N,
                                         None if residual is None else _vp(residual), _vp(out)), "mlq_ep_combine")
        return out


class EPMoELayer:
    """One MoE FFN whose experts [rank*E/world, (rank+1)*E/world) live on this rank.

    gate / up / down: this rank's expert tensors as raw GGUF bytes (uint8, expert-major,
    [E_local][rows][cols]); router: [E][N] fp32 (replicated), or raw bytes of type
    router_qt.  renorm: renormalise the top-k weights (qwen36_batch_forward) or not
    (moe_ffn)."""

    def __init__(self, rank, world, E, k, N, n_ff, gq, uq, dq, gate, up, down, router, router_qt=0, renorm=True,
                 backend=None, group=None, max_tokens=64):
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        self.rank, self.world, self.E, self.k, self.N, self.n_ff = rank, world, E, k, N, n_ff
        self.e_local = E // world
        # rows one rank may send one peer: a token sends at most one row per local expert
        self.max_tokens = max_tokens
        self.cap = max_tokens * min(k, self.e_local)
        self.gq, self.uq, self.dq = gq, uq, dq
        self.gate, self.up, self.down, self.router, self.router_qt = gate, up, down, router, router_qt
        self.gstride = n_ff * row_bytes(gq, N)
        self.ustride = n_ff * row_bytes(uq, N)
        self.dstride = N * row_bytes(dq, n_ff)
        self.renorm = renorm
        self.backend = backend if backend is not None else CudaBackend()
        self.group = group

    def exchange(self, send: torch.Tensor) -> torch.Tensor:
        """all-to-all with equal splits: block d of `send` goes to rank d, block r of the
        result came from rank r"""
        out = torch.empty_like(send)
        dist.all_to_all_single(out, send, group=self.group)
        return out

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"{x.shape[0]} tokens > max_tokens {self.max_tokens}")
        b = self.backend
        idx, w = b.route(self, x)
        pos, send = b.dispatch(self, idx, x)
        if self.world == 1:
            return b.combine(self, b.experts(self, send), pos, w, residual)
        recv = self.exchange(send)
        y = b.experts(self, recv)
        back = self.exchange(y)
        return b.combine(self, back, pos, w, residual)


def expert_slice(full: torch.Tensor, rank: int, world: int, E: int) -> torch.Tensor:
    """Rank's contiguous slice of an expert-major [E][...] byte tensor."""
    per = full.numel() // E
    el = E // world
    return full.reshape(-1)[rank * el * per:(rank + 1) * el * per]
