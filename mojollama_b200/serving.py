"""Continuous batching over the batch engine's paged KV cache.

The reference batches concurrent requests in an HTTP proxy in front of llama.cpp
(src/mojollama/scheduler.py:28-180: collect requests for a window, dispatch them, hand the
answers back); its own engines decode one request per call.  Here the batching happens at
the batch engine itself: every request owns a KVBlock (its page table and page pool, so
each sequence sits at its own position), and every ``step`` runs one ``batch_forward`` over
all running sequences -- each takes one token, prompt tokens while it is prefilling and its
own last sampled token afterwards -- followed by the library's sampler on the device
(``mlq_batch_forward_sample``).  Requests join and leave between steps: a finished request
frees its slot and the next queued request takes it, so the batch stays full while work is
queued.  The host reads back one token id per sequence per step (to return it and to end a
request on its stop token or length), nothing else.

With a ``PrefixCache`` a request whose prompt starts like an earlier one restores that
prompt's K/V rows from HBM (``KVSnapshot.restore``) and starts its prefill after them; a
request that finishes its prompt leaves a snapshot for later ones.

    eng = ContinuousBatcher(bc_builder, n_layers, nkh, hd, max_batch=8)
    r = eng.submit([1, 2, 3], max_new_tokens=16)
    eng.run()
    r.output                            # generated token ids
"""
from __future__ import annotations

import ctypes
from collections import deque
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from ._lib import core
from .bc import KVBlock
from .prefix_cache import KVSnapshot, PrefixCache


@dataclass
class Request:
    prompt: List[int]
    max_new_tokens: int
    temperature: float = 0.0
    stop_token: Optional[int] = None
    seed: int = 0
    rid: int = 0
    output: List[int] = field(default_factory=list)
    done: bool = False
    cached_prefix: int = 0          # prompt positions restored from the prefix cache


class PagedKV:
    """A sequence's KVBlock with only a page table and page pool (no reference-style 64-slot
    k/v mirror arrays): page_size slots per page, n_pages pages, in HBM."""

    def __init__(self, n_layers: int, nkh: int, hd: int, page_size: int, n_pages: int):
        self.lib = core()
        self.block = KVBlock()
        rc = self.lib.mlq_page_table_init(ctypes.byref(self.block.pt), n_pages, page_size, nkh, hd, n_layers)
        if rc != 0:
            raise RuntimeError(self.lib.mlq_last_error_message().decode())

    def reset(self):
        """back to position 0 with every page free"""
        pt = self.block.pt
        for i in range(1024):
            pt.table[i] = -1
        for i in range(pt.n_pages):
            pt.free_pages[i] = pt.n_pages - 1 - i
        pt.free_count = pt.n_pages
        self.block.seq_len[0] = 0

    def fast_forward(self, n: int):
        """map pages for positions [0, n) and continue at position n; the rows keep whatever
        the pool holds (zeros for a fresh pool), which is what a decode-throughput
        measurement at context n needs (the values do not change the work)"""
        pt = self.block.pt
        for i in range((n + pt.page_size - 1) // pt.page_size):
            if pt.table[i] < 0:
                page = self.lib.mlq_page_table_alloc(ctypes.byref(pt))
                if page < 0:
                    raise RuntimeError("page pool full")
                pt.table[i] = page
        self.block.seq_len[0] = n

    def free(self):
        if self.block.pt.pages:
            self.lib.mlq_page_table_destroy(ctypes.byref(self.block.pt))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class _Slot:
    def __init__(self, kv: PagedKV):
        self.kv = kv
        self.req: Optional[Request] = None
        self.pos = 0                  # next prompt index to feed while prefilling

    @property
    def prefilling(self) -> bool:
        return self.pos < len(self.req.prompt)


class ContinuousBatcher:
    """Token-level continuous batching of requests on one model (a BCBuilder whose BC
    describes the model; its logits pointer must hold max_batch rows)."""

    def __init__(self, builder, n_layers: int, nkh: int, hd: int, max_batch: int = 8, page_size: int = 16,
                 max_len: int = 1024, prefix_cache: Optional[PrefixCache] = None, stream=None):
        import torch
        if not 1 <= max_batch <= 64:
            raise ValueError("max_batch 1..64 (the batch engine's limit)")
        self.lib = core()
        self.builder = builder
        self.max_batch = max_batch
        self.max_len = max_len
        self.cache = prefix_cache
        n_pages = (max_len + page_size - 1) // page_size
        self.slots = [_Slot(PagedKV(n_layers, nkh, hd, page_size, n_pages)) for _ in range(max_batch)]
        self.queue: deque = deque()
        self.stream = stream
        self.d_tok = torch.zeros(max_batch, dtype=torch.int32, device="cuda")
        self.d_next = torch.zeros(max_batch, dtype=torch.int32, device="cuda")
        self.h_next = torch.zeros(max_batch, dtype=torch.int32, pin_memory=True)
        self.steps = 0
        self.cache_hits = 0
        self._rid = 0

    def submit(self, prompt, max_new_tokens: int, temperature: float = 0.0, stop_token: Optional[int] = None,
               seed: int = 0) -> Request:
        if len(prompt) == 0:
            raise ValueError("empty prompt")
        if len(prompt) + max_new_tokens > self.max_len:
            raise ValueError(f"prompt + new tokens exceed max_len {self.max_len}")
        self._rid += 1
        r = Request([int(t) for t in prompt], int(max_new_tokens), float(temperature), stop_token, seed, self._rid)
        self.queue.append(r)
        return r

    @property
    def active(self) -> int:
        return sum(1 for s in self.slots if s.req is not None)

    def _admit(self):
        for s in self.slots:
            if s.req is None and self.queue:
                r = self.queue.popleft()
                s.kv.reset()
                s.req, s.pos = r, 0
                if self.cache is not None:
                    snap = self.cache.get(tuple(r.prompt))
                    if isinstance(snap, KVSnapshot):
                        n = snap.usable_length(r.prompt)
                        if n > 0:
                            snap.restore(s.kv.block, n)
                            s.pos = n
                            r.cached_prefix = n
                            self.cache_hits += 1

    def step(self) -> int:
        """admit queued requests into free slots, run one token for every running sequence,
        retire finished requests; returns the number of sequences that ran"""
        import torch
        self._admit()
        run = [s for s in self.slots if s.req is not None]
        if not run:
            return 0
        B = len(run)
        tok = np.empty(B, np.int32)
        for i, s in enumerate(run):
            tok[i] = s.req.prompt[s.pos] if s.prefilling else s.req.output[-1]
        self.builder.kv_array([s.kv.block for s in run])
        stream = self.stream or torch.cuda.current_stream()
        with torch.cuda.stream(stream):
            self.d_tok[:B].copy_(torch.from_numpy(tok), non_blocking=True)
            # one temperature / seed per step (requests in one batch share them; greedy when 0)
            temp = max(s.req.temperature for s in run)
            rc = self.lib.mlq_batch_forward_sample(ctypes.byref(self.builder.bc), ctypes.c_void_p(self.d_tok.data_ptr()),
                                                   B, None, ctypes.c_float(temp), run[0].req.seed, self.steps,
                                                   ctypes.c_void_p(self.d_next.data_ptr()))
            if rc != 0:
                raise RuntimeError(f"batch_forward_sample failed ({rc}): {self.lib.mlq_last_error_message().decode()}")
            self.h_next[:B].copy_(self.d_next[:B], non_blocking=True)
        stream.synchronize()
        nxt = self.h_next[:B].numpy()
        self.steps += 1
        for i, s in enumerate(run):
            r = s.req
            if s.prefilling:
                s.pos += 1
                if s.prefilling:
                    continue
                # the prompt's last token just ran: its sample is the first generated token
                if self.cache is not None and self.cache.get(tuple(r.prompt)) is None:
                    self.cache.put(tuple(r.prompt), KVSnapshot.take(s.kv.block, r.prompt, len(r.prompt)))
            r.output.append(int(nxt[i]))
            if len(r.output) >= r.max_new_tokens or (r.stop_token is not None and r.output[-1] == r.stop_token):
                r.done = True
                s.req = None
        return B

    def run(self, max_steps: int = 1 << 30) -> None:
        n = 0
        while (self.queue or self.active) and n < max_steps:
            self.step()
            n += 1
