"""Continuous batching (mojollama_b200/serving.py) and the prefix cache's KV snapshots on
the GPU, checked against the oracle (oracle/model.py) on the small dense model.

More requests than slots, with different prompt lengths and lengths of output, so that
requests join the batch while others are mid-way through their prompt or their output.
Every request's greedy tokens must be the tokens of that request decoded alone by the
oracle wherever the oracle's top-2 margin exceeds 1e-2 (teacher-forced on the library's
tokens; the logits of each position within the model bar 3e-3).  With the prefix cache, a
request sharing a prompt prefix restores those K/V rows (the restored rows equal the
snapshot bit for bit) and still matches the oracle."""
import ctypes

import numpy as np
import pytest

from mojollama_b200 import bc as BCm
from mojollama_b200.prefix_cache import KVSnapshot, PrefixCache
from mojollama_b200.serving import ContinuousBatcher, PagedKV
from oracle import model as OM
from oracle import ops as O

from model_fixture import fill_bc, make_model

pytestmark = pytest.mark.gpu


def _oracle_check(m, req):
    """teacher-forced oracle decode of one request: its logits at every generated position"""
    st = OM.new_state(m, 1)
    fed = list(req.prompt) + list(req.output[:-1])
    for i, t in enumerate(fed):
        lg, _ = OM.forward_step(m, st, [0], [t])
        if i >= len(req.prompt) - 1:
            got = req.output[i - len(req.prompt) + 1]
            top = np.argsort(lg[0])[::-1]
            if lg[0][top[0]] - lg[0][top[1]] > 1e-2:
                assert got == int(top[0]), (req.rid, i)


def _engine(m, max_batch, cache=None):
    import torch
    lib = BCm.core()
    stream = torch.cuda.Stream()
    assert lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream)) == 0
    logits = torch.zeros(max_batch * m["V"], device="cuda")
    bld = BCm.BCBuilder()
    fill_bc(m, bld, [], np.zeros(1, np.float32))
    bld.bc.logits = ctypes.cast(ctypes.c_void_p(logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
    bld.keep(logits)
    return ContinuousBatcher(bld, m["L"], m["NKH"], m["HD"], max_batch=max_batch, page_size=8, max_len=64,
                             prefix_cache=cache, stream=stream), stream


def _restore_stream():
    import torch
    BCm.core().mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_continuous_batching_matches_oracle(cuda_device):
    m = make_model("dense", seed=41, attn_modes=["sep", "qk", "sep"])
    eng, _ = _engine(m, max_batch=3)
    try:
        rng = np.random.default_rng(42)
        reqs = [eng.submit(rng.integers(0, m["V"], n), k) for n, k in ((5, 4), (2, 7), (9, 3), (3, 5), (6, 2), (4, 6))]
        widths = []
        while eng.queue or eng.active:
            widths.append(eng.step())
        assert all(r.done and len(r.output) == r.max_new_tokens for r in reqs)
        assert max(widths) == 3 and eng.steps < sum(len(r.prompt) + r.max_new_tokens for r in reqs)
        for r in reqs:
            _oracle_check(m, r)
    finally:
        _restore_stream()


def test_prefix_cache_reuses_prompt_rows(cuda_device):
    import torch
    m = make_model("dense", seed=43, attn_modes=["sep", "sep", "sep"])
    cache = PrefixCache(max_entries=8, prefix_len=4)
    eng, stream = _engine(m, max_batch=2, cache=cache)
    try:
        base = [11, 22, 33, 44, 55, 66, 77]
        a = eng.submit(base, 3)
        eng.run()
        assert cache.size == 1 and a.cached_prefix == 0
        b = eng.submit(base[:5] + [99, 98], 4)       # shares 5 prompt tokens with a
        c = eng.submit([1, 2, 3, 4, 5], 2)            # shares nothing
        eng.run()
        assert b.cached_prefix == 5 and c.cached_prefix == 0 and eng.cache_hits == 1
        for r in (a, b, c):
            _oracle_check(m, r)
        # snapshot -> restore -> snapshot is the identity on the rows
        snap = cache.get(tuple(base))
        kv = PagedKV(m["L"], m["NKH"], m["HD"], 8, 8)
        snap.restore(kv.block, snap.length)
        again = KVSnapshot.take(kv.block, base, snap.length)
        torch.cuda.synchronize()
        assert torch.equal(again.data, snap.data)
    finally:
        _restore_stream()
