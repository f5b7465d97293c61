"""batch_forward on a capturable stream: from the second step of a shape the step is
replayed as a CUDA graph (mojollama_b200/csrc/forward.cu, run_graph_step), with device
tokens and device logits, as a serving loop drives it.  The other forward tests bind the
library to the legacy default stream, which cannot be captured, so they run the direct
launches only; these check the replayed step against the oracle on every step, across an
attention-length bucket boundary (64 -> 128 positions).  Also the next-token entry
mlq_batch_forward_sample (greedy: np.argmax of the step's logits, on the device)."""
import ctypes

import numpy as np
import pytest

from mojollama_b200 import bc as BCm
from oracle import model as OM
from oracle import ops as O
from oracle import sampling as OS

from model_fixture import fill_bc, make_model

pytestmark = pytest.mark.gpu
MODEL_TOL = 3e-3


def _greedy_ok(got, ref):
    for g, r in zip(np.atleast_2d(got), np.atleast_2d(ref)):
        top = np.argsort(r)[::-1]
        if r[top[0]] - r[top[1]] > 1e-2:
            assert int(np.argmax(g)) == int(top[0])


@pytest.mark.parametrize("modes,steps", [(["sep", "qk", "qkv"], 70), (["sep", "sep", "sep"], 20)])
def test_graph_replayed_steps_match_oracle(cuda_device, modes, steps):
    import torch
    lib = cuda_device
    m = make_model("dense", seed=31, attn_modes=modes)
    B, V = 3, m["V"]
    stream = torch.cuda.Stream()
    assert lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream)) == 0
    try:
        caches = [BCm.KVCache(m["L"], m["NKH"], m["HD"]) for _ in range(B)]
        d_logits = torch.zeros(B * V, device="cuda")
        bld = BCm.BCBuilder()
        fill_bc(m, bld, [c.block for c in caches], np.zeros(B * V, np.float32))
        bld.bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        bld.kv_array([c.block for c in caches])
        st = OM.new_state(m, B)
        rng = np.random.default_rng(32)
        d_tok = torch.zeros(B, dtype=torch.int32, device="cuda")
        for step in range(steps):
            toks = rng.integers(0, V, B).astype(np.int32)
            with torch.cuda.stream(stream):
                d_tok.copy_(torch.from_numpy(toks).cuda())
                rc = lib.mlq_batch_forward(ctypes.byref(bld.bc), ctypes.c_void_p(d_tok.data_ptr()), B, None)
            assert rc == 0, lib.mlq_last_error_message()
            stream.synchronize()
            got = d_logits.cpu().numpy().reshape(B, V)
            want, _ = OM.forward_step(m, st, list(range(B)), list(toks))
            assert O.rel_l2(got, want) < MODEL_TOL, (step, O.rel_l2(got, want))
            _greedy_ok(got, want)
        assert all(c.seq_len == steps for c in caches)
    finally:
        lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_batch_forward_sample_greedy_loop_stays_on_device(cuda_device):
    """A greedy decode loop whose tokens never leave the device: next_tokens is the tokens
    buffer itself; every step's tokens equal np.argmax of that step's logits, and the
    logits match the oracle fed the same tokens."""
    import torch
    lib = cuda_device
    m = make_model("dense", seed=33, attn_modes=["sep", "sep", "sep"])
    B, V = 2, m["V"]
    stream = torch.cuda.Stream()
    assert lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream)) == 0
    try:
        caches = [BCm.KVCache(m["L"], m["NKH"], m["HD"]) for _ in range(B)]
        d_logits = torch.zeros(B * V, device="cuda")
        bld = BCm.BCBuilder()
        fill_bc(m, bld, [c.block for c in caches], np.zeros(B * V, np.float32))
        bld.bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        bld.kv_array([c.block for c in caches])
        st = OM.new_state(m, B)
        d_tok = torch.tensor([5, 7], dtype=torch.int32, device="cuda")
        fed = [5, 7]
        for step in range(12):
            with torch.cuda.stream(stream):
                rc = lib.mlq_batch_forward_sample(ctypes.byref(bld.bc), ctypes.c_void_p(d_tok.data_ptr()), B, None,
                                                  0.0, 0, step, ctypes.c_void_p(d_tok.data_ptr()))
            assert rc == 0, lib.mlq_last_error_message()
            stream.synchronize()
            logits = d_logits.cpu().numpy().reshape(B, V)
            nxt = d_tok.cpu().numpy()
            assert np.array_equal(nxt, OS.argmax(logits)), step
            want, _ = OM.forward_step(m, st, list(range(B)), fed)
            assert O.rel_l2(logits, want) < MODEL_TOL, step
            fed = [int(t) for t in nxt]
    finally:
        lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
