"""GGUF reader and device loader (mojollama_b200/csrc/gguf.cu, mojollama_b200/gguf_loader.py).

The reference loads weights through gguf-py 0.19.0 (GGUFReader; turbo_engine_v7_moe.py
:425-618), so gguf-py is the pin: test files are written with gguf-py's GGUFWriter, and the
library's parse (tensor names, dims, types, offsets, sizes, metadata) must equal what
GGUFReader reads from the same file.  CPU tests cover the parse (no device work) and the
refusal of damaged files; GPU tests upload the data section and compare the device bytes
with GGUFReader's, dequantize on the device against gguf-py, and run a matmul straight
from the loaded bytes against the oracle."""
import ctypes
import os

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

from mojollama_b200 import gguf_loader as GL
from oracle import formats as F
from oracle import ops as O

Q = gguf.GGMLQuantizationType


def _write(path, big=False):
    rng = np.random.default_rng(3)
    w = gguf.GGUFWriter(str(path), arch="llama")
    w.add_custom_alignment(64)
    w.add_context_length(4096)
    w.add_uint64("test.u64", 1 << 40)
    w.add_int32("test.i32", -7)
    w.add_float32("test.eps", 1e-5)
    w.add_bool("test.flag", True)
    w.add_array("test.ints", [1, 2, 3, 4])
    w.add_array("test.names", ["a", "bb", "ccc"])
    w.add_string("test.name", "mojollama")
    tensors = {}

    def qt(name, t, shape, vals):
        raw = F.quantize(int(t), vals.astype(np.float32))
        be, bb = gguf.GGML_QUANT_SIZES[t]
        w.add_tensor(name, raw, raw_shape=shape[:-1] + (shape[-1] // be * bb,), raw_dtype=t)   # byte shape
        tensors[name] = (int(t), shape)

    qt("blk.0.attn_q.weight", Q.Q8_0, (128, 256), rng.standard_normal(128 * 256) * 0.02)
    qt("blk.0.ffn_gate_exps.weight", Q.Q4_K, (4, 64, 256), rng.standard_normal(4 * 64 * 256) * 0.02)
    qt("blk.0.ffn_down.weight", Q.Q6_K, (256, 256), rng.standard_normal(256 * 256) * 0.02)
    qt("output.weight", Q.MXFP4, (96, 256), rng.standard_normal(96 * 256) * 0.02)
    emb = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    w.add_tensor("token_embd.weight", emb)
    tensors["token_embd.weight"] = (0, (64, 256))
    norm = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    w.add_tensor("blk.0.attn_norm.weight", norm)
    tensors["blk.0.attn_norm.weight"] = (0, (256,))
    if big:   # several 64 MB staging chunks
        qt("blk.1.big.weight", Q.Q8_0, (2048 * 34, 2048), np.tile(rng.standard_normal(2048 * 64) * 0.02, 34 * 32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


def test_block_table_matches_gguf_py():
    """the library's (elements, bytes) per block for every type it sizes = gguf-py's"""
    import re
    src = open(os.path.join(os.path.dirname(GL.__file__), "csrc", "gguf.cu")).read()
    table = {int(t): (int(be), int(bb)) for t, be, bb in
             re.findall(r"case (\d+): be = (\d+); bb = (\d+); return true;", src)}
    assert len(table) >= 20
    for t, (be, bb) in table.items():
        assert gguf.GGML_QUANT_SIZES[Q(t)] == (be, bb), Q(t).name


def test_parse_matches_gguf_reader(tmp_path):
    path = tmp_path / "m.gguf"
    _write(path)
    r = gguf.GGUFReader(str(path))
    f = GL.GGUFFile(str(path))
    assert f.version == 3 and f.alignment == 64
    assert [t.name for t in f.tensors] == [t.name for t in r.tensors]
    for mine, ref in zip(f.tensors, r.tensors):
        assert mine.dims == tuple(int(d) for d in ref.shape)
        assert mine.type == int(ref.tensor_type)
        assert f.data_offset + mine.offset == ref.data_offset
        assert mine.bytes == ref.n_bytes
    assert f.kv("general.architecture") == "llama"
    assert f.kv("llama.context_length") == 4096
    assert f.kv("test.u64") == 1 << 40 and f.kv("test.i32") == -7 and f.kv("test.flag") is True
    assert abs(f.kv("test.eps") - 1e-5) < 1e-12
    assert f.kv("test.name") == "mojollama"
    assert f.kv("test.ints")[1] == 4 and f.kv("test.names") == (8, 3)
    assert f.kv("missing.key") is None
    # host views inside the mapping equal gguf-py's data
    for i, ref in enumerate(r.tensors):
        p = f.lib.mlq_gguf_tensor_data(f.h, i)
        got = np.ctypeslib.as_array((ctypes.c_uint8 * ref.n_bytes).from_address(p))
        assert np.array_equal(got, np.asarray(ref.data).view(np.uint8).reshape(-1))
    f.close()


@pytest.mark.parametrize("damage", ["magic", "truncate_header", "truncate_data", "version"])
def test_damaged_files_are_refused(tmp_path, damage):
    path = tmp_path / "m.gguf"
    _write(path)
    b = bytearray(path.read_bytes())
    if damage == "magic":
        b[0:4] = b"GGUX"
    elif damage == "truncate_header":
        b = b[:100]
    elif damage == "truncate_data":
        b = b[:len(b) - 1000]
    else:
        b[4:8] = (7).to_bytes(4, "little")
    path.write_bytes(bytes(b))
    with pytest.raises(ValueError):
        GL.GGUFFile(str(path))


@pytest.mark.gpu
def test_upload_and_use_on_device(cuda_device, tmp_path):
    import time

    import torch
    path = tmp_path / "m.gguf"
    tensors = _write(path, big=True)
    r = gguf.GGUFReader(str(path))
    t0 = time.perf_counter()
    m = GL.GGUFModel(str(path))
    dt = time.perf_counter() - t0
    print(f"uploaded {m.data_bytes / 1e6:.1f} MB in {dt * 1e3:.1f} ms ({m.data_bytes / dt / 1e9:.2f} GB/s)")
    dev = m.data.cpu().numpy()
    for ref in r.tensors:
        info = m.tensor(ref.name)
        got = dev[info.offset:info.offset + info.bytes]
        assert np.array_equal(got, np.asarray(ref.data).view(np.uint8).reshape(-1)), ref.name
    # dequantized on the device = gguf-py's dequantize
    for name in ("blk.0.attn_q.weight", "blk.0.ffn_down.weight", "token_embd.weight", "blk.0.attn_norm.weight",
                 "output.weight"):
        ref = next(t for t in r.tensors if t.name == name)
        want = gguf.dequantize(np.asarray(ref.data), ref.tensor_type).reshape(-1)
        got = m.f32(name).cpu().numpy().reshape(-1)
        assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32)), name
    # a matmul straight from the loaded bytes
    t, (rows, cols) = tensors["blk.0.attn_q.weight"]
    x = np.random.default_rng(9).standard_normal(cols).astype(np.float32)
    out = np.zeros(rows, np.float32)
    lib = cuda_device
    assert lib.mlq_matmul(ctypes.c_void_p(m.ptr("blk.0.attn_q.weight")), t, x.ctypes.data, out.ctypes.data, rows,
                          cols, 1) == 0
    raw = np.asarray(next(tt for tt in r.tensors if tt.name == "blk.0.attn_q.weight").data).view(np.uint8)
    assert O.rel_l2(out, O.gemv(raw.reshape(-1), t, x, rows, cols)[0]) < 1e-3
    # a K-quant head requantized to Q8_0 on the device = the oracle's Q8_0 rule on gguf-py's decode
    q = m.q8_0("blk.0.ffn_down.weight").cpu().numpy()
    ref = next(tt for tt in r.tensors if tt.name == "blk.0.ffn_down.weight")
    want = F.quantize_q8_0(gguf.dequantize(np.asarray(ref.data), ref.tensor_type).reshape(-1).astype(np.float32))
    assert np.array_equal(q, want)
    torch.cuda.synchronize()
    m.close()
