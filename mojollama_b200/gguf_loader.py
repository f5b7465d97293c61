"""GGUF model files on the device: the Python face of the library's GGUF reader and loader
(mlq_gguf_* in include/mojollama_b200.h, mojollama_b200/csrc/gguf.cu).

It stands where the reference's loader stands (src/mojollama/kernels/turbo_engine_v7_moe.py
:425-618), which reads the file with gguf-py's GGUFReader and keeps numpy views of the
mapped file (quantized tensors) or host F32 copies (norms, small tensors, the embedding).
Here the parse is native, the data section is streamed into HBM once, in its GGUF block
layout, and every tensor is a device address (``GGUFModel.ptr``) for the library's entry
points; 1-D and other small tensors become F32 on the device (``GGUFModel.f32``), and a
K-quant output head can be requantized to Q8_0 on the device as the reference does on the
host (``GGUFModel.q8_0``, turbo_engine_v7_moe.py:515-518).

    m = GGUFModel("model.gguf")            # parse + upload
    w = m.ptr("blk.0.attn_q.weight")       # device pointer, GGUF bytes
    info = m.tensor("blk.0.attn_q.weight") # name, dims (fastest first), type, offset, bytes
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from ._lib import core

GGUF_STRING, GGUF_ARRAY = 8, 9


class MlqGgufTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 128), ("n_dims", ctypes.c_int), ("dims", ctypes.c_int64 * 4),
                ("type", ctypes.c_int), ("offset", ctypes.c_uint64), ("bytes", ctypes.c_uint64)]


@dataclass
class TensorInfo:
    name: str
    dims: tuple            # as stored in the file: dims[0] is the contiguous dimension
    type: int              # ggml type code
    offset: int            # inside the data section
    bytes: int             # 0 when the library does not know the type's block layout

    @property
    def rows(self) -> int:
        n = 1
        for d in self.dims[1:]:
            n *= d
        return n

    @property
    def cols(self) -> int:
        return self.dims[0]


class GGUFFile:
    """A parsed, mapped GGUF file (no device work)."""

    def __init__(self, path: str):
        self.lib = core()
        self.path = path
        self.h = self.lib.mlq_gguf_open(path.encode())
        if not self.h:
            raise ValueError(self.lib.mlq_last_error_message().decode())
        self.version = self.lib.mlq_gguf_version(self.h)
        self.alignment = int(self.lib.mlq_gguf_alignment(self.h))
        self.data_offset = int(self.lib.mlq_gguf_data_offset(self.h))
        self.data_bytes = int(self.lib.mlq_gguf_data_bytes(self.h))
        self.tensors = []
        t = MlqGgufTensor()
        for i in range(int(self.lib.mlq_gguf_n_tensors(self.h))):
            assert self.lib.mlq_gguf_tensor(self.h, i, ctypes.byref(t)) == 0
            self.tensors.append(TensorInfo(t.name.decode(), tuple(t.dims[:t.n_dims]), t.type, int(t.offset),
                                           int(t.bytes)))
        self._index = {t.name: i for i, t in enumerate(self.tensors)}

    def tensor(self, name: str) -> TensorInfo:
        return self.tensors[self._index[name]]

    def __contains__(self, name: str) -> bool:
        return name in self._index

    def kv(self, key: str):
        """a scalar or string metadata value (None if absent; arrays: (item type, count))"""
        k = key.encode()
        t = self.lib.mlq_gguf_kv_type(self.h, k)
        if t < 0:
            return None
        if t == GGUF_STRING:
            n = self.lib.mlq_gguf_kv_str(self.h, k, None, 0)
            buf = ctypes.create_string_buffer(n + 1)
            self.lib.mlq_gguf_kv_str(self.h, k, buf, n + 1)
            return buf.raw[:n].decode("utf-8", errors="replace")
        if t == GGUF_ARRAY:
            it = ctypes.c_int()
            n = self.lib.mlq_gguf_kv_array(self.h, k, ctypes.byref(it))
            return (it.value, int(n))
        if t in (6, 12):
            v = ctypes.c_double()
            assert self.lib.mlq_gguf_kv_float(self.h, k, ctypes.byref(v)) == 0
            return v.value
        v = ctypes.c_int64()
        assert self.lib.mlq_gguf_kv_int(self.h, k, ctypes.byref(v)) == 0
        return bool(v.value) if t == 7 else int(v.value)

    def close(self):
        if self.h:
            self.lib.mlq_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GGUFModel(GGUFFile):
    """A GGUF file whose data section lives in HBM (one torch uint8 tensor on the current
    device, uploaded at construction)."""

    def __init__(self, path: str):
        import torch
        super().__init__(path)
        self.data = torch.empty(self.data_bytes + 256, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        rc = self.lib.mlq_gguf_upload(self.h, ctypes.c_void_p(self.data.data_ptr()), self.data_bytes + 256)
        if rc != 0:
            raise RuntimeError(self.lib.mlq_last_error_message().decode())
        self._keep = []

    def ptr(self, name: str) -> int:
        """device address of a tensor's GGUF bytes"""
        return self.data.data_ptr() + self.tensor(name).offset

    def f32(self, name: str):
        """the tensor dequantized to F32 on the device (torch tensor, shape as gguf-py reports
        it for the data: outermost dimension first)"""
        import torch
        t = self.tensor(name)
        n = t.rows * t.cols
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        rc = self.lib.mlq_dequantize(ctypes.c_void_p(self.ptr(name)), t.type, ctypes.c_void_p(out.data_ptr()), n)
        if rc != 0:
            raise RuntimeError(self.lib.mlq_last_error_message().decode())
        return out.view(*reversed(t.dims))

    def q8_0(self, name: str):
        """a quantized 2-D tensor requantized to Q8_0 on the device (dequantize, then the
        reference's Q8_0 rule), as the reference does for K-quant output heads on the host"""
        import torch
        t = self.tensor(name)
        f = self.f32(name).reshape(-1)
        q = torch.empty(f.numel() // 32 * 34, dtype=torch.uint8, device="cuda")
        rc = self.lib.mlq_quantize_q8_0(ctypes.c_void_p(f.data_ptr()), ctypes.c_void_p(q.data_ptr()), f.numel())
        if rc != 0:
            raise RuntimeError(self.lib.mlq_last_error_message().decode())
        self._keep.append(q)
        return q
