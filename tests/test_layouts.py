"""CPU checks of the byte layout of the structs the reference passes through ctypes
(cengine_batch_instr.c:160-207): the library's PageTable / KVBlock must match a
ctypes mirror field for field."""
import ctypes

from mojollama_b200 import core

cf = ctypes.POINTER(ctypes.c_float)
ci = ctypes.POINTER(ctypes.c_int)


class PageTable(ctypes.Structure):
    _fields_ = [("page_size", ctypes.c_int), ("n_pages", ctypes.c_int), ("pages", cf), ("table", ci),
                ("free_pages", ci), ("free_count", ctypes.c_int), ("_nkh", ctypes.c_int), ("_hd", ctypes.c_int),
                ("_n_layers", ctypes.c_int)]


class KVBlock(ctypes.Structure):
    _fields_ = [("k", cf), ("v", cf), ("n_blocks", ctypes.c_int), ("seq_len", ctypes.c_int * 64),
                ("block_map", (ctypes.c_int * 1024) * 64), ("pt", PageTable)]


def test_struct_sizes_match_reference_mirror():
    lib = core()
    lib.mlq_sizeof_page_table.restype = ctypes.c_size_t
    lib.mlq_sizeof_kv_block.restype = ctypes.c_size_t
    assert lib.mlq_sizeof_page_table() == ctypes.sizeof(PageTable)
    assert lib.mlq_sizeof_kv_block() == ctypes.sizeof(KVBlock)
    assert KVBlock.pt.offset == ctypes.sizeof(KVBlock) - ctypes.sizeof(PageTable)


def test_bc_struct_matches_package_mirror():
    """BC (cengine_batch_instr.c:536-589) as the library compiles it has the size of the
    package's ctypes mirror, which lists the reference's fields in order."""
    from mojollama_b200.bc import BC, KVBlock as PkgKV
    lib = core()
    assert lib.mlq_sizeof_bc() == ctypes.sizeof(BC)
    assert ctypes.sizeof(PkgKV) == ctypes.sizeof(KVBlock)
    assert BC.kv_array.offset < BC.logits.offset < BC.n_experts.offset
