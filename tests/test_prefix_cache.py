"""PrefixCache (mojollama_b200/prefix_cache.py) replays the reference's own PrefixCache:
tests/golden/prefix_cache_ops.json holds a seeded sequence of put / get / invalidate /
evict / clear operations run through the reference's class (src/mojollama/prefix_cache.py,
by tests/golden/gen_prefix_cache.py) with every result, size and key list; the library's
class must reproduce all of them.  Plus the reference's own smoke example
(prefix_cache.py:210-218) and the snapshot-length rule of KVSnapshot."""
import json
import os

import numpy as np

from mojollama_b200.prefix_cache import KVSnapshot, PrefixCache

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "prefix_cache_ops.json")


def test_replays_reference_operation_trace():
    for case in json.load(open(GOLD)):
        c = PrefixCache(max_entries=case["max_entries"], prefix_len=case["prefix_len"])
        for i, op in enumerate(case["ops"]):
            t = tuple(op["tokens"])
            if op["op"] == "put":
                c.put(t, op["value"])
                res = None
            elif op["op"] == "get":
                res = c.get(t)
            elif op["op"] == "invalidate":
                res = c.invalidate(t)
            elif op["op"] == "evict":
                res = c.evict()
            else:
                c.clear()
                res = None
            assert res == op["result"], (case["prefix_len"], i, op)
            assert c.size == op["size"]
            assert [list(k) for k in c.keys()] == op["keys"]


def test_reference_smoke_example():
    cache = PrefixCache(max_entries=4, prefix_len=4)
    cache.put((1, 2, 3, 4, 5, 6), "snapshot_A")
    cache.put((1, 2, 3, 7, 8, 9), "snapshot_B")
    assert cache.get((1, 2, 3, 4, 10, 11)) == "snapshot_A"
    assert cache.get((1, 2, 3, 7, 42, 99)) == "snapshot_B"
    assert cache.get((9, 9, 9, 9)) is None


def test_snapshot_usable_length():
    s = KVSnapshot((5, 6, 7, 8, 9), 5, None)
    assert s.usable_length([5, 6, 7, 8, 9, 10]) == 5
    assert s.usable_length([5, 6, 7, 8, 9]) == 4          # one prompt token is always run
    assert s.usable_length([5, 6, 1, 8, 9, 10]) == 2      # rows after a different token are not reused
    assert s.usable_length([1, 6]) == 0
    assert s.usable_length(np.array([5, 6, 7])) == 2
