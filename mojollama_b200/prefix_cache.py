"""Prefix cache over the library's paged KV: requests that share a prompt prefix reuse its
K/V rows instead of recomputing them.

``PrefixCache`` keeps the interface and matching rules of the reference's prefix cache
(src/mojollama/prefix_cache.py:24-162): an LRU of ``max_entries`` snapshots keyed by the
SHA-256 of the first ``prefix_len`` token ids (4-byte little-endian, comma-joined); ``get``
with at least ``prefix_len`` tokens is an exact lookup of that prefix, with fewer tokens a
scan for an entry that starts with them; ``put`` of an existing prefix replaces it and
promotes it; ``evict`` drops the least recently used entry; ``invalidate``, ``clear``,
``size`` and ``keys`` as there.  The reference stores engine-specific snapshots (whole host
KV arrays copied by ``snapshot_dense`` / ``restore_dense``); here a snapshot is
``KVSnapshot``: the first ``length`` positions of every layer's K and V rows, packed in HBM
by ``mlq_kv_snapshot`` and written back into another sequence's pages by
``mlq_kv_restore``.  ``usable_length`` returns how many positions of a snapshot a new
prompt may take: the snapshot's tokens must equal the prompt's up to that point (K/V at
position p depend on tokens 0..p only), and at least one prompt token is left to run so
the step that follows yields the logits of the prompt's last token.
"""
from __future__ import annotations

import ctypes
import hashlib
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, List, Optional, Tuple

from ._lib import core


class PrefixCache:
    """LRU prefix cache (the reference's PrefixCache API)."""

    def __init__(self, max_entries: int = 64, prefix_len: int = 8):
        self.max_entries = max_entries
        self.prefix_len = prefix_len
        self._cache: "OrderedDict[str, Tuple[Tuple[int, ...], Any]]" = OrderedDict()

    def put(self, tokens_tuple: Tuple[int, ...], kv_snapshot: Any) -> None:
        if not tokens_tuple:
            return
        key = self._hash(tuple(tokens_tuple[: self.prefix_len]))
        if key in self._cache:
            self._cache.move_to_end(key)
            self._cache[key] = (tuple(tokens_tuple), kv_snapshot)
            return
        if len(self._cache) >= self.max_entries:
            self._cache.popitem(last=False)
        self._cache[key] = (tuple(tokens_tuple), kv_snapshot)

    def get(self, tokens_tuple: Tuple[int, ...]) -> Optional[Any]:
        if not tokens_tuple:
            return None
        n = min(self.prefix_len, len(tokens_tuple))
        query = tuple(tokens_tuple[:n])
        if n == self.prefix_len:
            key = self._hash(query)
            hit = self._cache.get(key)
            if hit is not None and hit[0][: self.prefix_len] == query:
                self._cache.move_to_end(key)
                return hit[1]
            return None
        for key, (cached, snap) in list(self._cache.items()):
            if cached[:n] == query:
                self._cache.move_to_end(key)
                return snap
        return None

    def evict(self) -> int:
        if not self._cache:
            return 0
        self._cache.popitem(last=False)
        return 1

    def invalidate(self, tokens_tuple: Tuple[int, ...]) -> bool:
        if not tokens_tuple:
            return False
        prefix = tuple(tokens_tuple[: self.prefix_len])
        key = self._hash(prefix)
        hit = self._cache.get(key)
        if hit is not None and hit[0][: self.prefix_len] == prefix:
            del self._cache[key]
            return True
        return False

    def clear(self) -> None:
        self._cache.clear()

    @property
    def size(self) -> int:
        return len(self._cache)

    def keys(self) -> List[Tuple[int, ...]]:
        return [t for t, _ in self._cache.values()]

    @staticmethod
    def _hash(prefix: Tuple[int, ...]) -> str:
        raw = b",".join(int(t).to_bytes(4, "little", signed=True) for t in prefix)
        return hashlib.sha256(raw).hexdigest()


@dataclass
class KVSnapshot:
    """K/V rows of positions [0, length) of one sequence, [2][n_layers][length][row] fp32 in
    HBM, and the tokens that produced them."""
    tokens: Tuple[int, ...]
    length: int
    data: Any            # torch float32 tensor on the device

    @staticmethod
    def take(block, tokens, length: int) -> "KVSnapshot":
        """snapshot of a KVBlock (library KVBlock structure) after it ran `tokens`"""
        import torch
        pt = block.pt
        row = pt._nkh * pt._hd
        data = torch.empty(2 * pt._n_layers * max(length, 1) * row, dtype=torch.float32, device="cuda")
        lib = core()
        rc = lib.mlq_kv_snapshot(ctypes.byref(block), length, ctypes.c_void_p(data.data_ptr()))
        if rc != 0:
            raise RuntimeError(lib.mlq_last_error_message().decode())
        return KVSnapshot(tuple(int(t) for t in tokens[:length]), length, data)

    def restore(self, block, length: int) -> None:
        """write positions [0, length) (length <= self.length) into a fresh KVBlock"""
        if length > self.length:
            raise ValueError("restore beyond the snapshot")
        data = self.data
        if length < self.length:   # the packed layout is [2][L][len][row]: repack for a shorter length
            pt = block.pt
            row = pt._nkh * pt._hd
            data = self.data.view(2, pt._n_layers, self.length, row)[:, :, :length].contiguous()
        lib = core()
        rc = lib.mlq_kv_restore(ctypes.byref(block), length, ctypes.c_void_p(data.data_ptr()))
        if rc != 0:
            raise RuntimeError(lib.mlq_last_error_message().decode())

    def usable_length(self, prompt) -> int:
        n = 0
        limit = min(self.length, len(prompt) - 1)
        while n < limit and self.tokens[n] == int(prompt[n]):
            n += 1
        return n
