"""Writes tests/golden/prefix_cache_ops.json: a seeded sequence of put / get / invalidate /
evict / clear operations run through the reference's own PrefixCache
(src/mojollama/prefix_cache.py of the reference, imported from the checkout named by
MLQ_REFERENCE_DIR), with every result.  mojollama_b200.prefix_cache.PrefixCache must give
the same results (tests/test_prefix_cache.py).  Snapshots are stood in for by integers.

    MLQ_REFERENCE_DIR=<checkout> python tests/golden/gen_prefix_cache.py
"""
import importlib.util
import json
import os
import random

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "prefix_cache_ops.json")


def main():
    ref = os.environ["MLQ_REFERENCE_DIR"]
    spec = importlib.util.spec_from_file_location("ref_prefix_cache",
                                                  os.path.join(ref, "src", "mojollama", "prefix_cache.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = random.Random(11)
    cases = []
    for max_entries, prefix_len in ((4, 4), (3, 2), (8, 6), (2, 1)):
        cache = mod.PrefixCache(max_entries=max_entries, prefix_len=prefix_len)
        ops = []
        pool = [tuple(rng.randrange(5) for _ in range(rng.randrange(1, 9))) for _ in range(12)]
        for i in range(300):
            kind = rng.choices(["put", "get", "invalidate", "evict", "clear"], [40, 45, 8, 5, 2])[0]
            toks = list(rng.choice(pool))
            if rng.random() < 0.3:
                toks = toks[: rng.randrange(0, len(toks) + 1)]
            if kind == "put":
                cache.put(tuple(toks), i)
                res = None
            elif kind == "get":
                res = cache.get(tuple(toks))
            elif kind == "invalidate":
                res = cache.invalidate(tuple(toks))
            elif kind == "evict":
                res = cache.evict()
            else:
                cache.clear()
                res = None
            ops.append({"op": kind, "tokens": toks, "value": i, "result": res, "size": cache.size,
                        "keys": [list(k) for k in cache.keys()]})
        cases.append({"max_entries": max_entries, "prefix_len": prefix_len, "ops": ops})
    with open(OUT, "w") as f:
        json.dump(cases, f, separators=(",", ":"))
    print("wrote", OUT)


if __name__ == "__main__":
    main()
