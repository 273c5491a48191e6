"""Writes tests/golden/reference_kats.json: the known-answer vectors of the
reference's own tests for this path, restated as data.

Sources (forge-gpu project root):
  tests/radix_sort_test.rs:20-21   16 fixed keys, 4 bits, values 0..15
  tests/radix_sort_test.rs:57-66   xorshift32 seed 12345, n 10,000, keys & 0xFFFFF, 20 bits
  tests/radix_sort_test.rs:100-108 xorshift32 seed 42, n 5,000, keys & 0xFFFF, 16 bits,
                                   checked against a CPU stable sort_by_key (:111-113)
  tests/radix_sort_test.rs:145-168 find_cell_boundaries on [0,0,1,1,1,3,3,5], 8 cells
  tests/hashgrid_test.rs:9-33      4 particles, 10^3 grid, cell 1.0, query r=1.0
  tests/hashgrid_test.rs:42-85     1000 lattice points, 5^3 grid, cell 2.0, query (5,5,5) r=1.5

Expected outputs are what those tests assert (plus, for the sorts, the full
stable order a stable sort produces, which the reference's stable LSD
RadixSorter and std stable sort give). Run: python tests/golden/make_golden.py
"""
import json
import os


def xorshift32(seed, n, mask):
    s, out = seed, []
    for _ in range(n):
        s ^= (s << 13) & 0xFFFFFFFF
        s ^= s >> 17
        s ^= (s << 5) & 0xFFFFFFFF
        out.append(s & mask)
    return out


def stable(keys):
    order = sorted(range(len(keys)), key=lambda i: keys[i])  # Python sort is stable
    return [keys[i] for i in order], order


def main():
    kats = {}
    k16 = [15, 3, 7, 1, 9, 0, 12, 5, 8, 2, 14, 6, 11, 4, 13, 10]
    sk, sv = stable(k16)
    kats["radix_small"] = {"keys": k16, "num_bits": 4, "sorted_keys": sk, "sorted_vals": sv}
    for name, seed, n, mask, bits in (("radix_medium", 12345, 10000, 0xFFFFF, 20),
                                      ("radix_cpu_ref", 42, 5000, 0xFFFF, 16)):
        keys = xorshift32(seed, n, mask)
        sk, sv = stable(keys)
        kats[name] = {"seed": seed, "n": n, "mask": mask, "num_bits": bits, "keys_head": keys[:8],
                      "sorted_keys": sk, "sorted_vals": sv}
    S = 0xFFFFFFFF
    kats["cell_bounds"] = {"sorted": [0, 0, 1, 1, 1, 3, 3, 5], "num_cells": 8,
                           "start": [0, 2, S, 5, S, 7, S, S], "end": [2, 5, 0, 7, 0, 8, 0, 0]}
    kats["hashgrid_basic"] = {
        "cell_size": 1.0, "dims": [10, 10, 10], "origin": [0, 0, 0],
        "positions": [[5.0, 5.0, 5.0], [5.1, 5.0, 5.0], [5.5, 5.5, 5.5], [9.0, 9.0, 9.0]],
        "query": [5.0, 5.0, 5.0], "radius": 1.0, "must_contain": [0, 1, 2], "must_not_contain": [3]}
    pos = [[(i % 10) + 0.5, ((i // 10) % 10) + 0.5, (i // 100) + 0.5] for i in range(1000)]
    kats["hashgrid_uniform"] = {"cell_size": 2.0, "dims": [5, 5, 5], "origin": [0, 0, 0], "positions": pos,
                                "query": [5.0, 5.0, 5.0], "radius": 1.5, "min_hits": 4}
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(path, "w") as f:
        json.dump(kats, f)
    print("wrote", path)


if __name__ == "__main__":
    main()
