"""Generate the golden route-record fixtures from the reference's own kernels.

The reference's route.cuh (rows <= 8) and route_wide.cu (rows <= 64) are
compiled for the CPU by `make -C oracle ref` (oracle/ref_route_shim.h runs one
thread block as std::threads) and run on seeded top-k ids covering: one row,
8 rows (route.cu), 9..64 rows (route_wide.cu), every expert taking every row
(several tiles per expert), expert-parallel windows (expert_offset > 0, ids
outside the window -> -1), balanced dealing to either group (expert_offset -1
and -2), and top-k 1..8 at 32..384 experts.

Run from the repository root:  python tests/golden/make_golden.py
Writes tests/golden/route_cases.npz (ids, expected permuted and record per case).
"""

import ctypes
import os
import sys

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402


def main() -> None:
    O.build(ref=True)
    ref = O.ref_route_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libref_route.so is missing (needs the reference tree)")
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    rng = np.random.default_rng(20261201)
    cases = []
    shapes = [(1, 6, 384), (1, 8, 32), (6, 6, 384), (8, 8, 384), (8, 8, 64), (8, 3, 128), (9, 6, 384),
              (16, 6, 384), (16, 8, 256), (32, 8, 384), (48, 6, 384), (64, 8, 384), (64, 4, 32), (64, 8, 64)]
    for T, K, E in shapes:
        for variant in ("random", "all_rows", "ep_low", "ep_high", "deal0", "deal1"):
            if variant == "all_rows":
                pool = rng.permutation(E)[:K]
                ids = np.stack([rng.permutation(pool) for _ in range(T)])
            else:
                ids = np.stack([rng.permutation(E)[:K] for _ in range(T)])
            ids = ids.astype(np.int32)
            local, offset = E, 0
            if variant == "ep_low":
                local = E // 2
            elif variant == "ep_high":
                local, offset = E // 2, E // 2
            elif variant.startswith("deal"):  # balanced dealing: group -1 - offset
                offset = -1 - int(variant[-1])
            words = O.route_words(T, K, local)
            perm = np.empty((T, K), np.int32)
            rec = np.empty(words, np.int32)
            if T <= 8 and local % 32 == 0:
                barrier = np.zeros(1, np.uint32)
                ref.ref_route(P(ids), P(perm), P(rec), P(barrier), T, K, local, offset)
            else:
                ref.ref_route_wide(P(ids), P(perm), P(rec), T, K, local, offset)
            cases.append((ids, perm.copy(), rec.copy(), local, offset))
    out = {}
    for i, (ids, perm, rec, local, offset) in enumerate(cases):
        out[f"ids_{i}"] = ids
        out[f"perm_{i}"] = perm
        out[f"rec_{i}"] = rec
        out[f"meta_{i}"] = np.array([local, offset], np.int32)
    out["count"] = np.array([len(cases)], np.int32)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "route_cases.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {len(cases)} cases to {path}")


if __name__ == "__main__":
    main()
