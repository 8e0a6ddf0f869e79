"""Generates tests/golden/packer_golden.{npz,json} from the REFERENCE's own
host packer (SpeakOutLoudly/CUDA-Repo test/utils.h:91-229, compiled into
oracle/_ref/libref_packer.so by `make -C oracle ref`).

Inputs come from the oracle's seeded generator (and, for the known-answer
case, from the reference's own generator init_host_matrices_pruned,
test/utils.h:38-66).  Small cases store full arrays; larger ones store
FNV-1a-64 hashes of the inputs and outputs.  Run from the repo root:

    python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
import oracle as O  # noqa: E402


def edge_matrix() -> np.ndarray:
    """16 x 64 matrix exercising the compressor's zero rules: exactly two
    zeros, three zeros, four zeros, -0.0 as zero, subnormals, inf and nan as
    non-zero values, zeros in every position pair."""
    M, K = 16, 64
    a = O.normal_f16(M * K, 99, 0.0, 1.0).reshape(M, K).copy()
    pairs = [(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)]
    for m in range(M):
        for g in range(K // 4):
            kind = (m * 7 + g * 3) % 9
            grp = a[m, 4 * g:4 * g + 4]
            if kind < 6:
                z = pairs[kind]
                for i in z:
                    grp[i] = 0
            elif kind == 6:          # three zeros (one of them -0.0)
                grp[:] = [0x8000, grp[1], 0, 0]
            elif kind == 7:          # four zeros
                grp[:] = [0, 0x8000, 0, 0]
            else:                    # specials kept as values
                grp[:] = [0x0001, 0, 0x7c00 if g % 2 else 0x7e00, 0]
    return a.reshape(-1)


def main() -> None:
    if not O.ref_packer_available():
        raise SystemExit("oracle/_ref/libref_packer.so missing: run `make -C oracle ref` first")
    arrays = {}
    meta = {"generator": "tests/golden/make_golden.py", "packer": "reference test/utils.h via oracle/_ref",
            "cases": {}}

    # 1. known answer with the reference's own generator (ones, glibc rand mask)
    M = K = 256
    a = O.ref_init_pruned_ref(M, K)
    n, vals, raw = O.ref_compress_a(a, M, K)
    re = O.ref_reorder_metadata(raw, M, K)
    meta["cases"]["ref_known_answer_256"] = {
        "M": M, "K": K, "count": n, "fnv_a": hex(O.fnv1a64(a)), "fnv_vals": hex(O.fnv1a64(vals)),
        "fnv_meta_raw": hex(O.fnv1a64(raw)), "fnv_meta_reordered": hex(O.fnv1a64(re)),
        "meta_raw_first8": [int(x) for x in raw[:8]], "meta_reordered_first8": [int(x) for x in re[:8]],
    }

    # 2. small seeded case, full arrays
    M, K, N = 32, 128, 16
    a = O.prune_magnitude_2of4(O.normal_f16(M * K, 7, 0.0, 1.0), M, K)
    b = O.uniform_f16(K * N, 8, -1.0, 1.0)
    n, vals, raw = O.ref_compress_a(a, M, K)
    arrays.update(small_a=a, small_b=b, small_vals=vals, small_meta_raw=raw,
                  small_meta_reordered=O.ref_reorder_metadata(raw, M, K), small_b_packed=O.ref_pack_b(b, K, N))
    meta["cases"]["small"] = {"M": M, "K": K, "N": N, "count": n}

    # 3. edge patterns, full arrays
    M, K = 16, 64
    a = edge_matrix()
    n, vals, raw = O.ref_compress_a(a, M, K)
    arrays.update(edge_a=a, edge_vals=vals, edge_meta_raw=raw, edge_meta_reordered=O.ref_reorder_metadata(raw, M, K))
    meta["cases"]["edge"] = {"M": M, "K": K, "count": n}

    # 4/5. larger seeded cases, hashes only
    for name, (M, K, N, seed, astd) in {"config1": (256, 256, 128, 0, 1.0),
                                         "decode_slice": (256, 4096, 16, 3, 0.02)}.items():
        a = O.prune_magnitude_2of4(O.normal_f16(M * K, seed, 0.0, astd), M, K)
        b = O.uniform_f16(K * N, seed + 1, -1.0, 1.0)
        n, vals, raw = O.ref_compress_a(a, M, K)
        re = O.ref_reorder_metadata(raw, M, K)
        bp = O.ref_pack_b(b, K, N)
        meta["cases"][name] = {"M": M, "K": K, "N": N, "seed": seed, "a_std": astd, "count": n,
                               "fnv_a": hex(O.fnv1a64(a)), "fnv_b": hex(O.fnv1a64(b)),
                               "fnv_vals": hex(O.fnv1a64(vals)), "fnv_meta_raw": hex(O.fnv1a64(raw)),
                               "fnv_meta_reordered": hex(O.fnv1a64(re)), "fnv_b_packed": hex(O.fnv1a64(bp))}

    np.savez_compressed(os.path.join(HERE, "packer_golden.npz"), **arrays)
    with open(os.path.join(HERE, "packer_golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", sorted(arrays), "and", sorted(meta["cases"]))


if __name__ == "__main__":
    main()
