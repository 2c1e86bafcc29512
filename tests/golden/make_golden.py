"""Generate the golden vectors that pin the CPU oracle to the reference.

Run where the reference checkout is available (its directory is given with
--ref-dir) after ``make -C oracle ref``.  For every reference entry point
``mma_sp_wgmma_*.cu`` it parses the case table, then replays the suite exactly
as the reference does (one mt19937 seeded 1234 shared by the cases in table
order, wgmma_sp_raw_common.hpp:1123-1127) through the reference's own host
code (oracle/_ref/libsp24ref.so) and records:

  * sha256 of A (dense), B, A_c, the metadata bytes and C (fp32 bytes)
  * the metadata bytes of every case, C of the pattern cases, and A/B/C of
    the smallest random case, in golden.npz

plus known-answer compressions of an alternating six-pattern matrix for each
dtype (pins the e4m3 nibble table of wgmma_sp_raw_common.hpp:176-193), and
every case of the reference's mixed fp8 entry point mma_sp_m16n8k64_fp32fp8.cu
(A e5m2, B e4m3; through oracle/_ref/libsp24ref_fp8.so): dense A, B (row-major
K x N), A_c, metadata bytes and its fp32 CPU GEMM; and sha256 records of the
reference's four legacy warp-level entry points (mma_sp_m16n8k{16,32}_fp32
{fp16,bf16}.cu, through oracle/_ref/libsp24ref_legacy.so) at a small size and
at their own 2048^3 size.
The CuTe harness (wgmma_sp_demo_common.hpp) shares these host algorithms;
its suites are recorded the same way.

    python tests/golden/make_golden.py [--ref-dir REFERENCE_CHECKOUT]
"""
from __future__ import annotations

import argparse
import glob
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

PAIRS = [(0, 1), (0, 2), (0, 3), (1, 2), (1, 3), (2, 3)]


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def alternating_a(dt: int, m: int, k: int):
    """Group g of row r keeps pair PAIRS[(r + g) % 6]; values 1 + (r + 2g + i) % 7."""
    vals = np.zeros((m, k), np.float32)
    for r in range(m):
        for g in range(k // 4):
            i0, i1 = PAIRS[(r + g) % 6]
            vals[r, 4 * g + i0] = 1 + (r + 2 * g) % 7
            vals[r, 4 * g + i1] = -(1 + (r + 2 * g + 1) % 7)
    return oracle.from_float(dt, vals)


def main() -> None:
    ap = argparse.ArgumentParser()
    here = os.path.dirname(os.path.abspath(__file__))
    default_ref = os.environ.get("SP24_REF_DIR",
                                 os.path.join(here, "..", "..", "..", "reference"))
    ap.add_argument("--ref-dir", default=os.path.normpath(default_ref),
                    help="the reference checkout (SP24_REF_DIR, else ../reference beside the repo)")
    args = ap.parse_args()
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libsp24ref.so missing: run `make -C oracle ref`")
    r = oracle.ref_lib()
    suites = []
    arrays = {}
    for path in sorted(glob.glob(os.path.join(args.ref_dir, "mma_sp_wgmma_*.cu"))):
        parsed = oracle.parse_entry_point(path)
        if parsed is None:
            continue
        harness, dt, bn, cases = parsed
        name = os.path.basename(path)[:-3]
        gen = r.ref_gen_new(1234)
        rec = {"entry": name, "harness": harness, "dtype": dt, "block_n": bn, "cases": []}
        smallest = None
        for ci, (tag, m, n, k, pat) in enumerate(cases):
            a, b, ac, e, c = oracle.ref_host_case(gen, dt, m, n, k, pat)
            rec["cases"].append({"tag": tag, "m": m, "n": n, "k": k, "pattern": pat,
                                 "sha256": {"a": sha(a), "b": sha(b), "a_c": sha(ac),
                                            "meta": sha(e), "c": sha(c)}})
            arrays[f"{name}/{ci}/meta"] = e
            if pat:
                arrays[f"{name}/{ci}/c"] = c
            elif smallest is None or m * n * k < smallest[0]:
                smallest = (m * n * k, ci, a, b, c)
        r.ref_gen_free(gen)
        _, ci, a, b, c = smallest
        arrays[f"{name}/{ci}/a"] = a
        arrays[f"{name}/{ci}/b"] = b
        arrays[f"{name}/{ci}/c"] = c
        rec["full_case"] = ci
        suites.append(rec)
        print(f"{name}: {harness} dt={dt} BlockN={bn} cases={len(cases)}")

    kats = []
    for dt in (oracle.F16, oracle.BF16, oracle.E4M3):
        m, k = 128, 256
        a = alternating_a(dt, m, k)
        ac = np.empty((m, k // 2), oracle.BITS[dt])
        e = np.empty((m, k // 8), np.uint8)
        r.ref_compress(dt, a.ctypes.data, m, k, ac.ctypes.data, e.ctypes.data)
        kats.append({"name": f"alternating6_dt{dt}", "dtype": dt, "m": m, "k": k,
                     "sha256": {"a": sha(a), "a_c": sha(ac), "meta": sha(e)}})
        arrays[f"kat/alternating6_dt{dt}/meta"] = e
        arrays[f"kat/alternating6_dt{dt}/a_c"] = ac

    # The reference's mixed fp8 entry point (A e5m2, B e4m3, 16 x 8 x 64):
    # every case of its run_one(), through its own host code.
    legacy_fp8 = None
    if oracle.ref_fp8_available():
        s = oracle.ref_fp8_suite()
        for key in ("a", "b", "a_c", "meta", "c"):
            arrays[f"legacy_fp8/{key}"] = s[key]
        legacy_fp8 = {"entry": "mma_sp_m16n8k64_fp32fp8.cu", "seed": 123, "m": 16, "n": 8,
                      "k": 64, "a": "e5m2", "b": "e4m3", "tags": s["tags"],
                      "sha256": {key: sha(s[key]) for key in ("a", "b", "a_c", "meta", "c")}}

    # The legacy warp-level entry points (m16n8k16 / m16n8k32, fp16 / bf16):
    # each main replayed by its own host code at a small size (every array
    # hashed, C included) and at its own 2048^3 size (A, B, A_c and metadata
    # hashed; its CPU product is too slow to record here).
    legacy_mma_sp = None
    if oracle.ref_legacy_available():
        legacy_mma_sp = []
        for which, entry in enumerate(oracle.LEGACY_FILES):
            rec = {"entry": entry, "which": which, "dtype": oracle.legacy_dtype(which),
                   "seed": 42, "sizes": []}
            for (m, n, k, with_c) in ((64, 64, 128, True), (2048, 2048, 2048, False)):
                a, b, ac, e, c = oracle.ref_legacy_case(which, m, n, k, with_c)
                h = {"a": sha(a), "b": sha(b), "a_c": sha(ac), "meta_words": sha(e)}
                if with_c:
                    h["c"] = sha(c)
                rec["sizes"].append({"m": m, "n": n, "k": k, "sha256": h})
            legacy_mma_sp.append(rec)

    out = {"generator": "tests/golden/make_golden.py", "reference_seed": 1234,
           "suites": suites, "kats": kats, "legacy_fp8": legacy_fp8,
           "legacy_mma_sp": legacy_mma_sp}
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    size = os.path.getsize(os.path.join(HERE, "golden.npz"))
    print(f"wrote golden.json ({len(suites)} suites) and golden.npz ({size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
