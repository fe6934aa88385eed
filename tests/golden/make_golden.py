"""Regenerates tests/golden/kv_golden.npz.

Run in a container that has the reference checkout, after `make -C oracle`
(which compiles kv_cache/KV_int8_split_optimized.cu from the checkout into
oracle/_ref/libkvref_split.so):

    python tests/golden/make_golden.py

Contents
  * pattern_<H>_<S>_<D>: output of the reference's own fp32 host loop
    `cpu_reference` (KV_int8_split_optimized.cu:385-437) on the reference's own
    self-test inputs (:473-486) at several shapes -- executed from the
    reference build, not from the restatement.
  * rand_*: seeded N(0,1) data quantised per token, with the reference
    `cpu_reference` output for it (inputs stored, so the fixture does not depend
    on numpy's generator staying stable).
  * quant_*: quantiser edge cases (ties, zero rows, signed zeros, extremes,
    subnormals) with codes and scale bit patterns. The reference has no
    quantiser; these pin the north-star formula and were produced by the C
    oracle and checked bit-for-bit against an independent numpy restatement.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import pyoracle as po  # noqa: E402

PATTERN_SHAPES = [(4, 128, 64), (3, 129, 128), (2, 1, 64), (5, 257, 96), (1, 1000, 64), (8, 300, 128)]


def quant_cases() -> np.ndarray:
    D = 128
    rows = []
    rng = np.random.default_rng(5)
    rows.append(np.zeros(D, np.float32))                                  # all zero -> scale 0
    z = np.zeros(D, np.float32); z[::2] = -0.0; rows.append(z)             # signed zeros
    r = np.zeros(D, np.float32); r[0] = 127.0
    r[1:40] = np.arange(39, dtype=np.float32) + 0.5                        # exact .5 ties
    r[40:80] = -(np.arange(40, dtype=np.float32) + 0.5)
    rows.append(r)
    rows.append(np.full(D, 3.0e38, np.float32))                            # near FLT_MAX
    rows.append(np.full(D, 1.0e-45, np.float32) * np.sign(rng.standard_normal(D)).astype(np.float32))  # subnormal
    rows.append((rng.standard_normal(D) * 1e-30).astype(np.float32))       # tiny
    one = np.zeros(D, np.float32); one[7] = -2.5; rows.append(one)         # single nonzero
    for _ in range(25):
        rows.append(rng.standard_normal(D).astype(np.float32) * np.float32(rng.uniform(0.01, 100)))
    return np.stack(rows)


def main() -> None:
    ref = po.ref_lib("split")
    if ref is None:
        raise SystemExit("oracle/_ref/libkvref_split.so missing: run `make -C oracle` with the reference present")
    out: dict[str, np.ndarray] = {}
    for H, S, D in PATTERN_SHAPES:
        Q, K, V, ks, vs = po.reference_pattern(H, S, D)
        out[f"pattern_{H}_{S}_{D}"] = po.ref_cpu_reference(Q, K, V, ks, vs, H, S, D)

    H, S, D = 4, 96, 64
    rng = np.random.default_rng(17)
    q = rng.standard_normal((H, D), dtype=np.float32)
    K, ks = po.quantize_rows(rng.standard_normal((H, S, D), dtype=np.float32))
    V, vs = po.quantize_rows(rng.standard_normal((H, S, D), dtype=np.float32))
    out.update(rand_q=q, rand_k=K, rand_v=V, rand_ks=ks, rand_vs=vs,
               rand_out=po.ref_cpu_reference(q, K, V, ks, vs, H, S, D))

    x = quant_cases()
    codes, scales = po.quantize_rows(x)
    ncodes, nscales = po.quantize_rows_numpy(x)
    assert np.array_equal(codes, ncodes) and np.array_equal(scales.view(np.uint32), nscales.view(np.uint32))
    out.update(quant_x=x, quant_codes=codes, quant_scale_bits=scales.view(np.uint32))

    path = Path(__file__).with_name("kv_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
