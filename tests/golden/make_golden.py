"""Generates tests/golden/*.npz from the reference itself.

Runs the reference's own host model -- make_weights, make_q2, pack_q4, pack_q2_rowmajor, ref_value, ref_scale, ref_q2
and its check-input generators (uniform x, +bigx, +tinyx), all compiled from the reference's source by oracle/Makefile
into oracle/_ref/libvkbref.so -- on small tables seeded like its --check (std::mt19937(1234), src/bakeoff.cu:476), and
stores inputs and outputs. tests/test_oracle.py pins the numpy oracle against these files; the GPU parity tests use
them as known-answer vectors. Re-run (needs the reference source to build oracle/_ref):

    make -f oracle/Makefile && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", ".."))

from oracle import refbind  # noqa: E402


def main() -> None:
    if refbind.load() is None:
        raise SystemExit("oracle/_ref/libvkbref.so is missing: run make -f oracle/Makefile first")
    rng = refbind.Rng(1234)
    out = {}
    # Q4 and Q8 tables in the order the reference's check draws them: weights, then activations per case
    for name, N, K in (("a", 64, 256), ("odd", 33, 512)):
        for bits in (4, 8):
            codes, scales = rng.make_weights(N, K, bits)
            p = f"{name}_q{bits}_"
            out[p + "codes"], out[p + "scales"] = codes, scales
            if bits == 4:
                out[p + "packed"] = refbind.pack_q4(codes, scales, False)
                out[p + "packed_sab"] = refbind.pack_q4(codes, scales, True)
            cases = [(1, 0), (2, 0), (8, 0), (4, 1), (2, 2)]   # (M, kind): 0 uniform, 1 +bigx, 2 +tinyx
            for ci, (M, kind) in enumerate(cases):
                x = rng.uniform_x(M, K, 1e-3 if kind == 2 else 1.0)
                if kind == 1:
                    rng.bigx(x)
                val, mag = refbind.values(codes, scales, x)
                out[p + f"x{ci}"], out[p + f"val{ci}"], out[p + f"mag{ci}"] = x, val, mag
    # 2-bit, one token (the reference's 2-bit kernels are 1-token; src/bakeoff.cu:592-642)
    for name, N, K in (("a", 64, 256), ("odd", 33, 512)):
        codes, scales = rng.make_q2(N, K)
        p = f"{name}_q2_"
        out[p + "codes"], out[p + "scales"] = codes, scales
        out[p + "packed"] = refbind.pack_q2(codes, scales, False)
        out[p + "packed_sab"] = refbind.pack_q2(codes, scales, True)
        x = rng.uniform_x(1, K)
        val, mag = refbind.q2_values(codes, scales, x[0])
        out[p + "x0"], out[p + "val0"], out[p + "mag0"] = x, val[None, :], mag[None, :]
    # the survey's probe: mt19937(1234), 8192x2048 q4 -- first packed words and the first row's reference value
    rng2 = refbind.Rng(1234)
    codes, scales = rng2.make_weights(8192, 2048, 4)
    packed = refbind.pack_q4(codes[:2], scales[:2], False)
    x = rng2.uniform_x(1, 2048)
    val, mag = refbind.values(codes[:4], scales[:4], x)
    out["probe_packed_row0"] = packed[0]
    out["probe_codes_row0"], out["probe_scales_row0"] = codes[0], scales[0]
    out["probe_x"], out["probe_val"], out["probe_mag"] = x, val, mag
    np.savez_compressed(os.path.join(HERE, "reference_vectors.npz"), **out)
    print(f"wrote {len(out)} arrays to tests/golden/reference_vectors.npz")


if __name__ == "__main__":
    main()
