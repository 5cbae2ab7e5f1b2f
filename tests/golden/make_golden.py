#!/usr/bin/env python3
"""Generates the golden fixtures under tests/golden/ from the reference
runtime's own C code, compiled from its sources by oracle/Makefile into
oracle/_ref/ (scalar build: double-accumulating matvec; AVX2 build: the CI
configuration).  Run in a container where the reference sources exist:

    make -f oracle/Makefile all REF=<reference checkout> && python tests/golden/make_golden.py

Inputs are regenerated from seeds by in-c-test_b200/synth.py; each fixture
stores the seeds, a digest of the generated inputs (so a drifting generator is
caught) and the reference outputs.

Cases (shapes of the reference's own MLA gates):
  incremental  S=5, H=16, NH=2, DN=DR=DV=4, R=6, theta 1e4, eps 1e-6
               (src/mla_incremental_probe.c:33, :58)
  spec_q8      S=13, H=64, NH=4, DN=DR=DV=8, R=32, theta 1e4, eps 1e-6
               (src/spec_q8_lab_probe.c:44-47, :83)
  kimi         S=6, production dims, theta 8e5 (src/generate.c:11-18)
  kimi_50k     S=4, production dims, theta 5e4
For each: decode outputs after a state prefill of 2 rows (fp32 and Q8 state),
the Q8 state bytes, and the causal prefill output.
"""
from __future__ import annotations

import hashlib
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import kvl_pkg  # noqa: E402

kvl_pkg.load()
import kvl_b200.synth as SY  # noqa: E402
from oracle.oracle import REF_SCALAR_SO, REF_SO, Reference, cfg_of  # noqa: E402

CASES = {
    "incremental": dict(S=5, H=16, NH=2, DN=4, DR=4, DV=4, R=6, eps=1e-6, theta=10000.0, wstd=0.05, seed=101),
    "spec_q8": dict(S=13, H=64, NH=4, DN=8, DR=8, DV=8, R=32, eps=1e-6, theta=10000.0, wstd=0.036, seed=102),
    "kimi": dict(S=6, H=2048, NH=16, DN=128, DR=64, DV=128, R=512, eps=1e-5, theta=800000.0, wstd=0.02, seed=103),
    "kimi_50k": dict(S=4, H=2048, NH=16, DN=128, DR=64, DV=128, R=512, eps=1e-5, theta=50000.0, wstd=0.02,
                     seed=104),
}
PREFIX = 2


def case_inputs(c):
    s = c["seed"]
    H, NH, DN, DR, DV, R = c["H"], c["NH"], c["DN"], c["DR"], c["DV"], c["R"]
    w = [SY.normal_bf16(s, SY.S_WQ, (NH * (DN + DR), H), c["wstd"]),
         SY.normal_bf16(s, SY.S_WKVA, (R + DR, H), c["wstd"]),
         SY.f32_to_bf16_bits(1.0 + SY.normal(s, 40, R, 0.05)),
         SY.normal_bf16(s, SY.S_WKVB, (NH * (DN + DV), R), c["wstd"]),
         SY.normal_bf16(s, SY.S_WO, (H, NH * DV), c["wstd"])]
    x = SY.normal(s, SY.S_X, c["S"] * H, 0.5).reshape(c["S"], H)
    return w, x


def digest(arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    out_dir = pathlib.Path(__file__).resolve().parent
    refs = {"scalar": Reference(REF_SCALAR_SO), "avx2": Reference(REF_SO)}
    for name, c in CASES.items():
        w, x = case_inputs(c)
        cfg = cfg_of(c["H"], c["NH"], c["DN"], c["DR"], c["DV"], c["R"], c["eps"], c["theta"])
        rec = {"digest": np.array(digest(w + [x]))}
        for k, v in c.items():
            rec["cfg_" + k] = np.array(v)
        for tag, ref in refs.items():
            dec, (lat, rope) = ref.decode_sequence(x, cfg, w, prefix=PREFIX)
            dq8, (l8, ls, r16) = ref.decode_sequence(x, cfg, w, prefix=PREFIX, q8=True)
            rec[f"{tag}_decode"] = dec
            rec[f"{tag}_state_latent"] = lat
            rec[f"{tag}_state_rope"] = rope
            rec[f"{tag}_q8_decode"] = dq8
            rec[f"{tag}_q8_latent"] = l8
            rec[f"{tag}_q8_scale"] = ls
            rec[f"{tag}_q8_rope"] = r16
            rec[f"{tag}_prefill"] = ref.prefill(x, cfg, w)
        np.savez_compressed(out_dir / f"{name}.npz", **rec)
        print(name, "written", sum(v.nbytes for v in rec.values()), "bytes")


if __name__ == "__main__":
    main()
