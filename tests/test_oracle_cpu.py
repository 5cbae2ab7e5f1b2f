"""The CPU oracle (oracle/kvl_oracle.c) pinned to the reference runtime.

1. Against the golden fixtures in tests/golden/ (produced by the reference's own
   C code compiled from its sources, tests/golden/make_golden.py): bit-exact
   against the scalar build (double-accumulating matvec, src/ops.c:19-24) for
   decode outputs, fp32 state rows, Q8 state bytes and the causal prefill; within
   1e-4 relative of the AVX2 build (fp32 matvec, src/ops.c:31-50).
2. Against the compiled reference itself when oracle/_ref is present.
3. The attend core against an independent float64 numpy evaluation.
"""
from __future__ import annotations

import pathlib

import numpy as np
import pytest

from tests.golden.make_golden import CASES, PREFIX, case_inputs, digest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def _cfg(c):
    from oracle.oracle import cfg_of
    return cfg_of(c["H"], c["NH"], c["DN"], c["DR"], c["DV"], c["R"], c["eps"], c["theta"])


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_golden(orc, name):
    c = CASES[name]
    g = np.load(GOLDEN / f"{name}.npz")
    w, x = case_inputs(c)
    assert str(g["digest"]) == digest(w + [x]), "synthetic input generator drifted"
    cfg = _cfg(c)
    dec, (lat, rope) = orc.decode_sequence(x, cfg, w, prefix=PREFIX)
    np.testing.assert_array_equal(dec, g["scalar_decode"])
    np.testing.assert_array_equal(lat, g["scalar_state_latent"])
    np.testing.assert_array_equal(rope, g["scalar_state_rope"])
    dq8, (l8, ls, r16) = orc.decode_sequence(x, cfg, w, prefix=PREFIX, q8=True)
    np.testing.assert_array_equal(dq8, g["scalar_q8_decode"])
    np.testing.assert_array_equal(l8, g["scalar_q8_latent"])
    np.testing.assert_array_equal(ls.view(np.uint32), g["scalar_q8_scale"].view(np.uint32))
    np.testing.assert_array_equal(r16, g["scalar_q8_rope"])
    pre = orc.prefill(x, cfg, w)
    np.testing.assert_array_equal(pre, g["scalar_prefill"])
    # the AVX2 build accumulates the projections in fp32
    assert _rel(dec, g["avx2_decode"]) < 1e-4
    assert _rel(dq8, g["avx2_q8_decode"]) < 1e-2
    assert _rel(pre, g["avx2_prefill"]) < 1e-4


def test_decode_prefill_agreement_in_reference(name="incremental"):
    """The reference's own gate (src/mla_incremental_probe.c:105): compressed
    decode equals causal prefill within 2e-6, seen in the fixtures."""
    g = np.load(GOLDEN / f"{name}.npz")
    assert np.max(np.abs(g["scalar_decode"] - g["scalar_prefill"][PREFIX:])) <= 2e-6


@pytest.mark.parametrize("name", ["incremental", "spec_q8"])
def test_oracle_matches_live_reference(orc, ref_scalar, name):
    c = CASES[name]
    w, x = case_inputs(c)
    cfg = _cfg(c)
    want, _ = ref_scalar.decode_sequence(x, cfg, w, prefix=1)
    got, _ = orc.decode_sequence(x, cfg, w, prefix=1)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("name", ["incremental", "spec_q8"])
def test_oracle_against_reference_lower_layers(orc, ref_scalar, name):
    """The restatement against the reference's lower oracle layers (its V6a
    stack): the expanded-K/V state decode (src/mla_state.c:66-149, decoded from
    position 0) within 2e-6, the gate of src/mla_incremental_probe.c:105, and the
    materialised prefill (src/ops.c:105-192) within 2e-5
    (src/mla_streaming_probe.c:90)."""
    c = CASES[name]
    w, x = case_inputs(c)
    cfg = _cfg(c)
    got, _ = orc.decode_sequence(x, cfg, w, prefix=0)
    want = ref_scalar.decode_expanded(x, cfg, w)
    assert np.max(np.abs(got - want)) <= 2e-6
    mat = ref_scalar.prefill(x, cfg, w, materialized=True)
    assert np.max(np.abs(orc.prefill(x, cfg, w) - mat)) <= 2e-5


def test_attend_core_against_numpy(orc, S):
    L, NH, R, DR = 300, 4, 32, 8
    q = S.normal(7, 0, NH * (R + DR), 0.3).reshape(NH, R + DR)
    lat = S.normal(7, 1, L * R, 1.0).reshape(L, R)
    rope = S.normal(7, 2, L * DR, 1.0).reshape(L, DR)
    scale = 1.0 / np.sqrt(192.0)
    mix, lse = orc.attend_f32(q, lat, rope, scale)
    s = (q[:, :R].astype(np.float64) @ lat.T.astype(np.float64) +
         q[:, R:].astype(np.float64) @ rope.T.astype(np.float64)) * scale
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    want = (p / p.sum(axis=1, keepdims=True)) @ lat.astype(np.float64)
    assert np.max(np.abs(mix - want)) < 1e-5
    assert np.max(np.abs(lse - (m[:, 0] + np.log(p.sum(axis=1))))) < 1e-4


def test_quantiser_edge_cases(orc):
    """src/mla_compressed_q8_state.c:41-53: zero and non-finite rows give zeros
    with scale 1; ties round away from zero; values clamp to +-127."""
    rows = np.array([[0.0] * 4, [np.inf, 1, 2, 3], [127.0, 0.5, -0.5, -127.0], [1e-30, -1e-30, 0, 0]],
                    np.float32)
    q, s = orc.quantize_rows(rows)
    assert (q[0] == 0).all() and s[0] == 1.0
    assert (q[1] == 0).all() and s[1] == 1.0
    assert list(q[2]) == [127, 1, -1, -127] and s[2] == np.float32(1.0)
    assert list(q[3]) == [127, -127, 0, 0]
