"""The arithmetic of the int8 tensor-core Q8 attend, restated in numpy.

The Q8 decode kernel (attend_q8.cu) never converts the int8 rows: it splits the
absorbed query per head, and the softmax weights P' = p * scale per head and
128-row tile, into two int8 parts (v ~ s * (hi + lo / 256), s = max|v| / 127),
multiplies them with the int8 rows exactly (int32 sums) and rescales in fp32.
This restatement pins down that method's error against the CPU restatement of
src/mla_compressed_q8_state.c:216-238 on seeded inputs -- the GPU tests then
compare the kernel itself with the same restatement.
"""
from __future__ import annotations

import numpy as np

from tests.parity import assert_close

R, DR, NH, TILE = 512, 64, 16, 128
SCALE = 1.0 / np.sqrt(192.0)


def split16(v, amax):
    """v ~ s * (hi + lo / 256), hi/lo int8, s = amax / 127 (per row of amax)."""
    inv = np.where(amax > 0, 127.0 / np.where(amax > 0, amax, 1.0), 0.0)
    x = v * inv
    hi = np.rint(x)
    lo = np.clip(np.rint((x - hi) * 256.0), -127, 127)
    return hi, lo, amax / 127.0


def attend_q8_split(q, lat8, lscale, rope):
    """q [16][576] fp32, lat8 [L][512] int8, lscale [L], rope [L][64] fp32."""
    k8 = lat8.astype(np.int64)
    qh, ql, sq = split16(q[:, :R].astype(np.float64), np.abs(q[:, :R]).max(1, keepdims=True))
    s_int = qh.astype(np.int64) @ k8.T * 256 + ql.astype(np.int64) @ k8.T  # exact
    q_rope = q[:, R:].astype(np.float32)
    s = (lscale[None, :] * (sq / 256.0) * s_int + q_rope @ rope.T) * SCALE * np.log2(np.e)
    m = s.max(1, keepdims=True)
    pr = np.exp2(s - m)
    out = np.zeros((NH, R))
    for t0 in range(0, lat8.shape[0], TILE):
        pq = pr[:, t0:t0 + TILE] * lscale[None, t0:t0 + TILE]
        ph, pl, sp = split16(pq, np.abs(pq).max(1, keepdims=True))
        o_int = ph.astype(np.int64) @ k8[t0:t0 + TILE] * 256 + pl.astype(np.int64) @ k8[t0:t0 + TILE]
        out += (sp / 256.0) * o_int
    return out / pr.sum(1, keepdims=True)


def _inputs(S, seed, L, scale_lo=0.001, scale_hi=0.02, log_scale=False):
    lat8 = S.uniform_int8(seed, S.S_LAT, (L, R))
    if log_scale:
        lscale = (scale_hi * 10.0 ** S.uniform_f32(seed, S.S_SCALE, (L,), -4.0, 0.0)).astype(np.float32)
    else:
        lscale = S.uniform_f32(seed, S.S_SCALE, (L,), scale_lo, scale_hi)
    rope16 = S.normal_bf16(seed, S.S_ROPE, (L, DR))
    q = S.bf16_bits_to_f32(S.normal_bf16(seed, S.S_Q, (NH, R + DR), 0.1))
    return q, lat8, lscale, rope16


def test_split_method_matches_restatement(S, orc):
    """Config-3 value distributions, a ragged last tile."""
    q, lat8, lscale, rope16 = _inputs(S, 31, 1000)
    got = attend_q8_split(q, lat8, lscale, S.bf16_bits_to_f32(rope16))
    want, _ = orc.attend_q8(q, lat8, lscale, rope16, SCALE)
    r, _ = assert_close(got, want, rel=1e-4, mabs=1e-5, what="int8 split method")
    assert r < 1e-4


def test_split_method_wide_scale_range(S, orc):
    """Row scales over four decades below 0.02: small-scale rows get the
    fewest bits of the per-tile split, and the error stays far inside the
    BASELINE tolerance."""
    q, lat8, lscale, rope16 = _inputs(S, 32, 700, log_scale=True)
    got = attend_q8_split(q, lat8, lscale, S.bf16_bits_to_f32(rope16))
    want, _ = orc.attend_q8(q, lat8, lscale, rope16, SCALE)
    assert_close(got, want, rel=1e-4, mabs=1e-5, what="int8 split method, wide scales")
