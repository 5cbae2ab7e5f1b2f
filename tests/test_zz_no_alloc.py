"""kvl_mla_attend_bf16_noalloc: the single-sequence decode attend whose
scratch lives in a fixed device array, for callers that cannot allocate
device memory while they decode.

It must give what the allocating entry point (kvl_mla_attend_bf16 with a
plan) gives, and what the CPU restatement of the reference attend core
(src/mla_compressed_state.c:132-148) gives, within the parity tolerance of the
other tests (rel-L2 <= 1e-2, max-abs <= 2e-2), on consecutive calls that share
the array, and it must reject sizes its array cannot hold.  This file sorts last so that a failure
here comes after every other test has run; it also passes on its own in a
fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

R, DR, NH = 512, 64, 16
SCALE = 1.0 / np.sqrt(192.0)


def _inputs(S, seed, rows, batch=1):
    lat = S.normal_bf16(seed, S.S_LAT, (rows, R), 1.0)
    rope = S.normal_bf16(seed, S.S_ROPE, (rows, DR), 1.0)
    kv = np.concatenate([lat, rope], axis=1)
    q = S.bf16_bits_to_f32(S.normal_bf16(seed, S.S_Q, (batch, NH, R + DR), 0.1))
    return kv, q


def _allocating(K, torch, kv_t, q_t, rows, L, r0):
    out = torch.full((1, NH, R), float("nan"), device="cuda")
    lse = torch.full((1, NH), float("nan"), device="cuda")
    plan = K.AttendPlan([L], [r0], NH, R)
    assert plan.attend_bf16(out, lse, q_t, kv_t, rows, rope_dim=DR, scale=SCALE) == 0, K.last_error()
    assert plan.check() == 0, K.last_error()
    return out.cpu().numpy()[0], lse.cpu().numpy()[0]


def _noalloc(K, torch, kv_t, q_t, rows, L, r0, splits=0):
    out = torch.full((1, NH, R), float("nan"), device="cuda")
    lse = torch.full((1, NH), float("nan"), device="cuda")
    rc = K.load().kvl_mla_attend_bf16_noalloc(out.data_ptr(), lse.data_ptr(), q_t.data_ptr(), kv_t.data_ptr(),
                                              rows, L, r0, NH, R, DR, splits, float(SCALE), 0)
    torch.cuda.synchronize()
    return rc, out.cpu().numpy()[0], lse.cpu().numpy()[0]


def test_noalloc_matches_allocating_entry_point_on_consecutive_calls(K, S, orc, torch_cuda):
    torch = torch_cuda
    rows = 20000
    kv, q = _inputs(S, 31, rows)
    kv_t = torch.from_numpy(kv.view(np.int16)).cuda()
    q_t = torch.from_numpy(q).cuda()
    # Two calls in a row sharing the array: a long split sequence, then a
    # shorter one at another offset with fewer ranges, then a one-range call.
    for L, r0, splits in [(13000, 0, 0), (3001, 15000, 7), (100, 123, 0)]:
        rc, got, got_lse = _noalloc(K, torch, kv_t, q_t, rows, L, r0, splits)
        assert rc == 0, K.last_error()
        want, want_lse = _allocating(K, torch, kv_t, q_t, rows, L, r0)
        assert_close(got, want, what=f"noalloc L={L} splits={splits}")
        assert np.max(np.abs(got_lse - want_lse)) < 1e-2
        # the same call against the oracle's restatement of the reference attend
        lat = S.bf16_bits_to_f32(kv[r0:r0 + L, :R])
        rope = S.bf16_bits_to_f32(kv[r0:r0 + L, R:])
        ref_mix, ref_lse = orc.attend_f32(q[0], lat, rope, SCALE)
        assert_close(got, ref_mix, what=f"noalloc vs oracle L={L} splits={splits}")
        assert np.max(np.abs(got_lse - ref_lse)) < 2e-2, f"lse vs oracle L={L}"


def test_noalloc_rejects_sizes_beyond_its_array(K, S, torch_cuda):
    torch = torch_cuda
    rows = 512
    kv, q = _inputs(S, 32, rows)
    kv_t = torch.from_numpy(kv.view(np.int16)).cuda()
    q_t = torch.from_numpy(q).cuda()
    rc, _, _ = _noalloc(K, torch, kv_t, q_t, rows, 500, 0, splits=149)
    assert rc == -1 and "at most 148" in K.last_error()
    rc, _, _ = _noalloc(K, torch, kv_t, q_t, rows, 600, 0)
    assert rc == -1 and "sequence range" in K.last_error()
    rc = K.load().kvl_mla_attend_bf16_noalloc(0, 0, q_t.data_ptr(), kv_t.data_ptr(), rows, 10, 0, NH, R, DR, 0,
                                              float(SCALE), 0)
    assert rc == -1
