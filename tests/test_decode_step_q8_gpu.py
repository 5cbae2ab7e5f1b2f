"""The batched Q8 decode step (kvl_mla_decode_step_q8) against the reference
runtime's own kvl_mla_decode_compressed_q8_bf16
(src/mla_compressed_q8_state.c:161-255, compiled from its sources into
oracle/_ref) on the same weights, cached rows and tokens.

Cached rows are written straight into the reference state's public arrays
(int8 latent, fp32 scale, bf16 rope) and into the device pool in the same
layout.  Checked: every output row (rel-L2 <= 1e-2, max-abs <= 2e-2) and every
appended row -- its int8 latent agrees byte for byte except where the fp32
kv_a projection rounds differently (at least 98% equal, all within one
quantisation step), its scale to 1e-4 relative, its bf16 rope within the
output tolerance -- and the cached rows are untouched.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

H, NH, R, DR = 2048, 16, 512, 64


def _run(K, S, ref, torch, lens, seed, theta=50000.0):
    from oracle.oracle import cfg_of
    lib = K.load()
    cfg = K.make_config(H, NH, 128, DR, 128, R, 1e-5, theta)
    rcfg = cfg_of(H, NH, 128, DR, 128, R, 1e-5, theta)
    w = K.random_weights(cfg, seed, 0.02, norm_std=0.05)
    B = len(lens)
    row0 = np.concatenate([[0], np.cumsum([L + 1 for L in lens])[:-1]]).astype(np.int64)
    total = int(sum(L + 1 for L in lens)) + 128
    lat8 = np.zeros((total, R), np.int8)
    scale = np.ones(total, np.float32)
    rope = np.zeros((total, DR), np.uint16)
    for b, L in enumerate(lens):
        lat8[row0[b]:row0[b] + L] = S.uniform_int8(seed + 7 + b, S.S_LAT, (L, R))
        scale[row0[b]:row0[b] + L] = S.uniform_f32(seed + 7 + b, S.S_SCALE, (L,), 0.001, 0.02)
        rope[row0[b]:row0[b] + L] = S.normal_bf16(seed + 7 + b, S.S_ROPE, (L, DR), 1.0)
    x = S.bf16_bits_to_f32(S.normal_bf16(seed + 3, S.S_X, (B, H), 1.0))

    want, app = [], []
    for b, L in enumerate(lens):
        sl = slice(row0[b], row0[b] + L)
        out, q_new, s_new, r_new = ref.decode_q8_from_rows(x[b], rcfg, w.arrays, lat8[sl], scale[sl], rope[sl])
        want.append(out)
        app.append((q_new, s_new, r_new))

    dev = torch.device("cuda", 0)
    d_lat8 = torch.from_numpy(lat8).to(dev)
    d_scale = torch.from_numpy(scale).to(dev)
    d_rope = torch.from_numpy(rope.view(np.int16)).to(dev)
    ts = [torch.from_numpy(a.view(np.int16)).to(dev) for a in w.arrays]
    dw = K.KvlMlaDeviceWeights(*[t.data_ptr() for t in ts])
    plan = K.AttendPlan([L + 1 for L in lens], row0, NH, R)
    d_x = torch.from_numpy(x).to(dev)
    d_out = torch.empty((B, H), dtype=torch.float32, device=dev)
    d_row = torch.tensor([int(row0[b]) + L for b, L in enumerate(lens)], dtype=torch.int64, device=dev)
    d_pos = torch.tensor(lens, dtype=torch.int32, device=dev)
    ws = torch.empty(lib.kvl_mla_decode_step_workspace_bytes(C.byref(cfg), B), dtype=torch.uint8, device=dev)
    rc = lib.kvl_mla_decode_step_q8(C.byref(cfg), C.byref(dw), plan.h, d_out.data_ptr(), d_x.data_ptr(),
                                    d_lat8.data_ptr(), d_scale.data_ptr(), d_rope.data_ptr(), total,
                                    d_row.data_ptr(), d_pos.data_ptr(), B, ws.data_ptr(), C.c_void_p(0))
    assert rc == 0, K.last_error()
    torch.cuda.synchronize()
    assert plan.check() == 0, K.last_error()
    got = d_out.cpu().numpy()
    l8_after = d_lat8.cpu().numpy()
    sc_after = d_scale.cpu().numpy()
    rp_after = d_rope.cpu().numpy().view(np.uint16)
    new_l8 = np.stack([l8_after[row0[b] + L] for b, L in enumerate(lens)])
    want_l8 = np.stack([a[0] for a in app])
    for b, L in enumerate(lens):
        assert_close(got[b], want[b], what=f"Q8 decode step vs reference, seq {b} (L={L})")
        r = row0[b] + L
        assert abs(float(sc_after[r]) - app[b][1]) <= 1e-4 * abs(app[b][1]), f"appended scale, seq {b}"
        assert_close(S.bf16_bits_to_f32(rp_after[r]), S.bf16_bits_to_f32(app[b][2]), what=f"appended rope, seq {b}")
        np.testing.assert_array_equal(l8_after[row0[b]:row0[b] + L], lat8[row0[b]:row0[b] + L])
        np.testing.assert_array_equal(rp_after[row0[b]:row0[b] + L], rope[row0[b]:row0[b] + L])
    assert np.mean(new_l8 == want_l8) > 0.98
    assert np.max(np.abs(new_l8.astype(int) - want_l8.astype(int))) <= 1


def test_decode_step_q8_batch64_vs_reference(K, S, ref, torch_cuda):
    """64 ragged sequences at config-3 lengths (a 2048-row cap keeps the CPU
    reference within seconds): the tensor-core projections and the int8 attend."""
    lens = [int(v) for v in S.uniform_ints(211, S.S_LEN, 64, 1, 2048)]
    _run(K, S, ref, torch_cuda, lens, 211)


def test_decode_step_q8_long_sequence_vs_reference(K, S, ref, torch_cuda):
    """16 sequences, one at 8192 cached rows (config 3's longest); RoPE theta 800000."""
    lens = [8192] + [int(v) for v in S.uniform_ints(212, S.S_LEN, 15, 1, 600)]
    _run(K, S, ref, torch_cuda, lens, 212, theta=800000.0)


def test_decode_step_q8_small_batch_vs_reference(K, S, ref, torch_cuda):
    """Below 16 sequences: the per-token matvec path."""
    _run(K, S, ref, torch_cuda, [3000, 1, 129], 213)
