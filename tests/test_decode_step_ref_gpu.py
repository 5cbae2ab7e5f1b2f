"""The batched device decode step (kvl_mla_decode_step_bf16) against the
reference runtime's own kvl_mla_decode_compressed_bf16
(src/mla_compressed_state.c:86-161, compiled from its sources into
oracle/_ref) on the same weights, cached rows and tokens.

The cached rows are bf16 values written straight into the reference state's
public latent/rope arrays (exact in fp32), so both sides attend the same
rows.  Batches of 16 and more run the tcgen05 projections (split-K q, kv_a
and o GEMMs, batched per-head W_UK / W_UV products); one case carries a
sequence at 32768 cached rows, the config-4 length.  Checked: every output
row and every appended state row, within rel-L2 <= 1e-2 and max-abs <= 2e-2.
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
    total = int(sum(L + 1 for L in lens))
    pool = np.zeros((total + 128, R + DR), np.uint16)
    for b, L in enumerate(lens):
        pool[row0[b]:row0[b] + L] = S.normal_bf16(seed + 7 + b, S.S_LAT, (L, R + DR), 1.0)
    x = S.bf16_bits_to_f32(S.normal_bf16(seed + 3, S.S_X, (B, H), 1.0))

    want, app_lat, app_rope = [], [], []
    for b, L in enumerate(lens):
        rows = S.bf16_bits_to_f32(pool[row0[b]:row0[b] + L])
        out, lat_new, rope_new = ref.decode_from_rows(x[b], rcfg, w.arrays, rows[:, :R], rows[:, R:])
        want.append(out)
        app_lat.append(lat_new)
        app_rope.append(rope_new)

    dev = torch.device("cuda", 0)
    d_kv = torch.from_numpy(pool.view(np.int16)).to(dev)
    ts = [torch.from_numpy(a.view(np.int16)).to(dev) for a in w.arrays]
    dw = K.KvlMlaDeviceWeights(*[t.data_ptr() for t in ts])
    plan = K.AttendPlan([L + 1 for L in lens], row0, NH, R)
    d_x = torch.from_numpy(x).to(dev)
    d_out = torch.empty((B, H), dtype=torch.float32, device=dev)
    d_row = torch.tensor([int(row0[b]) + L for b, L in enumerate(lens)], dtype=torch.int64, device=dev)
    d_pos = torch.tensor(lens, dtype=torch.int32, device=dev)
    ws = torch.empty(lib.kvl_mla_decode_step_workspace_bytes(C.byref(cfg), B), dtype=torch.uint8, device=dev)
    rc = lib.kvl_mla_decode_step_bf16(C.byref(cfg), C.byref(dw), plan.h, d_out.data_ptr(), d_x.data_ptr(),
                                      d_kv.data_ptr(), total + 128, d_row.data_ptr(), d_pos.data_ptr(), B,
                                      ws.data_ptr(), C.c_void_p(0))
    assert rc == 0, K.last_error()
    torch.cuda.synchronize()
    assert plan.check() == 0, K.last_error()
    got = d_out.cpu().numpy()
    kv_after = d_kv.cpu().numpy().view(np.uint16)
    for b, L in enumerate(lens):
        assert_close(got[b], want[b], what=f"decode step vs reference, seq {b} (L={L})")
        row = S.bf16_bits_to_f32(kv_after[row0[b] + L])
        assert_close(row[:R], app_lat[b], what=f"appended latent, seq {b}")
        assert_close(row[R:], app_rope[b], what=f"appended rope, seq {b}")
        np.testing.assert_array_equal(kv_after[row0[b]:row0[b] + L], pool[row0[b]:row0[b] + L])


def test_decode_step_batch64_vs_reference(K, S, ref, torch_cuda):
    """64 ragged sequences: the tensor-core projections at a config-4-like batch."""
    lens = [int(v) for v in S.uniform_ints(201, S.S_LEN, 64, 1, 600)]
    _run(K, S, ref, torch_cuda, lens, 201)


def test_decode_step_long_sequence_vs_reference(K, S, ref, torch_cuda):
    """16 sequences (tensor-core path), one at 32768 cached rows; RoPE theta 800000."""
    lens = [32768] + [int(v) for v in S.uniform_ints(202, S.S_LEN, 15, 1, 300)]
    _run(K, S, ref, torch_cuda, lens, 202, theta=800000.0)


def test_decode_step_small_batch_vs_reference(K, S, ref, torch_cuda):
    """Below 16 sequences: the per-token matvec path."""
    _run(K, S, ref, torch_cuda, [5000, 1, 129], 203)
