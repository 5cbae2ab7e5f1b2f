"""Parity of the decode attend kernels (device-pointer C-ABI) against the CPU
restatement of src/mla_compressed_state.c:132-148 and
src/mla_compressed_q8_state.c:216-238, on seeded inputs.

Tolerance: rel-L2 <= 1e-2 and max-abs <= 2e-2 of the
fp32/double reference; lse within 1e-2 absolute.
"""
from __future__ import annotations

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

R, DR, NH = 512, 64, 16
SCALE = 1.0 / np.sqrt(192.0)


def bf16_pool(S, seed, rows, R=R, DR=DR):
    lat = S.normal_bf16(seed, S.S_LAT, (rows, R), 1.0)
    rope = S.normal_bf16(seed, S.S_ROPE, (rows, DR), 1.0)
    kv = np.concatenate([lat, rope], axis=1)
    return kv, S.bf16_bits_to_f32(lat), S.bf16_bits_to_f32(rope)


def q8_pool(S, seed, rows, R=R, DR=DR):
    lat8 = S.uniform_int8(seed, S.S_LAT, (rows, R))
    scale = S.uniform_f32(seed, S.S_SCALE, (rows,), 0.001, 0.02)
    rope = S.normal_bf16(seed, S.S_ROPE, (rows, DR), 1.0)
    return lat8, scale, rope


def absorbed_q(S, seed, batch, nh=NH, R=R, DR=DR, std=0.1):
    return S.bf16_bits_to_f32(S.normal_bf16(seed, S.S_Q, (batch, nh, R + DR), std))


def run_bf16(K, torch, kv, q, lens, row0, max_ctas=0, nh=NH, R=R, DR=DR):
    dev = torch.device("cuda:0")
    kv_t = torch.from_numpy(kv.view(np.int16)).to(dev)
    q_t = torch.from_numpy(q).to(dev)
    out = torch.full((len(lens), nh, R), float("nan"), device=dev)
    lse = torch.full((len(lens), nh), float("nan"), device=dev)
    plan = K.AttendPlan(lens, row0, nh, R, max_ctas)
    rc = plan.attend_bf16(out, lse, q_t, kv_t, kv.shape[0], rope_dim=DR, scale=SCALE)
    assert rc == 0, K.last_error()
    assert plan.check() == 0, K.last_error()
    return out.cpu().numpy(), lse.cpu().numpy(), plan.info()


def run_q8(K, torch, lat8, scale, rope, q, lens, row0, max_ctas=0, nh=NH, R=R, DR=DR):
    dev = torch.device("cuda:0")
    out = torch.full((len(lens), nh, R), float("nan"), device=dev)
    lse = torch.full((len(lens), nh), float("nan"), device=dev)
    plan = K.AttendPlan(lens, row0, nh, R, max_ctas)
    rc = plan.attend_q8(out, lse, torch.from_numpy(q).to(dev), torch.from_numpy(lat8).to(dev),
                        torch.from_numpy(scale).to(dev), torch.from_numpy(rope.view(np.int16)).to(dev),
                        lat8.shape[0], rope_dim=DR, scale=SCALE)
    assert rc == 0, K.last_error()
    assert plan.check() == 0, K.last_error()
    return out.cpu().numpy(), lse.cpu().numpy(), plan.info()


@pytest.mark.parametrize("L", [1, 7, 63, 64, 65, 130, 1024, 4097])
@pytest.mark.parametrize("max_ctas", [0, 1, 3])
def test_bf16_single_sequence(K, S, orc, torch_cuda, L, max_ctas):
    kv, lat, rope = bf16_pool(S, 1, L)
    q = absorbed_q(S, 1, 1)
    out, lse, info = run_bf16(K, torch_cuda, kv, q, [L], [0], max_ctas)
    mix, lse_ref = orc.attend_f32(q[0], lat, rope, SCALE)
    assert_close(out[0], mix, what=f"bf16 L={L} {info}")
    assert np.max(np.abs(lse[0] - lse_ref)) < 1e-2


def test_bf16_config1_parity(K, S, orc, torch_cuda):
    """one sequence, L=1024, latent/rope ~N(0,1), q ~N(0,0.1)."""
    kv, lat, rope = bf16_pool(S, 1, 1024)
    q = absorbed_q(S, 1, 1)
    out, _, _ = run_bf16(K, torch_cuda, kv, q, [1024], [0])
    mix, _ = orc.attend_f32(q[0], lat, rope, SCALE)
    r, m = assert_close(out[0], mix, what="config 1")
    print(f"config1 rel_l2={r:.3e} max_abs={m:.3e}")


@pytest.mark.parametrize("max_ctas", [0, 5, 1])
def test_bf16_ragged_batch(K, S, orc, torch_cuda, max_ctas):
    lens = [1, 700, 64, 3001, 129, 2048]
    gaps = [0, 17, 3, 100, 0, 64]
    row0, r = [], 0
    for n, g in zip(lens, gaps):
        r += g
        row0.append(r)
        r += n
    kv, lat, rope = bf16_pool(S, 2, r + 5)
    q = absorbed_q(S, 2, len(lens))
    out, lse, info = run_bf16(K, torch_cuda, kv, q, lens, row0, max_ctas)
    for b, (n, r0) in enumerate(zip(lens, row0)):
        mix, lse_ref = orc.attend_f32(q[b], lat[r0:r0 + n], rope[r0:r0 + n], SCALE)
        assert_close(out[b], mix, what=f"seq {b} L={n} {info}")
        assert np.max(np.abs(lse[b] - lse_ref)) < 1e-2


@pytest.mark.parametrize("L", [1, 100, 1000])
def test_garbage_after_sequence_end(K, S, orc, torch_cuda, L):
    """Rows after a sequence's end (inside its last 64-row tile) may hold any
    bits, NaN included; they must not leak into the output."""
    kv, lat, rope = bf16_pool(S, 6, L + 64)
    kv[L:] = 0x7FC0  # bf16 NaN
    q = absorbed_q(S, 6, 1)
    out, lse, _ = run_bf16(K, torch_cuda, kv, q, [L], [0])
    mix, _ = orc.attend_f32(q[0], lat[:L], rope[:L], SCALE)
    assert_close(out[0], mix, what=f"nan tail L={L}")
    lat8, scale, rope16 = q8_pool(S, 6, L + 64)
    scale[L:] = np.nan
    rope16[L:] = 0x7FC0
    out, _, _ = run_q8(K, torch_cuda, lat8, scale, rope16, q, [L], [0])
    mix, _ = orc.attend_q8(q[0], lat8[:L], scale[:L], rope16[:L], SCALE)
    assert_close(out[0], mix, what=f"q8 nan tail L={L}")


def test_bf16_peaked_scores(K, S, orc, torch_cuda):
    """Large scores exercise the online-softmax rescaling of the running max."""
    L = 2000
    kv, lat, rope = bf16_pool(S, 3, L)
    q = absorbed_q(S, 3, 1, std=1.5)
    out, _, _ = run_bf16(K, torch_cuda, kv, q, [L], [0], 4)
    mix, _ = orc.attend_f32(q[0], lat, rope, SCALE)
    assert_close(out[0], mix, what="peaked")


@pytest.mark.parametrize("L", [1, 65, 1024, 3000])
@pytest.mark.parametrize("max_ctas", [0, 2])
def test_q8_single_sequence(K, S, orc, torch_cuda, L, max_ctas):
    lat8, scale, rope = q8_pool(S, 4, L)
    q = absorbed_q(S, 4, 1)
    out, lse, info = run_q8(K, torch_cuda, lat8, scale, rope, q, [L], [0], max_ctas)
    mix, lse_ref = orc.attend_q8(q[0], lat8, scale, rope, SCALE)
    assert_close(out[0], mix, what=f"q8 L={L} {info}")
    assert np.max(np.abs(lse[0] - lse_ref)) < 1e-2


def test_q8_ragged_batch(K, S, orc, torch_cuda):
    """BASELINE config 3 shape, reduced: ragged lengths uniform in [512, 8192]."""
    lens = [int(v) for v in S.uniform_ints(3, S.S_LEN, 8, 512, 8192)]
    row0 = np.concatenate([[0], np.cumsum(lens)[:-1]]).tolist()
    rows = int(sum(lens))
    lat8, scale, rope = q8_pool(S, 3, rows)
    q = absorbed_q(S, 3, len(lens))
    out, _, info = run_q8(K, torch_cuda, lat8, scale, rope, q, lens, row0)
    for b, (n, r0) in enumerate(zip(lens, row0)):
        mix, _ = orc.attend_q8(q[b], lat8[r0:r0 + n], scale[r0:r0 + n], rope[r0:r0 + n], SCALE)
        assert_close(out[b], mix, what=f"q8 seq {b} L={n} {info}")


@pytest.mark.parametrize("nh,R,DR", [(2, 6, 4), (4, 32, 8), (16, 512, 32)])
def test_generic_shapes(K, S, orc, torch_cuda, nh, R, DR):
    """Non-production head shapes run the CUDA-core kernel."""
    L = 300
    kv, lat, rope = bf16_pool(S, 5, L, R, DR)
    q = absorbed_q(S, 5, 2, nh, R, DR)
    out, _, _ = run_bf16(K, torch_cuda, kv, q, [L, 100], [0, 200], 0, nh, R, DR)
    mix0, _ = orc.attend_f32(q[0], lat, rope, SCALE)
    mix1, _ = orc.attend_f32(q[1], lat[200:300], rope[200:300], SCALE)
    assert_close(out[0], mix0, what="generic seq0")
    assert_close(out[1], mix1, what="generic seq1")


def test_q8_peaked_scores(K, S, orc, torch_cuda):
    """Large scores move the running maximum often: the int8 kernel rescales
    its folded P'.V sums and splits P' against small tile maxima."""
    L = 2000
    lat8, scale, rope = q8_pool(S, 7, L)
    q = absorbed_q(S, 7, 1, std=1.5)
    out, lse, _ = run_q8(K, torch_cuda, lat8, scale, rope, q, [L], [0], 4)
    mix, lse_ref = orc.attend_q8(q[0], lat8, scale, rope, SCALE)
    assert_close(out[0], mix, what="q8 peaked")
    assert np.max(np.abs(lse[0] - lse_ref)) < 1e-2


def test_q8_wide_scale_range(K, S, orc, torch_cuda):
    """Row scales spanning four decades below the largest BASELINE scale (0.02,
    so the outputs keep the magnitude the absolute tolerance is set for): the
    per-tile split of P' = p * scale is taken against the largest |P'| of the
    tile, so the small-scale rows get the fewest bits."""
    L = 3000
    lat8, _, rope = q8_pool(S, 8, L)
    scale = (0.02 * 10.0 ** S.uniform_f32(8, S.S_SCALE, (L,), -4.0, 0.0)).astype(np.float32)
    q = absorbed_q(S, 8, 1)
    out, _, _ = run_q8(K, torch_cuda, lat8, scale, rope, q, [L], [0])
    mix, _ = orc.attend_q8(q[0], lat8, scale, rope, SCALE)
    assert_close(out[0], mix, what="q8 wide scale range")


def test_attend_rejects_misaligned_query(K, S, torch_cuda):
    """The decode kernels read the absorbed query as float4: a query that is
    not 16-byte aligned is refused before anything is launched."""
    dev = torch_cuda.device("cuda:0")
    L = 256
    kv, _, _ = bf16_pool(S, 9, L)
    base = torch_cuda.zeros(NH * (R + DR) + 1, device=dev)
    q_bad = base[1:].view(1, NH, R + DR)  # 4 bytes past a 16-byte boundary
    out = torch_cuda.zeros((1, NH, R), device=dev)
    plan = K.AttendPlan([L], [0], NH, R)
    rc = plan.attend_bf16(out, None, q_bad, torch_cuda.from_numpy(kv.view(np.int16)).to(dev), L)
    assert rc == -1 and "16-byte aligned" in K.last_error()
    lat8, scale, rope = q8_pool(S, 9, L)
    rc = plan.attend_q8(out, None, q_bad, torch_cuda.from_numpy(lat8).to(dev), torch_cuda.from_numpy(scale).to(dev),
                        torch_cuda.from_numpy(rope.view(np.int16)).to(dev), L)
    assert rc == -1 and "16-byte aligned" in K.last_error()
