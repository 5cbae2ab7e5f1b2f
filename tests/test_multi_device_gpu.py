"""One process, two GPUs: attend plans and states created on each device in
turn.  The tcgen05 attend kernels need more than 48 KB of dynamic shared
memory, an attribute that belongs to each device's context; the launches on
the second device must carry it too.  Checked against the CPU restatement of
the reference attend core (src/mla_compressed_state.c:132-148,
src/mla_compressed_q8_state.c:216-238) at the decode tolerance.  Needs two
GPUs; skipped otherwise."""
from __future__ import annotations

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

NH, R, DR = 16, 512, 64
SCALE = 1.0 / np.sqrt(192.0)


def test_attend_on_two_devices_in_one_process(K, S, orc, torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    lens, rows = [3000, 700], 3700
    row0 = [0, 3000]
    lat = S.normal_bf16(41, S.S_LAT, (rows, R), 1.0)
    rope = S.normal_bf16(41, S.S_ROPE, (rows, DR), 1.0)
    kv = np.concatenate([lat, rope], axis=1)
    lat8 = S.uniform_int8(42, S.S_LAT, (rows, R))
    sc = S.uniform_f32(42, S.S_SCALE, (rows,), 0.001, 0.02)
    q = S.bf16_bits_to_f32(S.normal_bf16(43, S.S_Q, (2, NH, R + DR), 0.1))
    for dev_i in (0, 1, 0, 1):
        torch.cuda.set_device(dev_i)
        dev = torch.device("cuda", dev_i)
        plan = K.AttendPlan(lens, row0, NH, R)
        kv_t = torch.from_numpy(kv.view(np.int16)).to(dev)
        q_t = torch.from_numpy(q).to(dev)
        out = torch.full((2, NH, R), float("nan"), device=dev)
        assert plan.attend_bf16(out, None, q_t, kv_t, rows) == 0, K.last_error()
        assert plan.check() == 0, K.last_error()
        o = out.cpu().numpy()
        out8 = torch.full((2, NH, R), float("nan"), device=dev)
        assert plan.attend_q8(out8, None, q_t, torch.from_numpy(lat8).to(dev), torch.from_numpy(sc).to(dev),
                              torch.from_numpy(rope.view(np.int16)).to(dev), rows) == 0, K.last_error()
        assert plan.check() == 0, K.last_error()
        o8 = out8.cpu().numpy()
        for b, (L, r0) in enumerate(zip(lens, row0)):
            want, _ = orc.attend_f32(q[b], S.bf16_bits_to_f32(lat[r0:r0 + L]), S.bf16_bits_to_f32(rope[r0:r0 + L]),
                                     SCALE)
            assert_close(o[b], want, what=f"bf16 attend on device {dev_i}, seq {b}")
            want8, _ = orc.attend_q8(q[b], lat8[r0:r0 + L], sc[r0:r0 + L], rope[r0:r0 + L], SCALE)
            assert_close(o8[b], want8, what=f"Q8 attend on device {dev_i}, seq {b}")
        del plan
    torch.cuda.set_device(0)
