"""Bit-exactness of the Q8 row helpers against the CPU restatement:
quantiser (src/mla_compressed_q8_state.c:34-55), dequantiser (:57-61) and
bf16 RNE with truncated Inf/NaN (:9-16)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _edge_rows(S, R=512):
    rows = [S.normal(11, 0, R, 1.0), np.zeros(R, np.float32), S.normal(11, 1, R, 1e-30),
            S.normal(11, 2, R, 3e4), np.full(R, 0.5, np.float32)]
    r = S.normal(11, 3, R, 1.0).copy()
    r[5] = np.inf
    rows.append(r)
    r = S.normal(11, 4, R, 1.0).copy()
    r[9] = np.nan
    rows.append(r)
    # exact .5 ties after scaling: amax 127 -> inv 1.0
    r = (np.arange(R, dtype=np.float32) % 255 - 127) + 0.5
    r[0] = 127.0
    rows.append(np.clip(r, -127, 127).astype(np.float32))
    return np.stack(rows).astype(np.float32)


def test_quantize_rows_bit_exact(K, S, orc, torch_cuda):
    torch = torch_cuda
    x = np.concatenate([_edge_rows(S), S.normal(12, 0, 256 * 512, 2.0).reshape(256, 512)])
    qd = torch.empty(x.shape, dtype=torch.int8, device="cuda")
    sd = torch.empty(x.shape[0], dtype=torch.float32, device="cuda")
    xd = torch.from_numpy(x).cuda()
    assert K.load().kvl_mla_q8_quantize_rows(qd.data_ptr(), sd.data_ptr(), xd.data_ptr(), x.shape[0], 512, 0) == 0
    torch.cuda.synchronize()
    q_ref, s_ref = orc.quantize_rows(x)
    np.testing.assert_array_equal(qd.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sd.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


def test_dequant_bit_exact(K, S, orc, torch_cuda):
    torch = torch_cuda
    rows = 4096
    q = S.uniform_int8(13, 0, (rows, 512))
    s = S.uniform_f32(13, 1, (rows,), 0.001, 0.02)
    out = torch.empty((rows, 512), dtype=torch.float32, device="cuda")
    assert K.load().kvl_mla_q8_dequant(out.data_ptr(), torch.from_numpy(q).cuda().data_ptr(),
                                       torch.from_numpy(s).cuda().data_ptr(), rows, 512, 0) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), orc.dequant(q, s).view(np.uint32))


def test_bf16_rne_bit_exact(K, S, orc, torch_cuda):
    torch = torch_cuda
    x = S.normal(14, 0, 1 << 16, 10.0)
    special = np.array([0x7F800000, 0xFF800000, 0x7FC00000, 0x7F800001, 0x7F80FFFF, 0x7FFF0000,
                        0x00000001, 0x80000000, 0x3F808000, 0x3F818000, 0x7F7FFFFF], dtype=np.uint32)
    x = np.concatenate([x, special.view(np.float32)])
    out = torch.empty(x.size, dtype=torch.int16, device="cuda")
    assert K.load().kvl_mla_bf16_rne(out.data_ptr(), torch.from_numpy(x).cuda().data_ptr(), x.size, 0) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), orc.bf16_rne(x))
