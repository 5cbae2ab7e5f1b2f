"""The split-KV combine on the GPU (kvl_mla_merge_partials, part-major arrays,
and kvl_mla_merge_packed, one [o | lse] record per part as an all-gather of each
GPU's buffers produces) against the numpy restatement of the combine
(o = sum_p exp(lse_p - M) o_p / sum_p exp(lse_p - M), lse = M + log sum):
1, 2, 7 and 148 parts (148 = one partial per SM of one long sequence), one and
three sequences, parts with very different lse.  Tolerance 1e-5 relative
(fp32 with a different summation order)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _case(seed, P, B, NH=16, R=512):
    rng = np.random.default_rng(seed)
    o = rng.standard_normal((P, B, NH, R)).astype(np.float32)
    lse = (rng.standard_normal((P, B, NH)) * 3.0).astype(np.float32)
    return o, lse


def _want(o, lse):
    from kvl_b200.parallel import merge_partials
    outs, lses = [], []
    for b in range(o.shape[1]):
        wo, wl = merge_partials(o[:, b].astype(np.float64), lse[:, b].astype(np.float64))
        outs.append(wo)
        lses.append(wl)
    return np.stack(outs), np.stack(lses)


@pytest.mark.parametrize("P,B", [(1, 1), (2, 3), (7, 3), (148, 1)])
def test_merge_partials_and_packed(K, torch_cuda, P, B):
    torch = torch_cuda
    lib = K.load()
    dev = torch.device("cuda", 0)
    o, lse = _case(100 + P * 10 + B, P, B)
    want_o, want_l = _want(o, lse)
    d_o = torch.from_numpy(o).to(dev)
    d_l = torch.from_numpy(lse).to(dev)
    out = torch.empty((B, 16, 512), device=dev)
    out_l = torch.empty((B, 16), device=dev)
    assert lib.kvl_mla_merge_partials(out.data_ptr(), out_l.data_ptr(), d_o.data_ptr(), d_l.data_ptr(), P, B, 16,
                                      512, None) == 0, K.last_error()
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), want_o, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out_l.cpu().numpy(), want_l, rtol=1e-5, atol=1e-5)
    # packed records: [P][B*16*512 + B*16]
    rec = np.concatenate([o.reshape(P, -1), lse.reshape(P, -1)], axis=1)
    d_rec = torch.from_numpy(np.ascontiguousarray(rec)).to(dev)
    out2 = torch.empty_like(out)
    out2_l = torch.empty_like(out_l)
    assert lib.kvl_mla_merge_packed(out2.data_ptr(), out2_l.data_ptr(), d_rec.data_ptr(), P, B, 16, 512,
                                    None) == 0, K.last_error()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out2.cpu().numpy(), out.cpu().numpy())
    np.testing.assert_array_equal(out2_l.cpu().numpy(), out_l.cpu().numpy())
