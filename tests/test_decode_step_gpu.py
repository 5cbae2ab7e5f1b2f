"""The batched device decode step (kvl_mla_decode_step_bf16: projections,
append of each token's row, attend over a plan, V up-projection, o_proj for a
batch of sequences of one bf16 pool) against the drop-in serial decode
(kvl_mla_decode_compressed_bf16, src/mla_compressed_state.c:86-161) on the
same weights, cached rows and tokens.

Batches below 16 run the per-token matvec kernels; 16 and more run the
tcgen05 GEMM projections (batched per-head products for W_UK and W_UV).
Tolerance: rel-L2 <= 1e-2, max-abs <= 2e-2.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu


def _run(K, S, torch, lens, seed):
    lib = K.load()
    H = 2048
    cfg = K.make_config(H, 16, 128, 64, 128, 512, 1e-5, 50000.0)
    w = K.random_weights(cfg, seed, 0.02, norm_std=0.05)
    xs = [S.normal(seed + 1 + b, S.S_X, (L + 1) * H, 1.0).reshape(L + 1, H) for b, L in enumerate(lens)]

    # reference: state prefill of the cached tokens, then one decode step each
    want, pools, appended = [], [], []
    for b, L in enumerate(lens):
        st = K.CompressedState(cfg, L + 1)
        assert st.prefill(xs[b][:L], w) == 0, K.last_error()
        rows = np.concatenate([st.latent(), st.rope()], axis=1)  # [L][576] fp32 mirror
        pools.append(S.f32_to_bf16_bits(rows.reshape(-1)).reshape(L, 576))
        rc, out = st.decode(xs[b][L], L, w)
        assert rc == 0, K.last_error()
        want.append(out)
        appended.append(np.concatenate([st.latent()[L], st.rope()[L]]))
        st.free()

    # device step: one pool with every sequence's cached rows and room for the new one
    dev = torch.device("cuda", 0)
    row0 = np.concatenate([[0], np.cumsum([L + 1 for L in lens])[:-1]]).astype(np.int64)
    total = int(sum(L + 1 for L in lens))
    pool = np.zeros((total + 128, 576), np.uint16)
    for b, L in enumerate(lens):
        pool[row0[b]:row0[b] + L] = pools[b]
    d_kv = torch.from_numpy(pool.view(np.int16)).to(dev)
    ts = [torch.from_numpy(a.view(np.int16)).to(dev) for a in w.arrays]
    dw = K.KvlMlaDeviceWeights(*[t.data_ptr() for t in ts])
    plan = K.AttendPlan([L + 1 for L in lens], row0, 16, 512)
    d_x = torch.from_numpy(np.stack([xs[b][L] for b, L in enumerate(lens)]).astype(np.float32)).to(dev)
    d_out = torch.empty((len(lens), H), dtype=torch.float32, device=dev)
    d_row = torch.tensor([int(row0[b]) + L for b, L in enumerate(lens)], dtype=torch.int64, device=dev)
    d_pos = torch.tensor(lens, dtype=torch.int32, device=dev)
    ws = torch.empty(lib.kvl_mla_decode_step_workspace_bytes(C.byref(cfg), len(lens)), dtype=torch.uint8, device=dev)
    rc = lib.kvl_mla_decode_step_bf16(C.byref(cfg), C.byref(dw), plan.h, d_out.data_ptr(), d_x.data_ptr(),
                                      d_kv.data_ptr(), total + 128, d_row.data_ptr(), d_pos.data_ptr(), len(lens),
                                      ws.data_ptr(), C.c_void_p(0))
    assert rc == 0, K.last_error()
    torch.cuda.synchronize()
    assert plan.check() == 0, K.last_error()
    got = d_out.cpu().numpy()
    for b in range(len(lens)):
        assert_close(got[b], want[b], what=f"decode step seq {b} (L={lens[b]})")
    # the appended rows match the drop-in's appended rows (stored as bf16);
    # the cached rows are untouched
    kv_after = d_kv.cpu().numpy().view(np.uint16)
    for b, L in enumerate(lens):
        row = (kv_after[row0[b] + L].astype(np.uint32) << 16).view(np.float32)
        assert_close(row, appended[b], what=f"appended row seq {b}")
        np.testing.assert_array_equal(kv_after[row0[b]:row0[b] + L], pools[b])


def test_decode_step_matvec_batch(K, S, torch_cuda):
    _run(K, S, torch_cuda, [100, 257, 1000], 91)


def test_decode_step_gemm_batch(K, S, torch_cuda):
    """20 ragged sequences (one with a single cached row): the tensor-core path."""
    lens = [1, 300] + [int(v) for v in S.uniform_ints(93, S.S_LEN, 18, 2, 260)]
    _run(K, S, torch_cuda, lens, 93)
