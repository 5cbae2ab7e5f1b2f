"""Context-parallel prefill (kvl_mla_prefill_cp_begin / kvl_mla_prefill_cp_end)
on one GPU: every rank of a world of 2, 4 or 8 runs in turn with its own
workspace and only its own rows (chunk r, then chunk 2 world - 1 - r), the
ranks' compressed rows are concatenated in rank order (what the all-gather
between the two calls produces), and the output rows each rank returns,
scattered back to their prompt positions, form the prompt's output.  Checked against the reference's own
streaming prefill (src/mla_prefill_streaming.c:78-206, oracle/_ref) within
rel-L2 <= 1e-2 and max-abs <= 2e-2, and against the single-GPU device prefill
(kvl_mla_prefill_dev), which uses the same kernels over other row ranges.  A
rank with fewer (head, query tile) items than SMs has its long items cut into
key-range pieces whose softmax partials are combined afterwards (every shape
below cuts on some rank; 2048 x 2 leaves rank 1 uncut), which re-associates
the softmax sums: against the one-GPU prefill the bound is rel-L2 <= 5e-3.
Bad splits are rejected."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

SHAPE = (2048, 16, 128, 64, 128, 512, 1e-5, 50000.0)


def _cp_prefill(K, torch, cfg, dw, xb, Sq, world):
    from kvl_b200.parallel import zigzag_chunks
    lib = K.load()
    dev = xb.device
    nbytes = lib.kvl_mla_prefill_workspace_bytes(C.byref(cfg), Sq)
    c = Sq // (2 * world)
    chunks = zigzag_chunks(Sq, world)
    xs = [torch.cat([xb[a0:a1], xb[b0:b1]]).contiguous() for (a0, a1), (b0, b1) in chunks]
    outs = [torch.full((2 * c, cfg.hidden_size), float("nan"), dtype=torch.float32, device=dev) for _ in range(world)]
    wss = [torch.empty(nbytes, dtype=torch.uint8, device=dev) for _ in range(world)]
    sends = [torch.empty((2 * c, 576), dtype=torch.int16, device=dev) for _ in range(world)]
    for r in range(world):
        rc = lib.kvl_mla_prefill_cp_begin(C.byref(cfg), C.byref(dw), xs[r].data_ptr(), Sq, r, world,
                                          sends[r].data_ptr(), wss[r].data_ptr(), nbytes, None)
        assert rc == 0, K.last_error()
    recv = torch.cat(sends)
    for r in range(world):
        rc = lib.kvl_mla_prefill_cp_end(C.byref(cfg), C.byref(dw), outs[r].data_ptr(), Sq, r, world,
                                        recv.data_ptr(), wss[r].data_ptr(), nbytes, None)
        assert rc == 0, K.last_error()
    torch.cuda.synchronize()
    out = np.full((Sq, cfg.hidden_size), np.nan, dtype=np.float32)
    for ((a0, a1), (b0, b1)), o in zip(chunks, outs):
        o = o.cpu().numpy()
        out[a0:a1] = o[:c]
        out[b0:b1] = o[c:]
    return out


@pytest.mark.parametrize("Sq,world", [(1024, 2), (1024, 4), (2048, 2), (4096, 8)])
def test_context_parallel_prefill(K, S, ref, torch_cuda, Sq, world):
    from oracle.oracle import cfg_of
    torch = torch_cuda
    lib = K.load()
    cfg = K.make_config(*SHAPE)
    w = K.random_weights(cfg, 71 + world, 0.02, norm_std=0.05)
    xbits = S.normal_bf16(71 + world, S.S_X, (Sq, SHAPE[0]), 1.0)
    dev = torch.device("cuda", 0)
    ts = [torch.from_numpy(a.view(np.int16)).to(dev) for a in w.arrays]
    dw = K.KvlMlaDeviceWeights(*[t.data_ptr() for t in ts])
    xb = torch.from_numpy(xbits.view(np.int16)).to(dev)
    got = _cp_prefill(K, torch, cfg, dw, xb, Sq, world)
    assert np.isfinite(got).all()
    # the single-GPU device prefill on the same inputs
    nbytes = lib.kvl_mla_prefill_workspace_bytes(C.byref(cfg), Sq)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    one = torch.empty((Sq, SHAPE[0]), dtype=torch.float32, device=dev)
    assert lib.kvl_mla_prefill_dev(C.byref(cfg), C.byref(dw), one.data_ptr(), xb.data_ptr(), Sq, ws.data_ptr(),
                                   nbytes, None) == 0, K.last_error()
    torch.cuda.synchronize()
    assert_close(got, one.cpu().numpy(), rel=5e-3, mabs=2e-2, what=f"cp x{world} vs one-GPU prefill")
    if Sq <= 1024:
        want = ref.prefill(S.bf16_bits_to_f32(xbits), cfg_of(*SHAPE), w.arrays)
        assert_close(got, want, what=f"cp x{world} vs reference prefill S={Sq}")


def test_context_parallel_prefill_rejects_bad_splits(K, torch_cuda):
    torch = torch_cuda
    lib = K.load()
    cfg = K.make_config(*SHAPE)
    dev = torch.device("cuda", 0)
    nbytes = lib.kvl_mla_prefill_workspace_bytes(C.byref(cfg), 1000)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    buf = torch.empty(4096 * 2048, dtype=torch.int16, device=dev)
    dw = K.KvlMlaDeviceWeights(*([buf.data_ptr()] * 5))
    # 1000 rows do not split into 4 chunks of a multiple of 128; rank out of range
    for Sq, r, world in [(1000, 0, 2), (1024, 2, 2), (1024, 0, 0)]:
        rc = lib.kvl_mla_prefill_cp_begin(C.byref(cfg), C.byref(dw), buf.data_ptr(), Sq, r, world, buf.data_ptr(),
                                          ws.data_ptr(), nbytes, None)
        assert rc == -1
