"""The tensor-core prefill path (tcgen05 GEMMs + causal flash kernel) against the
reference's own streaming prefill (src/mla_prefill_streaming.c:78-206, compiled
from its sources into oracle/_ref) on seeded inputs.

Covers the edges of the tiled path: a single token, lengths one short of / one
past a 128-token tile, a length that is not a multiple of the tile, the host
entry's chunked copy/compute pipeline (2 and 4 chunks, a ragged last chunk),
a hidden size whose K tail and output-column tail are not multiples of the
64-wide K step or the 256-wide N tile, and the device entry point
(`kvl_mla_prefill_dev`) against the host one.  Tolerance: rel-L2 <= 1e-2,
max-abs <= 2e-2.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

# (H, NH, DN, DR, DV, R, eps, theta): the Kimi attention shape with varying hidden size
KIMI = (2048, 16, 128, 64, 128, 512, 1e-5, 50000.0)


def _shape(H=2048, theta=50000.0):
    return (H,) + KIMI[1:6] + (KIMI[6], theta)


def _setup(K, S, shape, Sq, seed):
    H = shape[0]
    cfg = K.make_config(*shape)
    w = K.random_weights(cfg, seed, 0.02, norm_std=0.05)
    x = S.normal(seed, S.S_X, Sq * H, 1.0).reshape(Sq, H)
    return cfg, w, x


def _upload(torch, K, w, dev):
    """Device copies of the host bf16 weight bits + the KvlMlaDeviceWeights struct."""
    ts = [torch.from_numpy(a.view(np.int16)).to(dev) for a in w.arrays]
    return ts, K.KvlMlaDeviceWeights(*[t.data_ptr() for t in ts])


def _ref_prefill(ref, shape, x, w):
    from oracle.oracle import cfg_of
    return ref.prefill(x, cfg_of(*shape), w.arrays)


@pytest.mark.parametrize("Sq", [1, 2, 127, 128, 129, 1000, 1100, 2048, 4100])
def test_fast_prefill_lengths(K, S, ref, torch_cuda, Sq):
    shape = _shape()
    cfg, w, x = _setup(K, S, shape, Sq, 101 + Sq)
    out = np.zeros_like(x)
    rc = K.load().kvl_mla_prefill_bf16(K.ptr(out, K.f32p), K.ptr(x, K.f32p), Sq, C.byref(cfg), C.byref(w.c))
    assert rc == 0, K.last_error()
    assert np.isfinite(out).all()
    assert_close(out, _ref_prefill(ref, shape, x, w), what=f"fast prefill S={Sq}")


@pytest.mark.parametrize("H", [1024, 2056])
def test_fast_prefill_hidden_tails(K, S, ref, torch_cuda, H):
    shape = _shape(H=H, theta=800000.0)
    Sq = 300
    cfg, w, x = _setup(K, S, shape, Sq, 7 + H)
    out = np.zeros_like(x)
    rc = K.load().kvl_mla_prefill_bf16(K.ptr(out, K.f32p), K.ptr(x, K.f32p), Sq, C.byref(cfg), C.byref(w.c))
    assert rc == 0, K.last_error()
    assert_close(out, _ref_prefill(ref, shape, x, w), what=f"fast prefill H={H}")


@pytest.mark.parametrize("Sq", [513, 1100, 2048, 4100])
def test_device_entry_matches_host_entry(K, S, torch_cuda, Sq):
    """kvl_mla_prefill_dev (device bf16 x, device weights, caller workspace, one
    pass over the prompt) gives the host entry's result on the same inputs, bit
    for bit, also where the host entry pipelines its copies over 2 or 4 row
    chunks (1100, 2048, 4100 tokens): the same kernels, per row, per query tile."""
    torch = torch_cuda
    shape = _shape()
    cfg, w, x = _setup(K, S, shape, Sq, 55)
    lib = K.load()
    host = np.zeros_like(x)
    assert lib.kvl_mla_prefill_bf16(K.ptr(host, K.f32p), K.ptr(x, K.f32p), Sq, C.byref(cfg), C.byref(w.c)) == 0, \
        K.last_error()
    dev = torch.device("cuda", 0)
    keep, dw = _upload(torch, K, w, dev)
    xb = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    out = torch.empty((Sq, shape[0]), dtype=torch.float32, device=dev)
    ws_bytes = lib.kvl_mla_prefill_workspace_bytes(C.byref(cfg), Sq)
    assert ws_bytes > 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    rc = lib.kvl_mla_prefill_dev(C.byref(cfg), C.byref(dw), C.c_void_p(out.data_ptr()), C.c_void_p(xb.data_ptr()),
                                 Sq, C.c_void_p(ws.data_ptr()), C.c_size_t(ws_bytes), C.c_void_p(stream))
    assert rc == 0, K.last_error()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), host)


def test_device_entry_rejects_small_workspace(K, S, torch_cuda):
    torch = torch_cuda
    shape = _shape()
    Sq = 64
    cfg, w, x = _setup(K, S, shape, Sq, 56)
    lib = K.load()
    dev = torch.device("cuda", 0)
    keep, dw = _upload(torch, K, w, dev)
    xb = torch.from_numpy(x).to(dev).to(torch.bfloat16)
    out = torch.empty((Sq, shape[0]), dtype=torch.float32, device=dev)
    ws_bytes = lib.kvl_mla_prefill_workspace_bytes(C.byref(cfg), Sq)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    rc = lib.kvl_mla_prefill_dev(C.byref(cfg), C.byref(dw), C.c_void_p(out.data_ptr()), C.c_void_p(xb.data_ptr()),
                                 Sq, C.c_void_p(ws.data_ptr()), C.c_size_t(ws_bytes - 1), C.c_void_p(0))
    assert rc == -1
    assert "workspace" in K.last_error()
