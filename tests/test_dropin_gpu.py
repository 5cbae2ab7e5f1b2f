"""The drop-in C ABI (reference function names and structs) against the
reference runtime's own C implementation compiled from its sources
(oracle/_ref), on identical seeded inputs.

Mirrors the reference's MLA gates:
  src/mla_incremental_probe.c:32-110  decode / state-prefill / prefill agreement,
                                      bad-order rejection, reset
  src/spec_q8_lab_probe.c:43-183      block decode == serial decode (exactly),
                                      truncate rollback == fresh prefill (exactly),
                                      Q8 state decode vs fp32 decode <= 0.02
with this build's tolerance for reference parity (rel-L2 <= 1e-2,
max-abs <= 2e-2).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.parity import assert_close

pytestmark = pytest.mark.gpu

SHAPES = {
    # name: (H, NH, DN, DR, DV, R, eps, theta)
    "incremental_probe": (16, 2, 4, 4, 4, 6, 1e-6, 10000.0),
    "spec_q8_probe": (64, 4, 8, 8, 8, 32, 1e-6, 10000.0),
    "kimi": (2048, 16, 128, 64, 128, 512, 1e-5, 800000.0),
    "kimi_theta50k": (2048, 16, 128, 64, 128, 512, 1e-5, 50000.0),
}


def _weights(K, S, shape, seed, std):
    H, NH, DN, DR, DV, R, eps, theta = shape
    cfg = K.make_config(H, NH, DN, DR, DV, R, eps, theta)
    w = K.random_weights(cfg, seed, std, norm_std=0.05)
    return cfg, w


def _ref_cfg(shape):
    from oracle.oracle import cfg_of
    return cfg_of(*shape)


def _decode_all(K, cfg, w, x, prefix=0, q8=False):
    """Shim: state prefill of `prefix` rows, then serial decode of the rest."""
    lib = K.load()
    Sq = x.shape[0]
    st = K.KvlMlaCompressedQ8State() if q8 else K.KvlMlaCompressedState()
    base = "kvl_mla_compressed_q8_state" if q8 else "kvl_mla_compressed_state"
    assert getattr(lib, base + "_init")(C.byref(st), C.byref(cfg), Sq + 1) == 0, K.last_error()
    x = np.ascontiguousarray(x, np.float32)
    if prefix:
        rc = getattr(lib, base + "_prefill_bf16")(K.ptr(x, K.f32p), prefix, C.byref(cfg), C.byref(w.c),
                                                  C.byref(st))
        assert rc == 0, K.last_error()
    dec = lib.kvl_mla_decode_compressed_q8_bf16 if q8 else lib.kvl_mla_decode_compressed_bf16
    outs = np.zeros((Sq - prefix, cfg.hidden_size), np.float32)
    for t in range(prefix, Sq):
        rc = dec(K.ptr(outs[t - prefix], K.f32p), K.ptr(x[t], K.f32p), t, C.byref(cfg), C.byref(w.c),
                 C.byref(st))
        assert rc == 0, K.last_error()
    return outs, st, lib, base


@pytest.mark.parametrize("name", ["incremental_probe", "spec_q8_probe", "kimi", "kimi_theta50k"])
def test_decode_matches_reference(K, S, ref, torch_cuda, name):
    shape = SHAPES[name]
    Sq = 40 if shape[0] >= 2048 else 13
    prefix = 5
    cfg, w = _weights(K, S, shape, 21, 0.05 if shape[0] < 2048 else 0.02)
    x = S.normal(21, S.S_X, Sq * shape[0], 1.0).reshape(Sq, shape[0])
    got, st, lib, base = _decode_all(K, cfg, w, x, prefix)
    want, (rlat, rrope) = ref.decode_sequence(x, _ref_cfg(shape), w.arrays, prefix=prefix)
    assert_close(got, want, what=f"decode {name}")
    # The state rows (state prefill of the prefix, then one append per decoded
    # token) are the reference's bit for bit: the projection sums in the AVX2
    # build's order, RMSNorm and RoPE as the reference rounds them.
    R, DR = shape[5], shape[3]
    lat = np.ctypeslib.as_array(st.latent, shape=(Sq * R,)).reshape(Sq, R)
    rope = np.ctypeslib.as_array(st.rope, shape=(Sq * DR,)).reshape(Sq, DR)
    np.testing.assert_array_equal(lat.view(np.uint32), rlat.view(np.uint32))
    np.testing.assert_array_equal(rope.view(np.uint32), rrope.view(np.uint32))
    getattr(lib, base + "_free")(C.byref(st))


@pytest.mark.parametrize("name", ["incremental_probe", "spec_q8_probe", "kimi"])
def test_q8_decode_matches_reference(K, S, ref, torch_cuda, name):
    shape = SHAPES[name]
    Sq = 40 if shape[0] >= 2048 else 13
    cfg, w = _weights(K, S, shape, 22, 0.05 if shape[0] < 2048 else 0.02)
    x = S.normal(22, S.S_X, Sq * shape[0], 1.0).reshape(Sq, shape[0])
    got, st, lib, base = _decode_all(K, cfg, w, x, 5, q8=True)
    want, (rl8, rls, rrp) = ref.decode_sequence(x, _ref_cfg(shape), w.arrays, prefix=5, q8=True)
    assert_close(got, want, what=f"q8 decode {name}")
    # The mirrored state holds the reference's byte layout, and its rows are
    # the reference's bit for bit (int8 latent, fp32 row scale, bf16 rope).
    R, DR = shape[5], shape[3]
    l8 = np.ctypeslib.as_array(st.latent_q8, shape=(Sq * R,)).reshape(Sq, R)
    ls = np.ctypeslib.as_array(st.latent_scale, shape=(Sq,))
    rp = np.ctypeslib.as_array(st.rope_bf16, shape=(Sq * DR,)).reshape(Sq, DR)
    np.testing.assert_array_equal(l8, rl8)
    np.testing.assert_array_equal(ls.view(np.uint32), np.asarray(rls, np.float32).view(np.uint32))
    np.testing.assert_array_equal(rp, rrp)
    getattr(lib, base + "_free")(C.byref(st))


@pytest.mark.parametrize("name,Sq", [("incremental_probe", 5), ("incremental_probe", 257), ("spec_q8_probe", 64),
                                     ("kimi", 128), ("kimi_theta50k", 300)])
def test_prefill_matches_reference(K, S, ref, torch_cuda, name, Sq):
    shape = SHAPES[name]
    cfg, w = _weights(K, S, shape, 23, 0.05 if shape[0] < 2048 else 0.02)
    x = S.normal(23, S.S_X, Sq * shape[0], 1.0).reshape(Sq, shape[0])
    out = np.zeros_like(x)
    rc = K.load().kvl_mla_prefill_bf16(K.ptr(out, K.f32p), K.ptr(x, K.f32p), Sq, C.byref(cfg), C.byref(w.c))
    assert rc == 0, K.last_error()
    want = ref.prefill(x, _ref_cfg(shape), w.arrays)
    assert_close(out, want, what=f"prefill {name} S={Sq}")


def test_decode_equals_prefill_and_state_prefill(K, S, torch_cuda):
    """src/mla_incremental_probe.c:75-96: decode of every token, and state
    prefill of a prefix + decode of the next token, agree with causal prefill."""
    shape = SHAPES["spec_q8_probe"]
    cfg, w = _weights(K, S, shape, 24, 0.05)
    Sq = 9
    x = S.normal(24, S.S_X, Sq * shape[0], 1.0).reshape(Sq, shape[0])
    pre = np.zeros_like(x)
    assert K.load().kvl_mla_prefill_bf16(K.ptr(pre, K.f32p), K.ptr(x, K.f32p), Sq, C.byref(cfg),
                                         C.byref(w.c)) == 0
    dec, st, lib, base = _decode_all(K, cfg, w, x, 0)
    assert_close(dec, pre, what="decode vs prefill")
    getattr(lib, base + "_free")(C.byref(st))
    dec2, st, lib, base = _decode_all(K, cfg, w, x, 4)
    assert_close(dec2, pre[4:], what="state prefill + decode vs prefill")
    getattr(lib, base + "_free")(C.byref(st))


def test_block_and_rollback_exact(K, S, torch_cuda):
    """src/spec_q8_lab_probe.c:86-119, 173-176: block decode equals serial decode
    and a truncate rollback equals a fresh prefill, exactly (0.0)."""
    shape = SHAPES["spec_q8_probe"]
    cfg, w = _weights(K, S, shape, 25, 0.036)
    H = shape[0]
    Sq, PREFIX, BLOCK, ACCEPT = 13, 5, 4, 2
    x = S.normal(25, S.S_X, Sq * H, 0.2).reshape(Sq, H)
    repl = S.normal(25, 99, H, 0.2)
    lib = K.load()
    seq, st_seq, _, _ = _decode_all(K, cfg, w, x, 0)

    bs = K.KvlMlaCompressedState()
    assert lib.kvl_mla_compressed_state_init(C.byref(bs), C.byref(cfg), Sq + 1) == 0
    assert lib.kvl_mla_compressed_state_prefill_bf16(K.ptr(x, K.f32p), PREFIX, C.byref(cfg), C.byref(w.c),
                                                     C.byref(bs)) == 0
    block = np.zeros((BLOCK, H), np.float32)
    xb = np.ascontiguousarray(x[PREFIX:PREFIX + BLOCK])
    assert lib.kvl_mla_decode_compressed_block_bf16(K.ptr(block, K.f32p), K.ptr(xb, K.f32p), BLOCK, PREFIX,
                                                    C.byref(cfg), C.byref(w.c), C.byref(bs)) == 0
    assert np.max(np.abs(block - seq[PREFIX:PREFIX + BLOCK])) == 0.0

    assert lib.kvl_mla_compressed_state_truncate(C.byref(bs), PREFIX + ACCEPT) == 0
    rb = np.zeros(H, np.float32)
    assert lib.kvl_mla_decode_compressed_bf16(K.ptr(rb, K.f32p), K.ptr(repl, K.f32p), PREFIX + ACCEPT,
                                              C.byref(cfg), C.byref(w.c), C.byref(bs)) == 0
    fs = K.KvlMlaCompressedState()
    assert lib.kvl_mla_compressed_state_init(C.byref(fs), C.byref(cfg), Sq + 1) == 0
    assert lib.kvl_mla_compressed_state_prefill_bf16(K.ptr(x, K.f32p), PREFIX + ACCEPT, C.byref(cfg),
                                                     C.byref(w.c), C.byref(fs)) == 0
    rb_ref = np.zeros(H, np.float32)
    assert lib.kvl_mla_decode_compressed_bf16(K.ptr(rb_ref, K.f32p), K.ptr(repl, K.f32p), PREFIX + ACCEPT,
                                              C.byref(cfg), C.byref(w.c), C.byref(fs)) == 0
    assert np.max(np.abs(rb - rb_ref)) == 0.0

    # Q8: the same rollback, exactly; and Q8 vs fp32 decode within the lab gate.
    qs = K.KvlMlaCompressedQ8State()
    assert lib.kvl_mla_compressed_q8_state_init(C.byref(qs), C.byref(cfg), Sq + 1) == 0
    assert lib.kvl_mla_compressed_q8_state_prefill_bf16(K.ptr(x, K.f32p), PREFIX, C.byref(cfg), C.byref(w.c),
                                                        C.byref(qs)) == 0
    q8 = np.zeros((Sq - PREFIX, H), np.float32)
    for t in range(PREFIX, Sq):
        assert lib.kvl_mla_decode_compressed_q8_bf16(K.ptr(q8[t - PREFIX], K.f32p), K.ptr(x[t], K.f32p), t,
                                                     C.byref(cfg), C.byref(w.c), C.byref(qs)) == 0
    d = q8 - seq[PREFIX:]
    assert np.max(np.abs(d)) <= 0.02
    assert np.sqrt(np.sum(d * d) / np.sum(seq[PREFIX:] ** 2)) <= 0.02
    assert lib.kvl_mla_compressed_q8_state_truncate(C.byref(qs), PREFIX + ACCEPT) == 0
    qrb = np.zeros(H, np.float32)
    assert lib.kvl_mla_decode_compressed_q8_bf16(K.ptr(qrb, K.f32p), K.ptr(repl, K.f32p), PREFIX + ACCEPT,
                                                 C.byref(cfg), C.byref(w.c), C.byref(qs)) == 0
    qf = K.KvlMlaCompressedQ8State()
    assert lib.kvl_mla_compressed_q8_state_init(C.byref(qf), C.byref(cfg), Sq + 1) == 0
    assert lib.kvl_mla_compressed_q8_state_prefill_bf16(K.ptr(x, K.f32p), PREFIX + ACCEPT, C.byref(cfg),
                                                        C.byref(w.c), C.byref(qf)) == 0
    qrb_ref = np.zeros(H, np.float32)
    assert lib.kvl_mla_decode_compressed_q8_bf16(K.ptr(qrb_ref, K.f32p), K.ptr(repl, K.f32p), PREFIX + ACCEPT,
                                                 C.byref(cfg), C.byref(w.c), C.byref(qf)) == 0
    assert np.max(np.abs(qrb - qrb_ref)) == 0.0
    for st in (st_seq, bs, fs):
        lib.kvl_mla_compressed_state_free(C.byref(st))
    for st in (qs, qf):
        lib.kvl_mla_compressed_q8_state_free(C.byref(st))


def test_error_conventions(K, S, torch_cuda):
    """Bad order, capacity overflow, truncate beyond len, reset, double free."""
    shape = SHAPES["incremental_probe"]
    cfg, w = _weights(K, S, shape, 26, 0.05)
    lib = K.load()
    st = K.KvlMlaCompressedState()
    assert lib.kvl_mla_compressed_state_init(C.byref(st), C.byref(cfg), 2) == 0
    x = S.normal(26, 0, 16, 1.0)
    out = np.zeros(16, np.float32)
    call = lambda pos: lib.kvl_mla_decode_compressed_bf16(K.ptr(out, K.f32p), K.ptr(x, K.f32p), pos,
                                                          C.byref(cfg), C.byref(w.c), C.byref(st))
    assert call(1) == -1 and st.len == 0          # position != len
    assert call(0) == 0 and st.len == 1
    assert call(0) == -1 and st.len == 1          # bad order
    assert call(1) == 0 and st.len == 2
    assert call(2) == -1 and st.len == 2          # capacity overflow
    assert lib.kvl_mla_compressed_state_truncate(C.byref(st), 3) == -1
    assert lib.kvl_mla_compressed_state_truncate(C.byref(st), 1) == 0 and st.len == 1
    lib.kvl_mla_compressed_state_reset(C.byref(st))
    assert st.len == 0 and call(0) == 0
    lib.kvl_mla_compressed_state_free(C.byref(st))
    lib.kvl_mla_compressed_state_free(C.byref(st))  # double free is safe
    assert st.capacity == 0 and not st.latent


@pytest.mark.parametrize("prefix,block", [(1020, 8), (509, 8), (3, 16), (20000, 4)])
def test_block_decode_exact_kimi(K, S, torch_cuda, prefix, block):
    """The one-pass block decode equals `block` serial decodes bit for bit (outputs
    and the appended state rows) at the Kimi shape, where the attends are cut
    into several KV splits: 1021..1028 rows cross a 128-row tile boundary (8 and
    9 splits), 510..517 rows cross from 4 to 5 splits (the one-warp merge beside
    the block-wide one), 20001..20004 rows use every SM (148 splits), 4..19 rows
    one."""
    shape = (2048, 16, 128, 64, 128, 512, 1e-5, 800000.0)
    cfg, w = _weights(K, S, shape, 71, 0.02)
    H = shape[0]
    x = S.normal(71, S.S_X, (prefix + block) * H, 1.0).reshape(prefix + block, H)
    lib = K.load()
    outs, rows = [], []
    for use_block in (False, True):
        st = K.CompressedState(cfg, prefix + block)
        assert st.prefill(x[:prefix], w) == 0, K.last_error()
        out = np.zeros((block, H), np.float32)
        if use_block:
            xb = np.ascontiguousarray(x[prefix:])
            assert lib.kvl_mla_decode_compressed_block_bf16(K.ptr(out, K.f32p), K.ptr(xb, K.f32p), block, prefix,
                                                            C.byref(cfg), C.byref(w.c), C.byref(st.s)) == 0, \
                K.last_error()
        else:
            for t in range(block):
                rc, out[t] = st.decode(x[prefix + t], prefix + t, w)
                assert rc == 0, K.last_error()
        outs.append(out)
        rows.append((st.latent()[prefix:].copy(), st.rope()[prefix:].copy()))
        assert st.s.len == prefix + block
        st.free()
    np.testing.assert_array_equal(outs[1], outs[0])
    np.testing.assert_array_equal(rows[1][0], rows[0][0])
    np.testing.assert_array_equal(rows[1][1], rows[0][1])


@pytest.mark.parametrize("name", ["incremental_probe", "kimi"])
def test_layered_oracles(K, S, ref, torch_cuda, name):
    """The reference's lower oracle layers, run against the GPU path: its
    expanded-K/V state decode (src/mla_state.c:66-149; the mla_incremental_probe
    gate) against our compressed-state serial decode, and its materialised
    prefill (src/ops.c:105-192) against our prefill."""
    shape = SHAPES[name]
    Sq = 24 if shape[0] >= 2048 else 13
    cfg, w = _weights(K, S, shape, 31, 0.05 if shape[0] < 2048 else 0.02)
    x = S.normal(31, S.S_X, Sq * shape[0], 1.0).reshape(Sq, shape[0])
    got, st, lib, base = _decode_all(K, cfg, w, x, 0)
    getattr(lib, base + "_free")(C.byref(st))
    want = ref.decode_expanded(x, _ref_cfg(shape), w.arrays)
    assert_close(got, want, what=f"compressed decode vs expanded-state decode ({name})")
    out = np.zeros_like(x)
    assert lib.kvl_mla_prefill_bf16(K.ptr(out, K.f32p), K.ptr(x, K.f32p), Sq, C.byref(cfg), C.byref(w.c)) == 0, \
        K.last_error()
    mat = ref.prefill(x, _ref_cfg(shape), w.arrays, materialized=True)
    assert_close(out, mat, what=f"prefill vs materialised prefill ({name})")
