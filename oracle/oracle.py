"""ctypes wrappers of the CPU checkers (TEST INFRASTRUCTURE ONLY).

  Oracle     oracle/liboracle.so -- the restatement in kvl_oracle.c
  Reference  oracle/_ref/libkvl_ref.so (AVX2 build) or libkvl_ref_scalar.so --
             the reference runtime's own MLA sources compiled by oracle/Makefile

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker or the timed CPU baseline; the product library never
calls it.
"""
from __future__ import annotations

import ctypes as C
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libkvl_ref.so"
REF_SCALAR_SO = HERE / "_ref" / "libkvl_ref_scalar.so"

f32p = C.POINTER(C.c_float)
u16p = C.POINTER(C.c_uint16)
i8p = C.POINTER(C.c_int8)


class Cfg(C.Structure):
    """include/kvl/ops.h:17-26 (KvlMlaConfig)."""
    _fields_ = [("hidden_size", C.c_int), ("num_heads", C.c_int), ("qk_nope_dim", C.c_int),
                ("qk_rope_dim", C.c_int), ("v_head_dim", C.c_int), ("kv_lora_rank", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float)]


class W(C.Structure):
    """include/kvl/ops.h:28-34 (KvlMlaBF16)."""
    _fields_ = [("q_proj", u16p), ("kv_a_proj", u16p), ("kv_a_norm", u16p), ("kv_b_proj", u16p),
                ("o_proj", u16p)]


class State(C.Structure):
    """include/kvl/mla_compressed_state.h:7-14."""
    _fields_ = [("capacity", C.c_int), ("len", C.c_int), ("kv_lora_rank", C.c_int),
                ("qk_rope_dim", C.c_int), ("latent", f32p), ("rope", f32p)]


class Q8State(C.Structure):
    """include/kvl/mla_compressed_q8_state.h:8-16."""
    _fields_ = [("capacity", C.c_int), ("len", C.c_int), ("kv_lora_rank", C.c_int),
                ("qk_rope_dim", C.c_int), ("latent_q8", i8p), ("latent_scale", f32p),
                ("rope_bf16", u16p)]


def _p(a, t):
    return a.ctypes.data_as(t)


def cfg_of(H, NH, DN, DR, DV, R, eps, theta) -> Cfg:
    return Cfg(H, NH, DN, DR, DV, R, eps, theta)


def w_of(arrays) -> W:
    return W(*[_p(a, u16p) for a in arrays])


class Oracle:
    """The restatement (kvl_oracle.c)."""

    def __init__(self, path=ORACLE_SO):
        if not pathlib.Path(path).exists():
            raise RuntimeError(f"{path} missing: run `make -f oracle/Makefile oracle`")
        self.lib = C.CDLL(str(path))
        L = self.lib
        L.orc_f32_to_bf16_rne.restype = C.c_uint16
        L.orc_f32_to_bf16_rne.argtypes = [C.c_float]
        L.orc_bf16_to_f32.restype = C.c_float
        L.orc_bf16_to_f32.argtypes = [C.c_uint16]
        L.orc_f32_to_bf16_rne_n.argtypes = [u16p, f32p, C.c_size_t]
        L.orc_rope.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_float]
        L.orc_rope_table.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_float]
        L.orc_rmsnorm.argtypes = [f32p, f32p, u16p, C.c_int, C.c_float]
        L.orc_matvec.argtypes = [f32p, f32p, u16p, C.c_int, C.c_int]
        L.orc_quantize_row.argtypes = [i8p, f32p, f32p, C.c_int]
        L.orc_dequant.restype = C.c_float
        L.orc_dequant.argtypes = [C.c_int8, C.c_float]
        L.orc_dequant_n.argtypes = [f32p, i8p, f32p, C.c_int, C.c_int]
        L.orc_attend_f32.restype = C.c_int
        L.orc_attend_f32.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_float]
        L.orc_attend_q8.restype = C.c_int
        L.orc_attend_q8.argtypes = [f32p, f32p, f32p, f32p, i8p, f32p, u16p, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_float]
        L.orc_decode_f32.restype = C.c_int
        L.orc_decode_f32.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), u16p, u16p, u16p, u16p, u16p, f32p, f32p]
        L.orc_decode_q8.restype = C.c_int
        L.orc_decode_q8.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), u16p, u16p, u16p, u16p, u16p, i8p, f32p,
                                    u16p]
        L.orc_prefill.restype = C.c_int
        L.orc_prefill.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), u16p, u16p, u16p, u16p, u16p]
        L.orc_append_f32.argtypes = [f32p, f32p, f32p, C.c_int, C.POINTER(Cfg), u16p, u16p]
        L.orc_append_q8.argtypes = [i8p, f32p, u16p, f32p, C.c_int, C.POINTER(Cfg), u16p, u16p]

    # -- attend core (src/mla_compressed_state.c:132-148)
    def attend_f32(self, q, latent, rope, scale):
        """q [NH][R+DR] fp32, latent [L][R], rope [L][DR] -> (mix [NH][R], lse [NH])."""
        q = np.ascontiguousarray(q, np.float32)
        NH, RD = q.shape
        L, R = latent.shape
        DR = RD - R
        ql = np.ascontiguousarray(q[:, :R])
        qr = np.ascontiguousarray(q[:, R:])
        lat = np.ascontiguousarray(latent, np.float32)
        rp = np.ascontiguousarray(rope, np.float32)
        mix = np.zeros((NH, R), np.float32)
        lse = np.zeros(NH, np.float32)
        rc = self.lib.orc_attend_f32(_p(mix, f32p), _p(lse, f32p), _p(ql, f32p), _p(qr, f32p), _p(lat, f32p),
                                     _p(rp, f32p), L, NH, R, DR, scale)
        assert rc == 0
        return mix, lse

    def attend_q8(self, q, lat8, lscale, rope16, scale):
        q = np.ascontiguousarray(q, np.float32)
        NH, RD = q.shape
        L, R = lat8.shape
        DR = RD - R
        ql = np.ascontiguousarray(q[:, :R])
        qr = np.ascontiguousarray(q[:, R:])
        l8 = np.ascontiguousarray(lat8, np.int8)
        ls = np.ascontiguousarray(lscale, np.float32)
        r16 = np.ascontiguousarray(rope16, np.uint16)
        mix = np.zeros((NH, R), np.float32)
        lse = np.zeros(NH, np.float32)
        rc = self.lib.orc_attend_q8(_p(mix, f32p), _p(lse, f32p), _p(ql, f32p), _p(qr, f32p), _p(l8, i8p),
                                    _p(ls, f32p), _p(r16, u16p), L, NH, R, DR, scale)
        assert rc == 0
        return mix, lse

    # -- Q8 row helpers (src/mla_compressed_q8_state.c:9-16, 34-61)
    def quantize_rows(self, x):
        x = np.ascontiguousarray(x, np.float32)
        rows, R = x.shape
        q = np.zeros((rows, R), np.int8)
        s = np.zeros(rows, np.float32)
        for t in range(rows):
            self.lib.orc_quantize_row(_p(q[t], i8p), _p(s[t:t + 1], f32p), _p(x[t], f32p), R)
        return q, s

    def dequant(self, q, scale):
        q = np.ascontiguousarray(q, np.int8)
        rows, R = q.shape
        s = np.ascontiguousarray(scale, np.float32)
        out = np.zeros((rows, R), np.float32)
        self.lib.orc_dequant_n(_p(out, f32p), _p(q, i8p), _p(s, f32p), rows, R)
        return out

    def bf16_rne(self, x):
        x = np.ascontiguousarray(x, np.float32).ravel()
        out = np.zeros(x.shape, np.uint16)
        self.lib.orc_f32_to_bf16_rne_n(_p(out, u16p), _p(x, f32p), x.size)
        return out

    # -- whole steps
    def decode_f32(self, x, position, cfg: Cfg, warrays, latent, rope):
        out = np.zeros(cfg.hidden_size, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        rc = self.lib.orc_decode_f32(_p(out, f32p), _p(x, f32p), position, C.byref(cfg),
                                     *[_p(a, u16p) for a in warrays], _p(latent, f32p), _p(rope, f32p))
        assert rc == 0
        return out

    def decode_q8(self, x, position, cfg: Cfg, warrays, lat8, lscale, rope16):
        out = np.zeros(cfg.hidden_size, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        rc = self.lib.orc_decode_q8(_p(out, f32p), _p(x, f32p), position, C.byref(cfg),
                                    *[_p(a, u16p) for a in warrays], _p(lat8, i8p), _p(lscale, f32p),
                                    _p(rope16, u16p))
        assert rc == 0
        return out

    def prefill(self, x, cfg: Cfg, warrays):
        x = np.ascontiguousarray(x, np.float32)
        S = x.shape[0]
        out = np.zeros((S, cfg.hidden_size), np.float32)
        rc = self.lib.orc_prefill(_p(out, f32p), _p(x, f32p), S, C.byref(cfg), *[_p(a, u16p) for a in warrays])
        assert rc == 0
        return out

    def append_f32(self, x, position, cfg: Cfg, kv_a, kv_a_norm):
        R, DR = cfg.kv_lora_rank, cfg.qk_rope_dim
        lat = np.zeros(R, np.float32)
        rp = np.zeros(DR, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        self.lib.orc_append_f32(_p(lat, f32p), _p(rp, f32p), _p(x, f32p), position, C.byref(cfg),
                                _p(kv_a, u16p), _p(kv_a_norm, u16p))
        return lat, rp

    def append_q8(self, x, position, cfg: Cfg, kv_a, kv_a_norm):
        R, DR = cfg.kv_lora_rank, cfg.qk_rope_dim
        q = np.zeros(R, np.int8)
        s = np.zeros(1, np.float32)
        rp = np.zeros(DR, np.uint16)
        x = np.ascontiguousarray(x, np.float32)
        self.lib.orc_append_q8(_p(q, i8p), _p(s, f32p), _p(rp, u16p), _p(x, f32p), position, C.byref(cfg),
                               _p(kv_a, u16p), _p(kv_a_norm, u16p))
        return q, s[0], rp

    def decode_sequence(self, x, cfg: Cfg, warrays, prefix=0, q8=False):
        """Same protocol as Reference.decode_sequence, on the restatement."""
        x = np.ascontiguousarray(x, np.float32)
        S = x.shape[0]
        R, DR = cfg.kv_lora_rank, cfg.qk_rope_dim
        outs = np.zeros((S - prefix, cfg.hidden_size), np.float32)
        if q8:
            l8 = np.zeros((S, R), np.int8)
            ls = np.zeros(S, np.float32)
            r16 = np.zeros((S, DR), np.uint16)
            for t in range(prefix):
                l8[t], ls[t], r16[t] = self.append_q8(x[t], t, cfg, warrays[1], warrays[2])
            for t in range(prefix, S):
                outs[t - prefix] = self.decode_q8(x[t], t, cfg, warrays, l8, ls, r16)
            return outs, (l8, ls, r16)
        lat = np.zeros((S, R), np.float32)
        rope = np.zeros((S, DR), np.float32)
        for t in range(prefix):
            lat[t], rope[t] = self.append_f32(x[t], t, cfg, warrays[1], warrays[2])
        for t in range(prefix, S):
            outs[t - prefix] = self.decode_f32(x[t], t, cfg, warrays, lat, rope)
        return outs, (lat, rope)


class ExpandedState(C.Structure):
    """KvlMlaState of the reference (include/kvl/mla_state.h:13-22): the expanded
    fp32 K/V state of its V6a correctness oracle."""
    _fields_ = [("capacity", C.c_int), ("len", C.c_int), ("num_heads", C.c_int), ("qk_nope_dim", C.c_int),
                ("qk_rope_dim", C.c_int), ("v_head_dim", C.c_int), ("keys", f32p), ("values", f32p)]


class Reference:
    """The reference runtime's own MLA functions, compiled from its sources."""

    def __init__(self, path=REF_SO):
        if not pathlib.Path(path).exists():
            raise FileNotFoundError(str(path))
        self.path = pathlib.Path(path)
        self.lib = C.CDLL(str(path))
        L = self.lib
        for n, st in (("kvl_mla_compressed_state", State), ("kvl_mla_compressed_q8_state", Q8State)):
            getattr(L, n + "_init").argtypes = [C.POINTER(st), C.POINTER(Cfg), C.c_int]
            getattr(L, n + "_init").restype = C.c_int
            getattr(L, n + "_free").argtypes = [C.POINTER(st)]
            getattr(L, n + "_truncate").argtypes = [C.POINTER(st), C.c_int]
            getattr(L, n + "_truncate").restype = C.c_int
            getattr(L, n + "_prefill_bf16").argtypes = [f32p, C.c_int, C.POINTER(Cfg), C.POINTER(W), C.POINTER(st)]
            getattr(L, n + "_prefill_bf16").restype = C.c_int
            getattr(L, n + "_bytes").argtypes = [C.POINTER(st)]
            getattr(L, n + "_bytes").restype = C.c_size_t
        L.kvl_mla_decode_compressed_bf16.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), C.POINTER(W), C.POINTER(State)]
        L.kvl_mla_decode_compressed_bf16.restype = C.c_int
        L.kvl_mla_decode_compressed_block_bf16.argtypes = [f32p, f32p, C.c_int, C.c_int, C.POINTER(Cfg), C.POINTER(W),
                                                           C.POINTER(State)]
        L.kvl_mla_decode_compressed_block_bf16.restype = C.c_int
        L.kvl_mla_decode_compressed_q8_bf16.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), C.POINTER(W),
                                                        C.POINTER(Q8State)]
        L.kvl_mla_decode_compressed_q8_bf16.restype = C.c_int
        L.kvl_mla_prefill_bf16.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), C.POINTER(W)]
        L.kvl_mla_prefill_bf16.restype = C.c_int
        L.kvl_mla_prefill_materialized_bf16.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), C.POINTER(W)]
        L.kvl_mla_prefill_materialized_bf16.restype = C.c_int
        L.kvl_mla_state_init.argtypes = [C.POINTER(ExpandedState), C.POINTER(Cfg), C.c_int]
        L.kvl_mla_state_init.restype = C.c_int
        L.kvl_mla_state_free.argtypes = [C.POINTER(ExpandedState)]
        L.kvl_mla_decode_bf16.argtypes = [f32p, f32p, C.c_int, C.POINTER(Cfg), C.POINTER(W), C.POINTER(ExpandedState)]
        L.kvl_mla_decode_bf16.restype = C.c_int

    def decode_expanded(self, x, cfg, warrays):
        """Every token of x decoded from position 0 through the reference's
        expanded-K/V state (src/mla_state.c:66-149), the layer below the
        compressed state in its oracle stack."""
        x = np.ascontiguousarray(x, np.float32)
        S = x.shape[0]
        w = w_of(warrays)
        st = ExpandedState()
        assert self.lib.kvl_mla_state_init(C.byref(st), C.byref(cfg), S) == 0
        outs = np.zeros((S, cfg.hidden_size), np.float32)
        for t in range(S):
            assert self.lib.kvl_mla_decode_bf16(_p(outs[t], f32p), _p(x[t], f32p), t, C.byref(cfg), C.byref(w),
                                                C.byref(st)) == 0
        self.lib.kvl_mla_state_free(C.byref(st))
        return outs

    def prefill(self, x, cfg, warrays, materialized=False):
        x = np.ascontiguousarray(x, np.float32)
        S = x.shape[0]
        out = np.zeros((S, cfg.hidden_size), np.float32)
        w = w_of(warrays)
        fn = self.lib.kvl_mla_prefill_materialized_bf16 if materialized else self.lib.kvl_mla_prefill_bf16
        rc = fn(_p(out, f32p), _p(x, f32p), S, C.byref(cfg), C.byref(w))
        assert rc == 0
        return out

    def decode_from_rows(self, x, cfg, warrays, latent, rope):
        """One kvl_mla_decode_compressed_bf16 call for token x at position L
        against a state whose L cached rows are given (fp32 latent [L][R] and
        rope [L][DR], written into the public state arrays as the reference's
        lab tools do).  Returns (out [H], appended latent [R], appended rope [DR])."""
        x = np.ascontiguousarray(x, np.float32)
        L, R = latent.shape
        DR = rope.shape[1]
        w = w_of(warrays)
        st = State()
        assert self.lib.kvl_mla_compressed_state_init(C.byref(st), C.byref(cfg), L + 1) == 0
        np.ctypeslib.as_array(st.latent, shape=((L + 1) * R,))[:L * R] = np.asarray(latent, np.float32).reshape(-1)
        np.ctypeslib.as_array(st.rope, shape=((L + 1) * DR,))[:L * DR] = np.asarray(rope, np.float32).reshape(-1)
        st.len = L
        out = np.zeros(cfg.hidden_size, np.float32)
        rc = self.lib.kvl_mla_decode_compressed_bf16(_p(out, f32p), _p(x, f32p), L, C.byref(cfg), C.byref(w),
                                                     C.byref(st))
        assert rc == 0
        lat_new = np.ctypeslib.as_array(st.latent, shape=((L + 1) * R,))[L * R:].copy()
        rope_new = np.ctypeslib.as_array(st.rope, shape=((L + 1) * DR,))[L * DR:].copy()
        self.lib.kvl_mla_compressed_state_free(C.byref(st))
        return out, lat_new, rope_new

    def decode_q8_from_rows(self, x, cfg, warrays, lat8, lscale, rope16):
        """kvl_mla_decode_compressed_q8_bf16 for token x at position L against a
        Q8 state whose L cached rows are given (int8 [L][R], fp32 [L], bf16 bits
        [L][DR]).  Returns (out [H], appended int8 [R], scale, bf16 rope [DR])."""
        x = np.ascontiguousarray(x, np.float32)
        L, R = lat8.shape
        DR = rope16.shape[1]
        w = w_of(warrays)
        st = Q8State()
        assert self.lib.kvl_mla_compressed_q8_state_init(C.byref(st), C.byref(cfg), L + 1) == 0
        np.ctypeslib.as_array(st.latent_q8, shape=((L + 1) * R,))[:L * R] = np.asarray(lat8, np.int8).reshape(-1)
        np.ctypeslib.as_array(st.latent_scale, shape=(L + 1,))[:L] = np.asarray(lscale, np.float32)
        np.ctypeslib.as_array(st.rope_bf16, shape=((L + 1) * DR,))[:L * DR] = np.asarray(rope16, np.uint16).reshape(-1)
        st.len = L
        out = np.zeros(cfg.hidden_size, np.float32)
        rc = self.lib.kvl_mla_decode_compressed_q8_bf16(_p(out, f32p), _p(x, f32p), L, C.byref(cfg), C.byref(w),
                                                        C.byref(st))
        assert rc == 0
        q_new = np.ctypeslib.as_array(st.latent_q8, shape=((L + 1) * R,))[L * R:].copy()
        s_new = float(np.ctypeslib.as_array(st.latent_scale, shape=(L + 1,))[L])
        r_new = np.ctypeslib.as_array(st.rope_bf16, shape=((L + 1) * DR,))[L * DR:].copy()
        self.lib.kvl_mla_compressed_q8_state_free(C.byref(st))
        return out, q_new, s_new, r_new

    def decode_sequence(self, x, cfg, warrays, prefix=0, q8=False):
        """Prefill `prefix` rows then decode the remaining tokens one by one.
        Returns (outputs of the decoded tokens, final state arrays)."""
        x = np.ascontiguousarray(x, np.float32)
        S = x.shape[0]
        w = w_of(warrays)
        st = Q8State() if q8 else State()
        base = "kvl_mla_compressed_q8_state" if q8 else "kvl_mla_compressed_state"
        assert getattr(self.lib, base + "_init")(C.byref(st), C.byref(cfg), S) == 0
        if prefix > 0:
            assert getattr(self.lib, base + "_prefill_bf16")(_p(x, f32p), prefix, C.byref(cfg), C.byref(w),
                                                             C.byref(st)) == 0
        outs = np.zeros((S - prefix, cfg.hidden_size), np.float32)
        dec = self.lib.kvl_mla_decode_compressed_q8_bf16 if q8 else self.lib.kvl_mla_decode_compressed_bf16
        for t in range(prefix, S):
            rc = dec(_p(outs[t - prefix], f32p), _p(x[t], f32p), t, C.byref(cfg), C.byref(w), C.byref(st))
            assert rc == 0
        R, DR = cfg.kv_lora_rank, cfg.qk_rope_dim
        if q8:
            arrs = (np.ctypeslib.as_array(st.latent_q8, shape=(S * R,)).reshape(S, R).copy(),
                    np.ctypeslib.as_array(st.latent_scale, shape=(S,)).copy(),
                    np.ctypeslib.as_array(st.rope_bf16, shape=(S * DR,)).reshape(S, DR).copy())
        else:
            arrs = (np.ctypeslib.as_array(st.latent, shape=(S * R,)).reshape(S, R).copy(),
                    np.ctypeslib.as_array(st.rope, shape=(S * DR,)).reshape(S, DR).copy())
        getattr(self.lib, base + "_free")(C.byref(st))
        return outs, arrs


def reference_available(scalar=False) -> bool:
    return (REF_SCALAR_SO if scalar else REF_SO).exists()
