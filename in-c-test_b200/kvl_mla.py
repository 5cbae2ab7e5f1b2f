"""ctypes binding of libkvl_mla_cuda: the reference runtime's MLA state API
(include/kvl/mla_compressed_state.h, include/kvl/mla_compressed_q8_state.h,
kvl_mla_prefill_bf16 in include/kvl/ops.h) plus the device-pointer calls of
include/kvl/mla_cuda.h.

Function names, argument meaning and the 0 / -1 return convention are the
reference's; this module only adds numpy/torch conveniences.  It loads the
in-tree library and raises if it is missing -- there is no fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import pathlib

import numpy as np

LIB_PATH = pathlib.Path(__file__).resolve().parent / "lib" / "libkvl_mla_cuda.so"

u16p = C.POINTER(C.c_uint16)
f32p = C.POINTER(C.c_float)
i8p = C.POINTER(C.c_int8)
i32p = C.POINTER(C.c_int)
i64p = C.POINTER(C.c_int64)


class KvlMlaConfig(C.Structure):
    _fields_ = [("hidden_size", C.c_int), ("num_heads", C.c_int), ("qk_nope_dim", C.c_int),
                ("qk_rope_dim", C.c_int), ("v_head_dim", C.c_int), ("kv_lora_rank", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float)]


class KvlMlaBF16(C.Structure):
    _fields_ = [("q_proj", u16p), ("kv_a_proj", u16p), ("kv_a_norm", u16p), ("kv_b_proj", u16p),
                ("o_proj", u16p)]


class KvlMlaDeviceWeights(C.Structure):
    _fields_ = [("q_proj", C.c_void_p), ("kv_a_proj", C.c_void_p), ("kv_a_norm", C.c_void_p),
                ("kv_b_proj", C.c_void_p), ("o_proj", C.c_void_p)]


class KvlMlaCompressedState(C.Structure):
    _fields_ = [("capacity", C.c_int), ("len", C.c_int), ("kv_lora_rank", C.c_int),
                ("qk_rope_dim", C.c_int), ("latent", f32p), ("rope", f32p)]


class KvlMlaCompressedQ8State(C.Structure):
    _fields_ = [("capacity", C.c_int), ("len", C.c_int), ("kv_lora_rank", C.c_int),
                ("qk_rope_dim", C.c_int), ("latent_q8", i8p), ("latent_scale", f32p),
                ("rope_bf16", u16p)]


# Every symbol include/kvl/*.h declares, with its ctypes signature.
SIGNATURES = {
    # kvl/mla_compressed_state.h
    "kvl_mla_compressed_state_init": (C.c_int, [C.POINTER(KvlMlaCompressedState), C.POINTER(KvlMlaConfig), C.c_int]),
    "kvl_mla_compressed_state_reset": (None, [C.POINTER(KvlMlaCompressedState)]),
    "kvl_mla_compressed_state_truncate": (C.c_int, [C.POINTER(KvlMlaCompressedState), C.c_int]),
    "kvl_mla_compressed_state_free": (None, [C.POINTER(KvlMlaCompressedState)]),
    "kvl_mla_compressed_state_bytes": (C.c_size_t, [C.POINTER(KvlMlaCompressedState)]),
    "kvl_mla_compressed_state_prefill_bf16": (C.c_int, [f32p, C.c_int, C.POINTER(KvlMlaConfig),
                                                        C.POINTER(KvlMlaBF16), C.POINTER(KvlMlaCompressedState)]),
    "kvl_mla_decode_compressed_bf16": (C.c_int, [f32p, f32p, C.c_int, C.POINTER(KvlMlaConfig),
                                                 C.POINTER(KvlMlaBF16), C.POINTER(KvlMlaCompressedState)]),
    "kvl_mla_decode_compressed_block_bf16": (C.c_int, [f32p, f32p, C.c_int, C.c_int, C.POINTER(KvlMlaConfig),
                                                       C.POINTER(KvlMlaBF16), C.POINTER(KvlMlaCompressedState)]),
    # kvl/mla_compressed_q8_state.h
    "kvl_mla_compressed_q8_state_init": (C.c_int, [C.POINTER(KvlMlaCompressedQ8State), C.POINTER(KvlMlaConfig), C.c_int]),
    "kvl_mla_compressed_q8_state_reset": (None, [C.POINTER(KvlMlaCompressedQ8State)]),
    "kvl_mla_compressed_q8_state_truncate": (C.c_int, [C.POINTER(KvlMlaCompressedQ8State), C.c_int]),
    "kvl_mla_compressed_q8_state_free": (None, [C.POINTER(KvlMlaCompressedQ8State)]),
    "kvl_mla_compressed_q8_state_bytes": (C.c_size_t, [C.POINTER(KvlMlaCompressedQ8State)]),
    "kvl_mla_compressed_q8_state_prefill_bf16": (C.c_int, [f32p, C.c_int, C.POINTER(KvlMlaConfig),
                                                           C.POINTER(KvlMlaBF16), C.POINTER(KvlMlaCompressedQ8State)]),
    "kvl_mla_decode_compressed_q8_bf16": (C.c_int, [f32p, f32p, C.c_int, C.POINTER(KvlMlaConfig),
                                                    C.POINTER(KvlMlaBF16), C.POINTER(KvlMlaCompressedQ8State)]),
    # kvl/ops.h
    "kvl_mla_prefill_bf16": (C.c_int, [f32p, f32p, C.c_int, C.POINTER(KvlMlaConfig), C.POINTER(KvlMlaBF16)]),
    # kvl/mla_cuda.h
    "kvl_mla_cuda_last_error": (C.c_char_p, []),
    "kvl_mla_cuda_weight_cache": (C.c_int, [C.c_int]),
    "kvl_mla_cuda_state_device_bytes": (C.c_size_t, [C.c_void_p]),
    "kvl_mla_cuda_profile": (C.c_int, [C.c_int]),
    "kvl_mla_cuda_profile_read": (C.c_int, [C.c_char_p, C.c_size_t]),
    "kvl_mla_attend_plan_create": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, i32p, i64p, C.c_int, C.c_int, C.c_int]),
    "kvl_mla_attend_plan_destroy": (None, [C.c_void_p]),
    "kvl_mla_attend_plan_info": (C.c_int, [C.c_void_p, i32p, i32p, i32p]),
    "kvl_mla_attend_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                      C.c_int, C.c_int, C.c_int, C.c_float, C.c_void_p]),
    "kvl_mla_attend_q8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_float, C.c_void_p]),
    "kvl_mla_attend_bf16_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int,
                                              C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                              C.c_void_p]),
    "kvl_mla_attend_check": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kvl_mla_merge_partials": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                         C.c_int, C.c_void_p]),
    "kvl_mla_merge_packed": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.c_void_p]),
    "kvl_mla_peer_handle_bytes": (C.c_size_t, []),
    "kvl_mla_peer_group_create": (C.c_int, [C.POINTER(C.c_void_p), C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                            C.c_void_p]),
    "kvl_mla_peer_group_connect": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kvl_mla_merge_exchange": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "kvl_mla_peer_group_check": (C.c_int, [C.c_void_p, C.c_void_p]),
    "kvl_mla_peer_group_destroy": (None, [C.c_void_p]),
    "kvl_mla_attend_bf16_exchange": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                               C.c_void_p, C.c_int64, C.c_float, C.c_void_p]),
    "kvl_mla_decode_step_workspace_bytes": (C.c_size_t, [C.POINTER(KvlMlaConfig), C.c_int]),
    "kvl_mla_decode_step_bf16": (C.c_int, [C.POINTER(KvlMlaConfig), C.POINTER(KvlMlaDeviceWeights), C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p,
                                           C.c_int, C.c_void_p, C.c_void_p]),
    "kvl_mla_decode_step_q8": (C.c_int, [C.POINTER(KvlMlaConfig), C.POINTER(KvlMlaDeviceWeights), C.c_void_p,
                                         C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                         C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "kvl_mla_prefill_workspace_bytes": (C.c_size_t, [C.POINTER(KvlMlaConfig), C.c_int]),
    "kvl_mla_prefill_dev": (C.c_int, [C.POINTER(KvlMlaConfig), C.POINTER(KvlMlaDeviceWeights), C.c_void_p,
                                      C.c_void_p, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]),
    "kvl_mla_prefill_cp_begin": (C.c_int, [C.POINTER(KvlMlaConfig), C.POINTER(KvlMlaDeviceWeights), C.c_void_p,
                                           C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_size_t,
                                           C.c_void_p]),
    "kvl_mla_prefill_cp_end": (C.c_int, [C.POINTER(KvlMlaConfig), C.POINTER(KvlMlaDeviceWeights), C.c_void_p,
                                         C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_size_t,
                                         C.c_void_p]),
    "kvl_mla_q8_quantize_rows": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "kvl_mla_q8_dequant": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_void_p]),
    "kvl_mla_bf16_rne": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
}

_lib = None


def load(path: os.PathLike | str | None = None) -> C.CDLL:
    """Loads the in-tree CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = pathlib.Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `make -C in-c-test_b200/csrc` "
                           "(there is no CPU fallback)")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def last_error() -> str:
    return load().kvl_mla_cuda_last_error().decode()


class KvlError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise KvlError(f"{what} failed: {last_error()}")


def ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def make_config(H=2048, NH=16, DN=128, DR=64, DV=128, R=512, eps=1e-5, theta=800000.0) -> KvlMlaConfig:
    return KvlMlaConfig(H, NH, DN, DR, DV, R, eps, theta)


class Weights:
    """Host bf16 weights of one MLA layer (numpy uint16 arrays) + the C struct."""

    def __init__(self, q_proj, kv_a_proj, kv_a_norm, kv_b_proj, o_proj):
        self.arrays = [np.ascontiguousarray(a, dtype=np.uint16) for a in
                       (q_proj, kv_a_proj, kv_a_norm, kv_b_proj, o_proj)]
        self.c = KvlMlaBF16(*[ptr(a, u16p) for a in self.arrays])

    @property
    def q_proj(self):
        return self.arrays[0]

    @property
    def kv_a_proj(self):
        return self.arrays[1]

    @property
    def kv_a_norm(self):
        return self.arrays[2]

    @property
    def kv_b_proj(self):
        return self.arrays[3]

    @property
    def o_proj(self):
        return self.arrays[4]


def random_weights(cfg: KvlMlaConfig, seed: int, std: float = 0.02, norm_std: float = 0.0) -> Weights:
    from . import synth as S  # noqa: WPS433
    H, NH, DN, DR, DV, R = (cfg.hidden_size, cfg.num_heads, cfg.qk_nope_dim, cfg.qk_rope_dim,
                            cfg.v_head_dim, cfg.kv_lora_rank)
    q = S.normal_bf16(seed, S.S_WQ, (NH * (DN + DR), H), std)
    kva = S.normal_bf16(seed, S.S_WKVA, (R + DR, H), std)
    if norm_std > 0:
        kvan = S.f32_to_bf16_bits(1.0 + S.normal(seed, 40, R, norm_std))
    else:
        kvan = S.f32_to_bf16_bits(np.ones(R, np.float32))
    kvb = S.normal_bf16(seed, S.S_WKVB, (NH * (DN + DV), R), std)
    o = S.normal_bf16(seed, S.S_WO, (H, NH * DV), std)
    return Weights(q, kva, kvan, kvb, o)


class CompressedState:
    """Owner of a KvlMlaCompressedState created through the library."""

    def __init__(self, cfg: KvlMlaConfig, capacity: int, lib=None):
        self.lib = lib or load()
        self.cfg = cfg
        self.s = KvlMlaCompressedState()
        check(self.lib.kvl_mla_compressed_state_init(C.byref(self.s), C.byref(cfg), capacity), "state init")

    def prefill(self, x: np.ndarray, w: Weights) -> int:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return self.lib.kvl_mla_compressed_state_prefill_bf16(ptr(x, f32p), x.shape[0], C.byref(self.cfg),
                                                              C.byref(w.c), C.byref(self.s))

    def decode(self, x: np.ndarray, position: int, w: Weights) -> tuple[int, np.ndarray]:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(self.cfg.hidden_size, np.float32)
        rc = self.lib.kvl_mla_decode_compressed_bf16(ptr(out, f32p), ptr(x, f32p), position, C.byref(self.cfg),
                                                     C.byref(w.c), C.byref(self.s))
        return rc, out

    def latent(self) -> np.ndarray:
        n = self.s.len * self.s.kv_lora_rank
        return np.ctypeslib.as_array(self.s.latent, shape=(max(n, 1),))[:n].reshape(self.s.len, -1).copy()

    def rope(self) -> np.ndarray:
        n = self.s.len * self.s.qk_rope_dim
        return np.ctypeslib.as_array(self.s.rope, shape=(max(n, 1),))[:n].reshape(self.s.len, -1).copy()

    def free(self) -> None:
        self.lib.kvl_mla_compressed_state_free(C.byref(self.s))


def t_ptr(t) -> int:
    """Device pointer of a torch tensor (0 for None)."""
    return 0 if t is None else int(t.data_ptr())


class PeerGroup:
    """kvl_mla_peer_group_*: the split-KV combine across the GPUs of one node.
    `gather(bytes) -> list of bytes` gathers one byte string per rank in rank
    order (e.g. torch.distributed.all_gather_object)."""

    def __init__(self, rank, world, batch, gather, num_heads=16, kv_lora_rank=512, lib=None):
        self.lib = lib or load()
        n = self.lib.kvl_mla_peer_handle_bytes()
        handle = C.create_string_buffer(n)
        self.h = C.c_void_p()
        check(self.lib.kvl_mla_peer_group_create(C.byref(self.h), rank, world, batch, num_heads, kv_lora_rank,
                                                 handle), "peer group create")
        handles = gather(handle.raw)
        table = C.create_string_buffer(b"".join(handles), n * world)
        check(self.lib.kvl_mla_peer_group_connect(self.h, table), "peer group connect")

    def merge(self, out, lse, record, stream=0):
        return self.lib.kvl_mla_merge_exchange(self.h, t_ptr(out), t_ptr(lse), t_ptr(record), stream)

    def attend_exchange(self, plan, out, lse, q, kv, rows, scale=1.0 / np.sqrt(192.0), stream=0):
        """kvl_mla_attend_bf16_exchange: attend this rank's KV range with `plan`
        and combine across the group in the same call."""
        return self.lib.kvl_mla_attend_bf16_exchange(plan.h, self.h, t_ptr(out), t_ptr(lse), t_ptr(q), t_ptr(kv),
                                                     rows, float(scale), stream)

    def check(self, stream=0):
        return self.lib.kvl_mla_peer_group_check(self.h, stream)

    def close(self):
        if self.h:
            self.lib.kvl_mla_peer_group_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class AttendPlan:
    """kvl_mla_attend_plan_create wrapper (current CUDA device)."""

    def __init__(self, seq_len, seq_row0, num_heads=16, kv_lora_rank=512, max_ctas=0, lib=None):
        self.lib = lib or load()
        sl = np.ascontiguousarray(seq_len, dtype=np.int32)
        r0 = np.ascontiguousarray(seq_row0, dtype=np.int64)
        self.batch = int(sl.shape[0])
        self.num_heads = num_heads
        self.kv_lora_rank = kv_lora_rank
        self.h = C.c_void_p()
        check(self.lib.kvl_mla_attend_plan_create(C.byref(self.h), self.batch, ptr(sl, i32p), ptr(r0, i64p),
                                                  num_heads, kv_lora_rank, max_ctas), "plan create")

    def info(self):
        a, b, c = C.c_int(), C.c_int(), C.c_int()
        self.lib.kvl_mla_attend_plan_info(self.h, C.byref(a), C.byref(b), C.byref(c))
        return {"ctas": a.value, "partials": b.value, "segments": c.value}

    def attend_bf16(self, out, lse, q, kv, rows, rope_dim=64, scale=1.0 / np.sqrt(192.0), stream=0):
        return self.lib.kvl_mla_attend_bf16(self.h, t_ptr(out), t_ptr(lse), t_ptr(q), t_ptr(kv), rows,
                                            self.num_heads, self.kv_lora_rank, rope_dim, float(scale), stream)

    def attend_q8(self, out, lse, q, lat8, lscale, rope16, rows, rope_dim=64, scale=1.0 / np.sqrt(192.0), stream=0):
        return self.lib.kvl_mla_attend_q8(self.h, t_ptr(out), t_ptr(lse), t_ptr(q), t_ptr(lat8), t_ptr(lscale),
                                          t_ptr(rope16), rows, self.num_heads, self.kv_lora_rank, rope_dim,
                                          float(scale), stream)

    def check(self, stream=0):
        return self.lib.kvl_mla_attend_check(self.h, stream)

    def __del__(self):
        try:
            if self.h:
                self.lib.kvl_mla_attend_plan_destroy(self.h)
                self.h = C.c_void_p()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass
