"""The C-ABI library on a host without a GPU: it loads, exports every symbol
the headers in include/kvl/ declare, keeps the reference's struct layouts,
rejects invalid arguments with -1 exactly where the reference does, and has no
CPU fallback (compute calls fail without a device)."""
from __future__ import annotations

import ctypes as C
import pathlib
import re
import subprocess
import tempfile

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include" / "kvl").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"\b(kvl_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol(K):
    lib = K.load()
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    assert set(K.SIGNATURES) >= names


def test_struct_layouts_match_the_headers(K):
    """sizeof/offsetof from the C headers (compiled here) equal the ctypes
    layouts of the binding and of the reference-side stubs (oracle/oracle.py)."""
    from oracle import oracle as O
    src = r'''
#include <stdio.h>
#include <stddef.h>
#include "kvl/mla_compressed_state.h"
#include "kvl/mla_compressed_q8_state.h"
#include "kvl/mla_cuda.h"
int main(void) {
  printf("%zu %zu %zu\n", sizeof(KvlMlaConfig), offsetof(KvlMlaConfig, rms_eps), offsetof(KvlMlaConfig, rope_theta));
  printf("%zu %zu\n", sizeof(KvlMlaBF16), offsetof(KvlMlaBF16, o_proj));
  printf("%zu %zu %zu\n", sizeof(KvlMlaCompressedState), offsetof(KvlMlaCompressedState, latent),
         offsetof(KvlMlaCompressedState, rope));
  printf("%zu %zu %zu %zu\n", sizeof(KvlMlaCompressedQ8State), offsetof(KvlMlaCompressedQ8State, latent_q8),
         offsetof(KvlMlaCompressedQ8State, latent_scale), offsetof(KvlMlaCompressedQ8State, rope_bf16));
  return 0;
}
'''
    with tempfile.TemporaryDirectory() as td:
        c = pathlib.Path(td) / "abi.c"
        exe = pathlib.Path(td) / "abi"
        c.write_text(src)
        subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(c), "-o", str(exe)], check=True)
        lines = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = [list(map(int, ln.split())) for ln in lines if ln.strip()]
    for cfg_t in (K.KvlMlaConfig, O.Cfg):
        assert got[0] == [C.sizeof(cfg_t), cfg_t.rms_eps.offset, cfg_t.rope_theta.offset]
    for w_t in (K.KvlMlaBF16, O.W):
        assert got[1] == [C.sizeof(w_t), w_t.o_proj.offset]
    for s_t in (K.KvlMlaCompressedState, O.State):
        assert got[2] == [C.sizeof(s_t), s_t.latent.offset, s_t.rope.offset]
    for q_t in (K.KvlMlaCompressedQ8State, O.Q8State):
        assert got[3] == [C.sizeof(q_t), q_t.latent_q8.offset, q_t.latent_scale.offset, q_t.rope_bf16.offset]


def test_argument_validation_matches_reference(K):
    """src/mla_compressed_state.c:27-29, :41-42, :57-61, :92-95 and
    src/mla_prefill_streaming.c:80-85: -1 before any state change."""
    lib = K.load()
    cfg = K.make_config(16, 2, 4, 4, 4, 6, 1e-6, 1e4)
    st = K.KvlMlaCompressedState()
    assert lib.kvl_mla_compressed_state_init(C.byref(st), C.byref(cfg), 0) == -1
    bad = K.make_config(16, 2, 4, 3, 4, 6, 1e-6, 1e4)  # odd rope dim
    assert lib.kvl_mla_compressed_state_init(C.byref(st), C.byref(bad), 4) == -1
    assert lib.kvl_mla_compressed_state_truncate(None, 0) == -1
    st.len = 3
    assert lib.kvl_mla_compressed_state_truncate(C.byref(st), 4) == -1
    assert lib.kvl_mla_compressed_state_truncate(C.byref(st), 2) == 0 and st.len == 2
    lib.kvl_mla_compressed_state_reset(C.byref(st))
    assert st.len == 0
    assert lib.kvl_mla_decode_compressed_bf16(None, None, 0, C.byref(cfg), None, C.byref(st)) == -1
    assert lib.kvl_mla_prefill_bf16(None, None, 0, C.byref(cfg), None) == -1
    q8 = K.KvlMlaCompressedQ8State()
    assert lib.kvl_mla_compressed_q8_state_init(C.byref(q8), C.byref(cfg), -1) == -1
    assert lib.kvl_mla_compressed_state_bytes(None) == 0
    lib.kvl_mla_compressed_state_free(None)
    h = C.c_void_p()
    assert lib.kvl_mla_attend_plan_create(C.byref(h), 0, None, None, 16, 512, 0) == -1


def test_no_cpu_fallback(K):
    """Without a device the compute path reports failure instead of running on
    the CPU."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = K.load()
    cfg = K.make_config(16, 2, 4, 4, 4, 6, 1e-6, 1e4)
    st = K.KvlMlaCompressedState()
    assert lib.kvl_mla_compressed_state_init(C.byref(st), C.byref(cfg), 8) == -1
    assert st.capacity == 0 and not st.latent
    assert K.last_error() != ""
