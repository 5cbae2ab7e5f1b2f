"""The summation order of the kv_a projection on the matvec path, restated in
numpy and checked bit for bit against the reference's own AVX2 matvec.

The library's reference-order gemv (mla_kernels.cu, gemv_bf16_exact_kernel)
sums y = W x the way src/ops.c:31-50 does in its AVX2 build: eight fp32
accumulators, the one for i = l (mod 8) adding the rounded products w_i * x_i
(a multiply, then an add) in increasing i, then
((a0 + a4) + (a1 + a5)) + ((a2 + a6) + (a3 + a7)), then the products of a tail
past the last multiple of 8 added in order.  This test pins that order on the
CPU against the compiled reference (oracle/_ref/libkvl_ref.so); the GPU tests
then check the stored state rows, which depend on it, for equality with the
reference's.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from oracle.oracle import REF_SO, reference_available


def matvec_avx2_order(w_bits: np.ndarray, x: np.ndarray) -> np.ndarray:
    """w_bits [out][in] bf16 bit patterns, x [in] fp32 -> y [out] fp32."""
    out, n = w_bits.shape
    w = (w_bits.astype(np.uint32) << 16).view(np.float32)
    x = x.astype(np.float32)
    n8 = n // 8
    acc = np.zeros((out, 8), np.float32)
    for k in range(n8):
        prod = (w[:, 8 * k:8 * k + 8] * x[8 * k:8 * k + 8]).astype(np.float32)
        acc = (acc + prod).astype(np.float32)
    s = (acc[:, 0:4] + acc[:, 4:8]).astype(np.float32)
    y = ((s[:, 0] + s[:, 1]).astype(np.float32) + (s[:, 2] + s[:, 3]).astype(np.float32)).astype(np.float32)
    for i in range(8 * n8, n):
        y = (y + (w[:, i] * x[i]).astype(np.float32)).astype(np.float32)
    return y


@pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built (reference sources absent)")
@pytest.mark.parametrize("n_in,n_out", [(2048, 576), (2048, 64), (30, 7), (8, 3), (13, 5)])
def test_matvec_order_matches_reference_avx2(n_in, n_out):
    lib = C.CDLL(str(REF_SO))
    lib.kvl_matvec_bf16.restype = None
    lib.kvl_matvec_bf16.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]
    rng = np.random.default_rng(n_in * 1000 + n_out)
    w = (rng.standard_normal((n_out, n_in), dtype=np.float32) * 0.02)
    w_bits = (w.view(np.uint32) >> 16).astype(np.uint16)  # truncation: any bf16 pattern will do
    x = rng.standard_normal(n_in).astype(np.float32)
    want = np.zeros(n_out, np.float32)
    lib.kvl_matvec_bf16(want.ctypes.data, x.ctypes.data, np.ascontiguousarray(w_bits).ctypes.data, n_in, n_out)
    got = matvec_avx2_order(w_bits, x)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
