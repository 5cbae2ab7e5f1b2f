"""The decode attends at full BASELINE sizes against the CPU restatement
(src/mla_compressed_state.c:132-148, src/mla_compressed_q8_state.c:216-238):
config 5 (one sequence of 131,072 rows, split over every SM and merged) and
config 3 (64 Q8 sequences with the lengths of bench.py's
workload), plus the size-independent property that the split-KV result equals a
single pass over all rows (one CTA, no merge) to within the rounding of P.
Tolerance: rel-L2 <= 1e-2, max-abs <= 2e-2 against the reference; lse within 1e-2."""
from __future__ import annotations

import numpy as np
import pytest

from tests.parity import assert_close
from tests.test_attend_gpu import SCALE, absorbed_q, bf16_pool, q8_pool, run_bf16, run_q8

pytestmark = pytest.mark.gpu


def test_config5_full_length(K, S, orc, torch_cuda):
    L = 131072
    kv, lat, rope = bf16_pool(S, 5, L)
    q = absorbed_q(S, 55, 1)
    out, lse, info = run_bf16(K, torch_cuda, kv, q, [L], [0])
    assert info["partials"] >= 100
    mix, lse_ref = orc.attend_f32(q[0], lat, rope, SCALE)
    assert_close(out[0], mix, what="config 5 attend, split over the SMs")
    np.testing.assert_allclose(lse[0], lse_ref, atol=1e-2)
    one, lse1, info1 = run_bf16(K, torch_cuda, kv, q, [L], [0], max_ctas=1)
    assert info1["partials"] == 0
    rel = np.linalg.norm(out - one) / np.linalg.norm(one)
    assert rel < 2e-3, f"split vs single pass rel-L2 {rel:.2e}"
    np.testing.assert_allclose(lse, lse1, atol=1e-4)


def test_config3_full_batch(K, S, orc, torch_cuda):
    lens = [int(v) for v in S.uniform_ints(3, S.S_LEN, 64, 512, 8192)]
    row0 = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
    rows = int(sum(lens))
    lat8, scale, rope = q8_pool(S, 3, rows)
    q = absorbed_q(S, 33, len(lens))
    out, lse, info = run_q8(K, torch_cuda, lat8, scale, rope, q, lens, row0)
    got, want = [], []
    for b, n in enumerate(lens):
        r0 = int(row0[b])
        mix, lse_ref = orc.attend_q8(q[b], lat8[r0:r0 + n], scale[r0:r0 + n], rope[r0:r0 + n], SCALE)
        got.append(out[b])
        want.append(mix)
        np.testing.assert_allclose(lse[b], lse_ref, atol=1e-2)
    assert_close(np.stack(got), np.stack(want), what="config 3 Q8 attend, 64 sequences")
