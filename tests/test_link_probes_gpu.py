"""The drop-in at link level: the reference runtime's own MLA probe programs
(src/mla_incremental_probe.c, src/mla_streaming_probe.c,
src/spec_q8_lab_probe.c), compiled from the reference's sources by
oracle/Makefile's `probes` target and linked against libkvl_mla_cuda.so in
place of the reference's mla_compressed_state.c, mla_compressed_q8_state.c and
mla_prefill_streaming.c.  Each probe runs its own gates unchanged and must
print its PASS line:
  mla_incremental_probe  expanded-state, compressed-state and prefilled-history
                         decode against the causal prefill (max-abs <= 1e-6 /
                         2e-6, src/mla_incremental_probe.c:105-108)
  mla_streaming_probe    the streaming prefill against the reference's
                         materialised prefill (max-abs and rel-RMS <= 2e-5)
  spec_q8_lab_probe      block decode and truncate-rollback exactly equal to
                         serial decode (0.0), Q8 state within 0.02
                         (src/spec_q8_lab_probe.c:173-180)
The probes use the reference's small probe shapes, whose states keep fp32
rows on the device (the reference's state format)."""
from __future__ import annotations

import pathlib
import subprocess

import pytest

pytestmark = pytest.mark.gpu

PROBES = pathlib.Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "probes"
PASS = {"mla_incremental_probe": "PASS: expanded, compressed and batch-history MLA match causal prefill",
        "mla_streaming_probe": "mla_streaming_probe PASS",
        "spec_q8_lab_probe": "PASS: exact block rollback and hybrid INT8 MLA synthetic gate"}


@pytest.mark.parametrize("name", sorted(PASS))
def test_reference_probe_linked_against_the_cuda_library(torch_cuda, name):
    exe = PROBES / name
    if not exe.exists():
        pytest.skip("probes not built (reference sources absent when building)")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, f"{name} failed:\n{r.stdout}\n{r.stderr}"
    assert PASS[name] in r.stdout, r.stdout
