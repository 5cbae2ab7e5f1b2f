"""The split-KV combine across GPUs in one kernel (kvl_mla_merge_exchange: each
GPU stores its packed (o, lse) record into every GPU's exchange buffer over
NVLink, flags it, and merges the records of all ranks) against the numpy
restatement of the combine, over several consecutive calls (both buffer sets,
one rank made late on purpose by the host so the other waits), on two GPUs as
two processes.  Needs two GPUs; skipped otherwise."""
from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NH, R = 16, 512


def _records(call, world, B):
    out = []
    for r in range(world):
        rng = np.random.default_rng(1000 * call + r)
        o = rng.standard_normal((B, NH, R)).astype(np.float32)
        lse = (rng.standard_normal((B, NH)) * 2.0).astype(np.float32)
        out.append((o, lse))
    return out


def _worker(rank, world, port, B, calls, q):
    try:
        import sys
        import time
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        import torch
        import torch.distributed as dist
        import kvl_pkg
        kvl_pkg.load()
        import kvl_b200.kvl_mla as K
        from kvl_b200.parallel import merge_partials
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")

        def gather(b):
            lst = [None] * world
            dist.all_gather_object(lst, b)
            return lst

        pg = K.PeerGroup(rank, world, B, gather)
        dev = torch.device("cuda", rank)
        worst = 0.0
        for call in range(calls):
            recs = _records(call, world, B)
            o, lse = recs[rank]
            rec = torch.from_numpy(np.concatenate([o.ravel(), lse.ravel()])).to(dev)
            out = torch.empty((B, NH, R), device=dev)
            out_l = torch.empty((B, NH), device=dev)
            if rank == 1 and call % 2 == 1:
                time.sleep(0.05)  # the other rank's kernel waits for this one's flag
            assert pg.merge(out, out_l, rec) == 0, K.last_error()
            assert pg.check() == 0, K.last_error()
            for b in range(B):
                wo, wl = merge_partials(np.stack([r[0][b] for r in recs]).astype(np.float64),
                                        np.stack([r[1][b] for r in recs]).astype(np.float64))
                np.testing.assert_allclose(out[b].cpu().numpy(), wo, rtol=1e-5, atol=1e-5)
                np.testing.assert_allclose(out_l[b].cpu().numpy(), wl, rtol=1e-5, atol=1e-5)
                worst = max(worst, float(np.max(np.abs(out[b].cpu().numpy() - wo))))
        dist.barrier()
        pg.close()
        dist.destroy_process_group()
        q.put((rank, "ok", worst))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error: {e!r}", None))


@pytest.mark.parametrize("B", [1, 3])
def test_merge_exchange_two_gpus(torch_cuda, B):
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, B, 6, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in procs:
            results.append(q.get(timeout=240))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
    assert sorted(r[0] for r in results) == [0, 1]
    for rank, status, _ in results:
        assert status == "ok", f"rank {rank}: {status}"
