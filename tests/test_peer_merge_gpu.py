"""The split-KV combine across GPUs in one kernel (kvl_mla_merge_exchange: each
GPU stores its packed (o, lse) record into every GPU's exchange buffer over
NVLink, flags it, and merges the records of all ranks) against the numpy
restatement of the combine, over several consecutive calls (both buffer sets,
one rank made late on purpose by the host so the other waits), on two GPUs as
two processes.  The fused form (kvl_mla_attend_bf16_exchange: each GPU
attends its half of every sequence's KV and one kernel combines locally,
exchanges and merges) is checked against the CPU restatement of the attend
over the whole sequence (src/mla_compressed_state.c:132-148), at the decode
tolerance rel-L2 <= 1e-2, max-abs <= 2e-2.  Needs two GPUs; skipped otherwise."""
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


def _attend_worker(rank, world, port, lens, calls, q):
    try:
        import sys
        import time
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path.insert(0, root)
        import torch
        import torch.distributed as dist
        import kvl_pkg
        kvl_pkg.load()
        import kvl_b200.kvl_mla as K
        import kvl_b200.synth as S
        from oracle.oracle import Oracle
        from tests.parity import assert_close
        orc = Oracle()
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"tcp://127.0.0.1:{port}")

        def gather(b):
            lst = [None] * world
            dist.all_gather_object(lst, b)
            return lst

        B = len(lens)
        row0 = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        rows = int(np.sum(lens))
        lat = S.normal_bf16(7, S.S_LAT, (rows, R), 1.0)
        rope = S.normal_bf16(7, S.S_ROPE, (rows, 64), 1.0)
        kv = np.concatenate([lat, rope], axis=1)
        latf, ropef = S.bf16_bits_to_f32(lat), S.bf16_bits_to_f32(rope)
        # this rank's contiguous KV range of every sequence
        cut = [(r0 + (n * rank) // world, r0 + (n * (rank + 1)) // world) for n, r0 in zip(lens, row0)]
        plan = K.AttendPlan([b - a for a, b in cut], [a for a, _ in cut], NH, R)
        pg = K.PeerGroup(rank, world, B, gather)
        dev = torch.device("cuda", rank)
        kv_t = torch.from_numpy(kv.view(np.int16)).to(dev)
        scale = 1.0 / np.sqrt(192.0)
        for call in range(calls):
            qv = S.bf16_bits_to_f32(S.normal_bf16(100 + call, S.S_Q, (B, NH, R + 64), 0.1))
            q_t = torch.from_numpy(qv).to(dev)
            out = torch.full((B, NH, R), float("nan"), device=dev)
            out_l = torch.full((B, NH), float("nan"), device=dev)
            if rank == 1 and call % 2 == 1:
                time.sleep(0.05)
            assert pg.attend_exchange(plan, out, out_l, q_t, kv_t, rows, scale) == 0, K.last_error()
            assert pg.check() == 0, K.last_error()
            o, lv = out.cpu().numpy(), out_l.cpu().numpy()
            for b, (n, r0) in enumerate(zip(lens, row0)):
                mix, lse_ref = orc.attend_f32(qv[b], latf[r0:r0 + n], ropef[r0:r0 + n], scale)
                assert_close(o[b], mix, what=f"rank {rank} call {call} seq {b} L={n}")
                assert np.max(np.abs(lv[b] - lse_ref)) < 1e-2
        dist.barrier()
        pg.close()
        dist.destroy_process_group()
        q.put((rank, "ok", plan.info()))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error: {e!r}", None))


def _run_two(target, args):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, 2, port) + args + (q,)) for r in range(2)]
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


@pytest.mark.parametrize("lens", [[3000], [20000, 7, 130, 5000]])
def test_attend_exchange_two_gpus(torch_cuda, lens):
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_two(_attend_worker, (lens, 4))


@pytest.mark.parametrize("B", [1, 3])
def test_merge_exchange_two_gpus(torch_cuda, B):
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_two(_worker, (B, 6))


def _timeout_worker(rank, world, port, q):
    """Rank 1 skips one merge call.  Rank 0's kernel waits for rank 1's values,
    gives up after its bounded wait (2 s) and records the timeout, which
    kvl_mla_peer_group_check reports; rank 1 stays (launching nothing) until
    rank 0 has read that status.  Then both ranks destroy the group and create
    and connect a new one, whose merges are correct again -- the recovery the
    library documents."""
    try:
        import sys
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

        dev = torch.device("cuda", rank)
        B = 2

        def merge_once(pg, call):
            recs = _records(call, world, B)
            o, lse = recs[rank]
            rec = torch.from_numpy(np.concatenate([o.ravel(), lse.ravel()])).to(dev)
            out = torch.empty((B, NH, R), device=dev)
            out_l = torch.empty((B, NH), device=dev)
            assert pg.merge(out, out_l, rec) == 0, K.last_error()
            return out, out_l, recs

        pg = K.PeerGroup(rank, world, B, gather)
        merge_once(pg, 0)
        assert pg.check() == 0, K.last_error()
        dist.barrier()
        if rank == 0:
            merge_once(pg, 1)  # rank 1 never joins this call
            rc = pg.check()
            msg = K.last_error()
            assert rc == -1, "the wait for the absent rank did not run out"
            assert "did not arrive in time" in msg, msg
        dist.barrier()  # rank 1 leaves its buffer in place until rank 0 has read the status
        pg.close()
        pg = K.PeerGroup(rank, world, B, gather)
        out, out_l, recs = merge_once(pg, 2)
        assert pg.check() == 0, K.last_error()
        for b in range(B):
            wo, wl = merge_partials(np.stack([r[0][b] for r in recs]).astype(np.float64),
                                    np.stack([r[1][b] for r in recs]).astype(np.float64))
            np.testing.assert_allclose(out[b].cpu().numpy(), wo, rtol=1e-5, atol=1e-5)
        dist.barrier()
        pg.close()
        dist.destroy_process_group()
        q.put((rank, "ok", None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error: {e!r}", None))


def test_merge_exchange_timeout_and_recreate_two_gpus(torch_cuda):
    if torch_cuda.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    _run_two(_timeout_worker, ())
