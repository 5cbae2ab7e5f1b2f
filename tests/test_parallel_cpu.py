"""Multi-GPU host logic on CPU: sequence sharding, split-KV ranges and the
(o, lse) merge protocol, including a world_size-2 gloo run in which each rank
attends its half of the KV range with the oracle and the ranks all-gather and
merge their partials -- the protocol bench.py runs over NCCL with the attend
and merge kernels."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def test_shard_sequences_balances_and_is_deterministic():
    from kvl_b200.parallel import shard_sequences
    import kvl_b200.synth as S
    lens = [int(v) for v in S.uniform_ints(3, S.S_LEN, 64, 512, 8192)]
    for world in (1, 2, 4, 8):
        parts = shard_sequences(lens, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)
        assert parts == shard_sequences(lens, world)


def test_split_kv_covers_the_range():
    from kvl_b200.parallel import split_kv
    for L, world in [(131072, 8), (1000, 3), (5, 8)]:
        r = split_kv(L, world)
        assert len(r) == world and r[0][0] == 0 and r[-1][1] == L
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))


def _partials(orc, S, world):
    from kvl_b200.parallel import split_kv
    L, R, DR, NH = 900, 512, 64, 16
    q = S.bf16_bits_to_f32(S.normal_bf16(9, S.S_Q, (NH, R + DR), 0.1))
    lat = S.bf16_bits_to_f32(S.normal_bf16(9, S.S_LAT, (L, R)))
    rope = S.bf16_bits_to_f32(S.normal_bf16(9, S.S_ROPE, (L, DR)))
    scale = 1.0 / np.sqrt(192.0)
    full, full_lse = orc.attend_f32(q, lat, rope, scale)
    parts = [orc.attend_f32(q, lat[lo:hi], rope[lo:hi], scale) for lo, hi in split_kv(L, world)]
    return full, full_lse, parts


def test_merge_of_partials_equals_full_attend(orc, S):
    from kvl_b200.parallel import merge_partials
    full, full_lse, parts = _partials(orc, S, 4)
    o, lse = merge_partials(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]))
    assert np.max(np.abs(o - full)) < 1e-5
    assert np.max(np.abs(lse - full_lse)) < 1e-4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_q):
    import sys
    import pathlib
    root = pathlib.Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    import kvl_pkg
    kvl_pkg.load()
    import torch
    import torch.distributed as dist
    import kvl_b200.synth as S
    from kvl_b200.parallel import merge_partials
    from oracle.oracle import Oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full, full_lse, parts = _partials(Oracle(), S, world)
        o, lse = parts[rank]
        go = [torch.zeros(o.shape) for _ in range(world)]
        gl = [torch.zeros(lse.shape) for _ in range(world)]
        dist.all_gather(go, torch.from_numpy(o))
        dist.all_gather(gl, torch.from_numpy(lse))
        mo, ml = merge_partials(np.stack([t.numpy() for t in go]), np.stack([t.numpy() for t in gl]))
        result_q.put((rank, float(np.max(np.abs(mo - full))), float(np.max(np.abs(ml - full_lse)))))
    finally:
        dist.destroy_process_group()


def test_split_kv_merge_over_gloo_world2():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err_o, err_l in res:
        assert err_o < 1e-5 and err_l < 1e-4, (rank, err_o, err_l)


def test_zigzag_chunks_partition_and_balance():
    from kvl_b200.parallel import gathered_row_order, zigzag_chunks
    for S_len, world in [(4096, 1), (4096, 2), (4096, 4), (4096, 8), (48, 3)]:
        ch = zigzag_chunks(S_len, world)
        rows = sorted(r for a, b in ch for r in list(range(*a)) + list(range(*b)))
        assert rows == list(range(S_len))
        # causal work of a chunk [lo, hi): sum of (t + 1) over its query rows
        work = [sum(t + 1 for t in range(*a)) + sum(t + 1 for t in range(*b)) for a, b in ch]
        assert max(work) - min(work) <= (S_len // (2 * world)) ** 2
        order = gathered_row_order(S_len, world)
        assert sorted(order.tolist()) == list(range(S_len))
        # the row map the device reads the all-gather through (zigzag_tile,
        # gemm.cuh, per 128-row tile): prompt row t of chunk j = t // c sits at
        # gathered row 2j c + t % c (j < world) or (2 (2 world - 1 - j) + 1) c + t % c
        c = S_len // (2 * world)
        src = [(2 * (t // c) if t // c < world else 2 * (2 * world - 1 - t // c) + 1) * c + t % c
               for t in range(S_len)]
        assert (order[src] == np.arange(S_len)).all()
    with pytest.raises(ValueError):
        zigzag_chunks(100, 3)


# A small attention shape of the reference's own probes (H, NH, DN, DR, DV, R, eps, theta).
_CP_SHAPE = (64, 4, 8, 8, 8, 32, 1e-6, 10000.0)


def _cp_rank_main(rank, world, port, seq_len, result_q):
    """One rank of the context-parallel prefill protocol on CPU: append the
    rank's rows (the oracle's restatement of the reference's per-token append),
    all-gather them over gloo in rank order, place them by the gathered row
    order, then compute the rank's queries (the reference's streaming prefill
    attends row t over rows [0, t], which is the oracle's decode at t)."""
    import sys
    import pathlib
    root = pathlib.Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    import kvl_pkg
    kvl_pkg.load()
    import torch
    import torch.distributed as dist
    import kvl_b200.kvl_mla as K
    import kvl_b200.synth as S
    from kvl_b200.parallel import gathered_row_order, rank_rows
    from oracle.oracle import Oracle, cfg_of
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H, NH, DN, DR, DV, R, eps, theta = _CP_SHAPE
        cfg = cfg_of(*_CP_SHAPE)
        w = K.random_weights(K.make_config(*_CP_SHAPE), 61, 0.05)
        x = S.normal(61, S.S_X, seq_len * H, 1.0).reshape(seq_len, H)
        orc = Oracle()
        mine = [int(t) for t in rank_rows(seq_len, world, rank)]
        send = np.zeros((len(mine), R + DR), np.float32)
        for i, t in enumerate(mine):
            lat, rp = orc.append_f32(x[t], t, cfg, w.arrays[1], w.arrays[2])
            send[i, :R], send[i, R:] = lat, rp
        recv = [torch.zeros(send.shape) for _ in range(world)]
        dist.all_gather(recv, torch.from_numpy(send))
        rows = np.concatenate([t.numpy() for t in recv])
        pool = np.zeros_like(rows)
        pool[gathered_row_order(seq_len, world)] = rows
        latent = np.ascontiguousarray(pool[:, :R])
        rope = np.ascontiguousarray(pool[:, R:])
        out = {t: orc.decode_f32(x[t], t, cfg, w.arrays, latent, rope) for t in mine}
        result_q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_prefill_over_gloo(ref, world):
    """Every rank's rows of the zigzag context-parallel prefill equal the
    reference's own streaming prefill (src/mla_prefill_streaming.c:78-206) of
    the whole prompt, within the reference's decode-vs-prefill gate (2e-5)."""
    import multiprocessing as mp

    import kvl_pkg
    kvl_pkg.load()
    import kvl_b200.kvl_mla as K
    import kvl_b200.synth as S
    from oracle.oracle import cfg_of
    seq_len = 48
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cp_rank_main, args=(r, world, port, seq_len, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    H = _CP_SHAPE[0]
    w = K.random_weights(K.make_config(*_CP_SHAPE), 61, 0.05)
    x = S.normal(61, S.S_X, seq_len * H, 1.0).reshape(seq_len, H)
    want = ref.prefill(x, cfg_of(*_CP_SHAPE), w.arrays)
    seen = set()
    for rank, out in res:
        for t, o in out.items():
            assert t not in seen
            seen.add(t)
            assert np.max(np.abs(o - want[t])) < 2e-5, (rank, t)
    assert seen == set(range(seq_len))
