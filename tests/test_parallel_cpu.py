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
