"""CPU, 2 ranks over gloo: the N-split host logic.  Each rank computes only its output-column
shard (with the CPU oracle standing in for the GPU kernel) and the shards are all-gathered; the
result must equal the unsplit product bit for bit, as every column is computed the same way."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from invision_b200.nsplit import gather_columns, shard_bounds


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, K, N, silu, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from oracle import oracle as O

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(42)
        x = rng.standard_normal((M, K), dtype=np.float32)
        w = O.f32_to_bf16_rne((0.02 * rng.standard_normal((N, K))).astype(np.float32))
        half = N // 2 if silu else N
        n0, n1, per = shard_bounds(half, world, rank, 128)
        if silu:
            ws = np.concatenate([w[n0:n1], w[half + n0:half + n1]])
            g = O.linear_bf16(x, ws)
            h = n1 - n0
            ys = O.silu_mul(np.ascontiguousarray(g[:, :h]), np.ascontiguousarray(g[:, h:]))
        else:
            ys = O.linear_bf16(x, np.ascontiguousarray(w[n0:n1]))
        pad = np.zeros((M, per), np.float32)
        pad[:, : n1 - n0] = ys
        full = gather_columns(torch.from_numpy(pad), half).numpy()
        if rank == 0:
            ref = O.linear_bf16(x, w)
            if silu:
                ref = O.silu_mul(np.ascontiguousarray(ref[:, :half]), np.ascontiguousarray(ref[:, half:]))
            q.put(bool(np.array_equal(full, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M,K,N,silu", [(37, 64, 520, False), (9, 128, 2 * 300, True)])
def test_nsplit_two_ranks_bit_exact(M, K, N, silu):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, M, K, N, silu, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) is True


def test_shard_bounds_cover_exactly():
    for n in (1, 127, 128, 3072, 9216, 18432, 1000):
        for world in (1, 2, 3, 4, 8):
            cols = []
            pers = set()
            for r in range(world):
                n0, n1, per = shard_bounds(n, world, r, 128)
                assert per % 128 == 0 and n1 - n0 <= per
                cols.extend(range(n0, n1))
                pers.add(per)
            assert cols == list(range(n)) and len(pers) == 1


def _keep_worker(rank, world, port, M, K, segments, q):
    """Head-aligned shards kept on their ranks (ENVG_KEEP_SHARDED): each rank computes only its
    rows' columns, and a per-head consumer on each rank needs nothing from the other ranks."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from oracle import oracle as O
    from invision_b200.nsplit import segment_rows

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)
        x = rng.standard_normal((M, K), dtype=np.float32)
        N = sum(segments)
        w = O.f32_to_bf16_rne((0.02 * rng.standard_normal((N, K))).astype(np.float32))
        rows = segment_rows(segments, world, rank, 128)
        local = O.linear_bf16(x, np.ascontiguousarray(w[rows]))  # this rank's kept shard
        full = O.linear_bf16(x, w)
        ok = bool(np.array_equal(local, full[:, rows]))
        # Q, K, V (the first three blocks) in whole 128-wide heads, the same heads of each
        q_rows = rows[(rows >= 0) & (rows < segments[0])]
        k_rows = rows[(rows >= segments[0]) & (rows < 2 * segments[0])] - segments[0]
        ok = ok and np.array_equal(q_rows, k_rows) and len(q_rows) % 128 == 0 and q_rows[0] % 128 == 0
        # every row is held by exactly one rank (gathered here only to check the cover)
        allrows = [torch.zeros(0, dtype=torch.int64) for _ in range(world)]
        dist.all_gather_object(allrows, rows.tolist())
        flat = sorted(r for part in allrows for r in part)
        ok = ok and flat == list(range(N))
        q.put(ok)
    finally:
        dist.destroy_process_group()


def test_head_aligned_kept_shards_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    segments = (512, 512, 512, 768, 768)  # Q, K, V (4 heads of 128), gate, up
    procs = [ctx.Process(target=_keep_worker, args=(r, 2, port, 24, 128, segments, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    assert q.get(timeout=5) is True and q.get(timeout=5) is True
