"""Batch sharding logic on CPU: the partition, and the all-gather of (sign, logabs) over a
world-size-2 gloo process group, checked against the unsharded result. The per-rank
compute here is the CPU oracle (this machine has no GPU); on GPUs dist_slog runs the CUDA
library on each rank's slice and gathers with the same function."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fermix_b200 import sharded


def test_shard_bounds_partition():
    for B in (0, 1, 2, 7, 4096, 4097):
        for world in (1, 2, 3, 4, 8):
            bounds = [sharded.shard_bounds(B, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == B
            for (a0, a1), (b0, _) in zip(bounds, bounds[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in bounds]
            assert max(sizes) - min(sizes) <= 1 and sizes == sharded.shard_counts(B, world)
    with pytest.raises(ValueError):
        sharded.shard_bounds(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cases, errs):
    import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        for op, dtype, B, n in cases:
            rng = np.random.default_rng(B * 31 + n)
            A = rng.standard_normal((B, n, n))
            if np.dtype(dtype).kind == "c":
                A = A + 1j * rng.standard_normal((B, n, n))
            A = A.astype(dtype)
            if op == "slogpf":
                A = A - np.swapaxes(A, -1, -2)
            f = oracle.slogpf if op == "slogpf" else oracle.slogdet
            mine = sharded.local_slice(torch.from_numpy(A)).numpy()
            a0, a1 = sharded.shard_bounds(B, world, rank)
            assert np.array_equal(mine, A[a0:a1])
            s, l = f(mine) if len(mine) else (np.zeros(0, dtype), np.zeros(0, np.real(np.zeros(1, dtype)).dtype))
            S, L = sharded.all_gather_slog(torch.from_numpy(np.asarray(s)), torch.from_numpy(np.asarray(l)), B)
            s_all, l_all = f(A)
            assert np.array_equal(S.numpy(), s_all), (op, dtype, B)
            assert np.array_equal(L.numpy(), l_all), (op, dtype, B)
    except Exception as e:  # reported to the parent
        errs.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def test_all_gather_matches_unsharded_over_gloo():
    world = 2
    cases = [("slogdet", np.float32, 7, 12), ("slogpf", np.complex128, 4, 10), ("slogdet", np.float64, 1, 6),
             ("slogpf", np.float32, 0, 8)]
    ctx = mp.get_context("spawn")
    errs = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, cases, errs)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    msgs = []
    while not errs.empty():
        msgs.append(errs.get())
    for p in procs:
        if p.is_alive():
            p.kill()
    assert not msgs, msgs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.gpu
@pytest.mark.parametrize("op", ["slogdet", "slogpf"])
def test_multi_device_and_single_rank_dist_match_unsharded(op):
    """The GPU paths: slices on the visible devices (each device listed twice, so that a
    one-GPU box still runs two slices) and a one-rank NCCL group, against one call on the
    whole batch -- bit for bit, since every matrix is factorised by its own block."""
    import datetime

    import fermix_b200 as fx

    rng = np.random.default_rng(5)
    A = rng.standard_normal((37, 96, 96)).astype(np.float32)
    if op == "slogpf":
        A = A - np.swapaxes(A, -1, -2)
    ref = [t.cpu().numpy() for t in getattr(fx, op)(torch.from_numpy(A).cuda())]
    devs = [d for d in range(torch.cuda.device_count()) for _ in range(2)]
    s, l = sharded.multi_device_slog(op, torch.from_numpy(A), devices=devs)
    assert np.array_equal(s.cpu().numpy(), ref[0]) and np.array_equal(l.cpu().numpy(), ref[1])
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", 0))
    try:
        x = sharded.local_slice(torch.from_numpy(A).cuda())
        S, L, (s1, l1) = sharded.dist_slog(op, x, A.shape[0])
        assert np.array_equal(S.cpu().numpy(), ref[0]) and np.array_equal(L.cpu().numpy(), ref[1])
    finally:
        dist.destroy_process_group()
