"""Batch sharding over several GPUs.

Every matrix of a batch is independent, so the batch axis -- the reference's Pallas grid
axis ``grid=(B, ...)`` (src/fermix/_lu.py:459) -- is the one to shard: each GPU factorises
a contiguous slice of the batch with its own launches, gradients stay with the slice that
produced them, and only the (sign, logabs) pairs (B (k + 1) scalars) are gathered. No
other collective runs on the data path.

Two ways to run it:

* one process per GPU (torchrun / ``torch.distributed``): each rank calls
  :func:`dist_slog` on its local slice (``local_slice`` cuts it from a global batch) and
  gets the global (sign, logabs) back through one all-gather over the process group
  (NCCL on GPUs; the gather logic is the same over gloo on CPU tensors);
* one process driving several GPUs: :func:`multi_device_slog` splits a batch over the
  listed devices, launches each slice on that device's current stream, and copies the
  (sign, logabs) slices back to one device.
"""

import numpy as np
import torch

from . import api

OPS = {"slogdet": api.slogdet, "slogpf": api.slogpf}


def shard_bounds(batch, world, rank):
    """[start, stop) of rank's contiguous slice when `batch` items are split over `world`
    ranks as evenly as possible (the first batch % world ranks get one more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if batch < 0:
        raise ValueError("batch must be >= 0")
    q, r = divmod(int(batch), int(world))
    start = rank * q + min(rank, r)
    return start, start + q + (1 if rank < r else 0)


def shard_counts(batch, world):
    """Slice sizes of every rank under shard_bounds."""
    return [b - a for a, b in (shard_bounds(batch, world, r) for r in range(world))]


def local_slice(a, group=None):
    """This rank's slice of a global batch a (..., n, n), split along its first axis."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    a0, a1 = shard_bounds(a.shape[0], world, rank)
    return a[a0:a1]


def _as_real(t):
    return torch.view_as_real(t) if t.is_complex() else t


def all_gather_slog(sign, logabs, batch, group=None):
    """Concatenate every rank's (sign, logabs) slices, in rank order, into the global
    (batch,) arrays on every rank. The slices must follow shard_bounds(batch, world, .);
    each rank may hold a different number (zero included). One all-gather of the largest
    slice, zero-padded, with sign (as real parts) and logabs packed side by side in one
    buffer of logabs' real dtype."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    counts = shard_counts(batch, world)
    if sign.shape[0] != counts[rank] or logabs.shape[0] != counts[rank]:
        raise ValueError(f"rank {rank} holds {sign.shape[0]} results, its slice has {counts[rank]}")
    m = max(counts) if counts else 0
    ws = 2 if sign.is_complex() else 1
    sr = _as_real(sign).reshape(sign.shape[0], ws)
    pack = torch.zeros((m, ws + 1), dtype=logabs.dtype, device=logabs.device)
    pack[: sign.shape[0], :ws] = sr.to(logabs.dtype)
    pack[: sign.shape[0], ws] = logabs
    full = torch.empty((world * m, ws + 1), dtype=pack.dtype, device=pack.device)
    dist.all_gather_into_tensor(full, pack, group=group)
    if any(c != m for c in counts):
        full = torch.cat([full[r * m: r * m + c] for r, c in enumerate(counts)])
    S = full[:, :ws].contiguous()
    S = torch.view_as_complex(S) if sign.is_complex() else S.reshape(-1).to(sign.dtype)
    return S, full[:, ws].contiguous()


def dist_slog(op, a_local, batch, *, group=None, **kw):
    """(sign, logabs) of the whole sharded batch on every rank: this rank's slice a_local
    (shard_bounds of `batch` over the group, shape (b, n, n)) is factorised by `op`
    ("slogdet" or "slogpf", keyword arguments as those functions) on its own GPU, then the
    slices' results are all-gathered. Also returns the local (sign, logabs), which stay
    differentiable in a_local."""
    if op not in OPS:
        raise ValueError(f"op must be one of {sorted(OPS)}, got {op!r}")
    s, l = OPS[op](a_local, **kw)
    S, L = all_gather_slog(s.detach(), l.detach(), batch, group=group)
    return S, L, (s, l)


def multi_device_slog(op, a, devices=None, **kw):
    """(sign, logabs) of a batch a (B, n, n) split over several GPUs of this process:
    slice d of shard_bounds goes to devices[d] (default: every visible device), is
    factorised there on that device's current stream, and its (sign, logabs) are copied
    to the device of a (or devices[0] for a host tensor). The copies of a's slices are
    issued asynchronously from pinned memory when a is on the host."""
    if op not in OPS:
        raise ValueError(f"op must be one of {sorted(OPS)}, got {op!r}")
    if devices is None:
        devices = list(range(torch.cuda.device_count()))
    devices = [torch.device("cuda", d) if isinstance(d, int) else torch.device(d) for d in devices]
    if not devices:
        raise RuntimeError("no CUDA devices: fermix_b200 has no CPU fallback")
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
    if a.ndim != 3:
        raise ValueError(f"expected a (B, n, n) batch, got {tuple(a.shape)}")
    home = a.device if a.is_cuda else devices[0]
    if not a.is_cuda and not a.is_pinned():
        a = a.pin_memory()
    B = a.shape[0]
    pieces = []
    for d, dev in enumerate(devices):
        b0, b1 = shard_bounds(B, len(devices), d)
        if b1 == b0:
            continue
        with torch.cuda.device(dev):
            x = a[b0:b1].to(dev, non_blocking=True)
            s, l = OPS[op](x, **kw)
            pieces.append((s, l, dev))
    sign = torch.cat([s.to(home, non_blocking=True) for s, _, _ in pieces]) if pieces else None
    logabs = torch.cat([l.to(home, non_blocking=True) for _, l, _ in pieces]) if pieces else None
    for _, _, dev in pieces:
        torch.cuda.synchronize(dev)
    if sign is None:
        rd = torch.float32 if a.dtype in (torch.float32, torch.complex64) else torch.float64
        sign = torch.empty(0, dtype=a.dtype, device=home)
        logabs = torch.empty(0, dtype=rd, device=home)
    return sign, logabs
