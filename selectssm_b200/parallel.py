"""Multi-GPU partitioning of the scan: one process per GPU over torch.distributed.

The reference has no multi-device code; the partition follows from the math of
the recurrence (each (batch row, channel) is an independent scan; B and C are
shared by all channels of a batch row):

* Batch sharding (``shard_batch``): every rank scans its own batch rows with no
  communication in the forward.  The backward produces per-rank partial sums of
  the parameter gradients (A / A_log, D, dt bias, and the projections around the
  scan); ``allreduce_grads`` sums them with ONE all-reduce of a flattened buffer.
* Channel (d_inner) sharding (``shard_channels`` + ``replicated_bc``): every rank
  scans a contiguous slice of channels with B and C replicated.  dA, dD and the
  dt-bias gradient are per channel and stay local, but dB and dC are sums over
  all channels (src/selectssm/ssmrecscan.py:158-159), so their gradient is
  all-reduced in the backward -- ``replicated_bc`` inserts that reduction.
  ``MulticastBCSum`` fuses it into the backward kernel instead: partial sums go
  to every rank's copy through NVLink multicast (``multimem.red``).

Collectives use whatever backend the default process group has (NCCL over
NVLink on the B200 box; gloo in the CPU tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def world():
    """(rank, world_size) of the default group, or (0, 1) when not initialised."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def shard_range(n: int, rank: int, world_size: int):
    """Contiguous [start, stop) of n items owned by rank (sizes differ by at most 1)."""
    base, extra = divmod(n, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_batch(x: torch.Tensor, rank: int = None, world_size: int = None) -> torch.Tensor:
    """This rank's batch rows of a (B, ...) tensor."""
    r, w = world()
    rank = r if rank is None else rank
    world_size = w if world_size is None else world_size
    s, e = shard_range(x.shape[0], rank, world_size)
    return x[s:e]


def shard_channels(x: torch.Tensor, rank: int = None, world_size: int = None, dim: int = -1,
                   multiple: int = 8) -> torch.Tensor:
    """This rank's channel slice along ``dim``; slices are kept at multiples of
    ``multiple`` channels (the kernels need 16-byte aligned channel rows)."""
    r, w = world()
    rank = r if rank is None else rank
    world_size = w if world_size is None else world_size
    n = x.shape[dim]
    if n % multiple:
        raise ValueError(f"channel count {n} is not a multiple of {multiple}")
    s, e = shard_range(n // multiple, rank, world_size)
    return x.narrow(dim, s * multiple, (e - s) * multiple)


class _SumGradsAcrossRanks(torch.autograd.Function):
    """Identity forward on several tensors; the backward sums their incoming
    gradients over ranks with one all-reduce of a flattened buffer."""

    @staticmethod
    def forward(ctx, group, *xs):
        ctx.group = group
        return tuple(x.view_as(x) for x in xs)

    @staticmethod
    def backward(ctx, *gs):
        if not dist.is_initialized():
            return (None,) + gs
        flat = torch.cat([g.reshape(-1) for g in gs])
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=ctx.group)
        out, off = [], 0
        for g in gs:
            out.append(flat[off:off + g.numel()].view_as(g))
            off += g.numel()
        return (None,) + tuple(out)


class MulticastBCSum:
    """dB / dC of a d_inner-sharded scan, summed over ranks inside the backward
    kernel (``ssm_bwd_bc_multicast``) instead of by an all-reduce after it.

    A float32 buffer of 2 x (batch, seqlen, 16) is allocated in symmetric
    memory and bound to an NVLink multicast object; the kernel adds each
    tile's partial sums with ``multimem.red``, which the NVSwitch applies to
    every rank's copy.  Each backward: zero the local copy, a stream-ordered
    barrier (a one-element NCCL all-reduce), the kernel, a second barrier, then
    read the local copy.  ``available`` is False where the GPUs have no
    multicast support (then use ``replicated_bc``).  Collective: every rank of
    ``group`` constructs it with the same shape, and every rank's backward
    must run it (the barriers pair up across ranks).
    """

    def __init__(self, batch: int, seqlen: int, group=None, device=None):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.shape = (batch, seqlen, 16)
        n = batch * seqlen * 16
        self.buf = symm_mem.empty(2 * n, dtype=torch.float32, device=device)
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        self.mc = int(self.handle.multicast_ptr)
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.buf.device)

    @property
    def available(self) -> bool:
        return self.mc != 0

    def _barrier(self):
        # synchronous NCCL collective: the current stream waits for it, and it
        # completes only after every rank's stream reached it
        dist.all_reduce(self._flag, group=self.group)

    def begin(self, batch: int, seqlen: int) -> int:
        """Zero this rank's copy, wait for every rank to do so, and return the
        multicast address for the kernel."""
        if (batch, seqlen, 16) != self.shape:
            raise ValueError(f"MulticastBCSum was made for {self.shape[:2]}, the scan has {(batch, seqlen)}")
        if not self.available:
            raise RuntimeError("no NVLink multicast on this group; use parallel.replicated_bc")
        self.buf.zero_()
        self._barrier()
        return self.mc

    def end(self, dtype):
        """Wait for every rank's kernel; return (dB, dC) totals in ``dtype``."""
        self._barrier()
        n = self.buf.numel() // 2
        return (self.buf[:n].view(self.shape).to(dtype, copy=True),
                self.buf[n:].view(self.shape).to(dtype, copy=True))


def replicated_bc(Bm: torch.Tensor, Cm: torch.Tensor, group=None):
    """Mark B and C as replicated across a channel-sharded group: the gradients
    each rank computes from its channels are summed over ranks (one all-reduce
    for both)."""
    return _SumGradsAcrossRanks.apply(group, Bm, Cm)


class _PendingReduce:
    """An all-reduce in flight; wait() makes the current stream wait for it and
    copies the reduced values into the gradient tensors captured at the call
    (the parameters' .grad at that time)."""

    def __init__(self, work, flat, grads, scale):
        self.work, self.flat, self.grads, self.scale = work, flat, grads, scale

    def wait(self):
        if self.work is not None:
            self.work.wait()
        if self.scale is not None:
            self.flat /= self.scale
        off = 0
        for g in self.grads:
            n = g.numel()
            g.copy_(self.flat[off:off + n].view_as(g))
            off += n


def allreduce_grads(params, group=None, average: bool = False, async_op: bool = False):
    """Sum (or average) the .grad of ``params`` over ranks with a single
    all-reduce of one flattened buffer (batch sharding).  With async_op the
    reduction overlaps whatever the caller launches next; the returned handle's
    wait() finishes it (stream-ordered) and writes the results back."""
    ps = [p for p in params if p.grad is not None]
    if not ps or not dist.is_initialized():
        return None
    flat = torch.cat([p.grad.reshape(-1) for p in ps])
    work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
    pending = _PendingReduce(work if async_op else None, flat, [p.grad for p in ps],
                             dist.get_world_size(group) if average else None)
    if async_op:
        return pending
    pending.wait()
    return None
