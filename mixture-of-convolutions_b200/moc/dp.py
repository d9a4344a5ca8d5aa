"""Data parallelism for the MoC module: whole sequences per rank, one collective per step.

Every sequence is independent and the causal halo (kernel_size - 1 tokens) never
crosses a sequence boundary, so a rank that owns whole sequences computes its part of
the router, the convolution and every activation gradient without communication.  The
one exchange per step is the sum over ranks of the parameter gradients, conv_bases
[K, S, D] and router [K, Dz]: both are flattened into one fp32 buffer and summed by a
single all-reduce (NCCL on GPUs, gloo on CPU).  x, z, y, dx and dz never leave their GPU.

The reference trains in one process (its kernels are per-device); this module is the
scaling layer of this build, used by bench.py for the multi-GPU runs.
"""
from __future__ import annotations

import ctypes
from typing import Iterable, Sequence

import torch
import torch.distributed as dist

from . import _lib


def shard_fixed(batch: int, rank: int, world: int) -> slice:
    """The sequences [start, stop) of a fixed-length batch owned by `rank`: contiguous
    blocks, the first `batch % world` ranks holding one sequence more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if batch < 0:
        raise ValueError("batch must be non-negative")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def shard_varlen(cu_seqlens: Sequence[int] | torch.Tensor, rank: int, world: int):
    """Split a packed varlen batch into `world` contiguous runs of whole sequences,
    balanced by token count: rank r's run ends at the sequence boundary nearest to
    (r + 1) / world of the tokens.

    Returns (tok_start, tok_stop, local_cu_seqlens): the rank's slice of the packed
    token axis and its cu_seqlens rebased to start at 0 (int64, on the CPU)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    cu = torch.as_tensor(cu_seqlens).detach().to("cpu", torch.int64).reshape(-1)
    if cu.numel() < 1 or int(cu[0]) != 0 or bool((cu[1:] < cu[:-1]).any()):
        raise ValueError("cu_seqlens must start at 0 and be non-decreasing")
    n_seqs = cu.numel() - 1
    total = int(cu[-1])
    cuts = [0]
    for r in range(1, world):
        target = total * r / world
        j = int(torch.searchsorted(cu, torch.tensor(target, dtype=torch.float64).to(torch.int64)))
        j = min(max(j, 0), n_seqs)
        # the nearer of the boundaries around the target, never behind the previous cut
        if j > 0 and abs(int(cu[j - 1]) - target) <= abs(int(cu[j]) - target):
            j -= 1
        cuts.append(max(j, cuts[-1]))
    cuts.append(n_seqs)
    s0, s1 = cuts[rank], cuts[rank + 1]
    t0, t1 = int(cu[s0]), int(cu[s1])
    return t0, t1, cu[s0:s1 + 1] - t0


class GradAllReduce:
    """Sums parameter gradients over the ranks of `group` with one all-reduce of a
    persistent flat buffer, allocated once: fp32 for bf16 / fp16 / fp32 parameters
    (float64 parameters keep float64)."""

    def __init__(self, params: Iterable[torch.Tensor], group=None):
        self.params = list(params)
        if not self.params:
            raise ValueError("no parameters to reduce")
        dev = self.params[0].device
        self.sizes = [p.numel() for p in self.params]
        dtype = torch.float32
        for p in self.params:
            dtype = torch.promote_types(dtype, p.dtype)
        self.flat = torch.empty(sum(self.sizes), dtype=dtype, device=dev)
        self.group = group

    def __call__(self, grads: Sequence[torch.Tensor] | None = None) -> list[torch.Tensor]:
        """All-reduce `grads` (default: each parameter's .grad) in place; returns them."""
        grads = [p.grad for p in self.params] if grads is None else list(grads)
        if len(grads) != len(self.params) or any(g is None for g in grads):
            raise ValueError("one gradient per parameter is required")
        off = 0
        for g, n in zip(grads, self.sizes):
            self.flat[off:off + n].copy_(g.reshape(-1))
            off += n
        dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
        off = 0
        for g, n in zip(grads, self.sizes):
            g.copy_(self.flat[off:off + n].view_as(g))
            off += n
        return grads



class CommTimeout(RuntimeError):
    """A rank's all-reduce gave up waiting for its peers: that step's gradients were not
    summed.  Raised on every rank by ``NVLinkGradAllReduce.check``, after the communicator
    has been reset on every rank, so the next call pairs up again."""


def all_ranks_ok(ok: bool, group=None, device: torch.device | None = None) -> bool:
    """True on every rank when `ok` holds on every rank of `group` (one MIN all-reduce;
    every rank must call it)."""
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32)
    if dist.get_backend(group) == "nccl":
        flag = flag.to(device if device is not None else torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return int(flag.item()) == 1


class NVLinkGradAllReduce:
    """The same sum as GradAllReduce, by this library's own NVLink kernel instead of NCCL
    (``moc_comm_*`` in include/moc_b200.h): every rank's exchange buffer is opened by the
    others through CUDA IPC, and one kernel per call publishes this rank's gradients, waits
    (bounded) for the other ranks' and adds all of them in rank order, so every rank holds
    bitwise the same sum.  One process per GPU, all ranks on one node (peer access over
    NVLink / NVSwitch), at most 8 ranks, up to 4 gradient tensors.  Setup exchanges the IPC
    handles with ``all_gather_object`` over ``group``; each call is stream-ordered and can be
    captured in a CUDA graph.  Every rank must make the same calls in the same order."""

    def __init__(self, params: Iterable[torch.Tensor], group=None):
        self.params = list(params)
        if not 1 <= len(self.params) <= _lib.COMM_MAX_SEGMENTS:
            raise ValueError(f"between 1 and {_lib.COMM_MAX_SEGMENTS} parameters")
        dev = self.params[0].device
        if dev.type != "cuda":
            raise ValueError("NVLinkGradAllReduce needs CUDA parameters")
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        if world > _lib.COMM_MAX_RANKS:
            raise ValueError(f"at most {_lib.COMM_MAX_RANKS} ranks")
        self.device = dev
        self.group = group
        self._comm = None
        lib = _lib.load()
        # every step of the setup ends with an agreement over `group`, so a failure on one
        # rank raises on all of them instead of leaving the others waiting
        handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        comm = ctypes.c_void_p()
        with torch.cuda.device(dev):
            rc = lib.moc_comm_create(rank, world, sum(p.numel() for p in self.params), ctypes.byref(comm), handle)
        if rc == _lib.MOC_OK:
            self._comm = comm
        self._agree(rc == _lib.MOC_OK, "moc_comm_create", rc, group)
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        blob = ctypes.create_string_buffer(b"".join(handles), world * _lib.IPC_HANDLE_BYTES)
        with torch.cuda.device(dev):
            rc = lib.moc_comm_connect(comm, blob)
        self._agree(rc == _lib.MOC_OK, "moc_comm_connect", rc, group)
        self._self_check(group)

    def _self_check(self, group) -> None:
        """One sum of a probe buffer checked against torch.distributed's all-reduce, agreed
        over `group` (so a peer path that does not work raises on every rank)."""
        g = torch.Generator(device=self.device).manual_seed(1000 + dist.get_rank(group))
        probe = torch.randn(sum(p.numel() for p in self.params), generator=g, device=self.device)
        ref = probe.clone()
        dist.all_reduce(ref, group=group)
        segs, off = [], 0
        for p in self.params:
            segs.append(probe.narrow(0, off, p.numel()))
            off += p.numel()
        _lib.device_status(clear=True)
        self(segs)
        torch.cuda.synchronize(self.device)
        ok = _lib.device_status(clear=True) == 0 and bool(
            torch.allclose(probe, ref, rtol=1e-5, atol=1e-5 * float(ref.abs().max())))
        self._agree(ok, "the NVLink all-reduce self-check", _lib.MOC_OK, group)

    def _agree(self, ok: bool, what: str, rc: int, group) -> None:
        if all_ranks_ok(ok, group, self.device):
            return
        self.close(sync=False)
        if not ok:
            _lib.check(rc, what)
            raise RuntimeError(f"{what} failed on this rank")
        raise RuntimeError(f"{what} failed on another rank")

    def __call__(self, grads: Sequence[torch.Tensor] | None = None) -> list[torch.Tensor]:
        """All-reduce `grads` (default: each parameter's .grad) in place; returns them."""
        grads = [p.grad for p in self.params] if grads is None else list(grads)
        if len(grads) != len(self.params) or any(g is None for g in grads):
            raise ValueError("one gradient per parameter is required")
        for g, p in zip(grads, self.params):
            if not g.is_contiguous() or g.numel() != p.numel() or g.device != self.device:
                raise ValueError("gradients must be contiguous, parameter-shaped and on the parameters' device")
        n = len(grads)
        ptrs = (ctypes.c_void_p * n)(*[g.data_ptr() for g in grads])
        counts = (ctypes.c_int64 * n)(*[g.numel() for g in grads])
        dtypes = (ctypes.c_int32 * n)(*[_lib.dtype_code(g) for g in grads])
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().moc_comm_allreduce(self._comm, n, ptrs, counts, dtypes,
                                                      _lib.stream_of(self.device)), "moc_comm_allreduce")
        return grads

    def set_poll_limit(self, polls: int) -> None:
        """Polls of a peer's flag before a call gives up (0: the default, 2^22)."""
        _lib.check(_lib.load().moc_comm_set_poll_limit(self._comm, int(polls)), "moc_comm_set_poll_limit")

    def status(self, clear: bool = False) -> int:
        """MOC_STATUS_* bits this communicator's calls recorded (synchronous read)."""
        v = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().moc_comm_status(self._comm, ctypes.byref(v), int(clear)), "moc_comm_status")
        return v.value

    def _sync(self) -> None:
        torch.cuda.synchronize(self.device)

    def reset(self) -> None:
        """Zeroes this rank's flags, call counters and status (after a timeout, on every rank,
        with no call in flight anywhere)."""
        with torch.cuda.device(self.device):
            _lib.check(_lib.load().moc_comm_reset(self._comm, _lib.stream_of(self.device)), "moc_comm_reset")
        torch.cuda.synchronize(self.device)

    def check(self) -> None:
        """Step-boundary check, made by every rank: raises CommTimeout on every rank if any
        rank's call since the last check gave up waiting (its gradients were left unsummed).
        Before raising, every rank resets its communicator and the ranks meet at a barrier,
        so the next call pairs up again.  Synchronises this rank's device."""
        self._sync()
        bits = self.status(clear=True)
        if all_ranks_ok(bits == 0, self.group, self.device):
            return
        self.reset()
        dist.barrier(group=self.group)
        raise CommTimeout(
            "NVLink gradient all-reduce: a rank gave up waiting for its peers "
            f"(this rank's status {bits:#x}); the gradients of the calls since the last check are not summed"
        )

    def close(self, sync: bool = True) -> None:
        """Frees the exchange buffer (after every rank's last call has finished)."""
        if self._comm:
            if sync:
                torch.cuda.synchronize(self.device)
            with torch.cuda.device(self.device):
                rc = _lib.load().moc_comm_destroy(self._comm)
            self._comm = None
            _lib.check(rc, "moc_comm_destroy")
