"""Data-parallel runtime for the LoRA linears: one process per GPU, NCCL
over NVLink through torch.distributed.

Mirrors src/training/distributed.jl:

==========================  =========================================================
reference                   here
==========================  =========================================================
SingleProcessRuntime        :class:`SingleProcessRuntime` (distributed.jl:3)
init_distributed            :func:`init_distributed` (distributed.jl:148-189)
allreduce_mean!             :func:`allreduce_mean` (distributed.jl:214-219)
allreduce_gradients!        :func:`allreduce_gradients` (distributed.jl:224-241)
distributed_mean_scalar     :func:`distributed_mean_scalar` (distributed.jl:245-251)
distributed_barrier!        :func:`distributed_barrier` (distributed.jl:254-259)
close_distributed!          :func:`close_distributed` (distributed.jl:262-272)
distributed_sample_indices  :func:`distributed_sample_indices` (data/provider.jl:27-42)
==========================  =========================================================

The reference all-reduces every gradient after the whole backward, then
synchronises the device.  :class:`OverlappedGradReducer` instead launches the
fp32 sum all-reduces on a separate stream as soon as a layer's dA/dB (or a
bucket of layers' gradients) are written, so the exchange overlaps the
backward of earlier layers; the 1/world scale follows the sum, as in the
reference.  Only the adapter
gradients cross NVLink; the int8 weights are replicated and frozen.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta
from typing import List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist


@dataclass
class SingleProcessRuntime:
    rank: int = 0
    world_size: int = 1

    @property
    def is_main_process(self) -> bool:
        return True


@dataclass
class DistributedRuntime:
    rank: int
    world_size: int
    local_rank: int
    backend: str
    closed: bool = False

    @property
    def is_main_process(self) -> bool:
        return self.rank == 0


def _env_int(name: str, fallback: int) -> int:
    v = os.environ.get(name, "")
    return int(v) if v else int(fallback)


def init_distributed(enabled: bool = True, backend: str = "nccl", world_size: int = -1, rank: int = -1,
                     local_rank: int = -1, timeout_seconds: float = 300.0):
    """init_distributed (distributed.jl:148-189): WORLD_SIZE / RANK /
    LOCAL_RANK / MASTER_ADDR / MASTER_PORT from the environment.  NCCL is the
    data-path backend; "gloo" is accepted for CPU tests of the host logic."""
    if not enabled:
        return SingleProcessRuntime()
    if backend not in ("nccl", "gloo"):
        raise ValueError("only the NCCL distributed backend is supported (gloo for CPU tests)")
    world_size = world_size if world_size > 0 else _env_int("WORLD_SIZE", 1)
    rank = rank if rank >= 0 else _env_int("RANK", 0)
    local_rank = local_rank if local_rank >= 0 else _env_int("LOCAL_RANK", rank)
    if world_size <= 1:
        raise ValueError("distributed world size must be greater than one")
    if not (0 <= rank < world_size):
        raise ValueError(f"distributed rank {rank} is outside world size {world_size}")
    if local_rank < 0:
        raise ValueError("distributed local rank must be nonnegative")
    kw = {}
    if backend == "nccl":
        if not torch.cuda.is_available():
            raise RuntimeError("NCCL distributed training requires functional CUDA")
        torch.cuda.set_device(local_rank)
        kw["device_id"] = torch.device("cuda", local_rank)
    if not dist.is_initialized():
        dist.init_process_group(backend=backend, rank=rank, world_size=world_size,
                                timeout=timedelta(seconds=timeout_seconds), **kw)
    return DistributedRuntime(rank, world_size, local_rank, backend)


def _check_open(rt):
    if getattr(rt, "closed", False):
        raise ValueError("distributed runtime is closed")


def allreduce_mean(rt, array: torch.Tensor) -> torch.Tensor:
    """allreduce_mean! (distributed.jl:214-219): in-place sum, then *1/world."""
    if isinstance(rt, SingleProcessRuntime):
        return array
    _check_open(rt)
    dist.all_reduce(array, op=dist.ReduceOp.SUM)
    array.mul_(np.float32(1.0 / rt.world_size).item())
    return array


def allreduce_gradients(rt, gradients: Sequence[torch.Tensor]):
    """allreduce_gradients! (distributed.jl:224-241): sum every gradient
    (one grouped launch), then scale by 1/world."""
    if isinstance(rt, SingleProcessRuntime):
        return gradients
    _check_open(rt)
    if rt.backend == "nccl" and not all(g.is_cuda for g in gradients):
        raise ValueError("NCCL gradients must all be CUDA arrays")
    works = [dist.all_reduce(g, op=dist.ReduceOp.SUM, async_op=True) for g in gradients]
    for w in works:
        w.wait()
    scale = np.float32(1.0 / rt.world_size).item()
    for g in gradients:
        g.mul_(scale)
    return gradients


def distributed_mean_scalar(rt, value: float, device=None) -> float:
    if isinstance(rt, SingleProcessRuntime):
        return float(np.float32(value))
    dev = device if device is not None else (torch.device("cuda", rt.local_rank) if rt.backend == "nccl"
                                             else torch.device("cpu"))
    buf = torch.full((1,), float(value), dtype=torch.float32, device=dev)
    allreduce_mean(rt, buf)
    return float(buf.item())


def distributed_barrier(rt) -> None:
    """distributed_barrier! (distributed.jl:254-259): a one-float all-reduce."""
    if isinstance(rt, SingleProcessRuntime):
        return
    _check_open(rt)
    dev = torch.device("cuda", rt.local_rank) if rt.backend == "nccl" else torch.device("cpu")
    buf = torch.zeros((1,), dtype=torch.float32, device=dev)
    dist.all_reduce(buf)
    if rt.backend == "nccl":
        torch.cuda.synchronize(dev)


def close_distributed(rt) -> None:
    if isinstance(rt, SingleProcessRuntime) or rt.closed:
        return
    dist.destroy_process_group()
    rt.closed = True


def distributed_sample_indices(rng: np.random.Generator, count: int, batch_size: int, rank: int,
                               world_size: int) -> np.ndarray:
    """provider.jl:27-42: one global permutation, this rank's disjoint
    contiguous shard of ``batch_size`` entries (0-based here)."""
    if count <= 0:
        raise ValueError("sample count must be positive")
    if batch_size <= 0:
        raise ValueError("batch size must be positive")
    if world_size <= 0:
        raise ValueError("world size must be positive")
    if not (0 <= rank < world_size):
        raise ValueError("rank must be in 0:world_size-1")
    required = batch_size * world_size
    if required > count:
        raise ValueError(f"distributed batch requires {required} entries, found {count}")
    perm = rng.permutation(count)
    off = rank * batch_size
    return perm[off:off + batch_size]


class OverlappedGradReducer:
    """Per-layer (or bucketed) fp32 all-reduce of LoRA gradients on a side
    stream.

    Call :meth:`layer_done` with a layer's flat gradient buffer right after
    its backward kernels were enqueued on the compute stream; the side stream
    waits for them (an event), sums the buffer across ranks and scales it by
    1/world.  With ``bucket_bytes > 0`` the buffers are collected until a
    bucket holds that many bytes and then reduced together: one collective
    over their span when they are adjacent views of one buffer (as when the
    caller lays the gradients out in backward order), else one per buffer.
    :meth:`finish` reduces what is left and makes the compute stream wait for
    every reduction.  With the gloo backend (CPU tensors) the reductions run
    synchronously, which is what the host-logic tests exercise.
    """

    def __init__(self, rt, device: Optional[torch.device] = None, bucket_bytes: int = 0):
        self.rt = rt
        self.world = 1 if isinstance(rt, SingleProcessRuntime) else rt.world_size
        self.cuda = device is not None and device.type == "cuda" and self.world > 1
        self.stream = torch.cuda.Stream(device=device) if self.cuda else None
        self.pending: List = []
        self.scale = np.float32(1.0 / self.world).item()
        self.bucket_bytes = int(bucket_bytes)
        self.bucket: List[torch.Tensor] = []
        self.bucket_fill = 0
        self.collectives = 0   # all-reduce launches so far (for tests and reports)

    @staticmethod
    def _span(tensors: Sequence[torch.Tensor]) -> Optional[torch.Tensor]:
        """One 1-D view covering ``tensors`` when they are contiguous 1-D views
        of one storage that together tile an interval; else None."""
        t0 = tensors[0]
        if any(t.dim() != 1 or not t.is_contiguous() or t.dtype != t0.dtype for t in tensors):
            return None
        st = t0.untyped_storage()
        if any(t.untyped_storage().data_ptr() != st.data_ptr() for t in tensors):
            return None
        iv = sorted((t.storage_offset(), t.storage_offset() + t.numel()) for t in tensors)
        for (_, e), (b, _) in zip(iv, iv[1:]):
            if b != e:
                return None
        lo, hi = iv[0][0], iv[-1][1]
        return t0.new_empty(0).set_(st, lo, (hi - lo,), (1,))

    def _reduce(self, tensors: Sequence[torch.Tensor]) -> None:
        span = self._span(tensors) if len(tensors) > 1 else tensors[0]
        targets = [span] if span is not None else list(tensors)
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(targets[0].device))
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ev)
                for t in targets:
                    dist.all_reduce(t, op=dist.ReduceOp.SUM)
                    t.mul_(self.scale)
            for t in targets:
                t.record_stream(self.stream)
                self.pending.append(t)
        else:
            for t in targets:
                dist.all_reduce(t, op=dist.ReduceOp.SUM)
                t.mul_(self.scale)
        self.collectives += len(targets)

    def layer_done(self, flat_grad: torch.Tensor) -> None:
        if self.world == 1:
            return
        _check_open(self.rt)
        if self.bucket_bytes <= 0:
            self._reduce([flat_grad])
            return
        self.bucket.append(flat_grad)
        self.bucket_fill += flat_grad.numel() * flat_grad.element_size()
        if self.bucket_fill >= self.bucket_bytes:
            self._flush()

    def _flush(self) -> None:
        if self.bucket:
            self._reduce(self.bucket)
        self.bucket, self.bucket_fill = [], 0

    def finish(self) -> None:
        if self.world > 1:
            _check_open(self.rt)
            self._flush()
        if self.cuda and self.pending:
            torch.cuda.current_stream(self.pending[0].device).wait_stream(self.stream)
        self.pending.clear()
