"""Host logic of the data-parallel runtime (src/training/distributed.jl,
src/data/provider.jl:27-42) as gloo ranks on the CPU: world size 2, real
processes, no GPU."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    from reels_b200 import distributed as rd
    try:
        rt = rd.init_distributed(backend="gloo", timeout_seconds=60)
        out = {}
        # allreduce_mean of rank + 1 is 1.5 (test/gpu/distributed_worker.jl:17-22)
        t = torch.tensor([float(rank + 1)])
        rd.allreduce_mean(rt, t)
        out["mean"] = float(t.item())
        # grouped gradient all-reduce: sum then * 1/world
        grads = [torch.full((3, 2), float(rank + 1)), torch.arange(5, dtype=torch.float32) * (rank + 1)]
        rd.allreduce_gradients(rt, grads)
        out["g0"] = grads[0].tolist()
        out["g1"] = grads[1].tolist()
        # the per-layer reducer used by bench.py (CPU tensors: synchronous)
        red = rd.OverlappedGradReducer(rt, torch.device("cpu"))
        flat = torch.full((7,), float(10 * (rank + 1)))
        red.layer_done(flat)
        red.finish()
        out["flat"] = flat.tolist()
        # buckets: adjacent views of one buffer in backward order reduce as
        # one span; a view of another buffer reduces on its own
        buf = torch.arange(12, dtype=torch.float32) * (rank + 1)
        other = torch.full((3,), float(rank + 1))
        red = rd.OverlappedGradReducer(rt, torch.device("cpu"), bucket_bytes=32)
        red.layer_done(buf[8:12])
        red.layer_done(buf[4:8])        # 32 bytes: one collective over buf[4:12]
        red.layer_done(buf[0:4])
        red.layer_done(other)           # left for finish(): not adjacent, two collectives
        red.finish()
        out["bucket_buf"] = buf.tolist()
        out["bucket_other"] = other.tolist()
        out["bucket_collectives"] = red.collectives
        out["scalar"] = rd.distributed_mean_scalar(rt, 2.0 * (rank + 1))
        # every rank draws the same permutation and takes a disjoint shard
        out["shard"] = rd.distributed_sample_indices(np.random.default_rng(7), 20, 4, rank, world).tolist()
        rd.distributed_barrier(rt)
        rd.close_distributed(rt)
        q.put((rank, out))
    except Exception as e:  # surfaced to the parent
        q.put((rank, repr(e)))


def test_two_rank_gloo_runtime():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r], dict), res[r]
    for r in range(2):
        assert res[r]["mean"] == 1.5
        assert res[r]["g0"] == [[1.5, 1.5]] * 3
        assert res[r]["g1"] == [0.0, 1.5, 3.0, 4.5, 6.0]
        assert res[r]["flat"] == [15.0] * 7
        assert res[r]["bucket_buf"] == [1.5 * i for i in range(12)]
        assert res[r]["bucket_other"] == [1.5] * 3
        assert res[r]["bucket_collectives"] == 3
        assert res[r]["scalar"] == 3.0
    a, b = set(res[0]["shard"]), set(res[1]["shard"])
    assert len(a) == 4 and len(b) == 4 and not (a & b)


def test_single_process_runtime_is_identity():
    from reels_b200 import distributed as rd
    rt = rd.init_distributed(enabled=False)
    g = [torch.ones(3)]
    assert rd.allreduce_gradients(rt, g)[0].tolist() == [1.0, 1.0, 1.0]
    assert rd.distributed_mean_scalar(rt, 2.5) == 2.5
    red = rd.OverlappedGradReducer(rt, None)
    red.layer_done(g[0])
    red.finish()
    assert g[0].tolist() == [1.0, 1.0, 1.0]


@pytest.mark.parametrize("args,match", [
    (dict(count=0, batch_size=1, rank=0, world_size=1), "count"),
    (dict(count=5, batch_size=3, rank=0, world_size=2), "requires 6"),
    (dict(count=5, batch_size=1, rank=2, world_size=2), "rank"),
])
def test_sample_indices_errors(args, match):
    from reels_b200 import distributed as rd
    with pytest.raises(ValueError, match=match):
        rd.distributed_sample_indices(np.random.default_rng(0), **args)


def test_init_rejects_bad_world():
    from reels_b200 import distributed as rd
    with pytest.raises(ValueError):
        rd.init_distributed(backend="gloo", world_size=1, rank=0)
    with pytest.raises(ValueError):
        rd.init_distributed(backend="mpi", world_size=2, rank=0)
    with pytest.raises(ValueError):
        rd.init_distributed(backend="gloo", world_size=2, rank=3)


def _failing_worker(rank, world, port, q):
    """Rank 1 leaves before the gradient exchange (it exits between steps,
    with nothing in flight); rank 0 must see an error from its next
    collective within the process group's timeout instead of waiting."""
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    import time
    from reels_b200 import distributed as rd
    rt = rd.init_distributed(backend="gloo", timeout_seconds=5)
    rd.distributed_barrier(rt)  # both ranks are up
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the message is sent before the process goes
        os._exit(0)  # a rank that dies between steps
    t0 = time.time()
    try:
        rd.allreduce_gradients(rt, [torch.ones(4)])
        q.put((rank, "no error"))
    except Exception as e:  # the failure, surfaced on the host
        q.put((rank, ("error", type(e).__name__, time.time() - t0)))


def test_peer_failure_surfaces_as_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=90) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()  # this test's own child, by handle
    assert res[1] == "left"
    assert isinstance(res[0], tuple) and res[0][0] == "error", res[0]
    assert res[0][2] < 60  # bounded by the process-group timeout, not a hang


def test_closed_runtime_refuses_collectives():
    from reels_b200 import distributed as rd
    rt = rd.DistributedRuntime(rank=0, world_size=2, local_rank=0, backend="gloo")
    rt.closed = True
    with pytest.raises(ValueError, match="closed"):
        rd.allreduce_gradients(rt, [torch.ones(2)])
    with pytest.raises(ValueError, match="closed"):
        rd.allreduce_mean(rt, torch.ones(2))
