"""Failure cases of the row-sharded table on CPU ranks (gloo), made on the host, no GPU involved:

  * a non-finite output gradient on one rank makes the clip norm non-finite on every rank, so all ranks take the
    reference's skip decision together (smlm/train.py:686-704: skip the step, reset the row stores);
  * a rank that leaves between steps (exits without a word) or raises inside the exchange makes the other ranks'
    next sharded call end with an error within the process group's timeout instead of waiting for good.

The owner-side compute is the torch stand-in of test_sharded_host (the CUDA kernels are covered by the GPU tests).
"""
import datetime
import math
import os
import time

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from smlm_b200.sharded import RowShard, sharded_embedding_bag, sharded_sq_norm
from test_sharded_host import PlainStore, TorchShardOps, batches, free_port

R, D, N, KK = 64, 8, 16, 4
PG_TIMEOUT_S = 5


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))


def _step(rank, world, ops, grad_fault=None):
    """One sharded forward + backward; returns the global squared norm of the row gradients."""
    V, idx, w, g = batches(world, R, D, N, KK)
    shard = RowShard(R, world, rank)
    table = shard.take(V).clone().requires_grad_()
    store = PlainStore(shard.count, D)
    out = sharded_embedding_bag(idx[rank], w[rank].clone().requires_grad_(), table, shard, None, ops=ops,
                                store=store)
    grad = g[rank].clone()
    if grad_fault is not None:
        grad[3, 5] = grad_fault
    out.backward(grad)
    return sharded_sq_norm(store._acc.square().sum(), None, world)


def nan_worker(rank, world, port, fault_rank, value, q):
    _init(rank, world, port)
    try:
        sq = _step(rank, world, TorchShardOps(), grad_fault=value if rank == fault_rank else None)
        q.put((rank, "norm", float(sq)))
        # the next step on clean gradients is finite again on every rank (the store was dropped, as on a skip)
        q.put((rank, "next", float(_step(rank, world, TorchShardOps()))))
    except Exception as e:
        q.put((rank, "error", f"{type(e).__name__}: {e}"))
    finally:
        dist.destroy_process_group()


class RaisingOps(TorchShardOps):
    """Owner compute that fails on one rank after the lookups were exchanged (the others then wait for its
    partial bags)."""

    def __init__(self, fail):
        self.fail = fail

    def bag_forward(self, idx, w, table, base):
        if self.fail:
            raise RuntimeError("injected owner failure")
        return super().bag_forward(idx, w, table, base)


def leave_worker(rank, world, port, leaver, how, q):
    _init(rank, world, port)
    if rank == leaver:
        _step(rank, world, TorchShardOps())          # one complete step together, then leave between steps
        if how == "raise":
            try:
                _step(rank, world, RaisingOps(fail=True))
            except RuntimeError as e:
                q.put((rank, "raised", str(e)))
        q.close()
        q.join_thread()                              # flush the queue before the hard exit
        os._exit(0 if how == "exit" else 1)          # no goodbye: the others find out in their next collective
    try:
        _step(rank, world, TorchShardOps())
        t0 = time.monotonic()
        try:
            _step(rank, world, TorchShardOps())
            q.put((rank, "no error", time.monotonic() - t0))
        except Exception as e:                       # gloo: connection closed by the peer, or the timeout
            q.put((rank, "error", time.monotonic() - t0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(target, world, args, limit_s=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.monotonic() + limit_s
    for p in procs:
        p.join(max(0.0, deadline - time.monotonic()))
    hung = [p.pid for p in procs if p.is_alive()]
    for p in procs:
        if p.is_alive():
            p.kill()                                 # our own child, by its exact pid
            p.join()
    while not q.empty():
        results.append(q.get())
    assert not hung, f"ranks still running after {limit_s} s: {hung}"
    return results


@pytest.mark.parametrize("world,fault_rank,value", [(2, 1, float("nan")), (3, 0, float("inf")),
                                                    (3, 2, float("nan"))])
def test_nonfinite_gradient_seen_by_every_rank(world, fault_rank, value):
    res = _run(nan_worker, world, (fault_rank, value))
    errors = [r for r in res if r[1] == "error"]
    assert not errors, errors
    norms = {r[0]: r[2] for r in res if r[1] == "norm"}
    nxt = {r[0]: r[2] for r in res if r[1] == "next"}
    assert sorted(norms) == list(range(world)) and sorted(nxt) == list(range(world))
    assert all(not math.isfinite(v) for v in norms.values()), norms      # every rank skips the step
    assert all(math.isfinite(v) for v in nxt.values()), nxt
    assert len(set(nxt.values())) == 1                                   # and agrees on the next norm


@pytest.mark.parametrize("world,leaver,how", [(2, 1, "exit"), (3, 0, "exit"), (2, 0, "raise"), (3, 2, "raise")])
def test_lost_rank_ends_the_others_next_step_with_an_error(world, leaver, how):
    res = _run(leave_worker, world, (leaver, how))
    others = {r[0]: (r[1], r[2]) for r in res if r[0] != leaver}
    assert sorted(others) == [r for r in range(world) if r != leaver], res
    for rank, (what, elapsed) in others.items():
        assert what == "error", f"rank {rank}: {what}"
        assert elapsed < PG_TIMEOUT_S + 30, f"rank {rank} took {elapsed:.1f} s to notice"
    if how == "raise":
        assert any(r[0] == leaver and r[1] == "raised" for r in res), res
