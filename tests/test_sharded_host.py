"""Host logic of the row-sharded value table on CPU ranks (gloo, 2, 3 and 4 processes): row ranges, the all-gather /
all-to-all routing of lookups, partial bags and weight gradients, the owner-order sums, the sharded clip norm and
the replicated-gradient all-reduce. The owner-side compute is a plain torch stand-in here (the CUDA kernels are
covered by the GPU tests); the result of P ranks must equal one rank over the concatenated batches."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from smlm_b200.sharded import RowShard, allreduce_replicated_grads, sharded_embedding_bag, sharded_sq_norm


class TorchShardOps:
    """Owner-side compute in torch on CPU (test stand-in for the CUDA kernels)."""

    @staticmethod
    def _local(idx, table, base):
        """Local rows, other shards' lookups pointed at an appended zero row."""
        rows = table.shape[0]
        loc = idx.long() - base
        own = (loc >= 0) & (loc < rows)
        padded = torch.cat([table.detach(), torch.zeros(1, table.shape[1])])
        return torch.where(own, loc, torch.full_like(loc, rows)), own, padded

    def bag_forward(self, idx, w, table, base):
        loc, own, padded = self._local(idx, table, base)
        out = torch.zeros(idx.shape[0], table.shape[1])
        for j in range(idx.shape[1]):
            out = out + (w[:, j] * own[:, j]).unsqueeze(-1) * padded[loc[:, j]]
        return out

    def bag_backward(self, g, idx, w, table, base, store):
        loc, own, padded = self._local(idx, table, base)
        g = g.float()
        gw = torch.where(own, torch.einsum("nd,nkd->nk", g, padded[loc]), torch.zeros(()))
        if store is not None:
            n, k = idx.shape
            sel = own.reshape(-1)
            rows = loc.reshape(-1)[sel]
            contrib = (w.unsqueeze(-1) * g.unsqueeze(1)).reshape(n * k, -1)[sel]
            store._acc.index_add_(0, rows, contrib)
            store._touched[rows] = True
        return gw

    def slot_sum(self, x):
        t = x[0].clone()
        for s in range(1, x.shape[0]):
            t = t + x[s]
        return t


class PlainStore:
    def __init__(self, rows, d):
        self._acc = torch.zeros(rows, d)
        self._touched = torch.zeros(rows, dtype=torch.bool)
        self._sqnorm = torch.zeros(rows)
        self.clean = False


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def batches(world, R, D, N, Kk):
    gen = torch.Generator().manual_seed(7)
    V = torch.randn(R, D, generator=gen)
    idx = torch.randint(0, R, (world, N, Kk), generator=gen)
    idx[:, :, 0] = idx[:, :, 1]                             # repeated rows inside a token
    w = torch.softmax(torch.randn(world, N, Kk, generator=gen), -1)
    g = torch.randn(world, N, D, generator=gen)
    return V, idx, w, g


def worker(rank, world, port, R, D, N, Kk, errors):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V, idx, w, g = batches(world, R, D, N, Kk)
        shard = RowShard(R, world, rank)
        table = shard.take(V).clone().requires_grad_()
        store = PlainStore(shard.count, D)
        wr = w[rank].clone().requires_grad_()
        out = sharded_embedding_bag(idx[rank], wr, table, shard, None, ops=TorchShardOps(), store=store)
        out.backward(g[rank])
        # one rank over the concatenated batches
        ref_out = torch.einsum("nk,nkd->nd", w[rank], V[idx[rank]])
        ref_gw = torch.einsum("nd,nkd->nk", g[rank], V[idx[rank]])
        acc = torch.zeros(R, D)
        acc.index_add_(0, idx.reshape(-1), (w.unsqueeze(-1) * g.unsqueeze(2)).reshape(-1, D))
        touched = torch.zeros(R, dtype=torch.bool)
        touched[idx.reshape(-1)] = True
        torch.testing.assert_close(out, ref_out, rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(wr.grad, ref_gw, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(store._acc, shard.take(acc), rtol=1e-5, atol=1e-5)
        assert torch.equal(store._touched, shard.take(touched))
        assert table.grad is None                            # row gradients live in the store only
        # sharded clip norm: sum of the ranks' squared norms, in rank order, identical on every rank
        total = sharded_sq_norm(store._acc.square().sum(), None, world)
        torch.testing.assert_close(total, acc.square().sum(), rtol=1e-5, atol=1e-5)
        # replicated gradients are summed, sharded tables are left alone
        m = torch.nn.Linear(3, 2)
        big = torch.nn.Parameter(torch.zeros(shard.count, 2))
        big.row_shard = shard
        m.register_parameter("values", big)
        m.weight.grad = torch.full((2, 3), float(rank + 1))
        m.bias.grad = torch.full((2,), 1.0)
        big.grad = torch.full((shard.count, 2), float(rank + 1))
        allreduce_replicated_grads(m)
        assert torch.equal(m.weight.grad, torch.full((2, 3), float(world * (world + 1) // 2)))
        assert torch.equal(m.bias.grad, torch.full((2,), float(world)))
        assert torch.equal(big.grad, torch.full((shard.count, 2), float(rank + 1)))
        # no-grad forward takes the same route
        with torch.no_grad():
            out2 = sharded_embedding_bag(idx[rank], w[rank], table, shard, None, ops=TorchShardOps())
        assert torch.equal(out2, out.detach())
    except Exception as e:                                   # reported by the parent
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,R", [(2, 1000), (3, 50), (3, 4), (4, 130)])
def test_sharded_bag_equals_one_rank(world, R):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    mp.start_processes(worker, args=(world, free_port(), R, 16, 64, 8, errors), nprocs=world, join=True,
                       start_method="spawn")
    assert errors.empty()


def test_row_shard_partition():
    for rows in (0, 1, 4, 50, 1000, 16_777_216):
        for world in (1, 2, 3, 8):
            shards = [RowShard(rows, world, r) for r in range(world)]
            assert sum(s.count for s in shards) == rows
            nxt = 0
            for s in shards:
                assert s.base == min(rows, nxt) and s.count >= 0
                nxt = s.base + s.count
                for row in (s.base, s.base + s.count - 1):
                    if s.count:
                        assert s.owner(row) == s.rank
    with pytest.raises(ValueError):
        RowShard(2 ** 31, 2, 0)
    with pytest.raises(ValueError):
        RowShard(10, 2, 2)
