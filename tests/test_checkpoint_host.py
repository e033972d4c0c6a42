"""Checkpoints of a row-sharded table in the unsharded layout, on CPU ranks (gloo, 2 and 3 processes): the gathered
model and optimizer state dicts equal the one-process ones bit for bit (fp32, bf16, int8 / uint8 and int32 per-row
state; the smlm.lazy_row_adam.v1, smlm.row_wise.v1, torch and OptimizerSet layouts), the gather takes several
rounds when rows exceed its chunk, empty shards pass, and loading a full state dict gives each rank its own rows
back. A rank whose optimizer state has another structure makes every rank raise instead of waiting."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from smlm_b200.checkpoint import (gather_rows, load_unsharded_model_state, load_unsharded_optimizer_state,
                                  shard_optimizer_state, unshard_optimizer_state, unsharded_model_state,
                                  unsharded_optimizer_state)
from smlm_b200.sharded import RowShard
from smlm_b200.sparse_values import OptimizerSet


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class Layer(torch.nn.Module):
    """A value table (row-sharded when `shard` is given) beside replicated parameters and a buffer."""

    def __init__(self, full_values, shard=None, group=None):
        super().__init__()
        self.proj = torch.nn.Linear(4, 3)
        self.register_buffer("running", torch.arange(5, dtype=torch.float32))
        vals = full_values if shard is None else shard.take(full_values)
        self.values = torch.nn.Embedding(vals.shape[0], vals.shape[1])
        with torch.no_grad():
            self.values.weight.copy_(vals)
            self.proj.weight.copy_(torch.linspace(-1, 1, 12).view(3, 4))
            self.proj.bias.copy_(torch.tensor([0.5, -0.25, 2.0]))
        if shard is not None:
            self.values.weight.row_shard = shard
            self.values.weight.shard_group = group


class DictOpt:
    """An optimizer stand-in that returns / takes a given state dict in the library's table formats (the CUDA
    optimizers themselves need GPU tables)."""

    def __init__(self, params, sd):
        self.param_groups = [{"params": list(params)}]
        self.sd = sd

    def state_dict(self):
        return self.sd

    def load_state_dict(self, sd):
        self.sd = sd


def lazy_adam_state(rows, d, int8=False, bf16=False):
    """A smlm.lazy_row_adam.v1 state dict for one full table of `rows` rows (seeded, distinct per row)."""
    gen = torch.Generator().manual_seed(rows * 7 + d)
    if int8:
        st = {"step": torch.tensor(3.0),
              "exp_avg": torch.randint(-127, 128, (rows, d), generator=gen, dtype=torch.int8),
              "exp_avg_sq": torch.randint(0, 256, (rows, d), generator=gen, dtype=torch.uint8),
              "exp_avg_scale": torch.rand(rows, generator=gen),
              "exp_avg_sq_scale": torch.rand(rows, generator=gen)}
        dt = "int8"
    else:
        mdt = torch.bfloat16 if bf16 else torch.float32
        st = {"step": torch.tensor(3.0), "exp_avg": torch.randn(rows, d, generator=gen).to(mdt),
              "exp_avg_sq": torch.rand(rows, d, generator=gen).to(mdt)}
        dt = "bf16" if bf16 else "fp32"
    return {"format": "smlm.lazy_row_adam.v1", "state_dtype": dt, "shapes": [[rows, d]],
            "param_groups": [{"lr": 1e-3, "betas": (0.9, 0.98), "eps": 1e-8, "weight_decay": 0.0,
                              "name": "memory_values", "base_lr": 1e-3, "params": [0]}],
            "state": [st]}


def row_wise_state(rows):
    gen = torch.Generator().manual_seed(rows)
    return {"format": "smlm.row_wise.v1", "kind": "rowrms", "shapes": [[rows, 6]],
            "param_groups": [{"lr": 1e-2, "beta2": 0.95, "eps": 1e-8, "weight_decay": 0.0, "name": "memory_values",
                              "base_lr": 1e-2}],
            "state": [{"step": torch.tensor(2.0), "v": torch.rand(rows, generator=gen),
                       "n": torch.randint(0, 9, (rows,), generator=gen, dtype=torch.int32)}]}


def local_of(sd, shard):
    """The rank-local state dict a sharded optimizer holds: per-row entries cut to the shard, local shapes."""
    out = dict(sd)
    out["state"] = [{k: (shard.take(v).clone() if k != "step" and v.ndim >= 1 else v.clone())
                     for k, v in sd["state"][0].items()}]
    out["shapes"] = [[shard.count] + list(sd["shapes"][0][1:])]
    return out


def assert_same(a, b, path="sd"):
    """Two state dicts equal bit for bit (tensors: dtype, shape and bits)."""
    assert type(a) is type(b) or (isinstance(a, (list, tuple)) and isinstance(b, (list, tuple))), path
    if torch.is_tensor(a):
        assert a.dtype == b.dtype and a.shape == b.shape, f"{path}: {a.dtype}{tuple(a.shape)} vs {b.dtype}{tuple(b.shape)}"
        assert torch.equal(a.cpu(), b.cpu()), path
    elif isinstance(a, dict):
        assert a.keys() == b.keys(), f"{path}: keys {sorted(a)} vs {sorted(b)}"
        for k in a:
            assert_same(a[k], b[k], f"{path}[{k!r}]")
    elif isinstance(a, (list, tuple)):
        assert len(a) == len(b), path
        for i, (x, y) in enumerate(zip(a, b)):
            assert_same(x, y, f"{path}[{i}]")
    else:
        assert a == b, f"{path}: {a!r} vs {b!r}"


def worker(rank, world, port, R, D, dst, errors):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = RowShard(R, world, rank)
        full_v = torch.randn(R, D, generator=torch.Generator().manual_seed(5))
        # raw gather: every dtype, several rounds (chunk of 3 rows' bytes), empty shards
        for t in (full_v, full_v.to(torch.bfloat16), (full_v * 50).to(torch.int8),
                  torch.arange(R, dtype=torch.int32), torch.arange(R * 2, dtype=torch.uint8).view(R, 2)[:, :1]):
            got = gather_rows(shard.take(t).contiguous(), shard, None, dst, chunk_bytes=3 * t[:1].numel()
                              * t.element_size())
            if rank == dst:
                assert_same(got, t.contiguous(), "gather_rows")
            else:
                assert got is None
        # model state: the sharded model's unsharded state dict is the one-process model's
        one = Layer(full_v)
        model = Layer(full_v, shard)
        sd = unsharded_model_state(model, dst=dst, chunk_bytes=1000)
        if rank == dst:
            assert_same(sd, {k: v.detach() for k, v in one.state_dict().items()}, "model")
            torch.save(sd, os.path.join(os.environ["CKPT_DIR"], "model.pt"))
        else:
            assert sd is None
        dist.barrier()
        # load (no collective): memory-mapped full file, each rank keeps its rows
        fresh = Layer(torch.zeros(R, D), shard)
        with torch.no_grad():
            fresh.proj.weight.zero_()
            fresh.proj.bias.zero_()
        full = torch.load(os.path.join(os.environ["CKPT_DIR"], "model.pt"), mmap=True, weights_only=True)
        load_unsharded_model_state(fresh, full)
        assert torch.equal(fresh.values.weight.detach(), shard.take(full_v))
        assert torch.equal(fresh.proj.weight.detach(), one.proj.weight.detach())
        assert torch.equal(fresh.proj.bias.detach(), one.proj.bias.detach())
        # optimizer states: table formats (fp32 / bf16 / int8 lazy Adam, rowrms), unshard -> full, shard -> local
        p = model.values.weight
        for full_sd in (lazy_adam_state(R, D), lazy_adam_state(R, D, bf16=True), lazy_adam_state(R, D, int8=True),
                        row_wise_state(R)):
            if full_sd["format"] == "smlm.row_wise.v1":
                full_sd["shapes"] = [[R, D]]
            loc = local_of(full_sd, shard)
            got = unshard_optimizer_state(loc, [p], dst=dst, chunk_bytes=64)
            if rank == dst:
                assert_same(got, full_sd, full_sd["format"])
            else:
                assert got is None
            assert_same(shard_optimizer_state(full_sd, [p]), loc, "shard_optimizer_state")
        # torch's own Adam over the sharded table and a replicated parameter, inside an OptimizerSet with a table
        # optimizer: the gathered state equals one Adam step over the full table
        grad_full = torch.randn(R, D, generator=torch.Generator().manual_seed(9))
        ref = Layer(full_v)
        ref_adam = torch.optim.Adam([ref.values.weight, ref.proj.weight], lr=1e-2)
        ref.values.weight.grad = grad_full.clone()
        ref.proj.weight.grad = torch.ones(3, 4)
        ref_adam.step()
        adam = torch.optim.Adam([model.values.weight, model.proj.weight], lr=1e-2)
        model.values.weight.grad = shard.take(grad_full).clone()
        model.proj.weight.grad = torch.ones(3, 4)
        adam.step()
        table_sd = lazy_adam_state(R, D)
        table_opt = DictOpt([p], local_of(table_sd, shard))
        both = OptimizerSet(adam, table_opt)
        got = unsharded_optimizer_state(both, dst=dst, chunk_bytes=100)
        if rank == dst:
            want = {"format": "smlm.optimizer_set.v1",
                    "optimizers": [{"type": "Adam", "state_dict": ref_adam.state_dict()},
                                   {"type": "DictOpt", "state_dict": table_sd}]}
            assert_same(got, want, "OptimizerSet")
            torch.save(got, os.path.join(os.environ["CKPT_DIR"], "opt.pt"))
        else:
            assert got is None
        dist.barrier()
        full_opt = torch.load(os.path.join(os.environ["CKPT_DIR"], "opt.pt"), mmap=True, weights_only=True)
        adam2 = torch.optim.Adam([model.values.weight, model.proj.weight], lr=1e-2)
        table2 = DictOpt([p], None)
        load_unsharded_optimizer_state(OptimizerSet(adam2, table2), full_opt)
        assert_same(adam2.state_dict(), adam.state_dict(), "Adam reloaded")
        assert_same(table2.sd, local_of(table_sd, shard), "table state reloaded")
        # a rank with another state structure: every rank raises (no rank left waiting in a gather)
        bad = local_of(lazy_adam_state(R, D), shard)
        if rank == world - 1:
            del bad["state"][0]["exp_avg_sq"]
        with pytest.raises(ValueError, match="differs between the ranks"):
            unshard_optimizer_state(bad, [p], dst=dst)
        # a full state dict for another table size is refused before any copy
        with pytest.raises(ValueError):
            shard_optimizer_state(lazy_adam_state(R + 1, D), [p])
    except Exception as e:                                   # reported by the parent
        errors.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,R,dst", [(2, 37, 0), (3, 50, 2), (3, 2, 1)])
def test_unsharded_checkpoint(world, R, dst, tmp_path):
    os.environ["CKPT_DIR"] = str(tmp_path)
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    mp.start_processes(worker, args=(world, free_port(), R, 6, dst, errors), nprocs=world, join=True,
                       start_method="spawn")
    assert errors.empty()
