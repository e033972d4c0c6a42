"""Checkpoints through the real CUDA optimizers (smlm_b200.checkpoint) on one GPU: a table marked as row-sharded over
a one-rank NCCL group (its one shard is the whole table) saves through the gather path and loads through the
per-rank slicing path. The saved state dicts equal the model's and the optimizers' own bit for bit (LazyRowAdam
with fp32 and int8 moments, RowWiseOptimizer, fused AdamW inside an OptimizerSet), and a fresh model and optimizer
loaded from the files take the next step bit-identically. Gathers over several ranks are covered on gloo ranks
(tests/test_checkpoint_host.py). Runs in a spawned process, so the NCCL group never lives in the test process."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _same(a, b, path):
    if torch.is_tensor(a):
        assert torch.is_tensor(b) and a.dtype == b.dtype and a.shape == b.shape, path
        assert torch.equal(a.detach().cpu(), b.detach().cpu()), path
    elif isinstance(a, dict):
        assert a.keys() == b.keys(), path
        for k in a:
            _same(a[k], b[k], f"{path}[{k!r}]")
    elif isinstance(a, (list, tuple)):
        assert len(a) == len(b), path
        for i, (x, y) in enumerate(zip(a, b)):
            _same(x, y, f"{path}[{i}]")
    else:
        assert a == b, f"{path}: {a!r} vs {b!r}"


def _build(kind, seed):
    from smlm_b200.row_optim import RowWiseOptimizer
    from smlm_b200.sharded import RowShard
    from smlm_b200.sparse_values import LazyRowAdam, OptimizerSet
    torch.manual_seed(seed)
    model = torch.nn.Module()
    model.proj = torch.nn.Linear(16, 8).cuda()
    model.values = torch.nn.Embedding(1000, 64).cuda()
    table = model.values.weight
    table.row_shard = RowShard(table.shape[0], 1, 0)
    table.shard_group = None
    if kind == "rowrms":
        topt = RowWiseOptimizer([table], lr=1e-2, kind="rowrms", beta2=0.95)
    else:
        topt = LazyRowAdam([table], lr=1e-2, betas=(0.9, 0.98), state_dtype=kind)
    dense = torch.optim.AdamW(model.proj.parameters(), lr=1e-3, fused=True)
    return model, OptimizerSet(dense, topt)


def _step(model, opt, step):
    from smlm_b200.sparse_values import row_store
    gen = torch.Generator().manual_seed(100 + step)
    rows = torch.randperm(1000, generator=gen)[:300].cuda()
    st = row_store(model.values.weight)
    st.acc[rows] = torch.randn(300, 64, generator=gen).cuda()
    st.touched[rows] = True
    for p in model.proj.parameters():
        p.grad = torch.randn(p.shape, generator=gen).cuda()
    opt.step()
    opt.zero_grad(set_to_none=True)


def worker(rank, port, tmp, errors):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    try:
        from smlm_b200.checkpoint import (load_unsharded_model_state, load_unsharded_optimizer_state,
                                          unsharded_model_state, unsharded_optimizer_state)
        for kind in ("fp32", "int8", "rowrms"):
            model, opt = _build(kind, 0)
            for s in range(2):
                _step(model, opt, s)
            msd = unsharded_model_state(model, chunk_bytes=64 * 1024)
            osd = unsharded_optimizer_state(opt, chunk_bytes=64 * 1024)
            _same(msd, model.state_dict(), f"{kind} model")
            _same(osd, opt.state_dict(), f"{kind} optimizer")
            torch.save(msd, os.path.join(tmp, f"{kind}_model.pt"))
            torch.save(osd, os.path.join(tmp, f"{kind}_opt.pt"))
            fresh, fresh_opt = _build(kind, 1)
            load_unsharded_model_state(fresh, torch.load(os.path.join(tmp, f"{kind}_model.pt"), mmap=True,
                                                         weights_only=True))
            load_unsharded_optimizer_state(fresh_opt, torch.load(os.path.join(tmp, f"{kind}_opt.pt"), mmap=True,
                                                                 weights_only=True))
            _step(model, opt, 2)
            _step(fresh, fresh_opt, 2)
            _same(fresh.state_dict(), model.state_dict(), f"{kind} model after a step")
            _same(fresh_opt.state_dict(), opt.state_dict(), f"{kind} optimizer after a step")
    except Exception as e:                                   # reported by the parent
        errors.put(f"{type(e).__name__}: {e}")
        raise
    finally:
        dist.destroy_process_group()


def test_checkpoint_round_trip_with_cuda_optimizers(tmp_path):
    ctx = mp.get_context("spawn")
    errors = ctx.Queue()
    mp.start_processes(worker, args=(free_port(), str(tmp_path), errors), nprocs=1, join=True,
                       start_method="spawn")
    assert errors.empty()
