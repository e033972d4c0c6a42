"""Row-sharded product-key memory on 2 GPUs (one process per GPU; skipped with fewer GPUs), with the exchange by
NCCL collectives and fused through peer memory: two ranks with the table split by rows equal one GPU running the
same layer on the concatenated batches — outputs, the rows' accumulated gradients, the replicated parameters'
summed gradients, the clip norm, and the table after two LazyRowAdam steps."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
WORLD = 2


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_layer(group=None, exchange="nccl"):
    from smlm_b200.pkm import ProductKeyMemory
    torch.manual_seed(0)
    return ProductKeyMemory(64, 64, n_keys=64, heads=4, knn=16, k_dim=64, query_norm="none", swilu=False,
                            value_grad="row_sparse", shard_group=group, shard_exchange=exchange)


def data(steps, N):
    gen = torch.Generator().manual_seed(11)
    return [(torch.randn(WORLD, N, 64, generator=gen), torch.randn(WORLD, N, 64, generator=gen))
            for _ in range(steps)]


def run_step(mem, opt, x, g, autocast):
    from smlm_b200.sparse_values import clip_row_sparse
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        out = mem(x)
    out.backward(g)
    norm = clip_row_sparse([mem.values.weight], 0.5)
    return out.detach(), norm


def worker(rank, port, autocast, exchange, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from smlm_b200.sharded import allreduce_replicated_grads
        from smlm_b200.sparse_values import LazyRowAdam, row_store
        ref = make_layer().to(dev)                                   # one GPU, full table
        mem = make_layer(dist.group.WORLD, exchange).to(dev)
        sd = {k: v for k, v in ref.state_dict().items() if k != "values.weight"}
        mem.load_state_dict(sd, strict=False)
        with torch.no_grad():
            mem.values.weight.copy_(mem.shard.take(ref.values.weight))
        o_ref = LazyRowAdam([ref.values.weight], lr=1e-2, betas=(0.9, 0.98))
        o_mem = LazyRowAdam([mem.values.weight], lr=1e-2, betas=(0.9, 0.98))
        for x, g in data(2, 96):
            out_r, norm_r = run_step(ref, o_ref, x.reshape(-1, 64).to(dev), g.reshape(-1, 64).to(dev), autocast)
            out_m, norm_m = run_step(mem, o_mem, x[rank].to(dev), g[rank].to(dev), autocast)
            allreduce_replicated_grads(mem)
            torch.testing.assert_close(out_m, out_r.view(WORLD, -1, 64)[rank], rtol=1e-5, atol=1e-6)
            torch.testing.assert_close(norm_m, norm_r, rtol=1e-5, atol=1e-6)
            st_r, st_m = row_store(ref.values.weight), row_store(mem.values.weight)
            torch.testing.assert_close(st_m.acc, mem.shard.take(st_r.acc), rtol=1e-5, atol=1e-6)
            assert torch.equal(st_m.touched, mem.shard.take(st_r.touched))
            # replicated parameters: the per-rank gradients summed; under bf16 autocast each rank's contraction
            # rounds to bf16 before the sum (a few bf16 ulps of the largest entry)
            tol = 2.0 ** -6 if autocast else 1e-4
            for name in ("keys", "query_proj.weight", "query_proj.bias"):
                pr, pm = ref.get_parameter(name), mem.get_parameter(name)
                torch.testing.assert_close(pm.grad, pr.grad, rtol=tol, atol=tol * float(pr.grad.abs().max()))
            o_ref.step()
            o_mem.step()
            torch.testing.assert_close(mem.values.weight, mem.shard.take(ref.values.weight), rtol=1e-5, atol=1e-6)
            for m in (ref, mem):
                m.zero_grad(set_to_none=True)
        x = getattr(mem.values.weight, "peer_exchange", None)
        if x is not None:
            assert exchange == "p2p"
            x.close()
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, f"{type(e).__name__}: {e}"))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("autocast", [False, True])
@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
def test_sharded_layer_equals_one_gpu(autocast, exchange):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(worker, args=(free_port(), autocast, exchange, q), nprocs=WORLD, join=True,
                       start_method="spawn")
    res = dict(q.get() for _ in range(WORLD))
    assert res == {r: "ok" for r in range(WORLD)}, res
