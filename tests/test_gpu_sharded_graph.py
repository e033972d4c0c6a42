"""The row-sharded paths that run as CUDA graphs, on 2 GPUs (one process per GPU; skipped with fewer GPUs):

  * the row-sharded training step (peer exchange with owner buckets and device-side epochs, NCCL all-gather of the
    output gradients and all-reduce of the replicated gradients, LazyRowAdam(capturable=True), capturable AdamW)
    captured once with smlm_b200.graph_step.GraphedStep and replayed equals the same steps run eagerly;
  * greedy decoding of a model whose product-key memories share one row-sharded table (GraphDecoder, the whole
    step one CUDA graph, the exchange inside it) equals the same model on one GPU with the whole table, in fp32 and
    under bf16 autocast (where the sharded inference bag fuses the swilu product into the exchange's sum)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
WORLD = 2
needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < WORLD,
                               reason="needs 2 GPUs")


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run(fn, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(fn, args=(free_port(), q) + args, nprocs=WORLD, join=True, start_method="spawn")
    res = dict(q.get() for _ in range(WORLD))
    assert res == {r: "ok" for r in range(WORLD)}, res


def setup(rank, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    return dev


def close_exchanges(*tables):
    for t in tables:
        x = getattr(t, "peer_exchange", None)
        if x is not None:
            x.close()


# ------------------------------------------------------------------------------------ graphed training step
def graph_worker(rank, port, q):
    dev = setup(rank, port)
    try:
        from smlm_b200.graph_step import GraphedStep
        from smlm_b200.pkm import ProductKeyMemory
        from smlm_b200.sharded import allreduce_replicated_grads
        from smlm_b200.sparse_values import LazyRowAdam, OptimizerSet, clip_row_sparse

        def layer():
            torch.manual_seed(0)
            m = ProductKeyMemory(128, 128, n_keys=128, heads=4, knn=32, k_dim=256, query_norm="none", swilu=False,
                                 value_grad="row_sparse", shard_group=dist.group.WORLD).to(dev)
            t = m.values.weight
            dense = [p for p in m.parameters() if p is not t]
            opt = OptimizerSet(torch.optim.AdamW(dense, lr=1e-3, fused=True, capturable=True),
                               LazyRowAdam([t], lr=1e-2, betas=(0.9, 0.98), capturable=True))
            return m, opt

        def step(m, opt, x, g):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = m(x)
            out.backward(g)
            allreduce_replicated_grads(m)
            norm = clip_row_sparse([m.values.weight], 1.0)
            opt.step()
            opt.zero_grad(set_to_none=True)
            return out.detach(), norm

        gen = torch.Generator().manual_seed(100 + rank)
        batches = [(torch.randn(512, 128, generator=gen).to(dev), torch.randn(512, 128, generator=gen).to(dev))
                   for _ in range(4)]
        mg, og = layer()
        gstep = GraphedStep(lambda x, g: step(mg, og, x, g), list(batches[0]), og.opts, warmup=1)
        me, oe = layer()
        out_e = [step(me, oe, *batches[0])]
        outs_g = []
        for i in range(1, 4):
            out_e.append(step(me, oe, *batches[i]))
            o, n = gstep(*batches[i])
            outs_g.append((o.clone(), n.clone()))
        torch.cuda.synchronize()
        for i, ((oe_i, ne_i), (og_i, ng_i)) in enumerate(zip(out_e[1:], outs_g)):
            assert torch.equal(og_i, oe_i), f"step {i + 1}: layer output"
            assert torch.equal(ng_i, ne_i), f"step {i + 1}: clip norm"
        assert torch.equal(mg.values.weight, me.values.weight)
        torch.testing.assert_close(mg.keys, me.keys, rtol=1e-6, atol=1e-7)
        del gstep
        close_exchanges(mg.values.weight, me.values.weight)
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, f"{type(e).__name__}: {e}"))
        raise
    finally:
        dist.destroy_process_group()


@needs_two
def test_graphed_sharded_step_equals_eager():
    run(graph_worker)


# --------------------------------------------------------------------------------------- sharded decoding
def decode_worker(rank, port, q, autocast):
    dev = setup(rank, port)
    try:
        from smlm_b200.decode import GraphDecoder
        from smlm_b200.model import ModelConfig, Transformer
        cfg = ModelConfig(vocab_size=512, d_model=128, n_layers=4, n_heads=4, ffn_hidden=256, max_seq_len=64,
                          mem_layers=[1, 3], mem_n_keys=128, mem_heads=2, mem_knn=16, mem_k_dim=256,
                          mem_share_values=True, mem_value_grad="row_sparse")
        torch.manual_seed(0)
        ref = Transformer(cfg).to(dev).eval()
        shd = Transformer(cfg, shard_group=dist.group.WORLD).to(dev).eval()
        table_keys = [k for k in ref.state_dict() if k.endswith("ffn.values.weight")]
        shd.load_state_dict({k: v for k, v in ref.state_dict().items() if k not in table_keys}, strict=False)
        st = shd.memory_layers()[0]
        with torch.no_grad():
            st.values.weight.copy_(st.shard.take(ref.memory_layers()[0].values.weight))
        prompt = torch.randint(0, 512, (3, 10), generator=torch.Generator().manual_seed(rank)).to(dev)
        logs = []
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            for m in (ref, shd):
                dec = GraphDecoder(m, 3, max_len=40)
                steps = [dec.prefill(prompt)[:, -1:].float()]
                toks = []
                for _ in range(12):
                    toks.append(dec.tokens.clone())
                    dec.step()
                    steps.append(dec.logits.float().clone())
                logs.append((steps, toks))
        torch.cuda.synchronize()
        (ls_r, tk_r), (ls_s, tk_s) = logs
        tol = dict(rtol=2e-2, atol=2e-2) if autocast else dict(rtol=1e-4, atol=1e-4)
        # the same greedy tokens fed in both: compare the logits step by step while the tokens agree
        for i, (a, b) in enumerate(zip(ls_s, ls_r)):
            torch.testing.assert_close(a, b, **tol, msg=f"step {i}")
            if i < len(tk_r) and not torch.equal(tk_s[i], tk_r[i]):
                break
        assert torch.equal(tk_s[0], tk_r[0])
        close_exchanges(st.values.weight)
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, f"{type(e).__name__}: {e}"))
        raise
    finally:
        dist.destroy_process_group()


@needs_two
@pytest.mark.parametrize("autocast", [False, True])
def test_sharded_graph_decode_equals_one_gpu(autocast):
    run(decode_worker, autocast)
