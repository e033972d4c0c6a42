"""A whole training step captured as one CUDA graph (smlm_b200.graph_step.GraphedStep) and the capturable lazy
Adam it needs: replays give exactly the parameters, moments and outputs of the same steps run eagerly (one layer
with the fused deferred step; a model whose three memory layers share one table, with two accumulated
micro-batches, so several backward passes write the accumulator and the plain step runs), and the device-buffer
scalars give exactly the by-value step."""
import pytest
import torch

from smlm_b200.graph_step import GraphedStep
from smlm_b200.model import ModelConfig, Transformer
from smlm_b200.optim import build_optimizer, clip_grads
from smlm_b200.pkm import ProductKeyMemory
from smlm_b200.sparse_values import LazyRowAdam, OptimizerSet, clip_row_sparse

pytestmark = pytest.mark.gpu
DEV = "cuda"


def layer(seed=0):
    torch.manual_seed(seed)
    return ProductKeyMemory(128, 128, n_keys=64, heads=4, knn=16, k_dim=256, query_norm="none", swilu=False,
                            value_grad="row_sparse").to(DEV)


def step(mem, opt, x, g):
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = mem(x)
    out.backward(g)
    norm = clip_row_sparse([mem.values.weight], 1.0)
    torch.nn.utils.clip_grad_norm_([p for p in mem.parameters() if p.grad is not None], 1.0, foreach=True)
    opt.step()
    opt.zero_grad(set_to_none=True)
    return norm


def make(mem, capturable=True):
    table = mem.values.weight
    dense = [p for p in mem.parameters() if p is not table]
    return OptimizerSet(torch.optim.AdamW(dense, lr=1e-3, betas=(0.9, 0.98), weight_decay=0.0, fused=True,
                                          capturable=capturable),
                        LazyRowAdam([table], lr=1e-2, betas=(0.9, 0.98), eps=1e-8, capturable=capturable))


def test_graphed_steps_equal_eager_steps():
    gen = torch.Generator().manual_seed(3)
    data = [(torch.randn(300, 128, generator=gen).to(DEV), torch.randn(300, 128, generator=gen).to(DEV))
            for _ in range(6)]
    ma, mb = layer(), layer()
    oa, ob = make(ma), make(mb)
    norms_a = [step(ma, oa, x, g).clone() for x, g in data]
    gs = GraphedStep(lambda x, g: step(mb, ob, x, g), list(data[0]), ob.opts, warmup=1)   # warm-up = step 1
    norms_b = [None] + [gs(x, g).clone() for x, g in data[1:]]
    for a, b in zip(norms_a[1:], norms_b[1:]):
        assert torch.equal(a, b)
    for (n, pa), pb in zip(ma.named_parameters(), mb.parameters()):
        assert torch.equal(pa, pb), n
    lt_a, lt_b = oa.opts[1], ob.opts[1]
    for k in ("exp_avg", "exp_avg_sq"):
        assert torch.equal(lt_a.state[ma.values.weight][k], lt_b.state[mb.values.weight][k])
    assert int(lt_a.state[ma.values.weight]["step"]) == int(lt_b.state[mb.values.weight]["step"]) == 6


def test_device_scalars_equal_by_value_step():
    """LazyRowAdam(capturable=True) (scalars read from device memory) and the by-value fused step give the same
    table and moments bit for bit, over steps whose bias corrections differ (dense parameters frozen, so both
    layers read the same rows)."""
    gen = torch.Generator().manual_seed(4)
    mems = [layer(1), layer(1)]
    opts = []
    for m, cap in zip(mems, (False, True)):
        for p in m.parameters():
            p.requires_grad_(p is m.values.weight)
        opts.append(LazyRowAdam([m.values.weight], lr=1e-2, betas=(0.9, 0.98), capturable=cap))
    for _ in range(4):
        x = torch.randn(200, 128, generator=gen).to(DEV)
        g = torch.randn(200, 128, generator=gen).to(DEV)
        for m, o in zip(mems, opts):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = m(x)
            out.backward(g)
            clip_row_sparse([m.values.weight], 0.5)
            o.step()
    assert torch.equal(mems[0].values.weight, mems[1].values.weight)
    for k in ("exp_avg", "exp_avg_sq"):
        assert torch.equal(opts[0].state[mems[0].values.weight][k], opts[1].state[mems[1].values.weight][k])


def test_graphed_model_step_with_shared_table_equals_eager():
    """Three memory layers reading one shared table, two micro-batches per step (six backward passes into the
    table's row store, the accumulator written, then the plain lazy Adam step with device scalars): the graphed
    steps give the eager steps' losses, parameters and moments bit for bit."""
    cfg = ModelConfig(vocab_size=256, d_model=64, n_layers=6, n_heads=4, ffn_hidden=128, max_seq_len=32,
                      mem_layers=[1, 3, 5], mem_n_keys=32, mem_heads=2, mem_knn=8, mem_k_dim=64,
                      mem_share_values=True, mem_value_grad="row_sparse")
    models = []
    for _ in range(2):
        torch.manual_seed(7)
        with torch.device(DEV):
            models.append(Transformer(cfg))
    opts = [build_optimizer(m, lr=1e-3, value_lr=3e-3, weight_decay=0.1, betas=(0.9, 0.95), capturable=True)
            for m in models]
    gen = torch.Generator().manual_seed(8)
    data = [torch.randint(0, 256, (4, 17), generator=gen).to(DEV) for _ in range(5)]

    def train(model, opt, seqs):
        total = torch.zeros((), device=DEV)
        for a in range(2):
            x = seqs[2 * a:2 * a + 2]
            with torch.autocast("cuda", dtype=torch.bfloat16):
                _, loss = model(x[:, :-1], x[:, 1:])
            (loss / 2).backward()
            total += loss.detach() / 2
        clip_grads(model, 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return total

    gs = GraphedStep(lambda seqs: train(models[1], opts[1], seqs), [data[0]], opts[1].opts, warmup=1)
    losses_b = [None] + [gs(seqs).clone() for seqs in data[1:]]
    losses_a = [train(models[0], opts[0], seqs).clone() for seqs in data]
    for a, b in zip(losses_a[1:], losses_b[1:]):
        assert torch.equal(a, b)
    for (n, pa), pb in zip(models[0].named_parameters(), models[1].parameters()):
        assert torch.equal(pa, pb), n
    table_a = models[0].memory_layers()[0].values.weight
    table_b = models[1].memory_layers()[0].values.weight
    lazy_a = next(o for o in opts[0].opts if table_a in o.state)
    lazy_b = next(o for o in opts[1].opts if table_b in o.state)
    for k in ("exp_avg", "exp_avg_sq"):
        assert torch.equal(lazy_a.state[table_a][k], lazy_b.state[table_b][k])
    assert int(lazy_a.state[table_a]["step"]) == int(lazy_b.state[table_b]["step"]) == 5
