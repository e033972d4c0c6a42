"""A whole training step captured as one CUDA graph (smlm_b200.graph_step.GraphedStep) and the capturable lazy
Adam it needs: replays give exactly the parameters, moments and outputs of the same steps run eagerly, and the
device-buffer scalars give exactly the by-value step."""
import pytest
import torch

from smlm_b200.graph_step import GraphedStep
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
