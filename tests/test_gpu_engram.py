"""Engram n-gram memory on the CUDA kernels (smlm_b200.engram) against the reference's PyTorch path (golden fixture
engram.npz, made by tests/golden/make_golden.py from smlm/engram.py with impl="torch") and the reference's own model
tests (tests/test_engram.py): hash rows bit-exact, module outputs / gradients / table accumulator / one lazy Adam
step within fp32 tolerance, causality, KV-cache chunks, only read rows change."""
import numpy as np
import pytest
import torch

import smlm_b200.engram as E
from oracle import oracle as O
from smlm_b200 import kernels as K
from smlm_b200.model import ModelConfig, Transformer
from smlm_b200.optim import build_optimizer, clip_grads
from smlm_b200.sparse_values import LazyRowAdam, row_store
from util import close, golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def identity_vocabulary(monkeypatch):
    """Token compression needs the GPT-2 vocabulary (tiktoken), which is not reachable offline: the identity map
    stands in (hash, module and training take the compressed ids as given). fp32 convolutions (no TF32)."""
    monkeypatch.setattr(E, "canonical_ids", lambda vocab: (torch.arange(vocab, dtype=torch.int64), vocab))
    old = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32 = old


def test_hash_kernel_bit_exact():
    g = golden("engram.npz")
    for v in (0, 1):
        c = torch.from_numpy(g[f"v{v}_c"]).to(DEV)
        rows = K.ngram_rows(c, 2, torch.from_numpy(g[f"v{v}_mult"]).to(DEV), [2, 3], 2, 101)
        assert np.array_equal(rows.cpu().numpy(), g[f"v{v}_rows"])
    # larger, more orders and heads, large ids: against the oracle
    gen = torch.Generator().manual_seed(3)
    ng = E.NgramHash(50304, orders=(2, 3, 4), heads=8, rows=524287, seed=7)
    c = torch.randint(0, 50304, (3, ng.history + 1000), generator=gen)
    got = ng.to(DEV)(c.to(DEV)).cpu().numpy()
    assert np.array_equal(got, O.ngram_rows(c.numpy(), ng.history, ng.mult.cpu().numpy(), [2, 3, 4], 8, 524287))


@pytest.mark.parametrize("v", [0, 1])
def test_module_matches_reference_path(v):
    g = golden("engram.npz")
    head_dim = int(g[f"v{v}_head_dim"])
    e = E.EngramMemory(32, 4, head_dim, 101, conv_kernel=4, dilation=3).to(DEV)
    state = {k[len(f"v{v}_param_"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith(f"v{v}_param_")}
    e.load_state_dict(state)
    x = torch.from_numpy(g[f"v{v}_x"]).to(DEV).requires_grad_()
    y = e(x, torch.from_numpy(g[f"v{v}_rows"]).to(DEV))
    y.backward(torch.from_numpy(g[f"v{v}_g"]).to(DEV))
    close(y.detach().cpu(), g[f"v{v}_y"])
    close(x.grad.cpu(), g[f"v{v}_x_grad"])
    close(e.w_k.weight.grad.cpu(), g[f"v{v}_wk_grad"])
    close(e.w_v.weight.grad.cpu(), g[f"v{v}_wv_grad"])
    close(e.conv.weight.grad.cpu(), g[f"v{v}_conv_grad"])
    close(e.h_norm.weight.grad.cpu(), g[f"v{v}_hnorm_grad"])
    st = row_store(e.values.weight)
    close(st.acc.cpu(), g[f"v{v}_acc"])
    assert torch.equal(st.touched.cpu(), torch.from_numpy(g[f"v{v}_touched"]))
    opt = LazyRowAdam([e.values.weight], lr=1e-3, betas=(0.9, 0.98), eps=1e-8)
    opt.step()
    close(e.values.weight.detach().cpu(), g[f"v{v}_values_after"])


def tiny(seed=0, head_dim=8, **kw):
    cfg = ModelConfig(vocab_size=512, d_model=32, n_layers=4, n_heads=4, ffn_hidden=64, max_seq_len=64,
                      eng_layers=[0, 2], eng_heads=2, eng_head_dim=head_dim, eng_rows=101, **kw)
    torch.manual_seed(seed)
    return Transformer(cfg).to(DEV)


def test_causal_and_kv_cache_chunks():
    m = tiny().eval()
    with torch.no_grad():                       # a non-zero convolution, so that its cache is exercised too
        for e in m.engram_layers():
            e.conv.weight.normal_(std=0.3)
    gen = torch.Generator().manual_seed(1)
    x = torch.randint(0, 512, (2, 40), generator=gen).to(DEV)
    y = x.clone()
    y[:, 25:] = torch.randint(0, 512, (2, 15), generator=gen).to(DEV)
    with torch.no_grad():
        full = m(x)
        torch.testing.assert_close(m(y)[:, :25], full[:, :25])
        caches = [dict() for _ in range(m.cfg.n_layers)]
        steps = [m(x[:, a:a + n], kv_caches=caches, pos0=a) for a, n in ((0, 7), (7, 1), (8, 1), (9, 12), (21, 19))]
    torch.testing.assert_close(torch.cat(steps, 1), full, rtol=1e-4, atol=1e-5)


def test_only_read_rows_change_and_own_learning_rates():
    m = tiny()
    pc = m.param_counts()
    assert pc["memory_values"] == 2 * 4 * 101 * 8
    assert pc["active_non_embedding_per_token"] == pc["dense_body"] + 2 * 4 * 8
    e = m.engram_layers()[0]
    before = e.values.weight.detach().clone()
    opt = build_optimizer(m, 1e-2, 3e-3, 0.1, eng_value_lr=5e-3)
    assert {g["name"]: g["lr"] for g in opt.param_groups}["engram_values"] == 5e-3
    x = torch.randint(0, 512, (2, 17), generator=torch.Generator().manual_seed(2)).to(DEV)
    _, loss = m(x[:, :-1], x[:, 1:])
    loss.backward()
    clip_grads(m, 1.0)
    opt.step()
    c = torch.cat([torch.full((2, 2), m.ngram.pad, device=DEV), m.ngram.canon[x[:, :-1]]], 1)
    read = torch.zeros(e.values.weight.shape[0], dtype=torch.bool, device=DEV)
    read[m.ngram(c).reshape(-1)] = True
    after = e.values.weight.detach()
    assert torch.equal(after[~read], before[~read])
    assert not torch.equal(after[read], before[read])


def test_dense_variant_same_forward():
    sp, de = tiny(), tiny(eng_value_grad="dense")
    de.load_state_dict(sp.state_dict())
    x = torch.randint(0, 512, (2, 17), generator=torch.Generator().manual_seed(4)).to(DEV)
    torch.testing.assert_close(de(x), sp(x))
    opt = build_optimizer(de, 1e-2, 3e-3, 0.1)
    groups = {g["name"]: g for g in opt.param_groups}
    tab = de.engram_layers()[0].values.weight
    assert any(p is tab for p in groups["engram_values"]["params"]) and groups["engram_values"]["weight_decay"] == 0
