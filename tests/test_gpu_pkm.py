"""The PKM layer (smlm_b200.pkm.ProductKeyMemory on the CUDA kernels) against the reference's PyTorch path
(oracle/torch_path.py, run on the CPU) and the golden layer fixtures: config-1 shapes, fp32."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import torch_path as TP
from smlm_b200.model import ModelConfig, Transformer
from smlm_b200.optim import build_optimizer, clip_grads
from smlm_b200.pkm import ProductKeyMemory
from smlm_b200.sparse_values import LazyRowAdam, row_sparse_tables, row_store
from util import close, golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def config1_pair(N=2048, n_keys=256, seed=0):
    """8x256 tokens, d_model 384, H=4, k_dim 256, knn 32, 256 sub-keys per half (65,536
    rows), no BatchNorm / swilu, row-sparse values; the same parameters in both implementations."""
    ref = TP.TorchPKM(384, 384, n_keys=n_keys, heads=4, knn=32, k_dim=256, query_norm="none", swilu=False,
                      canonical=True)
    TP.init_like_reference(ref, seed)
    mem = ProductKeyMemory(384, 384, n_keys=n_keys, heads=4, knn=32, k_dim=256, query_norm="none", swilu=False,
                           value_grad="row_sparse").to(DEV)
    mem.load_state_dict(ref.state_dict())
    gen = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(N, 384, generator=gen)
    gout = torch.randn(N, 384, generator=gen)
    return ref, mem, x, gout


def boundary_gap_ulps(q, keys, knn):
    """Per row (n*h): the fp32-ulp gap at the two selection boundaries of the exact scores (oracle)."""
    s1, s2 = O.subkey_scores_f32(q, keys)
    gaps = []
    for s in (s1, s2):
        srt = -np.sort(-s.reshape(-1, s.shape[-1]), -1)
        a, b = srt[:, knn - 1], srt[:, knn]
        gaps.append(np.abs(a - b) / np.spacing(np.abs(a)))
    return np.minimum(gaps[0], gaps[1])


def test_layer_fp32_step_matches_reference_path():
    """Forward, backward and one lazy Adam step of the config-1 layer against the reference's PyTorch path.
    Indices: bit-exact against the oracle's fixed-order fp32 pipeline on the same queries; against the
    reference's einsum scores equal except at near-ties (boundary gap <= 4 ulp, counted, < 1% of rows).
    Outputs, row accumulator, keys / query gradients and updated rows within rel 1e-5,
    with the reference run on the same selection."""
    ref, mem, x, gout = config1_pair()
    mem.record = True
    xd = x.to(DEV)
    out = mem(xd)
    out.backward(gout.to(DEV))
    idx = mem.last_indices.cpu()
    with torch.no_grad():
        q = mem.query_proj(xd).view(-1, 4, 256).cpu()
    o1, o2 = O.subkey_scores_f32(q.numpy(), mem.keys.detach().cpu().numpy())
    _, oidx, _ = O.select(o1, o2, 32, bf16=False)
    assert np.array_equal(idx.numpy(), oidx)
    with torch.no_grad():
        _, idx_r = ref.get_indices(ref.query_proj(x).view(-1, 4, 256))
    rows_diff = (idx.sort(-1).values != idx_r.sort(-1).values).any(-1).reshape(-1)
    n_diff = int(rows_diff.sum())
    if n_diff:
        gaps = boundary_gap_ulps(q.numpy(), mem.keys.detach().cpu().numpy(), 32)
        assert (gaps[rows_diff.numpy()] <= 4).all(), "index differences away from near-ties"
    assert n_diff <= 0.01 * rows_diff.numel()
    ref.forced_indices = idx
    out_r = ref(x)
    out_r.backward(gout)
    close(out.detach().cpu(), out_r.detach(), msg="layer output")
    st, st_r = row_store(mem.values.weight), TP.row_store(ref.values.weight)
    assert torch.equal(st.touched.cpu(), st_r.touched)
    close(st.acc.cpu(), st_r.acc, msg="row accumulator")
    close(mem.keys.grad.cpu(), ref.keys.grad, msg="keys grad")
    close(mem.query_proj.weight.grad.cpu(), ref.query_proj.weight.grad, msg="query grad")
    close(mem.query_proj.bias.grad.cpu(), ref.query_proj.bias.grad, msg="query bias grad")
    # Adam on the gradient each path really holds would amplify summation-order noise of near-zero gradients
    # (the first step moves by ~lr * sign(g)); the step itself is compared on one accumulator
    st_r.acc.copy_(st.acc.cpu())
    opt, opt_r = LazyRowAdam([mem.values.weight], lr=1e-3, betas=(0.9, 0.98)), \
        TP.TorchLazyRowAdam([ref.values.weight], lr=1e-3, betas=(0.9, 0.98))
    opt.step()
    opt_r.step()
    close(mem.values.weight.detach().cpu(), ref.values.weight.detach(), msg="updated rows")
    assert not st.touched.any() and torch.count_nonzero(st.acc) == 0


@pytest.mark.parametrize("v", [0, 1])
def test_layer_golden(v):
    """The reference layer's own outputs (golden): forward, backward into the row store and keys / query, one
    lazy Adam step."""
    g = golden("layer.npz")
    n_keys, heads, knn, k_dim, d, N, bn, swilu = (int(x) for x in g[f"v{v}_cfg"])
    mem = ProductKeyMemory(d, d, n_keys=n_keys, heads=heads, knn=knn, k_dim=k_dim,
                           query_norm="batchnorm" if bn else "none", swilu=bool(swilu),
                           value_grad="row_sparse").to(DEV)
    pre = f"v{v}_param_"
    mem.load_state_dict({k[len(pre):]: torch.from_numpy(g[k]) for k in g.files if k.startswith(pre)})
    mem.record = True
    out = mem(torch.from_numpy(g[f"v{v}_x"]).to(DEV))
    out.backward(torch.from_numpy(g[f"v{v}_gout"]).to(DEV))
    assert torch.equal(mem.last_indices.cpu().sort(-1).values, torch.from_numpy(g[f"v{v}_idx"]).sort(-1).values)
    close(out.detach().cpu(), g[f"v{v}_out"], msg="out")
    st = row_store(mem.values.weight)
    close(st.acc.cpu(), g[f"v{v}_acc"], msg="acc")
    assert torch.equal(st.touched.cpu(), torch.from_numpy(g[f"v{v}_touched"]))
    close(mem.keys.grad.cpu(), g[f"v{v}_keys_grad"], msg="keys grad")
    close(mem.query_proj.weight.grad.cpu(), g[f"v{v}_qw_grad"], msg="query grad")
    close(mem.query_proj.bias.grad.cpu(), g[f"v{v}_qb_grad"], msg="query bias grad")
    opt = LazyRowAdam([mem.values.weight], lr=1e-3, betas=(0.9, 0.98), eps=1e-8)
    opt.step()
    close(mem.values.weight.detach().cpu(), g[f"v{v}_values_after"], msg="values after step")
    close(opt.state[mem.values.weight]["exp_avg"].cpu(), g[f"v{v}_m_after"], msg="exp_avg")


def test_layer_bf16_autocast_selection_equals_reference_selection():
    """Under bf16 autocast the layer scores with the fused tensor-core kernel; its selection equals the oracle's
    canonical selection on the kernel's bf16 sub-key scores bit for bit, and those scores are the reference's
    bf16 einsum scores to within one bf16 step."""
    from smlm_b200 import kernels as K
    ref, mem, x, gout = config1_pair(N=512)
    mem.record = True
    xx = x.to(DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = mem(xx)
    out.float().backward(gout.to(DEV))
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        q = mem.query_proj(xx).view(-1, 4, 256)
    with torch.no_grad():
        _, idx, w, s1, s2 = K.score_select(q.to(torch.bfloat16), mem.keys.to(torch.bfloat16), 32, dump=True)
        e1, e2 = mem.subkey_scores(q.to(torch.bfloat16))
    assert torch.equal(mem.last_indices, idx)
    osc, oidx, ow = O.select(s1.cpu().contiguous().view(torch.int16).numpy().view(np.uint16),
                             s2.cpu().contiguous().view(torch.int16).numpy().view(np.uint16), 32, bf16=True)
    assert np.array_equal(mem.last_indices.cpu().numpy(), oidx)
    np.testing.assert_allclose(mem.last_weights.cpu().numpy(), ow, rtol=0, atol=1e-6)
    assert float((s1 == e1).float().mean()) > 0.99 and float((s2 == e2).float().mean()) > 0.99
    assert mem.keys.grad is not None and mem.keys.grad.abs().sum() > 0


def tiny(value_grad="row_sparse", seed=0):
    cfg = ModelConfig(vocab_size=128, d_model=32, n_layers=4, n_heads=4, ffn_hidden=64, max_seq_len=64,
                      mem_layers=[0, 2, 3], mem_n_keys=16, mem_heads=2, mem_knn=4, mem_k_dim=16,
                      mem_share_values=True, mem_value_grad=value_grad)
    torch.manual_seed(seed)
    return Transformer(cfg).to(DEV)


def test_model_training_step_only_changes_read_rows():
    """Three memory layers sharing one table, two micro-batches, clip + OptimizerSet step: rows that were not
    read keep their values and Adam state (the reference's tests/test_sparse_values.py:73-104)."""
    m = tiny()
    opt = build_optimizer(m, 1e-2, 2.4e-2, 0.1)
    table = m.memory_layers()[0].values.weight
    lazy = opt.opts[1]
    assert isinstance(lazy, LazyRowAdam) and row_sparse_tables(m) == [table]
    for step in range(3):
        before = table.detach().clone()
        read = set()
        torch.manual_seed(step + 1)
        for _ in range(2):
            for x in m.memory_layers():
                x.record = True
            idx = torch.randint(0, 128, (2, 12), device=DEV)
            _, loss = m(idx[:, :-1], idx[:, 1:])
            (loss / 2).backward()
            for x in m.memory_layers():
                read |= set(x.last_indices.reshape(-1).tolist())
        rows = torch.tensor(sorted(read), device=DEV)
        assert set(torch.nonzero(row_store(table).touched).squeeze(1).tolist()) == read
        clip_grads(m, 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        unread = torch.ones(table.shape[0], dtype=torch.bool, device=DEV)
        unread[rows] = False
        assert torch.equal(table.detach()[unread], before[unread])
        assert not torch.equal(table.detach()[rows], before[rows])
        assert int(lazy.state[table]["step"]) == step + 1
        assert not row_store(table).touched.any() and torch.count_nonzero(row_store(table).acc) == 0


def test_frozen_table_and_table_only_training():
    for frozen in ("table", "rest"):
        m = tiny()
        table = m.memory_layers()[0].values.weight
        for p in m.parameters():
            p.requires_grad_((p is not table) if frozen == "table" else (p is table))
        before = {n: p.detach().clone() for n, p in m.named_parameters()}
        opt = build_optimizer(m, 1e-2, 1e-2, 0.0)
        idx = torch.randint(0, 128, (2, 12), device=DEV)
        _, loss = m(idx[:, :-1], idx[:, 1:])
        loss.backward()
        clip_grads(m, 1.0)
        opt.step()
        changed = {n for n, p in m.named_parameters() if not torch.equal(p.detach(), before[n])}
        if frozen == "table":
            assert "layers.0.ffn.values.weight" not in changed and not hasattr(table, "row_store")
            assert any("query_proj" in n for n in changed)
        else:
            assert changed == {"layers.0.ffn.values.weight"}


@pytest.mark.parametrize("kind", ["fp32", "bf16", "q4"])
def test_decode_graph_bit_identical(kind):
    """Decoding with captured memory-layer graphs gives logits bit-identical to the eager path (the reference's
    tests/test_kernels.py:257-277)."""
    m = tiny().eval()
    m.set_memory_inference_table(kind)
    x = torch.randint(0, 128, (1, 8), generator=torch.Generator().manual_seed(2)).to(DEV)

    def decode():
        caches = [dict() for _ in range(m.cfg.n_layers)]
        outs = [m(x[:, :4], kv_caches=caches, pos0=0).float()]
        for i in range(4, 8):
            outs.append(m(x[:, i:i + 1], kv_caches=caches, pos0=i).float())
        return torch.cat(outs, 1)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        eager = decode()
        m.set_memory_decode_graphs(True)
        graph = decode()
        graph2 = decode()
        m.set_memory_decode_graphs(False)
    assert torch.equal(graph, eager) and torch.equal(graph2, eager)


def test_kv_cache_decode_matches_full_forward():
    m = tiny().eval()
    x = torch.randint(0, 128, (1, 30), device=DEV)
    with torch.no_grad():
        full = m(x)
        caches = [dict() for _ in range(m.cfg.n_layers)]
        steps = [m(x[:, :10], kv_caches=caches, pos0=0)]
        for t in range(10, 30):
            steps.append(m(x[:, t:t + 1], kv_caches=caches, pos0=t))
    torch.testing.assert_close(torch.cat(steps, 1), full, rtol=1e-4, atol=1e-5)
