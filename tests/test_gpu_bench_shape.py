"""Parity of the benchmark's dominant kernel at the benchmark's own sizes: the deferred row sums fused with lazy
Adam (bb_rowsum_kernel<..., ROWS_ADAM> + bb_fixup_kernel) on a table above 2^31 elements, and one whole layer
step at the headline shape (16,777,216 x 384 fp32 table, 32,768 tokens, bf16 autocast scoring) with sampled rows
checked against the oracle. The oracle forms each row's sum with the kernel's chunk schedule over all lookups
(oracle.bag_rows_subset), then applies the oracle's lazy Adam (reference: smlm/sparse_values.py:270-305,
smlm/host_rows.c:63-80; the reference's own large-offset test is tests/test_kernels.py:324)."""
import gc

import numpy as np
import pytest
import torch

from oracle import oracle as O
from smlm_b200 import kernels as K

pytestmark = pytest.mark.gpu
DEV = "cuda"


def chunk_of(m):
    """Sorted positions per work chunk of the row-sum kernels for m lookups."""
    return 256 if m >= 1 << 20 else 64


def free_device_memory():
    gc.collect()
    torch.cuda.empty_cache()


def oracle_adam_rows(g, idx, w, rows, sample, p0, m0, v0, scale, step, lr, b1, b2, eps):
    """The oracle's updated (p, m, v) of the rows in `sample` (numpy, in place on copies of p0 / m0 / v0)."""
    sums = O.bag_rows_subset(g, idx, w, rows, sample, chunk=chunk_of(idx.size))
    p, m, v = p0.copy(), m0.copy(), v0.copy()
    O.lazy_adam(p, m, v, sums, np.ones(sample.size, np.uint8), scale, step, lr, b1, b2, eps)
    return p, m, v


def test_fused_deferred_adam_above_2g_elements():
    """6M x 384 table (2.3 G elements): lookups past row 5.6M (row * 384 > 2^31), 8 hot rows taking 20% of the
    reads (runs crossing many 256-position chunks), a clip factor from a device tensor; every touched row and
    both its moments equal the oracle bit for bit, untouched probe rows keep all three."""
    free_device_memory()
    rows, D, N, Kk = 6_000_000, 384, 4096, 256
    gen = torch.Generator(device=DEV).manual_seed(21)
    p = torch.randn(rows, D, device=DEV, generator=gen) * D ** -0.5
    m = torch.randn(rows, D, device=DEV, generator=gen) * 1e-3
    v = torch.rand(rows, D, device=DEV, generator=gen) * 1e-5
    idx = torch.randint(rows - 400_000, rows, (N, Kk), device=DEV, generator=gen)
    idx[:, :16] = torch.randint(0, rows, (N, 16), device=DEV, generator=gen)
    hot = torch.randint(5_600_000, rows, (8,), device=DEV, generator=gen)
    sel = torch.rand(N, Kk, device=DEV, generator=gen) < 0.2
    idx[sel] = hot[torch.randint(0, 8, (int(sel.sum()),), device=DEV, generator=gen)]
    w = torch.softmax(torch.randn(N, Kk, device=DEV, generator=gen), -1)
    g = torch.randn(N, D, device=DEV, generator=gen)
    touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
    sq = torch.zeros(rows, device=DEV)
    _, pend = K.bag_backward_deferred(g, idx, w, p, touched, sq)
    uniq = torch.unique(idx)
    assert int(uniq.max()) * D > 2 ** 31
    assert int(touched.sum()) == uniq.numel() and bool(touched[uniq].all())
    probe = torch.tensor([0, 1, rows // 2, rows - 400_001, 5_599_999], device=DEV)
    probe = probe[~touched[probe]]
    assert probe.numel() > 0
    p0, m0, v0 = (t[uniq].cpu().numpy() for t in (p, m, v))
    before = [t[probe].clone() for t in (p, m, v)]
    scale = torch.tensor(0.37, device=DEV)
    K.lazy_adam_deferred_step(p, m, v, touched, pend, scale, 3, 1e-2, 0.9, 0.98, 1e-8)
    assert not touched.any()
    op, om, ov = oracle_adam_rows(g.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), rows, uniq.cpu().numpy(),
                                  p0, m0, v0, float(scale), 3, 1e-2, 0.9, 0.98, 1e-8)
    for name, got, want in (("param", p, op), ("exp_avg", m, om), ("exp_avg_sq", v, ov)):
        g_rows = got[uniq].cpu().numpy()
        bad = int((g_rows != want).any(-1).sum())
        assert bad == 0, f"{name}: {bad} of {uniq.numel()} touched rows differ from the oracle"
    for t, b in zip((p, m, v), before):
        assert torch.equal(t[probe], b)
    del p, m, v, pend
    free_device_memory()


def test_headline_layer_step_sampled_rows():
    """One layer step at the benchmark's headline shape through the public API (ProductKeyMemory with row-sparse
    values, bf16 autocast, value clipping, LazyRowAdam on the fused deferred path), after a first step so that the
    moments are nonzero: 8,192 sampled touched rows (and the largest touched row) equal the oracle's lazy Adam on
    the oracle's chunked sums of the layer's own selection, bit for bit in the row and both moments; 256 sampled
    tokens' outputs equal the oracle's value bag bit for bit; unread probe rows keep row and moments."""
    from smlm_b200.pkm import ProductKeyMemory
    from smlm_b200.sparse_values import LazyRowAdam, clip_row_sparse, row_store
    free_device_memory()
    n_keys, N, D, H, knn = 4096, 32768, 384, 4, 32
    R = n_keys ** 2
    torch.manual_seed(0)
    with torch.device(DEV):
        mem = ProductKeyMemory(D, D, n_keys=n_keys, heads=H, knn=knn, k_dim=256, query_norm="none", swilu=False,
                               value_grad="row_sparse")
        with torch.no_grad():
            mem.query_proj.weight.normal_(0, 0.02)
            mem.keys.normal_(0, 128 ** -0.5)
    table = mem.values.weight
    opt = LazyRowAdam([table], lr=1e-3, betas=(0.9, 0.98), eps=1e-8)
    gen = torch.Generator(device=DEV).manual_seed(3)
    xs = [torch.randn(N, D, device=DEV, generator=gen) for _ in range(2)]
    gs = [torch.randn(N, D, device=DEV, generator=gen) for _ in range(2)]

    def forward_backward(x, g):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = mem(x)
        out.backward(g)
        clip_row_sparse([table], 1.0)
        return out

    forward_backward(xs[0], gs[0])
    opt.step()
    mem.record = True
    out = forward_backward(xs[1], gs[1]).detach()
    st = row_store(table)
    assert st.pending is not None, "the step did not take the fused deferred path"
    idx = mem.last_indices.view(N, H * knn)
    w = mem.last_weights.view(N, H * knn)
    uniq = torch.unique(idx)
    pick = torch.randperm(uniq.numel(), generator=torch.Generator().manual_seed(5))[:8192].to(DEV)
    sample = torch.unique(torch.cat([uniq[pick], uniq[-1:]]))
    assert int(sample[-1]) * D > 2 ** 31
    # forward: 256 tokens' outputs against the oracle's bag over the rows they read (the table is unchanged
    # until the step)
    tok = torch.randperm(N, generator=torch.Generator().manual_seed(6))[:256].to(DEV)
    t_rows, t_inv = torch.unique(idx[tok], return_inverse=True)
    ref_out, bad = O.bag_forward(t_inv.cpu().numpy(), w[tok].cpu().numpy(), table.detach()[t_rows].cpu().numpy())
    assert bad == 0 and np.array_equal(out[tok].cpu().numpy(), ref_out)
    # optimizer step: sampled rows against the oracle
    state = opt.state[table]
    p0, m0, v0 = (t[sample].cpu().numpy() for t in (table.detach(), state["exp_avg"], state["exp_avg_sq"]))
    read = torch.zeros(R, dtype=torch.bool, device=DEV)
    read[uniq] = True
    probe = torch.randint(0, R, (4096,), device=DEV, generator=gen)
    probe = probe[~read[probe]]
    before = [t[probe].clone() for t in (table.detach(), state["exp_avg"], state["exp_avg_sq"])]
    scale = float(st.grad_scale)
    opt.step()
    op, om, ov = oracle_adam_rows(gs[1].cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), R,
                                  sample.cpu().numpy(), p0, m0, v0, scale, 2, 1e-3, 0.9, 0.98, 1e-8)
    for name, got, want in (("param", table.detach(), op), ("exp_avg", state["exp_avg"], om),
                            ("exp_avg_sq", state["exp_avg_sq"], ov)):
        g_rows = got[sample].cpu().numpy()
        nbad = int((g_rows != want).any(-1).sum())
        assert nbad == 0, f"{name}: {nbad} of {sample.numel()} sampled rows differ from the oracle"
    for t, b in zip((table.detach(), state["exp_avg"], state["exp_avg_sq"]), before):
        assert torch.equal(t[probe], b)
    del mem, opt, state, table, st
    free_device_memory()
