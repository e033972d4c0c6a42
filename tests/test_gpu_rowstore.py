"""The RowStore's clean mode (untouched rows count as zero, first touches are written, the step leaves consumed
rows alone, clip norms from per-row squared norms) gives exactly what the exact, reference-semantics mode gives."""
import pytest
import torch

from smlm_b200 import kernels as K
from smlm_b200.pkm import ProductKeyMemory
from smlm_b200.sparse_values import LazyRowAdam, clip_row_sparse, row_store
from util import skewed_indices

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_first_touch_writes_and_row_norms():
    """Untouched rows hold garbage: with first-touch writes the result on the touched rows equals accumulating
    into zeros, the per-row squared norms are the rows' norms, and a second call accumulates."""
    gen = torch.Generator().manual_seed(1)
    rows, D, N = 4096, 384, 512
    table = torch.randn(rows, D, generator=gen) * D ** -0.5
    idx = skewed_indices(rows, N, 128, gen)
    w = torch.softmax(torch.randn(N, 128, generator=gen), -1)
    g = torch.randn(N, D, generator=gen)
    garbage = torch.randn(rows, D, generator=gen).to(DEV)
    touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
    sq = torch.zeros(rows, device=DEV)
    acc = garbage.clone()
    args = (g.to(DEV), idx.to(DEV), w.to(DEV), table.to(DEV))
    K.bag_backward_rows(*args, acc, touched, row_sqnorm=sq, first_touch_writes=True)
    ref = torch.zeros(rows, D, device=DEV)
    ref_t = torch.zeros(rows, dtype=torch.bool, device=DEV)
    K.bag_backward_rows(*args, ref, ref_t)
    assert torch.equal(touched, ref_t)
    assert torch.equal(acc[touched], ref[touched])
    assert torch.equal(acc[~touched], garbage[~touched])           # untouched rows not written
    torch.testing.assert_close(sq[touched], ref[touched].square().sum(-1), rtol=1e-5, atol=1e-6)
    # second micro-batch: touched rows accumulate, newly touched ones are written
    idx2 = skewed_indices(rows, N, 128, gen)
    args2 = (g.to(DEV), idx2.to(DEV), w.to(DEV), table.to(DEV))
    K.bag_backward_rows(*args2, acc, touched, row_sqnorm=sq, first_touch_writes=True)
    K.bag_backward_rows(*args2, ref, ref_t)
    assert torch.equal(acc[touched], ref[touched])
    torch.testing.assert_close(sq[touched], ref[touched].square().sum(-1), rtol=1e-5, atol=1e-6)
    n1 = K.touched_norm(acc, touched, row_sqnorm=sq)
    n2 = float(ref.double().norm())
    assert abs(float(n1) - n2) <= 1e-6 * n2


def test_keep_acc_step_equals_zeroing_step():
    gen = torch.Generator().manual_seed(2)
    rows, D = 2000, 64
    p = torch.randn(rows, D, generator=gen)
    acc = torch.randn(rows, D, generator=gen)
    touched = torch.rand(rows, generator=gen) < 0.4
    outs = []
    for keep in (False, True):
        pp, m, v, a, t = p.clone().to(DEV), torch.zeros(rows, D, device=DEV), torch.zeros(rows, D, device=DEV), \
            acc.clone().to(DEV), touched.clone().to(DEV)
        K.lazy_adam_step(pp, m, v, a, t, 1.0, 1, 1e-3, 0.9, 0.98, 1e-8, keep_acc=keep)
        outs.append((pp, m, v, a, t))
    for x, y in zip(outs[0][:3], outs[1][:3]):
        assert torch.equal(x, y)
    assert torch.equal(outs[1][3], acc.to(DEV))                 # kept
    assert torch.count_nonzero(outs[0][3][touched.to(DEV)]) == 0
    assert not outs[0][4].any() and not outs[1][4].any()


def test_clean_store_equals_exact_store_over_steps():
    """Two identical layers, two micro-batches per step, three steps: one store is never read from outside (clean
    mode), the other is read after every backward (exact mode). Tables, moments and clip norms agree."""
    mems = []
    for _ in range(2):
        torch.manual_seed(0)
        mems.append(ProductKeyMemory(64, 64, n_keys=64, heads=4, knn=16, k_dim=32, query_norm="none",
                                     swilu=False, value_grad="row_sparse").to(DEV))
    mems[1].load_state_dict(mems[0].state_dict())
    opts = [LazyRowAdam([m.values.weight], lr=1e-2, betas=(0.9, 0.98)) for m in mems]
    gen = torch.Generator().manual_seed(3)
    for step in range(3):
        norms = []
        for mb in range(2):
            x = torch.randn(300, 64, generator=gen).to(DEV)
            g = torch.randn(300, 64, generator=gen).to(DEV)
            for i, m in enumerate(mems):
                m(x).backward(g)
                if i == 1:
                    row_store(m.values.weight).acc       # read from outside: exact mode
        assert row_store(mems[0].values.weight).clean and not row_store(mems[1].values.weight).clean
        for m in mems:
            norms.append(float(clip_row_sparse([m.values.weight], 0.05)))
        assert abs(norms[0] - norms[1]) <= 1e-5 * norms[1]
        for m in mems:
            row_store(m.values.weight).grad_scale = 0.5        # identical clip factor in both
        for o in opts:
            o.step()
        assert torch.equal(mems[0].values.weight, mems[1].values.weight)
        for k in ("exp_avg", "exp_avg_sq"):
            assert torch.equal(opts[0].state[mems[0].values.weight][k], opts[1].state[mems[1].values.weight][k])
    # exposing the clean store yields the exact accumulator (all zero after the last step)
    st = row_store(mems[0].values.weight)
    assert torch.count_nonzero(st.acc) == 0 and not st.touched.any()


def test_deferred_rows_materialize_and_fused_step_bit_exact():
    """A deferred backward (row norms and touched marks now, rows later) materialises exactly the rows the
    write path produces, and the fused sum-and-Adam step equals materialising then stepping, bit for bit;
    hot rows make runs cross the 256-position work chunks."""
    gen = torch.Generator().manual_seed(4)
    rows, D, N, Kk = 20000, 384, 4096, 256                       # N K >= 2^20: 256-position chunks
    table = torch.randn(rows, D, generator=gen) * D ** -0.5
    idx = skewed_indices(rows, N, Kk, gen)
    w = torch.softmax(torch.randn(N, Kk, generator=gen), -1)
    g = torch.randn(N, D, generator=gen)
    T, I, W, G = (x.to(DEV) for x in (table, idx, w, g))
    # write path into a clean store
    acc_w = torch.randn(rows, D, generator=gen).to(DEV)          # stale garbage: first-touch writes ignore it
    t_w = torch.zeros(rows, dtype=torch.bool, device=DEV)
    sq_w = torch.zeros(rows, device=DEV)
    gw_w = K.bag_backward_rows(G, I, W, T, acc_w, t_w, row_sqnorm=sq_w, first_touch_writes=True)
    # deferred path
    t_d = torch.zeros(rows, dtype=torch.bool, device=DEV)
    sq_d = torch.zeros(rows, device=DEV)
    gw_d, pend = K.bag_backward_deferred(G, I, W, T, t_d, sq_d)
    assert torch.equal(t_d, t_w) and torch.equal(sq_d[t_d], sq_w[t_w]) and torch.equal(gw_d, gw_w)
    acc_d = torch.randn(rows, D, generator=gen).to(DEV)
    K.bag_rows_materialize(pend, acc_d)
    assert torch.equal(acc_d[t_d], acc_w[t_w])
    # fused step == materialise + lazy Adam step, with a clip factor and a bf16 value copy
    p0 = torch.randn(rows, D, generator=gen).to(DEV)
    m0 = (torch.randn(rows, D, generator=gen) * 1e-3).to(DEV)
    v0 = (torch.rand(rows, D, generator=gen) * 1e-5).to(DEV)
    scale = torch.tensor(0.37, device=DEV)
    outs = []
    for fused in (False, True):
        p, m, v = p0.clone(), m0.clone(), v0.clone()
        copy = p0.bfloat16()
        touched = t_w.clone()
        if fused:
            K.lazy_adam_deferred_step(p, m, v, touched, pend, scale, 3, 1e-2, 0.9, 0.98, 1e-8, value_copy=copy)
        else:
            K.lazy_adam_step(p, m, v, acc_w.clone(), touched, scale, 3, 1e-2, 0.9, 0.98, 1e-8, value_copy=copy,
                             keep_acc=True)
        assert not touched.any()
        outs.append((p, m, v, copy))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    assert torch.equal(outs[1][0][~t_w], p0[~t_w])               # unread rows untouched


@pytest.mark.parametrize("kind", ["rowrms", "rowadagrad"])
def test_deferred_rowwise_step_bit_exact(kind):
    """The row-wise step fused with a deferred backward's row sums equals materialising the rows and running
    rowwise_step, bit for bit (parameters, row state, step counts), with a clip factor; hot rows make runs cross
    the 256-position work chunks (the fix-up pass); unread rows and their state stay as they were."""
    gen = torch.Generator().manual_seed(6)
    rows, D, N, Kk = 20000, 384, 4096, 256
    table = torch.randn(rows, D, generator=gen) * D ** -0.5
    idx = skewed_indices(rows, N, Kk, gen)
    w = torch.softmax(torch.randn(N, Kk, generator=gen), -1)
    g = torch.randn(N, D, generator=gen)
    T, I, W, G = (x.to(DEV) for x in (table, idx, w, g))
    t_d = torch.zeros(rows, dtype=torch.bool, device=DEV)
    sq_d = torch.zeros(rows, device=DEV)
    _, pend = K.bag_backward_deferred(G, I, W, T, t_d, sq_d)
    acc = torch.zeros(rows, D, device=DEV)
    K.bag_rows_materialize(pend, acc)
    p0 = torch.randn(rows, D, generator=gen).to(DEV)
    v0 = (torch.rand(rows, generator=gen) * 1e-3).to(DEV)
    n0 = torch.randint(0, 5, (rows,), generator=gen, dtype=torch.int32).to(DEV)
    scale = torch.tensor(0.61, device=DEV)
    outs = []
    for fused in (False, True):
        p, v, n = p0.clone(), v0.clone(), n0.clone()
        touched = t_d.clone()
        if fused:
            K.rowwise_deferred_step(p, touched, v, n if kind == "rowrms" else None, pend, scale, 1e-2, 0.95, 1e-8,
                                    kind)
        else:
            K.rowwise_step(p, acc.clone(), touched, v, n if kind == "rowrms" else None, scale, 1e-2, 0.95, 1e-8,
                           kind, keep_acc=True)
        assert not touched.any()
        outs.append((p, v, n))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    assert torch.equal(outs[1][0][~t_d], p0[~t_d]) and torch.equal(outs[1][1][~t_d], v0[~t_d])
    assert not torch.equal(outs[1][0][t_d], p0[t_d])


def test_single_backward_steps_fused_equal_exact_store():
    """One backward per step (the fused path: the accumulator is never written) against a store read from
    outside after every backward (exact mode), three steps with clipping: tables and moments bit-identical."""
    mems = []
    for _ in range(2):
        torch.manual_seed(0)
        mems.append(ProductKeyMemory(64, 64, n_keys=64, heads=4, knn=16, k_dim=32, query_norm="none",
                                     swilu=False, value_grad="row_sparse").to(DEV))
    mems[1].load_state_dict(mems[0].state_dict())
    opts = [LazyRowAdam([m.values.weight], lr=1e-2, betas=(0.9, 0.98)) for m in mems]
    gen = torch.Generator().manual_seed(5)
    for step in range(3):
        x = torch.randn(300, 64, generator=gen).to(DEV)
        g = torch.randn(300, 64, generator=gen).to(DEV)
        for i, m in enumerate(mems):
            m(x).backward(g)
            if i == 1:
                row_store(m.values.weight).acc                   # exact mode
        assert row_store(mems[0].values.weight).pending is not None
        norms = [float(clip_row_sparse([m.values.weight], 0.05)) for m in mems]
        assert abs(norms[0] - norms[1]) <= 1e-5 * norms[1]
        for m in mems:
            row_store(m.values.weight).grad_scale = 0.5
        for o in opts:
            o.step()
        assert row_store(mems[0].values.weight).pending is None
        assert torch.equal(mems[0].values.weight, mems[1].values.weight)
        for k in ("exp_avg", "exp_avg_sq"):
            assert torch.equal(opts[0].state[mems[0].values.weight][k], opts[1].state[mems[1].values.weight][k])
