"""Edge cases of the CUDA path: empty batches through every entry point and the layer (nothing launched, empty
outputs, state unchanged), one-lookup bags (Engram's shape), rows wider than the deferred row-sum path takes
(512) and its exact fallback, the smallest tables a selection accepts."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from smlm_b200 import kernels as K
from smlm_b200.pkm import ProductKeyMemory
from smlm_b200.sparse_values import LazyRowAdam, row_store
from util import close

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_empty_batches():
    rows, D = 1000, 64
    gen = torch.Generator(device=DEV).manual_seed(0)
    table = torch.randn(rows, D, device=DEV, generator=gen)
    idx = torch.zeros(0, 8, dtype=torch.long, device=DEV)
    w = torch.zeros(0, 8, device=DEV)
    assert K.bag_forward(idx, w, table).shape == (0, D)
    assert K.bag_infer(idx, w, table, pre=torch.zeros(0, D, device=DEV), out_bf16=True).shape == (0, D)
    acc = torch.ones(rows, D, device=DEV)
    touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
    gw = K.bag_backward_rows(torch.zeros(0, D, device=DEV), idx, w, table, acc, touched)
    assert gw.shape == (0, 8) and bool((acc == 1).all()) and not bool(touched.any())
    s = torch.zeros(0, 4, 64, dtype=torch.bfloat16, device=DEV)
    for out, shape in zip(K.pk_select(s, s, 8), [(0, 4, 8)] * 3):
        assert out.shape == shape
    q = torch.zeros(0, 4, 256, dtype=torch.bfloat16, device=DEV)
    keys = torch.randn(4, 2, 64, 128, device=DEV, generator=gen).bfloat16()
    for out in K.score_select(q, keys, 8):
        assert out.shape == (0, 4, 8)
    torch.cuda.synchronize()


@pytest.mark.parametrize("autocast", [False, True])
def test_empty_batch_through_the_layer_and_step(autocast):
    torch.manual_seed(0)
    mem = ProductKeyMemory(64, 64, n_keys=64, heads=4, knn=8, k_dim=256, query_norm="none", swilu=False,
                           value_grad="row_sparse").to(DEV)
    opt = LazyRowAdam([mem.values.weight], lr=1e-2)
    before = mem.values.weight.detach().clone()
    x = torch.zeros(0, 64, device=DEV, requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        out = mem(x)
    assert out.shape == (0, 64)
    out.float().sum().backward()
    assert row_store(mem.values.weight).touched_rows() == 0
    opt.step()
    assert torch.equal(mem.values.weight.detach(), before)


def test_one_lookup_bags_scalar_rows_and_width_limit():
    """K = 1 (one row per bag, as Engram reads); D = 302 (not a multiple of 4: the scalar path, 10 values per
    lane); D = 384 through an unaligned view of a larger table (the scalar path too); bit-exact bags, accumulator
    under the kernel's chunk schedule. Rows wider than 512 values are refused, not cut."""
    from test_gpu_bag import chunk_positions
    gen = torch.Generator().manual_seed(3)
    for rows, D, N, Kk, unaligned in ((4000, 24, 5000, 1, False), (3000, 302, 64, 40, False),
                                      (3000, 384, 64, 40, True)):
        table = torch.randn(rows, D, generator=gen) * D ** -0.5
        idx = torch.randint(0, rows, (N, Kk), generator=gen)
        w = torch.rand(N, Kk, generator=gen)
        g = torch.randn(N, D, generator=gen)
        if unaligned:
            flat = torch.zeros(rows * D + 1, device=DEV)
            td = flat[1:].view(rows, D)
            td.copy_(table)
            assert td.data_ptr() % 16 != 0
        else:
            td = table.to(DEV)
        out = K.bag_forward(idx.to(DEV), w.to(DEV), td).cpu()
        ref, _ = O.bag_forward(idx.numpy(), w.numpy(), table.numpy())
        assert torch.equal(out, torch.from_numpy(ref))
        acc = torch.zeros(rows, D, device=DEV)
        touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
        gw = K.bag_backward_rows(g.to(DEV), idx.to(DEV), w.to(DEV), td, acc, touched).cpu()
        acc_o, t_o = np.zeros((rows, D), np.float32), np.zeros(rows, np.uint8)
        gw_o = O.bag_backward(g.numpy(), idx.numpy(), w.numpy(), table.numpy(), acc_o, t_o,
                              chunk=chunk_positions(N * Kk))
        assert torch.equal(acc.cpu(), torch.from_numpy(acc_o))
        assert torch.equal(touched.cpu(), torch.from_numpy(t_o.astype(bool)))
        close(gw, gw_o)
    wide = torch.zeros(100, 600, device=DEV)
    idx = torch.zeros(4, 2, dtype=torch.long, device=DEV)
    with pytest.raises(ValueError, match="wider"):
        K.bag_backward_rows(torch.zeros(4, 600, device=DEV), idx, torch.ones(4, 2, device=DEV), wide,
                            torch.zeros(100, 600, device=DEV), torch.zeros(100, dtype=torch.bool, device=DEV))
    with pytest.raises(ValueError, match="at most 512"):
        ProductKeyMemory(600, 600, n_keys=16, heads=2, knn=4, k_dim=32, query_norm="none", swilu=False,
                         value_grad="row_sparse")


def test_scalar_rows_through_the_layer_match_exact_store():
    """A 302-wide value table (scalar rows, no deferred row sums) trains like the reference semantics: two
    layers, one read from outside after every backward (exact store), equal after three LazyRowAdam steps."""
    mems = []
    for _ in range(2):
        torch.manual_seed(0)
        mems.append(ProductKeyMemory(302, 302, n_keys=32, heads=2, knn=8, k_dim=64, query_norm="none",
                                     swilu=False, value_grad="row_sparse").to(DEV))
    opts = [LazyRowAdam([m.values.weight], lr=1e-2) for m in mems]
    gen = torch.Generator().manual_seed(9)
    for _ in range(3):
        x = torch.randn(50, 302, generator=gen).to(DEV)
        g = torch.randn(50, 302, generator=gen).to(DEV)
        for i, m in enumerate(mems):
            m(x).backward(g)
            if i == 1:
                row_store(m.values.weight).acc
        for o in opts:
            o.step()
    assert torch.equal(mems[0].values.weight, mems[1].values.weight)


def test_smallest_tables_select_all_keys():
    """knn == n_keys (every sub-key of a half selected) for the exact selection and the fused kernel."""
    gen = torch.Generator().manual_seed(2)
    q = torch.randn(40, 2, 128, generator=gen).bfloat16().to(DEV)
    keys = (torch.randn(2, 2, 8, 64, generator=gen) * 0.1).bfloat16().to(DEV)
    sc, idx, w, s1, s2 = K.score_select(q, keys, 8, dump=True)
    from util import bits_of_bf16
    osc, oidx, ow = O.select(bits_of_bf16(s1), bits_of_bf16(s2), 8, bf16=True)
    assert np.array_equal(idx.cpu().numpy(), oidx) and np.array_equal(bits_of_bf16(sc), osc)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_small_batch_bag_ring_wraps(dtype):
    """Few tokens with many lookups: the small-batch bag's four in-flight chunks of 32 lookups wrap around its
    ring (K = 300: ten chunks, the last one partial), rows out of range in between are skipped and flagged."""
    gen = torch.Generator().manual_seed(12)
    rows, D, N, Kk = 5000, 64, 7, 300
    table = torch.randn(rows, D, generator=gen) * D ** -0.5
    idx = torch.randint(0, rows, (N, Kk), generator=gen)
    w = torch.rand(N, Kk, generator=gen)
    t = table.to(dtype)
    out = K.bag_forward(idx.to(DEV), w.to(DEV), t.to(DEV)).cpu()
    from util import bits_of_bf16
    if dtype == torch.bfloat16:
        ref, _ = O.bag_forward(idx.numpy(), w.numpy(), bits_of_bf16(t), bf16=True)
    else:
        ref, _ = O.bag_forward(idx.numpy(), w.numpy(), table.numpy())
    assert torch.equal(out, torch.from_numpy(ref))
    bad = idx.clone()
    bad[3, 100] = rows
    with pytest.raises(IndexError, match="out of range"):
        K.bag_forward(bad.to(DEV), w.to(DEV), t.to(DEV))
