"""The sparse selection backward: the per-sub-key lookups it emits carry exactly the dense selection backward's
nonzero gradients, and dq / dkeys computed from them (a value bag over the keys and its row-sparse backward) agree
with the exact contraction of the dense gradients within fp32-accumulation + one bf16 rounding, as the
reference's autocast einsum backward (reference: kernels.py:253-266, pkm.py:117-123)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from smlm_b200 import kernels as K
from util import close, exact_contractions, within_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def selection(N, H, NK, knn, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    s1 = torch.randn(N, H, NK, generator=gen).to(dtype).to(DEV)
    s2 = torch.randn(N, H, NK, generator=gen).to(dtype).to(DEV)
    _, idx, w = K.pk_select(s1, s2, knn)
    g_w = torch.randn(N, H, knn, generator=gen).to(DEV)
    g_s = torch.randn(N, H, knn, generator=gen).to(dtype).to(DEV)
    return idx, w, g_w, g_s


def scatter_entries(rows, ew, N, H, NK):
    """(N H 2, knn) lookups -> dense (N, H, NK) ds1, ds2 (the -1 rows of repeated sub-keys carry nothing)."""
    first = rows >= 0
    dense = torch.zeros(N * H * 2, NK, dtype=ew.dtype, device=DEV)
    r = torch.nonzero(first)[:, 0]
    dense[r, rows[first] % NK] = ew[first]                    # each sub-key once per (token, head, half)
    dense = dense.view(N, H, 2, NK)
    return dense[:, :, 0], dense[:, :, 1]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_entries_carry_the_dense_gradients(dtype):
    N, H, NK, knn = 1024, 4, 256, 32
    idx, w, g_w, g_s = selection(N, H, NK, knn, dtype, 1)
    ds1, ds2 = K.select_backward(idx, w, g_w, g_s, NK, dtype)
    rows, ew = K.select_grad_entries(idx, w, g_w, g_s, NK, dtype)
    assert rows.shape == (N * H * 2, knn) and ew.dtype == dtype
    # first occurrences: row (head * 2 + half) * NK + the pair's sub-key in that half; later ones: -1, weight 0
    r = rows.view(N, H, 2, knn)
    e = ew.view(N, H, 2, knn)
    hh = torch.arange(H, device=DEV).view(1, H, 1)
    for c, sub in ((0, idx // NK), (1, idx % NK)):
        later = torch.zeros_like(sub, dtype=torch.bool)
        for j in range(1, knn):
            later[..., j] = (sub[..., :j] == sub[..., j:j + 1]).any(-1)
        assert torch.equal(r[:, :, c], torch.where(later, torch.full_like(sub, -1), (hh * 2 + c) * NK + sub))
        assert torch.count_nonzero(e[:, :, c][later]) == 0
    # each sub-key's gradient sits on its first occurrence, bit for bit the dense value
    d1, d2 = scatter_entries(rows, ew, N, H, NK)
    assert torch.equal(d1, ds1) and torch.equal(d2, ds2)


@pytest.mark.parametrize("N,H,NK,half", [(1024, 4, 256, 64), (4096, 4, 4096, 128)])
def test_sparse_contractions_match_exact_dense(N, H, NK, half):
    knn = 32
    gen = torch.Generator().manual_seed(5)
    q = (torch.randn(N, H, 2 * half, generator=gen)).bfloat16().to(DEV)
    keys = (torch.randn(H, 2, NK, half, generator=gen) * half ** -0.5).bfloat16().to(DEV)
    idx, w, g_w, g_s = selection(N, H, NK, knn, torch.bfloat16, 6)
    ds1, ds2 = K.select_backward(idx, w, g_w, g_s, NK, torch.bfloat16)
    dq, dk = K.scoring_backward_sparse(q, keys, idx, w, g_w, g_s)
    assert dq.dtype == torch.bfloat16 and dk.dtype == torch.bfloat16
    assert dq.shape == q.shape and dk.shape == keys.shape
    edq, mq, edk, mk = exact_contractions(ds1, ds2, q, keys)
    within_bf16(dq, edq, mq, "dq")
    within_bf16(dk, edk, mk, "dkeys")
    # the cuBLAS contraction of the dense gradients (the reference's autocast backward) meets the same bound
    ref_dk = torch.stack([torch.einsum("nhk,nhd->hkd", ds1, q[..., :half]),
                          torch.einsum("nhk,nhd->hkd", ds2, q[..., half:])], 1)
    within_bf16(ref_dk, edk, mk, "dense dkeys")
    # keys no selection reads get exactly zero
    used = torch.zeros(H * 2 * NK, dtype=torch.bool, device=DEV)
    rows, ew = K.select_grad_entries(idx, w, g_w, g_s, NK, torch.bfloat16)
    used[rows.view(-1)[(rows.view(-1) >= 0) & (ew.view(-1) != 0)]] = True
    assert torch.count_nonzero(dk.view(H * 2 * NK, half)[~used]) == 0


def test_sparse_backward_is_deterministic():
    N, H, NK, half, knn = 2048, 4, 1024, 128, 32
    gen = torch.Generator().manual_seed(7)
    q = torch.randn(N, H, 2 * half, generator=gen).bfloat16().to(DEV)
    keys = torch.randn(H, 2, NK, half, generator=gen).bfloat16().to(DEV)
    idx, w, g_w, g_s = selection(N, H, NK, knn, torch.bfloat16, 8)
    a = K.scoring_backward_sparse(q, keys, idx, w, g_w, g_s)
    b = K.scoring_backward_sparse(q, keys, idx, w, g_w, g_s)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_shard_entry_points_match_oracle(idx_dtype):
    """The row-shard bag forward / backward over global indices equal the oracle on the local rows, with the
    other shards' lookups removed, bit for bit (same summation order and chunk schedule); bf16 grad_out; those
    lookups get gw 0 and mark nothing."""
    gen = torch.Generator().manual_seed(9)
    R, D, N, Kk = 12000, 128, 2048, 64
    base, rows = 4000, 3000
    idx = torch.randint(0, R, (N, Kk), generator=gen)
    hot = torch.randint(base, base + rows, (4,), generator=gen)
    m = torch.rand(N, Kk, generator=gen) < 0.25
    idx[m] = hot[torch.randint(0, 4, (int(m.sum()),), generator=gen)]
    idx[0] = -1                                       # padding lookups are skipped as well
    w = torch.randn(N, Kk, generator=gen)
    g = torch.randn(N, D, generator=gen).bfloat16()
    shard = torch.randn(rows, D, generator=gen)
    local = idx - base
    local = torch.where((local >= 0) & (local < rows), local, torch.full_like(local, -1))
    # forward
    out = K.shard_bag_forward(idx.to(idx_dtype).to(DEV), w.to(DEV), shard.to(DEV), base)
    o_out, _ = O.bag_forward(local.numpy(), w.numpy(), shard.numpy())
    assert np.array_equal(out.cpu().numpy(), o_out)
    # backward into a pre-filled accumulator
    acc0 = torch.randn(rows, D, generator=gen)
    acc = acc0.clone().to(DEV)
    touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
    gw = K.shard_bag_backward_rows(g.to(DEV), idx.to(idx_dtype).to(DEV), w.to(DEV), shard.to(DEV), base, acc,
                                   touched)
    o_acc = acc0.numpy().copy()
    o_t = np.zeros(rows, np.uint8)
    P = 256 if N * Kk >= 1 << 20 else 64
    o_gw = O.bag_backward(g.float().numpy(), local.numpy(), w.numpy(), shard.numpy(), o_acc, o_t, chunk=P)
    assert np.array_equal(acc.cpu().numpy(), o_acc)
    assert np.array_equal(touched.cpu().numpy(), o_t.astype(bool))
    close(gw.cpu(), o_gw)                              # dot products: lane partials + a warp tree
    assert torch.count_nonzero(gw.cpu()[local < 0]) == 0


def test_slot_sum_order():
    gen = torch.Generator().manual_seed(10)
    x = (torch.randn(5, 1001, generator=gen) * torch.logspace(-3, 3, 5).view(5, 1)).to(DEV)
    ref = x[0].clone()
    for s in range(1, 5):
        ref = ref + x[s]
    assert torch.equal(K.slot_sum(x), ref)
    y = x[:, :1000].contiguous()                     # vectorised path (count % 4 == 0)
    ref4 = y[0].clone()
    for s in range(1, 5):
        ref4 = ref4 + y[s]
    assert torch.equal(K.slot_sum(y), ref4)
