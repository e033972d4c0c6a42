"""The fused tensor-core scoring + selection kernel (score_tc.cu): its bf16 sub-key scores equal the bf16 einsum
of the reference's autocast path to within one bf16 rounding step (fp32 summation order differs), and its
selection equals the oracle's canonical selection on its own scores bit for bit."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from smlm_b200 import kernels as K
from util import bits_of_bf16, exact_contractions, within_bf16

pytestmark = pytest.mark.gpu
DEV = "cuda"


def inputs(N, H, NK, half, seed):
    gen = torch.Generator().manual_seed(seed)
    q = (torch.randn(N, H, 2 * half, generator=gen)).bfloat16()
    keys = (torch.randn(H, 2, NK, half, generator=gen) * half ** -0.5).bfloat16()
    return q.to(DEV), keys.to(DEV)


def einsum_scores(q, keys):
    half = keys.shape[-1]
    s1 = torch.einsum("nhd,hkd->nhk", q[..., :half], keys[:, 0])
    s2 = torch.einsum("nhd,hkd->nhk", q[..., half:], keys[:, 1])
    return s1, s2


@pytest.mark.parametrize("N,H,NK,half,knn", [
    (128, 1, 128, 128, 32), (1000, 4, 1024, 128, 32), (300, 2, 256, 64, 8), (77, 3, 200, 128, 5),
    (4096, 4, 4096, 128, 32), (1, 4, 512, 128, 32), (257, 1, 40, 64, 4)])
def test_fused_selection_bit_exact_on_its_scores(N, H, NK, half, knn):
    q, keys = inputs(N, H, NK, half, N + NK)
    sc, idx, w, s1, s2 = K.score_select(q, keys, knn, dump=True)
    osc, oidx, ow = O.select(bits_of_bf16(s1), bits_of_bf16(s2), knn, bf16=True)
    assert np.array_equal(bits_of_bf16(sc), osc)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=0, atol=1e-6)
    # the kernel's scores are the bf16 GEMM scores: within one bf16 step of cuBLAS's, almost always equal
    e1, e2 = einsum_scores(q, keys)
    for a, b in ((s1, e1), (s2, e2)):
        a, b = a.float(), b.float()
        ulp = torch.where(b == 0, torch.full_like(b, 2.0 ** -133), b.abs() * 2.0 ** -7)
        assert bool(((a - b).abs() <= ulp).all())
        assert float((a == b).float().mean()) > 0.99


def test_fused_matches_unfused_selection():
    """Same selection as einsum + pk_select wherever the two bf16 score tensors agree on the row."""
    q, keys = inputs(2048, 4, 1024, 128, 5)
    sc, idx, w, s1, s2 = K.score_select(q, keys, 32, dump=True)
    e1, e2 = einsum_scores(q, keys)
    psc, pidx, pw = K.pk_select(e1, e2, 32)
    same = ((s1 == e1).all(-1) & (s2 == e2).all(-1)).cpu()
    assert float(same.float().mean()) > 0.5
    assert torch.equal(idx.cpu()[same], pidx.cpu()[same])
    assert torch.equal(sc.cpu()[same], psc.cpu()[same])


def test_fused_determinism_and_ties():
    """Coarse keys / queries produce exact score ties at every stage; two runs are bit-identical and equal the
    oracle on the kernel's scores."""
    gen = torch.Generator().manual_seed(9)
    N, H, NK, half = 512, 2, 512, 128
    q = torch.randint(-2, 3, (N, H, 2 * half), generator=gen).bfloat16().to(DEV)
    keys = (torch.randint(-1, 2, (H, 2, NK, half), generator=gen).float() / 8).bfloat16().to(DEV)
    a = K.score_select(q, keys, 32, dump=True)
    b = K.score_select(q, keys, 32)
    assert torch.equal(a[1], b[1]) and torch.equal(a[0], b[0]) and torch.equal(a[2], b[2])
    osc, oidx, _ = O.select(bits_of_bf16(a[3]), bits_of_bf16(a[4]), 32, bf16=True)
    assert np.array_equal(a[1].cpu().numpy(), oidx)


def test_score_select_backward_matches_unfused():
    """ScoreSelect's backward on its own selection equals the exact (float64) contraction of the dense selection
    backward's bf16 score gradients within one bf16 rounding plus fp32 accumulation error, the bound the
    reference's autocast einsum backward meets; on every (token, head) whose selection and selected scores the
    einsum + PKSelect path reproduces, dq rows agree with that path's within twice that bound."""
    N, H, NK, half, knn = 512, 4, 256, 128, 32
    q, keys = inputs(N, H, NK, half, 3)
    gen = torch.Generator().manual_seed(4)
    gw = torch.randn(N, H, knn, generator=gen).to(DEV)
    qa, ka = q.clone().requires_grad_(), keys.clone().requires_grad_()
    sc, idx, w = K.ScoreSelect.apply(qa, ka, knn)
    (w * gw).sum().backward()
    # the fused path against the exact contraction of its own selection's dense score gradients
    ds1, ds2 = K.select_backward(idx, w.detach(), gw, torch.zeros_like(sc), NK, torch.bfloat16)
    edq, mq, edk, mk = exact_contractions(ds1, ds2, q, keys)
    within_bf16(qa.grad, edq, mq, "dq")
    within_bf16(ka.grad, edk, mk, "dkeys")
    assert qa.grad.abs().sum() > 0 and ka.grad.abs().sum() > 0
    # the unfused path (einsum scores + PKSelect): dq of a (token, head) depends on that row's selection only
    qb, kb = q.clone().requires_grad_(), keys.clone().requires_grad_()
    s1, s2 = einsum_scores(qb, kb)
    sc2, idx2, w2 = K.PKSelect.apply(s1, s2, knn)
    (w2 * gw).sum().backward()
    same = (idx == idx2).all(-1) & (sc == sc2).all(-1)
    assert float(same.float().mean()) > 0.5
    n_cmp = int(same.sum())
    assert n_cmp > 0
    ds1b, ds2b = K.select_backward(idx2, w2.detach(), gw, torch.zeros_like(sc), NK, torch.bfloat16)
    edqb, mqb, _, _ = exact_contractions(ds1b, ds2b, q, keys)
    within_bf16(qb.grad, edqb, mqb, "unfused dq")
    a, b = qa.grad.double()[same], qb.grad.double()[same]
    bound = 2 * (edq[same].abs() * 2.0 ** -8 + mq[same] * 2.0 ** -16) + 1e-30
    assert bool(((a - b).abs() <= bound).all()), f"dq differs on rows with the same selection ({n_cmp} rows)"


@pytest.mark.parametrize("N", [1024, 8])
def test_fused_scores_against_fp32_contraction(N):
    """The bf16 sub-key scores (N = 1024: the tensor-core kernel; N = 8: the few-token SIMT kernel) against a
    float64 CPU contraction of the same bf16 operands: every score lies within one bf16 rounding of the exact value
    plus fp32 accumulation error, and nearly all of them are the exact value rounded once to bf16 (round to
    nearest even)."""
    H, NK, half = 4, 1024, 128
    q, keys = inputs(N, H, NK, half, 17)
    _, _, _, s1, s2 = K.score_select(q, keys, 32, dump=True)
    qc, kc = q.double().cpu(), keys.double().cpu()
    for c, s in ((0, s1), (1, s2)):
        qh = qc[..., c * half:(c + 1) * half]
        exact = torch.einsum("nhd,hkd->nhk", qh, kc[:, c])
        mag = torch.einsum("nhd,hkd->nhk", qh.abs(), kc[:, c].abs())
        got = s.double().cpu()
        err = (got - exact).abs()
        assert bool((err <= exact.abs() * 2.0 ** -8 + mag * 2.0 ** -16 + 1e-30).all())
        once = exact.float().bfloat16().double()           # rounded to fp32 (exact here), then once to bf16
        assert float((got == once).double().mean()) > 0.99


@pytest.mark.parametrize("n_small", [64, 130, 600])
def test_key_range_splits_match_full_sweep(n_small):
    """Few token tiles (decoding, short prompts) split each (tile, head)'s key tiles over several CTAs, each with
    its own top lists, merged by the pair kernel. A token's scores do not depend on the other tokens of its tile,
    so the first n_small tokens alone (split sweep) select exactly what they select inside a batch of 37 tiles x
    4 heads = 148 units (one unsplit sweep per unit)."""
    q, keys = inputs(37 * 128, 4, 4096, 128, 11)
    full = K.score_select(q, keys, 32)
    part = K.score_select(q[:n_small].contiguous(), keys, 32)
    for a, b in zip(part, full):
        assert torch.equal(a, b[:n_small])


@pytest.mark.parametrize("n_small", [1, 3, 16])
def test_few_token_path_against_tensor_core_sweep(n_small):
    """Calls of at most 16 tokens (decoding) score on the SIMT cores (score_small_kernel: an fp32 fmaf chain per
    sub-key, rounded once to bf16) instead of the tensor cores. Their scores are the tensor-core sweep's up to the
    order of the fp32 additions: within one bf16 step, equal almost everywhere; on every (token, head) whose scores
    agree the selection, weights and order are identical; and on its own scores the selection is the oracle's."""
    q, keys = inputs(37 * 128, 4, 4096, 128, 11)
    full = K.score_select(q, keys, 32, dump=True)
    part = K.score_select(q[:n_small].contiguous(), keys, 32, dump=True)
    fs1, fs2 = (x[:n_small].float() for x in full[3:])
    ps1, ps2 = (x.float() for x in part[3:])
    qs, kf = q[:n_small].float(), keys.float()
    for c, (a, b) in enumerate(((ps1, fs1), (ps2, fs2))):
        # one bf16 rounding of either sum, plus the fp32 accumulation error of a 128-term sum (which dominates
        # where the terms cancel)
        mag = torch.einsum("nhd,hkd->nhk", qs[..., c * 128:(c + 1) * 128].abs(), kf[:, c].abs())
        bound = (a.abs() + b.abs()) * 2.0 ** -8 + mag * 2.0 ** -16 + 2.0 ** -133
        assert bool(((a - b).abs() <= bound).all())
        assert float((a == b).float().mean()) > 0.999
    same = ((ps1 == fs1).all(-1) & (ps2 == fs2).all(-1))
    assert int(same.sum()) > 0
    for a, b in zip(part[:3], full[:3]):
        assert torch.equal(a[same], b[:n_small][same])
    osc, oidx, ow = O.select(bits_of_bf16(part[3]), bits_of_bf16(part[4]), 32, bf16=True)
    assert np.array_equal(bits_of_bf16(part[0]), osc)
    assert np.array_equal(part[1].cpu().numpy(), oidx)
    np.testing.assert_allclose(part[2].cpu().numpy(), ow, rtol=0, atol=1e-6)
