"""Selection and scoring kernels on the GPU: bit-identical scores / indices / order to the C oracle (canonical
order: score descending, index ascending), the reference's golden selections on tie-free rows, weights within
1e-6 (the reference's own bound, its tests/test_kernels.py:152)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from smlm_b200 import kernels as K
from util import bf16_from_bits, bits_of_bf16, golden, tie_free_rows

pytestmark = pytest.mark.gpu
DEV = "cuda"


def gpu_vs_oracle(s1, s2, knn):
    """s1, s2 torch (CPU) bf16 or fp32 -> asserts the GPU equals the oracle bit for bit."""
    bf16 = s1.dtype == torch.bfloat16
    sc, idx, w = K.pk_select(s1.to(DEV), s2.to(DEV), knn)
    if bf16:
        osc, oidx, ow = O.select(bits_of_bf16(s1), bits_of_bf16(s2), knn, bf16=True)
        assert np.array_equal(bits_of_bf16(sc), osc)
    else:
        osc, oidx, ow = O.select(s1.numpy(), s2.numpy(), knn, bf16=False)
        assert np.array_equal(sc.cpu().numpy(), osc)
    assert np.array_equal(idx.cpu().numpy(), oidx)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=0, atol=1e-6)
    return sc, idx, w


def test_pk_select_bf16_golden():
    g = golden("select_bf16.npz")
    for c in range(int(g["n_cases"])):
        N, H, NK, knn = (int(x) for x in g[f"c{c}_shape"])
        s1, s2 = bf16_from_bits(g[f"c{c}_s1"]), bf16_from_bits(g[f"c{c}_s2"])
        sc, idx, w = gpu_vs_oracle(s1, s2, knn)
        assert np.array_equal(bits_of_bf16(sc), g[f"c{c}_triton_scores"])    # the reference kernel's scores
        free = tie_free_rows(s1, s2, knn, bf16=True)
        oi = np.sort(idx.cpu().numpy().reshape(-1, knn), -1)
        ti = np.sort(g[f"c{c}_triton_idx"].reshape(-1, knn), -1)
        assert np.array_equal(oi[free], ti[free])
        np.testing.assert_allclose(w.cpu().numpy(), g[f"c{c}_triton_w"], rtol=0, atol=1e-6)


def test_pk_select_f32_golden():
    g = golden("select_f32.npz")
    for c in range(int(g["n_cases"])):
        N, H, NK, knn, kd = (int(x) for x in g[f"c{c}_shape"])
        s1, s2 = torch.from_numpy(g[f"c{c}_s1"]), torch.from_numpy(g[f"c{c}_s2"])
        sc, idx, w = gpu_vs_oracle(s1, s2, knn)
        assert np.array_equal(sc.cpu().numpy(), g[f"c{c}_scores"])
        assert np.array_equal(np.sort(idx.cpu().numpy(), -1), np.sort(g[f"c{c}_idx"], -1))


@pytest.mark.parametrize("N,H,NK,knn", [(4096, 4, 512, 32), (1024, 4, 1024, 32), (1024, 4, 4096, 32),
                                         (1, 4, 1024, 32), (300, 3, 100, 5), (64, 2, 16, 16), (50, 4, 24, 1),
                                         (257, 4, 65536, 32)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pk_select_random_vs_oracle(N, H, NK, knn, dtype):
    gen = torch.Generator().manual_seed(N + NK + knn)
    s1 = torch.randn(N, H, NK, generator=gen).to(dtype)
    s2 = torch.randn(N, H, NK, generator=gen).to(dtype)
    gpu_vs_oracle(s1, s2, knn)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("levels", [2, 5, 17])
def test_pk_select_many_ties(dtype, levels):
    """Scores on a coarse grid: ties at every stage, including pairs outside the dominance-pruned candidate set
    that tie with the knn-th score; the lower index must win everywhere."""
    gen = torch.Generator().manual_seed(levels)
    N, H, NK, knn = 512, 4, 256, 32
    s1 = (torch.randint(0, levels, (N, H, NK), generator=gen).float() / levels).to(dtype)
    s2 = (torch.randint(0, levels, (N, H, NK), generator=gen).float() / levels).to(dtype)
    gpu_vs_oracle(s1, s2, knn)
    z = torch.zeros(N, H, NK, dtype=dtype)
    z[:, :, 7] = -0.0                                       # -0 and +0 tie
    gpu_vs_oracle(z, z.clone(), knn)


@pytest.mark.parametrize("N,H,NK,half", [(300, 4, 256, 128), (64, 3, 16, 8), (77, 2, 100, 13), (4100, 4, 64, 128)])
def test_subkey_scores_f32_bit_exact(N, H, NK, half):
    gen = torch.Generator().manual_seed(N)
    q = torch.randn(N, H, 2 * half, generator=gen)
    keys = torch.randn(H, 2, NK, half, generator=gen) * half ** -0.5
    s1, s2 = K.subkey_scores_f32(q.to(DEV), keys.to(DEV))
    o1, o2 = O.subkey_scores_f32(q.numpy(), keys.numpy())
    assert np.array_equal(s1.cpu().numpy(), o1) and np.array_equal(s2.cpu().numpy(), o2)


def test_exact_fp32_pipeline_indices_bit_exact():
    """End to end in fp32: fmaf-chain scores + selection on the GPU = the C oracle's pipeline, index for index."""
    gen = torch.Generator().manual_seed(11)
    N, H, NK, half, knn = 2048, 4, 256, 128, 32
    q = torch.randn(N, H, 2 * half, generator=gen) * 0.5
    keys = torch.randn(H, 2, NK, half, generator=gen) * half ** -0.5
    s1, s2 = K.subkey_scores_f32(q.to(DEV), keys.to(DEV))
    sc, idx, w = K.pk_select(s1, s2, knn)
    o1, o2 = O.subkey_scores_f32(q.numpy(), keys.numpy())
    osc, oidx, ow = O.select(o1, o2, knn, bf16=False)
    assert np.array_equal(idx.cpu().numpy(), oidx) and np.array_equal(sc.cpu().numpy(), osc)


def test_select_backward_vs_oracle_and_golden():
    g = golden("select_backward.npz")
    N, H, NK, knn = (int(x) for x in g["shape"])
    s1, s2 = bf16_from_bits(g["s1"]).to(DEV).requires_grad_(), bf16_from_bits(g["s2"]).to(DEV).requires_grad_()
    gg = torch.from_numpy(g["g"]).to(DEV)
    sc, idx, w = K.PKSelect.apply(s1, s2, knn)
    (w * gg).sum().backward()
    e1, e2 = bf16_from_bits(g["ds1"]).float(), bf16_from_bits(g["ds2"]).float()
    scale = float(e1.abs().max())
    torch.testing.assert_close(s1.grad.cpu().float(), e1, rtol=2 ** -7, atol=2 ** -8 * scale)
    torch.testing.assert_close(s2.grad.cpu().float(), e2, rtol=2 ** -7, atol=2 ** -8 * scale)
    for dtype in (torch.bfloat16, torch.float32):
        gen = torch.Generator().manual_seed(3)
        N, H, NK, knn = 512, 4, 256, 32
        a = torch.randn(N, H, NK, generator=gen).to(dtype).to(DEV)
        b = torch.randn(N, H, NK, generator=gen).to(dtype).to(DEV)
        _, idx, w = K.pk_select(a, b, knn)
        gw = torch.randn(N, H, knn, generator=gen).to(DEV)
        gs = torch.randn(N, H, knn, generator=gen).to(dtype).to(DEV)
        d1, d2 = K.select_backward(idx, w, gw, gs, NK, dtype)
        bf = dtype == torch.bfloat16
        enc = (lambda t: bits_of_bf16(t)) if bf else (lambda t: t.cpu().numpy())
        o1, o2 = O.select_backward(idx.cpu().numpy(), w.cpu().numpy(), gw.cpu().numpy(), enc(gs), NK, bf16=bf)
        dec = (lambda a_: bf16_from_bits(a_).float()) if bf else torch.from_numpy
        r1, r2 = dec(o1), dec(o2)
        tol = dict(rtol=2 ** -7, atol=2 ** -8 * float(r1.abs().max())) if bf else dict(rtol=1e-5, atol=1e-6)
        torch.testing.assert_close(d1.cpu().float(), r1, **tol)
        torch.testing.assert_close(d2.cpu().float(), r2, **tol)


def test_product_key_topk_equals_bruteforce():
    """The reference's tests/test_pkm.py:16-37 on the GPU kernels: the product-key search returns exactly the
    top-k of a brute-force search over all n_keys^2 keys, every score belonging to its index."""
    gen = torch.Generator().manual_seed(1)
    for n_keys, knn in ((16, 8), (16, 16), (32, 5), (8, 1), (64, 32)):
        H, half = 3, 8
        keys = torch.randn(H, 2, n_keys, half, generator=gen)
        q = torch.randn(200, H, 2 * half, generator=gen)
        s1, s2 = K.subkey_scores_f32(q.to(DEV), keys.to(DEV))
        sc, idx, _ = K.pk_select(s1, s2, knn)
        full = (s1[..., :, None] + s2[..., None, :]).reshape(200, H, -1)
        bf, bi = full.topk(knn, dim=-1)
        assert torch.equal(sc, bf)
        assert torch.equal(idx.sort(-1).values, bi.sort(-1).values)
