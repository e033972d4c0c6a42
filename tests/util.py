"""Shared helpers of the tests (no GPU needed to import)."""
import os

import numpy as np
import torch

from conftest import GOLDEN


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def bf16_from_bits(b):
    """uint16 numpy bit patterns -> torch bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def bits_of_bf16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def close(a, b, rtol=1e-5, atol=1e-5, msg=""):
    """assert_close relative to the reference's scale (the reference's tests/test_kernels.py:48-52)."""
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    scale = max(1.0, float(b.abs().max())) if b.numel() else 1.0
    torch.testing.assert_close(a / scale, b / scale, rtol=rtol, atol=atol, msg=msg)


def skewed_indices(rows, N, K, gen):
    """Uniform rows plus 20% of the reads on 8 hot rows, so that runs of equal rows cross work chunks
    (the reference's tests/test_kernels.py:55-61)."""
    idx = torch.randint(0, rows, (N, K), generator=gen)
    hot = torch.randint(0, rows, (8,), generator=gen)
    mask = torch.rand(N, K, generator=gen) < 0.2
    idx[mask] = hot[torch.randint(0, 8, (int(mask.sum()),), generator=gen)]
    return idx


def tie_free_rows(s1, s2, knn, bf16):
    """Rows (flattened n*h) where no unselected pair of the knn x knn product ties with the knn-th selected
    score under (score desc) alone: on those rows every correct selector returns the same index set."""
    s1 = torch.as_tensor(s1).float()
    s2 = torch.as_tensor(s2).float()
    N, H, NK = s1.shape
    a1, _ = s1.sort(-1, descending=True)
    a2, _ = s2.sort(-1, descending=True)
    a1, a2 = a1[..., :knn], a2[..., :knn]
    alls = (a1.unsqueeze(-1) + a2.unsqueeze(-2))
    if bf16:
        alls = alls.bfloat16().float()
    alls = alls.view(N * H, -1)
    srt, _ = alls.sort(-1, descending=True)
    T = srt[:, knn - 1:knn]
    n_eq_total = (alls == T).sum(-1)
    n_eq_sel = (srt[:, :knn] == T).sum(-1)
    # half-level ties at the knn-th sub-key score also make the index set ambiguous
    h1 = (s1.view(N * H, NK) == a1.reshape(N * H, knn)[:, -1:]).sum(-1) > 1
    h2 = (s2.view(N * H, NK) == a2.reshape(N * H, knn)[:, -1:]).sum(-1) > 1
    return ((n_eq_total == n_eq_sel) & ~h1 & ~h2).numpy()


def exact_contractions(ds1, ds2, q, keys):
    """float64 dq, dkeys and the magnitudes sum |term| of the dense contractions."""
    half = keys.shape[-1]
    d1, d2 = ds1.double(), ds2.double()
    qd, kd = q.double(), keys.double()
    dq = torch.cat([torch.einsum("nhk,hkd->nhd", d1, kd[:, 0]), torch.einsum("nhk,hkd->nhd", d2, kd[:, 1])], -1)
    mq = torch.cat([torch.einsum("nhk,hkd->nhd", d1.abs(), kd[:, 0].abs()),
                    torch.einsum("nhk,hkd->nhd", d2.abs(), kd[:, 1].abs())], -1)
    dk = torch.stack([torch.einsum("nhk,nhd->hkd", d1, qd[..., :half]),
                      torch.einsum("nhk,nhd->hkd", d2, qd[..., half:])], 1)
    mk = torch.stack([torch.einsum("nhk,nhd->hkd", d1.abs(), qd[..., :half].abs()),
                      torch.einsum("nhk,nhd->hkd", d2.abs(), qd[..., half:].abs())], 1)
    return dq, mq, dk, mk


def within_bf16(ours, exact, mag, what):
    """|ours - exact| <= one bf16 rounding of the result + fp32 accumulation error (2^-16 of sum |term|)."""
    err = (ours.double() - exact).abs()
    bound = exact.abs() * 2.0 ** -8 + mag * 2.0 ** -16 + 1e-30
    bad = err > bound
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} entries off, max err {float(err.max())}"
