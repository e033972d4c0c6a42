"""Row-sparse optimizer kernels on the GPU: bit-identical to the reference's own C row loops (host_rows.c,
compiled into oracle/_ref) and to the C oracle, within rel 1e-5 of the reference's PyTorch path (golden)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import torch_path as TP
from smlm_b200 import kernels as K
from smlm_b200.row_optim import RowWiseOptimizer
from smlm_b200.sparse_values import LazyRowAdam, clip_row_sparse, row_store
from util import close, golden, skewed_indices

pytestmark = pytest.mark.gpu
DEV = "cuda"


def random_state(rows, D, seed, frac=0.3):
    gen = torch.Generator().manual_seed(seed)
    p = torch.randn(rows, D, generator=gen) * D ** -0.5
    m = torch.randn(rows, D, generator=gen) * 1e-3
    v = torch.rand(rows, D, generator=gen) * 1e-5
    acc = torch.randn(rows, D, generator=gen)
    touched = torch.rand(rows, generator=gen) < frac
    acc[~touched] = 0
    return p, m, v, acc, touched


@pytest.mark.parametrize("rows,D", [(4096, 384), (1000, 16), (777, 23), (50, 1)])
@pytest.mark.parametrize("scale", [1.0, 0.37])
def test_lazy_adam_bit_exact_vs_reference_c_loop(rows, D, scale):
    p, m, v, acc, touched = random_state(rows, D, rows + D)
    step, lr, b1, b2, eps = 7, 2.4e-3, 0.9, 0.95, 1e-8
    gp, gm, gv, gacc, gt = (t.clone().to(DEV) for t in (p, m, v, acc, touched))
    K.lazy_adam_step(gp, gm, gv, gacc, gt, torch.tensor(scale, device=DEV), step, lr, b1, b2, eps)
    o = [t.numpy().copy() for t in (p, m, v, acc)]
    ot = touched.numpy().astype(np.uint8)
    O.lazy_adam(o[0], o[1], o[2], o[3], ot.copy(), scale, step, lr, b1, b2, eps)
    for a, b in zip((gp, gm, gv, gacc), o):
        assert torch.equal(a.cpu(), torch.from_numpy(b))
    assert not gt.any()
    assert torch.equal(gp.cpu()[~touched], p[~touched])                    # unread rows untouched
    if O.ref_lib() is not None:
        r = [t.numpy().copy() for t in (p, m, v, acc)]
        O.ref_lazy_adam(r[0], r[1], r[2], r[3], ot.copy(), scale, step, lr, b1, b2, eps)
        for a, b in zip((gp, gm, gv), r):
            assert torch.equal(a.cpu(), torch.from_numpy(b))


def test_lazy_adam_golden_three_steps():
    """LazyRowAdam (CUDA) against the reference's LazyRowAdam (torch path): three steps, clip factor 0.5 at the
    second; unread rows and their state bit-identical, accumulator and mask cleared."""
    g = golden("lazy_adam.npz")
    p = torch.nn.Parameter(torch.from_numpy(g["base"]).to(DEV))
    opt = LazyRowAdam([p], lr=float(g["lr"]), betas=(float(g["beta1"]), float(g["beta2"])), eps=float(g["eps"]))
    for step in range(3):
        st = row_store(p)
        st.acc.copy_(torch.from_numpy(g[f"acc{step}"]))
        st.touched.copy_(torch.from_numpy(g[f"touched{step}"]))
        st.grad_scale = torch.tensor(float(g[f"scale{step}"]), device=DEV)
        before = p.detach().clone()
        opt.step()
        assert not st.touched.any() and torch.count_nonzero(st.acc) == 0
        unread = ~torch.from_numpy(g[f"touched{step}"]).to(DEV)
        assert torch.equal(p.detach()[unread], before[unread])
        close(p.detach().cpu(), g[f"p{step}"], msg="values")
        s = opt.state[p]
        close(s["exp_avg"].cpu(), g[f"m{step}"], msg="exp_avg")
        close(s["exp_avg_sq"].cpu(), g[f"v{step}"], msg="exp_avg_sq")
        assert int(s["step"]) == step + 1


def test_lazy_adam_value_copy_and_state_dict_round_trip():
    p = torch.nn.Parameter(torch.randn(300, 32, device=DEV))
    opt = LazyRowAdam([p], lr=1e-2, betas=(0.9, 0.98), value_copy_dtype=torch.bfloat16)
    st = row_store(p)
    rows = torch.tensor([1, 5, 7, 299], device=DEV)
    st.acc[rows] = torch.randn(4, 32, device=DEV)
    st.touched[rows] = True
    opt.step()
    assert torch.equal(p.value_copy[rows], p.detach()[rows].bfloat16())
    sd = opt.state_dict()
    assert sd["format"] == "smlm.lazy_row_adam.v1"
    q = torch.nn.Parameter(p.detach().clone())
    opt2 = LazyRowAdam([q], lr=1e-2, betas=(0.9, 0.98))
    opt2.load_state_dict(sd)
    for o, t in ((opt, p), (opt2, q)):
        s = row_store(t)
        s.acc[rows] = 1.0
        s.touched[rows] = True
        o.step()
    assert torch.equal(p, q)


@pytest.mark.parametrize("kind", ["rowrms", "rowadagrad"])
def test_rowwise_golden_and_c_loop(kind):
    """The reference's RowWiseOptimizer visits (golden): equal to its C loop to fp32 rounding of q (q is summed
    in double in a different order), to its torch formulas within rel 1e-5."""
    g = golden("rowwise.npz")
    p = torch.nn.Parameter(torch.from_numpy(g["initial"]).to(DEV))
    opt = RowWiseOptimizer([p], lr=float(g["lr"]), kind=kind, beta2=float(g["beta2"]), eps=float(g["eps"]))
    for s in range(4):
        st = row_store(p)
        st.acc.copy_(torch.from_numpy(g[f"{kind}_acc{s}"]))
        st.touched.copy_(torch.from_numpy(g[f"{kind}_touched{s}"]))
        before = p.detach().clone()
        opt.step()
        unread = ~torch.from_numpy(g[f"{kind}_touched{s}"]).to(DEV)
        assert torch.equal(p.detach()[unread], before[unread])
        assert torch.count_nonzero(st.acc) == 0 and not st.touched.any()
    for c in ("0", "1"):
        np.testing.assert_allclose(p.detach().cpu().numpy(), g[f"{kind}_c{c}_p"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(opt.state[p]["v"].cpu().numpy(), g[f"{kind}_c{c}_v"], rtol=1e-5, atol=1e-9)
    if kind == "rowrms":
        assert np.array_equal(opt.state[p]["n"].cpu().numpy(), g["rowrms_c1_n"])


@pytest.mark.parametrize("kind", ["rowrms", "rowadagrad"])
@pytest.mark.parametrize("D", [384, 128, 640, 23])
def test_rowwise_vs_oracle_large(kind, D):
    """Widths: 3 and 1 register groups per lane, rows read twice (640 > 512), scalar lanes (23 % 4 != 0)."""
    rows = 20000
    p, _, _, acc, touched = random_state(rows, D, 3, frac=0.5)
    v = torch.rand(rows) * 1e-2
    n = torch.randint(0, 5, (rows,), dtype=torch.int32)
    gp, gacc, gt, gv, gn = (t.clone().to(DEV) for t in (p, acc, touched, v, n))
    K.rowwise_step(gp, gacc, gt, gv, gn if kind == "rowrms" else None, 0.8, 1e-2, 0.95, 1e-8, kind)
    o = [t.numpy().copy() for t in (p, acc, v, n)]
    O.rowwise(o[0], o[1], touched.numpy().astype(np.uint8), o[2], o[3], 0.8, kind, 0.95, 1e-8, 1e-2)
    np.testing.assert_allclose(gp.cpu().numpy(), o[0], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(gv.cpu().numpy(), o[2], rtol=1e-6, atol=0)
    if kind == "rowrms":
        assert np.array_equal(gn.cpu().numpy(), o[3])
    assert torch.equal(gp.cpu()[~touched], p[~touched]) and not gt.any() and not gacc.any()


def test_touched_norm_and_clip():
    rows, D = 50000, 384
    _, _, _, acc, touched = random_state(rows, D, 9)
    n = K.touched_norm(acc.to(DEV), touched.to(DEV))
    ref = O.touched_norm(acc.numpy(), touched.numpy().astype(np.uint8))
    assert abs(float(n) - ref) <= 1e-6 * ref
    assert abs(float(n) - float(acc.double().norm())) <= 1e-6 * ref
    # clipping: the coefficient multiplies the gradient inside the step
    tabs = [torch.nn.Parameter(torch.randn(rows, D, device=DEV)) for _ in range(2)]
    for t in tabs:
        st = row_store(t)
        st.acc.copy_(acc.to(DEV))
        st.touched.copy_(touched.to(DEV))
    total = clip_row_sparse(tabs, 1.0)
    torch.testing.assert_close(float(total), float(np.sqrt(2) * ref), rtol=1e-6, atol=0)
    coef = row_store(tabs[0]).grad_scale
    assert torch.is_tensor(coef) and coef.is_cuda
    torch.testing.assert_close(float(coef), min(1.0, 1.0 / (float(total) + 1e-6)), rtol=1e-6, atol=0)


def test_lazy_step_matches_reference_torch_path_after_clip():
    """Clip + lazy step against the reference's torch path (TorchLazyRowAdam restated in oracle/torch_path.py)."""
    rows, D, N = 4096, 64, 64
    gen = torch.Generator().manual_seed(5)
    base = torch.randn(rows, D, generator=gen) * D ** -0.5
    p_ref = torch.nn.Parameter(base.clone())
    p_gpu = torch.nn.Parameter(base.clone().to(DEV))
    ref_opt = TP.TorchLazyRowAdam([p_ref], lr=1e-3, betas=(0.9, 0.98))
    opt = LazyRowAdam([p_gpu], lr=1e-3, betas=(0.9, 0.98))
    for step in range(2):
        idx = skewed_indices(rows, N, 128, gen).reshape(-1)
        grads = torch.randn(idx.numel(), D, generator=gen)
        sr = TP.row_store(p_ref)
        sr.acc.index_put_((idx,), grads, accumulate=True)
        sr.touched[idx] = True
        sg = row_store(p_gpu)
        sg.acc.copy_(sr.acc.to(DEV))
        sg.touched.copy_(sr.touched.to(DEV))
        nr = TP.clip_row_sparse([p_ref], 5.0)
        ng = clip_row_sparse([p_gpu], 5.0)
        torch.testing.assert_close(float(ng), float(nr), rtol=1e-5, atol=0)
        ref_opt.step()
        opt.step()
        close(p_gpu.detach().cpu(), p_ref.detach(), msg="values")
        close(opt.state[p_gpu]["exp_avg"].cpu(), ref_opt.state(p_ref)["exp_avg"], msg="exp_avg")
