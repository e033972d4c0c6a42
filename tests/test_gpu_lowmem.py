"""LazyRowAdam with compact moments (bf16, or int8 codes with row scales) on the GPU: bit-identical to the oracle,
and so to the reference's Triton kernel, on the reference's 12-step scenario; the reference's semantics tests
(unread rows keep every state tensor, empty steps, state budget, positive variance never coded 0, cancellation)
(reference: kernels.py:445-515, sparse_values.py:193-255, tests/test_lowmem_values.py)."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from smlm_b200 import kernels as K
from smlm_b200.sparse_values import LazyRowAdam, row_store
from util import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
MODES = ("fp32", "bf16", "int8")


def apply_gradient(table, opt, rows, gradient, scale=1.0):
    """The reference's scripts/check_lowmem.py apply_gradient: rows' accumulator set, then one step."""
    st = row_store(table)
    st.acc[rows] = gradient
    st.touched[rows] = True
    st.grad_scale = scale
    opt.step()


def state_copy(opt, table):
    return {k: v.detach().clone() for k, v in opt.state[table].items() if k != "step" and torch.is_tensor(v)}


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


@pytest.mark.parametrize("mode", ["bf16", "int8"])
@pytest.mark.parametrize("dim", [23, 384])
def test_matches_oracle_and_reference_kernel(mode, dim):
    g = golden("lazy_adam_lowmem.npz")
    key = f"{mode}_{dim}"
    table = torch.nn.Parameter(torch.from_numpy(g[f"{key}_initial"].astype(np.float32)).to(DEV))
    opt = LazyRowAdam([table], lr=float(g["lr"]), betas=(float(g["beta1"]), float(g["beta2"])),
                      eps=float(g["eps"]), state_dtype=mode)
    R = table.shape[0]
    i8 = mode == "int8"
    p = g[f"{key}_initial"].astype(np.float32).copy()
    m = np.zeros((R, dim), np.int8 if i8 else np.uint16)
    v = np.zeros((R, dim), np.uint8 if i8 else np.uint16)
    ms, vs = np.zeros(R, np.float32), np.zeros(R, np.float32)
    for step in range(12):
        rows = torch.from_numpy(g[f"{key}_rows{step}"])
        grads = torch.from_numpy(g[f"{key}_grads{step}"])
        scale = float(g[f"{key}_scale{step}"])
        apply_gradient(table, opt, rows.to(DEV), grads.to(DEV), torch.tensor(scale, device=DEV))
        acc = np.zeros((R, dim), np.float32)
        acc[rows.numpy()] = grads.numpy()
        touched = np.zeros(R, np.uint8)
        touched[rows.numpy()] = 1
        O.lazy_adam_lowmem(p, m, v, ms, vs, acc, touched, scale, step + 1, float(g["lr"]), float(g["beta1"]),
                           float(g["beta2"]), float(g["eps"]), i8)
        s = opt.state[table]
        assert np.array_equal(table.detach().cpu().numpy(), p), f"values, step {step}"
        gm = s["exp_avg"].cpu()
        gv = s["exp_avg_sq"].cpu()
        if i8:
            assert np.array_equal(gm.numpy(), m) and np.array_equal(gv.numpy(), v)
            assert np.array_equal(s["exp_avg_scale"].cpu().numpy(), ms)
            assert np.array_equal(s["exp_avg_sq_scale"].cpu().numpy(), vs)
        else:
            assert np.array_equal(gm.view(torch.int16).numpy().view(np.uint16), m)
            assert np.array_equal(gv.view(torch.int16).numpy().view(np.uint16), v)
    t = f"{key}_triton"                                        # the reference kernel's final state
    assert np.array_equal(p, g[f"{t}_p11"])


@pytest.mark.parametrize("mode", ["bf16", "int8"])
def test_reference_named_entry_point(mode):
    """kernels.lazy_adam_step_lowmem (the reference's name and argument order, kernels.py:493-515) equals
    lazy_adam_lowmem_step bit for bit over three steps, and consumes the rows (touched cleared, acc rows zeroed)."""
    gen = torch.Generator().manual_seed(11)
    R, D = 300, 384
    i8 = mode == "int8"
    p0 = torch.randn(R, D, generator=gen).to(DEV)
    p1 = p0.clone()

    def moments():
        return (torch.zeros(R, D, dtype=torch.int8 if i8 else torch.bfloat16, device=DEV),
                torch.zeros(R, D, dtype=torch.uint8 if i8 else torch.bfloat16, device=DEV),
                torch.zeros(R, device=DEV) if i8 else None, torch.zeros(R, device=DEV) if i8 else None)
    sa, sb = moments(), moments()
    for step in range(1, 4):
        rows = torch.randperm(R, generator=gen)[:100].to(DEV)
        grad = torch.randn(100, D, generator=gen).to(DEV)
        accs, marks = [], []
        for _ in range(2):
            acc = torch.zeros(R, D, device=DEV)
            acc[rows] = grad
            mark = torch.zeros(R, dtype=torch.bool, device=DEV)
            mark[rows] = True
            accs.append(acc)
            marks.append(mark)
        K.lazy_adam_step_lowmem(p0, sa[0], sa[1], accs[0], marks[0], 0.5, step, 1e-2, 0.9, 0.98, 1e-8, mode,
                                exp_avg_scale=sa[2], exp_avg_sq_scale=sa[3])
        K.lazy_adam_lowmem_step(p1, sb[0], sb[1], sb[2], sb[3], accs[1], marks[1], 0.5, step, 1e-2, 0.9, 0.98, 1e-8)
        assert same_bits(p0, p1), f"values, step {step}"
        for a, b in zip(sa, sb):
            if a is not None:
                assert same_bits(a, b), f"state, step {step}"
        assert not marks[0].any() and not accs[0].any()
    with pytest.raises(ValueError):
        K.lazy_adam_step_lowmem(p0, sa[0], sa[1], accs[0], marks[0], 1.0, 4, 1e-2, 0.9, 0.98, 1e-8,
                                "int8" if not i8 else "bf16")


@pytest.mark.parametrize("mode", MODES)
def test_unread_rows_preserve_every_state_tensor(mode):
    gen = torch.Generator().manual_seed(71)
    table = torch.nn.Parameter(torch.randn(19, 13, generator=gen).to(DEV))
    opt = LazyRowAdam([table], lr=0.01, state_dtype=mode)
    for step, visited in enumerate([list(range(19)), [1, 5, 8], [2, 9], [1, 5, 18]]):
        rows = torch.tensor(visited, device=DEV)
        before = table.detach().clone()
        previous = state_copy(opt, table)
        apply_gradient(table, opt, rows, torch.randn(len(visited), 13, generator=gen).to(DEV),
                       torch.tensor(0.25, device=DEV))
        unread = torch.ones(19, dtype=torch.bool, device=DEV)
        unread[rows] = False
        assert same_bits(table.detach()[unread], before[unread])
        current = state_copy(opt, table)
        for k in previous:
            assert same_bits(current[k][unread], previous[k][unread]), k
        assert int(opt.state[table]["step"]) == step + 1
        assert table.grad is None
        st = row_store(table)
        assert not st.touched.any() and torch.count_nonzero(st.acc) == 0 and st.grad_scale == 1.0


@pytest.mark.parametrize("mode", MODES)
def test_empty_step_changes_nothing_but_the_count(mode):
    table = torch.nn.Parameter(torch.ones(7, 11, device=DEV))
    opt = LazyRowAdam([table], lr=0.01, state_dtype=mode)
    apply_gradient(table, opt, torch.tensor([3], device=DEV), torch.ones(1, 11, device=DEV))
    before, previous = table.detach().clone(), state_copy(opt, table)
    opt.step()
    assert same_bits(before, table.detach())
    for k, v in previous.items():
        assert same_bits(v, opt.state[table][k]), k
    assert int(opt.state[table]["step"]) == 2                  # global step count, as the reference's kernel path


@pytest.mark.parametrize("mode,bytes_per_row", [("fp32", 8 * 32), ("bf16", 4 * 32), ("int8", 2 * 32 + 8)])
def test_state_storage_matches_budget(mode, bytes_per_row):
    table = torch.nn.Parameter(torch.zeros(48, 32, device=DEV))
    opt = LazyRowAdam([table], lr=0.01, state_dtype=mode)
    apply_gradient(table, opt, torch.tensor([0], device=DEV), torch.zeros(1, 32, device=DEV))
    s = opt.state[table]
    assert sum(v.numel() * v.element_size() for k, v in s.items() if k != "step") == 48 * bytes_per_row
    expected = {"fp32": (torch.float32, torch.float32), "bf16": (torch.bfloat16, torch.bfloat16),
                "int8": (torch.int8, torch.uint8)}[mode]
    assert (s["exp_avg"].dtype, s["exp_avg_sq"].dtype) == expected


def test_int8_positive_variance_never_rounds_to_zero():
    table = torch.nn.Parameter(torch.zeros(1, 3, device=DEV))
    opt = LazyRowAdam([table], lr=0.003, state_dtype="int8")
    apply_gradient(table, opt, torch.tensor([0], device=DEV), torch.tensor([[1e6, 1e-6, 0.0]], device=DEV))
    v = opt.state[table]["exp_avg_sq"]
    assert v[0, 0] == 255 and v[0, 1] == 1 and v[0, 2] == 0


def test_int8_cancellation_retains_small_positive_variance():
    tables = {mode: torch.nn.Parameter(torch.zeros(1, 2, device=DEV)) for mode in ("fp32", "int8")}
    opts = {mode: LazyRowAdam([t], lr=0.003, state_dtype=mode) for mode, t in tables.items()}
    for values in ([1000.0, 0.0], [-900.0, 1.0], [0.0, 0.0]):
        for mode, t in tables.items():
            apply_gradient(t, opts[mode], torch.tensor([0], device=DEV), torch.tensor([values], device=DEV))
    assert opts["int8"].state[tables["int8"]]["exp_avg_sq"][0, 1] > 0
    assert torch.isfinite(tables["int8"]).all()
    torch.testing.assert_close(tables["int8"][:, 1], tables["fp32"][:, 1], rtol=0.05, atol=1e-6)


@pytest.mark.parametrize("mode", ["bf16", "int8"])
@pytest.mark.parametrize("D", [384, 1000])
def test_keep_acc_and_value_copy(mode, D):
    """The clean-store variant (accumulator rows left in place) and the bf16 value copy give the same table and
    state as the zeroing variant; wide rows take the two-pass path."""
    gen = torch.Generator().manual_seed(5)
    rows = 600
    p0 = torch.randn(rows, D, generator=gen) * 0.05
    acc0 = torch.randn(rows, D, generator=gen)
    touched0 = torch.rand(rows, generator=gen) < 0.4
    outs = []
    for keep in (False, True):
        table = torch.nn.Parameter(p0.clone().to(DEV))
        opt = LazyRowAdam([table], lr=1e-2, state_dtype=mode, value_copy_dtype=torch.bfloat16)
        s = opt._state(table)
        acc, touched = acc0.clone().to(DEV), touched0.clone().to(DEV)
        for step in range(2):
            K.lazy_adam_lowmem_step(table.data, s["exp_avg"], s["exp_avg_sq"], s.get("exp_avg_scale"),
                                    s.get("exp_avg_sq_scale"), acc, touched, 1.0, step + 1, 1e-2, 0.9, 0.95, 1e-8,
                                    value_copy=table.value_copy, keep_acc=keep)
            if not keep:
                assert torch.count_nonzero(acc[touched0.to(DEV)]) == 0
            touched.copy_(touched0.to(DEV))
            acc.copy_(acc0.to(DEV))
        outs.append((table.detach().clone(), table.value_copy.clone(), state_copy(opt, table)))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][1], outs[0][0].bfloat16())
    for k in outs[0][2]:
        assert same_bits(outs[0][2][k], outs[1][2][k]), k
