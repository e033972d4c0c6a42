"""Values bf16 with an fp32 master (LazyRowAdam(value_copy_dtype=torch.bfloat16)): the value
bag and its weight gradient read the bf16 copy, the optimizer updates the fp32 master and refreshes the copy's
rows. Against the reference's fp32 PyTorch path (oracle/torch_path.py) on the same selection the layer stays
within rel 2e-2 (the north star's tolerance for a bf16 value table), and the copy follows the master."""
import pytest
import torch

from oracle import torch_path as TP
from smlm_b200 import kernels as K
from smlm_b200.pkm import ProductKeyMemory
from smlm_b200.sparse_values import LazyRowAdam, clip_row_sparse, row_store
from util import close

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2              # bf16 value table against an fp32 reference


def pair(N=2048, n_keys=256, seed=0):
    ref = TP.TorchPKM(384, 384, n_keys=n_keys, heads=4, knn=32, k_dim=256, query_norm="none", swilu=False,
                      canonical=True)
    TP.init_like_reference(ref, seed)
    mem = ProductKeyMemory(384, 384, n_keys=n_keys, heads=4, knn=32, k_dim=256, query_norm="none", swilu=False,
                           value_grad="row_sparse").to(DEV)
    mem.load_state_dict(ref.state_dict())
    gen = torch.Generator().manual_seed(seed + 1)
    return ref, mem, [torch.randn(N, 384, generator=gen) for _ in range(2)], \
        [torch.randn(N, 384, generator=gen) for _ in range(2)]


def test_bf16_value_copy_layer_within_tolerance_of_fp32_reference():
    """Two steps (fp32 scoring, so that both paths select alike; the reference is given the layer's selection):
    outputs, keys and query gradients within rel 2e-2 of the fp32 reference; the row accumulator (independent
    of the table) and the updated fp32 master within rel 1e-5; the copy equals the master rounded to bf16."""
    ref, mem, xs, gs = pair()
    table = mem.values.weight
    opt = LazyRowAdam([table], lr=1e-3, betas=(0.9, 0.98), value_copy_dtype=torch.bfloat16)
    opt_r = TP.TorchLazyRowAdam([ref.values.weight], lr=1e-3, betas=(0.9, 0.98))
    mem.record = True
    for step in range(2):
        out = mem(xs[step].to(DEV))
        # the forward read the bf16 copy: bit for bit the bag over the bf16-rounded table
        idx = mem.last_indices.view(out.shape[0], -1)
        w = mem.last_weights.view(out.shape[0], -1)
        assert torch.equal(out.detach(), K.bag_forward(idx, w, table.detach().bfloat16()))
        out.backward(gs[step].to(DEV))
        ref.forced_indices = mem.last_indices.cpu()
        out_r = ref(xs[step])
        out_r.backward(gs[step])
        close(out.detach().cpu(), out_r.detach(), rtol=TOL, atol=TOL, msg=f"step {step}: layer output")
        close(mem.keys.grad.cpu(), ref.keys.grad, rtol=TOL, atol=TOL, msg=f"step {step}: keys grad")
        close(mem.query_proj.weight.grad.cpu(), ref.query_proj.weight.grad, rtol=TOL, atol=TOL,
              msg=f"step {step}: query grad")
        st, st_r = row_store(table), TP.row_store(ref.values.weight)
        assert torch.equal(st.touched.cpu(), st_r.touched)
        close(st.acc.cpu(), st_r.acc, msg=f"step {step}: row accumulator")
        st_r.acc.copy_(st.acc.cpu())                  # the step itself compared on one accumulator
        opt.step()
        opt_r.step()
        close(table.detach().cpu(), ref.values.weight.detach(), msg=f"step {step}: updated master rows")
        assert torch.equal(table.value_copy, table.detach().bfloat16())
        for p, pr in ((mem.keys, ref.keys), (mem.query_proj.weight, ref.query_proj.weight),
                      (mem.query_proj.bias, ref.query_proj.bias)):
            p.grad = None                             # no optimizer on the dense parameters: both keep them
            pr.grad = None


def test_value_copy_refreshed_after_torch_writes_the_master():
    """A change to the master through torch (an in-place op, load_state_dict) is seen before the next read."""
    _, mem, xs, gs = pair(N=512)
    table = mem.values.weight
    LazyRowAdam([table], lr=1e-3, value_copy_dtype=torch.bfloat16)
    with torch.no_grad():
        table.mul_(-2.0)
    mem.record = True
    with torch.no_grad():
        out = mem(xs[0].to(DEV))
    idx = mem.last_indices.view(out.shape[0], -1)
    w = mem.last_weights.view(out.shape[0], -1)
    assert torch.equal(out, K.bag_forward(idx, w, table.detach().bfloat16()))
    state = {k: v.clone() for k, v in mem.state_dict().items()}
    state["values.weight"].normal_()
    mem.load_state_dict(state)
    out = mem(xs[1].to(DEV))
    idx = mem.last_indices.view(out.shape[0], -1)
    w = mem.last_weights.view(out.shape[0], -1)
    assert torch.equal(out.detach(), K.bag_forward(idx, w, table.detach().bfloat16()))


def test_value_copy_fused_deferred_step_under_bf16_autocast():
    """The benchmark's path with the copy: bf16 autocast scoring, deferred row sums fused with lazy Adam, value
    clipping. The step refreshes exactly the updated rows of the copy; the untouched rows of master and copy stay
    as they were."""
    _, mem, xs, gs = pair(N=4096, n_keys=512)
    table = mem.values.weight
    opt = LazyRowAdam([table], lr=1e-3, betas=(0.9, 0.98), value_copy_dtype=torch.bfloat16)
    for step in range(3):
        before = table.detach().clone()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = mem(xs[step % 2].to(DEV))
        out.backward(gs[step % 2].to(DEV))
        st = row_store(table)
        assert st.pending is not None
        clip_row_sparse([table], 1.0)
        st.sync()
        read = st._touched.clone()
        opt.step()
        assert torch.equal(table.detach()[~read], before[~read])
        assert torch.equal(table.value_copy, table.detach().bfloat16())
        mem.zero_grad(set_to_none=True)
