"""Value tables in host RAM (smlm_b200.host_values, smlm_b200.host_optim): the table, its accumulator and its
optimizer state stay in host RAM, mapped into the GPU's address space, and the kernels gather, accumulate and step
the rows there. Trains like the same model with its table on the GPU (the reference's own checks:
tests/test_host_values.py, tests/test_hot_rows.py, tests/test_host_optim.py): losses, reads, accumulated row
gradients, clip norms, parameters and optimizer states after three steps of three micro-batches, for fp32, bf16 and
int8 moments; unread rows keep their values and state bit for bit; HOT rows and the GACC step accumulator (with
overflow) train like rows in RAM under rowrms; a single layer with a host table equals the GPU table bit for bit."""
import pytest
import torch
from torch import nn

from smlm_b200.host_optim import HostLazyRowAdam, value_table_memory_by_device
from smlm_b200.host_values import HostEmbedding, enable_host_values, enable_hot_rows, enable_step_rows, host_timings
from smlm_b200.model import ModelConfig, Transformer
from smlm_b200.optim import build_optimizer, clip_grads
from smlm_b200.pkm import ProductKeyMemory
from smlm_b200.row_optim import RowWiseOptimizer
from smlm_b200.sparse_values import LazyRowAdam, clip_row_sparse, row_store

pytestmark = pytest.mark.gpu
DEV = "cuda"
MODES = ["fp32", "bf16", "int8"]
TOL = dict(rtol=1e-4, atol=2e-6)        # the reference's GPU fp32 tolerance (changed reduction order)


def tiny(share=True, seed=39):
    cfg = ModelConfig(vocab_size=64, d_model=32, n_layers=4, n_heads=4, ffn_hidden=48, max_seq_len=24,
                      mem_layers=[0, 2, 3], mem_n_keys=16, mem_heads=2, mem_knn=4, mem_k_dim=16,
                      mem_share_values=share, mem_value_grad="row_sparse")
    torch.manual_seed(seed)
    return Transformer(cfg)


def paired(share=True):
    normal, host = tiny(share), tiny(share)
    host.load_state_dict(normal.state_dict())
    enable_host_values(host)
    return normal.to(DEV), host.to(DEV)


def table_of(model):
    return model.memory_layers()[0].values.weight


def close(a, b, **kw):
    torch.testing.assert_close(a.detach().cpu(), b.detach().cpu(), **dict(TOL, **kw))


def optimizer_for(opt, param):
    return next(o for o in opt.opts if any(p is param for g in o.param_groups for p in g["params"]))


def decoded(state, mode):
    m, v = state["exp_avg"].float().cpu(), state["exp_avg_sq"].float().cpu()
    if mode == "int8":
        m = m.sign() * (m / 127).square() * state["exp_avg_scale"].cpu()[:, None]
        v = (v / 255 * state["exp_avg_sq_scale"].cpu()[:, None]).square().square()
    return m, v


@pytest.mark.parametrize("mode", MODES)
def test_host_training_matches_gpu_table(tmp_path, mode):
    normal, host = paired()
    assert table_of(host).device.type == "cpu" and table_of(normal).is_cuda
    opts = [build_optimizer(m, lr=3e-4, value_lr=7e-4, weight_decay=0.03, value_state=mode) for m in (normal, host)]
    assert isinstance(optimizer_for(opts[1], table_of(host)), HostLazyRowAdam)
    gen = torch.Generator().manual_seed(103)
    for m in (normal, host):
        for mem in m.memory_layers():
            mem.record = True
    for step in range(3):
        for _ in range(3):
            tokens = torch.randint(0, 64, (2, 8), generator=gen).to(DEV)
            losses, reads = [], []
            for m in (normal, host):
                _, loss = m(tokens[:, :-1], tokens[:, 1:])
                (loss / 3).backward()
                losses.append(loss)
                reads.append([mem.last_indices.cpu() for mem in m.memory_layers()])
            close(losses[1], losses[0], rtol=2e-6, atol=2e-7)
            assert all(torch.equal(a, b) for a, b in zip(*reads))
            close(row_store(table_of(host)).acc, row_store(table_of(normal)).acc)
            assert torch.equal(row_store(table_of(host)).touched, row_store(table_of(normal)).touched.cpu())
        for (name, p), (_, h) in zip(normal.named_parameters(), host.named_parameters()):
            if p is table_of(normal):
                assert p.grad is None and h.grad is None
            else:
                close(h.grad, p.grad, msg=name)
        norms = [clip_grads(m, 1e-3) for m in (normal, host)]
        for a, b in zip(norms[1], norms[0]):
            close(a, b)
        for opt in opts:
            opt.step()
            opt.zero_grad(set_to_none=True)
        for (name, p), (_, h) in zip(normal.named_parameters(), host.named_parameters()):
            close(h, p, msg=name)
        a = optimizer_for(opts[0], table_of(normal)).state[table_of(normal)]
        b = optimizer_for(opts[1], table_of(host)).state[table_of(host)]
        assert int(a["step"]) == int(b["step"]) == step + 1
        assert all(v.device.type == "cpu" for v in b.values() if torch.is_tensor(v))
        # the clip norms come from differently ordered sums (per-row squared norms on the GPU path, the host
        # accumulator here), so the states agree to fp32 rounding, not bit for bit
        for x, y in zip(decoded(b, mode), decoded(a, mode)):
            if mode == "fp32":
                scale = y.abs().max().clamp_min(1e-30)
                close(x / scale, y / scale, atol=1e-5)
            else:
                scale = y.abs().amax(dim=1, keepdim=True).clamp_min(1e-30)
                close(x / scale, y / scale, rtol=1e-4, atol=0.008 if mode == "bf16" else 0.018)
        st = row_store(table_of(host))
        assert not st.touched.any() and torch.count_nonzero(st.acc) == 0 and st.grad_scale == 1.0
    path = tmp_path / "model.pt"
    torch.save(host.state_dict(), path)
    restored = Transformer(host.cfg).to(DEV).eval()
    restored.load_state_dict(torch.load(path, weights_only=True, map_location=DEV), strict=True)
    host.eval()
    with torch.no_grad():
        close(restored(tokens[:, :-1]), host(tokens[:, :-1]))
    assert not getattr(table_of(restored), "host_values", False)
    assert set(host_timings(host)) == {"unique", "indices_d2h", "gather", "rows_h2d", "gradients_d2h", "scatter"}


@pytest.mark.parametrize("mode", MODES)
def test_unread_rows_keep_values_and_state(mode):
    model = enable_host_values(tiny()).to(DEV)
    memory, table = model.memory_layers()[0], table_of(model)
    opt = build_optimizer(model, lr=3e-4, value_lr=7e-4, weight_decay=0.03, value_state=mode)
    lazy = optimizer_for(opt, table)
    gen = torch.Generator().manual_seed(122)
    visits = [torch.arange(table.shape[0]).view(-1, 1), torch.tensor([[1, 1, 5], [5, 9, 1]]),
              torch.tensor([[3, 3, 9], [11, 3, 11]])]
    for step, indices in enumerate(visits):
        previous = table.detach().clone()
        before = {k: v.clone() for k, v in lazy.state[table].items() if k != "step"}
        w = torch.randn(indices.shape, generator=gen).to(DEV).requires_grad_()
        g = torch.randn(indices.shape[0], table.shape[1], generator=gen).to(DEV)
        memory.read_values(indices.to(DEV), w).backward(g)
        unread = torch.ones(table.shape[0], dtype=torch.bool)
        unread[indices.unique()] = False
        assert torch.equal(row_store(table).touched, ~unread)
        clip_grads(model, 0.25)
        opt.step()
        opt.zero_grad(set_to_none=True)
        assert torch.equal(table[unread], previous[unread])
        for key, value in before.items():
            assert torch.equal(lazy.state[table][key][unread], value[unread]), key
        assert int(lazy.state[table]["step"]) == step + 1
        assert not row_store(table).touched.any() and torch.count_nonzero(row_store(table).acc) == 0


def test_single_layer_host_table_bit_identical_to_gpu_table():
    """One ProductKeyMemory, bf16 autocast scoring, two LazyRowAdam steps (no clipping, whose norm sums run in
    another order on the two paths): outputs, the weight gradients' effect on the keys, the accumulated rows and
    the updated table are the same bits with the table in host RAM."""
    torch.manual_seed(0)
    a = ProductKeyMemory(64, 64, n_keys=64, heads=2, knn=16, k_dim=256, query_norm="none", swilu=False,
                         value_grad="row_sparse")
    b = ProductKeyMemory(64, 64, n_keys=64, heads=2, knn=16, k_dim=256, query_norm="none", swilu=False,
                         value_grad="row_sparse")
    b.load_state_dict(a.state_dict())
    holder = nn.Module()
    holder.mem = b
    enable_host_values(holder)
    a, b = a.to(DEV), b.to(DEV)
    oa = LazyRowAdam([a.values.weight], lr=1e-2, betas=(0.9, 0.98))
    ob = HostLazyRowAdam([b.values.weight], lr=1e-2, betas=(0.9, 0.98))
    gen = torch.Generator().manual_seed(1)
    for _ in range(2):
        x = torch.randn(300, 64, generator=gen).to(DEV)
        g = torch.randn(300, 64, generator=gen).to(DEV)
        outs = []
        for m in (a, b):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = m(x)
            out.backward(g)
            outs.append(out.detach())
        assert torch.equal(outs[0], outs[1])
        assert torch.equal(a.keys.grad, b.keys.grad)
        assert torch.equal(row_store(a.values.weight).acc.cpu(), row_store(b.values.weight).acc)
        oa.step()
        ob.step()
        assert torch.equal(a.values.weight.detach().cpu(), b.values.weight.detach())
        for m in (a, b):
            m.zero_grad(set_to_none=True)


def make_holder(initial, hot_frac=None, reads=None, capacity=None, keep_values=True, kind="rowrms", overlap=False):
    emb = HostEmbedding(nn.Embedding(*initial.shape, _weight=initial.clone()))
    emb.weight.pk_value_param = True
    model = nn.Module()
    model.values = emb
    model = model.to(DEV)
    if hot_frac:
        enable_hot_rows(model, reads, hot_frac, torch.device(DEV))
    if capacity:
        enable_step_rows(model, capacity, torch.device(DEV), keep_values=keep_values, overlap=overlap)
    return model, RowWiseOptimizer([emb.weight], lr=0.05, kind=kind)


@pytest.mark.parametrize("width", [16, 384, 512])
@pytest.mark.parametrize("kind", ["rowrms", "rowadagrad"])
def test_gacc_step_from_gathered_rows_is_bit_identical(width, kind):
    """Without clipping and with one backward per step, the row-wise step gives the same bits whether the rows'
    gradients sit in the host accumulator, in GACC slots that read the rows from the host table, or in GACC slots
    that keep the rows the forward gathered (the step updates them on the GPU, writes them back, and the next step
    reads them from that cache), with the write-back overlapped with the next step or not; with a capacity below
    the rows a step reads, the overflow rows take the host path in the same step. Widths 16 / 384 / 512: one, three
    and four register groups per lane (the value bags take rows of up to 512 values)."""
    gen = torch.Generator().manual_seed(width)
    initial = torch.randn(300, width, generator=gen)
    holders = [make_holder(initial, kind=kind), make_holder(initial, capacity=400, keep_values=False, kind=kind),
               make_holder(initial, capacity=400, kind=kind), make_holder(initial, capacity=30, kind=kind),
               make_holder(initial, capacity=400, kind=kind, overlap=True),
               make_holder(initial, capacity=30, kind=kind, overlap=True)]
    outs = None
    for step in range(4):
        idx = torch.randint(0, 300, (40, 6), generator=gen).to(DEV)
        w = torch.rand(40, 6, generator=gen).to(DEV)
        outs = []
        for model, opt in holders:
            out = model.values.bag(idx, w)
            out.square().sum().backward()
            outs.append(out.detach())
        assert all(torch.equal(o, outs[0]) for o in outs[1:])     # rows read from the cache: the same values
        assert row_store(holders[3][0].values.weight).steprows.spilled() is not None
        assert row_store(holders[2][0].values.weight).steprows.current() is not None
        if step:
            assert row_store(holders[2][0].values.weight).steprows.cache()[0] is not None
        for _, opt in holders:
            opt.step()
        for model, _ in holders:
            model.values.flush()                                   # the overlapped write-backs reach the table
        ref, ref_state = holders[0][0].values.weight.detach(), holders[0][1].state_dict()["state"][0]
        for model, opt in holders[1:]:
            assert torch.equal(model.values.weight.detach(), ref)
            st = opt.state_dict()["state"][0]
            assert torch.equal(st["v"], ref_state["v"])
            if kind == "rowrms":
                assert torch.equal(st["n"], ref_state["n"])


@pytest.mark.parametrize("hot_frac,capacity,overlap", [(0.3, None, False), (None, 40, False), (0.3, 25, False),
                                                       (None, 40, True), (0.3, 25, True)])
def test_hot_rows_and_gacc_train_like_rows_in_ram(hot_frac, capacity, overlap):
    """rowrms on a host table: HOT rows on the GPU and / or the GACC step accumulator (capacity 25 / 40 rows: steps
    read more rows, so the overflow path runs) give the same outputs, clip norms, rows and row state as all rows
    in RAM; state_dict writes the hot rows back (reference: tests/test_hot_rows.py)."""
    gen = torch.Generator().manual_seed(0)
    initial = torch.randn(200, 16, generator=gen)
    reads = torch.randint(0, 1000, (200,), generator=gen)
    (plain, opt_a), (other, opt_b) = make_holder(initial), make_holder(initial, hot_frac, reads, capacity,
                                                                      overlap=overlap)
    spilled = False
    for _ in range(4):
        idx = torch.randint(0, 200, (12, 5), generator=gen).to(DEV)
        w = torch.rand(12, 5, generator=gen).to(DEV).requires_grad_(True)
        outs = []
        for model in (plain, other):
            out = model.values.bag(idx, w)
            out.square().sum().backward()
            outs.append(out.detach())
        torch.testing.assert_close(outs[1], outs[0], rtol=1e-6, atol=1e-6)
        if capacity:
            spilled |= row_store(other.values.weight).steprows.spilled() is not None
        norms = [clip_row_sparse([m.values.weight], 1.0) for m in (plain, other)]
        torch.testing.assert_close(norms[1], norms[0], rtol=1e-5, atol=1e-6)
        opt_a.step()
        opt_b.step()
    if capacity:
        assert spilled
    table = other.state_dict()["values.weight"]             # flushes the GPU rows into the table
    torch.testing.assert_close(table, plain.values.weight.detach(), rtol=1e-5, atol=1e-6)
    if hot_frac:
        # loading a table refreshes the HOT rows' device copies
        saved = {k: v.clone() for k, v in other.state_dict().items()}
        other.values.hot.values.add_(1.0)
        other.load_state_dict(saved)
        hot = other.values.hot
        assert torch.equal(hot.values.cpu(), other.values.weight.detach()[hot.rows.cpu()])
    sa, sb = opt_a.state_dict()["state"][0], opt_b.state_dict()["state"][0]
    assert sa.keys() == sb.keys() == {"step", "v", "n"}
    torch.testing.assert_close(sb["v"], sa["v"], rtol=1e-5, atol=1e-9)
    assert torch.equal(sb["n"], sa["n"])


def test_hot_rows_need_a_row_wise_optimizer_and_memory_split():
    gen = torch.Generator().manual_seed(3)
    initial = torch.randn(64, 8, generator=gen)
    emb = HostEmbedding(nn.Embedding(*initial.shape, _weight=initial.clone()))
    emb.weight.pk_value_param = True
    model = nn.Module()
    model.values = emb
    enable_hot_rows(model, torch.arange(64), 0.25, torch.device(DEV))
    opt = HostLazyRowAdam([emb.weight], lr=1e-3)
    emb.bag(torch.tensor([[1, 2]], device=DEV), torch.ones(1, 2, device=DEV)).sum().backward()
    with pytest.raises(ValueError, match="row-wise"):
        opt.step()
    split = value_table_memory_by_device(tiny(), "fp32")
    assert split["host"]["table_bytes"] == 0 and split["device"]["table_bytes"] > 0
