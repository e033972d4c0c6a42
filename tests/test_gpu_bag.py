"""Value bag kernels on the GPU against the CPU oracle (bit for bit where the order is fixed) and against the
reference's golden outputs (rel 1e-5 fp32; the reference's TOL, its tests/test_kernels.py:36)."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import oracle as O
from smlm_b200 import kernels as K
from util import bf16_from_bits, bits_of_bf16, close, golden, skewed_indices

pytestmark = pytest.mark.gpu
DEV = "cuda"


def chunk_positions(m):
    """The backward's work-chunk size (bag.cu chunk_positions): needed to replay its exact summation order."""
    return 256 if m >= (1 << 20) else 64


def make(rows, D, N, K_, seed, skew=True, dtype=torch.float32):
    gen = torch.Generator().manual_seed(seed)
    table = (torch.randn(rows, D, generator=gen) * D ** -0.5)
    idx = skewed_indices(rows, N, K_, gen) if skew else torch.randint(0, rows, (N, K_), generator=gen)
    w = torch.softmax(torch.randn(N, K_, generator=gen), -1)
    g = torch.randn(N, D, generator=gen)
    if dtype == torch.bfloat16:
        table = table.bfloat16()
    return table, idx, w, g


@pytest.mark.parametrize("rows,D,N,K_,dtype", [
    (512, 32, 16, 128, torch.float32), (4096, 384, 64, 128, torch.float32), (4096, 384, 64, 128, torch.bfloat16),
    (1000, 23, 8, 40, torch.float32), (1000, 23, 8, 40, torch.bfloat16), (300, 1, 4, 5, torch.float32),
    (2048, 96, 32, 96, torch.float32), (4096, 64, 32, 48, torch.float32), (777, 1000, 6, 33, torch.float32)])
def test_bag_forward_bit_exact_vs_oracle(rows, D, N, K_, dtype):
    table, idx, w, _ = make(rows, D, N, K_, rows + D, dtype=dtype)
    wt = w.to(dtype)
    out = K.bag_forward(idx.to(DEV), wt.to(DEV), table.to(DEV)).cpu()
    if dtype == torch.bfloat16:
        ref, _ = O.bag_forward(idx.numpy(), wt.float().numpy(), bits_of_bf16(table), bf16=True)
    else:
        ref, _ = O.bag_forward(idx.numpy(), w.numpy(), table.numpy())
    assert torch.equal(out, torch.from_numpy(ref))


def test_bag_forward_golden():
    g = golden("bag.npz")
    out = K.bag_forward(torch.from_numpy(g["idx"]).to(DEV), torch.from_numpy(g["w"]).to(DEV),
                        torch.from_numpy(g["table"]).to(DEV)).cpu()
    close(out, g["out"])
    wb = torch.from_numpy(g["w"]).bfloat16()
    out_b = K.bag_forward(torch.from_numpy(g["idx"]).to(DEV), wb.to(DEV), bf16_from_bits(g["table_bf16"]).to(DEV))
    close(out_b.cpu(), g["out_bf16_table"])


@pytest.mark.parametrize("rows", [512 ** 2, 1024 ** 2])
def test_bag_forward_large_vs_embedding_bag(rows):
    table, idx, w, _ = make(rows, 384, 4096, 128, 3)
    t, i, ww = table.to(DEV), idx.to(DEV), w.to(DEV)
    ref = F.embedding_bag(i, t, per_sample_weights=ww, mode="sum")
    close(K.bag_forward(i, ww, t), ref)
    tb = t.bfloat16()
    ref_b = F.embedding_bag(i, tb.float(), per_sample_weights=ww, mode="sum")
    close(K.bag_forward(i, ww, tb), ref_b)


@pytest.mark.parametrize("rows,D,N,K_,dtype", [
    (512, 32, 16, 128, torch.float32), (65536, 384, 256, 128, torch.float32), (4096, 384, 64, 128, torch.bfloat16),
    (1000, 23, 8, 40, torch.float32), (64, 8, 300, 128, torch.float32), (4096, 96, 8192, 128, torch.float32)])
def test_bag_backward_vs_oracle(rows, D, N, K_, dtype):
    """acc bit-exact under the kernel's chunked summation schedule; gw to fp32 rounding; touched exact.
    The accumulator starts pre-filled (as in the reference's test)."""
    table, idx, w, g = make(rows, D, N, K_, rows * 3 + D, dtype=dtype)
    wt = w.to(dtype)
    acc = torch.ones(rows, D, device=DEV)
    touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
    gw = K.bag_backward_rows(g.to(DEV), idx.to(DEV), wt.to(DEV), table.to(DEV), acc, touched).cpu()
    acc_o = np.ones((rows, D), np.float32)
    t_o = np.zeros(rows, np.uint8)
    tab_np = bits_of_bf16(table) if dtype == torch.bfloat16 else table.numpy()
    gw_o = O.bag_backward(g.numpy(), idx.numpy(), wt.float().numpy(), tab_np, acc_o, t_o,
                          bf16=dtype == torch.bfloat16, chunk=chunk_positions(N * K_))
    assert torch.equal(acc.cpu(), torch.from_numpy(acc_o))
    assert torch.equal(touched.cpu(), torch.from_numpy(t_o.astype(bool)))
    close(gw, gw_o)


def test_bag_backward_golden():
    g = golden("bag.npz")
    rows, D = g["table"].shape
    acc = torch.ones(rows, D, device=DEV)
    touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
    gw = K.bag_backward_rows(torch.from_numpy(g["g"]).to(DEV), torch.from_numpy(g["idx"]).to(DEV),
                             torch.from_numpy(g["w"]).to(DEV), torch.from_numpy(g["table"]).to(DEV), acc, touched)
    close(gw.cpu(), g["gw"])
    close(acc.cpu(), g["acc"])
    assert torch.equal(touched.cpu(), torch.from_numpy(g["touched"]))


def test_bag_backward_deterministic_and_matches_torch_large():
    """262k x 384 table, 4096 tokens x 128 reads with hot rows (runs span many chunks): two runs are
    bit-identical, and agree with the PyTorch reference accumulation (index_put_) to rel 1e-5."""
    rows, D, N = 512 ** 2, 384, 4096
    table, idx, w, g = make(rows, D, N, 128, 99)
    t, i, ww, gg = table.to(DEV), idx.to(DEV), w.to(DEV), g.to(DEV)
    outs = []
    for _ in range(2):
        acc = torch.zeros(rows, D, device=DEV)
        touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
        gw = K.bag_backward_rows(gg, i, ww, t, acc, touched)
        outs.append((acc, touched, gw))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][2], outs[1][2])
    ref = torch.zeros(rows, D, device=DEV)
    flat = i.reshape(-1)
    ref.index_put_((flat,), gg.repeat_interleave(128, 0) * ww.reshape(-1, 1), accumulate=True)
    close(outs[0][0], ref)
    ref_gw = (t[flat].view(N, 128, D) * gg[:, None, :]).sum(-1)
    close(outs[0][2], ref_gw)
    tref = torch.zeros(rows, dtype=torch.bool, device=DEV)
    tref[flat] = True
    assert torch.equal(outs[0][1], tref)


def test_bag_backward_weight_grad_only():
    """acc / touched None (frozen table): only the per-sample-weight gradient."""
    table, idx, w, g = make(1000, 64, 16, 32, 5)
    gw = K.bag_backward_rows(g.to(DEV), idx.to(DEV), w.to(DEV), table.to(DEV), None, None).cpu()
    close(gw, (table[idx] * g[:, None, :]).sum(-1))


def test_out_of_range_rows_are_flagged_not_trapped():
    table, idx, w, g = make(100, 16, 4, 8, 1)
    idx[1, 3] = 100
    with pytest.raises(IndexError, match="out of range"):
        K.bag_forward(idx.to(DEV), w.to(DEV), table.to(DEV))
    idx[1, 3] = -1
    acc = torch.zeros(100, 16, device=DEV)
    touched = torch.zeros(100, dtype=torch.bool, device=DEV)
    with pytest.raises(IndexError, match="out of range"):
        K.bag_backward_rows(g.to(DEV), idx.to(DEV), w.to(DEV), table.to(DEV), acc, touched)
    torch.cuda.synchronize()     # the context is still usable
    assert int(touched.sum()) > 0


@pytest.mark.parametrize("K_", [96, 48, 40])
@pytest.mark.parametrize("kind", ["fp32", "bf16", "q4"])
def test_bag_infer_vs_oracle(K_, kind):
    """Inference bag with the fused swilu product and bf16 output, partial last lookup blocks."""
    gen = torch.Generator().manual_seed(7)
    rows, D, N = 4096, 64, 32
    table = torch.randn(rows, D, generator=gen) * D ** -0.5
    idx = torch.randint(0, rows, (N, K_), generator=gen)
    w = torch.softmax(torch.randn(N, K_, generator=gen), -1)
    pre = torch.randn(N, D, generator=gen).bfloat16()
    if kind == "fp32":
        t, sc, tab_np, tt = table, None, table.numpy(), "f32"
    elif kind == "bf16":
        t, sc = table.bfloat16(), None
        tab_np, tt = bits_of_bf16(t), "bf16"
    else:
        t, sc = K.quantize_q4(table.to(DEV))
        p_o, s_o = O.quantize_q4(table.numpy())
        assert np.array_equal(t.cpu().numpy(), p_o) and np.array_equal(sc.cpu().view(torch.int16).numpy().view(np.uint16), s_o)
        tab_np, tt = p_o, "q4"
    s_np = None if sc is None else sc.cpu().view(torch.int16).numpy().view(np.uint16)
    dev = lambda x: None if x is None else x.to(DEV)  # noqa: E731
    plain = K.bag_infer(idx.to(DEV), w.to(DEV), dev(t), dev(sc)).cpu()
    ref_plain = O.bag_infer(idx.numpy(), w.numpy(), tab_np, tt, scales=s_np)
    assert torch.equal(plain, torch.from_numpy(ref_plain))              # same fmaf order: bit for bit
    sw = K.bag_infer(idx.to(DEV), w.to(DEV), dev(t), dev(sc), pre=pre.to(DEV)).cpu()
    ref_sw = O.bag_infer(idx.numpy(), w.numpy(), tab_np, tt, scales=s_np, pre=bits_of_bf16(pre))
    close(sw, ref_sw)
    ob = K.bag_infer(idx.to(DEV), w.to(DEV), dev(t), dev(sc), pre=pre.to(DEV), out_bf16=True).cpu()
    scale = float(np.abs(ref_sw).max())
    torch.testing.assert_close(ob.float(), torch.from_numpy(ref_sw).bfloat16().float(), rtol=2 ** -7,
                               atol=2 ** -8 * scale)
    if kind != "q4":
        close(K.bag_forward(idx.to(DEV), w.to(DEV), t.to(DEV)).cpu(), ref_plain)


def test_bag_infer_golden():
    g = golden("infer.npz")
    idx, w = torch.from_numpy(g["idx"]).to(DEV), torch.from_numpy(g["w"]).to(DEV)
    pre = bf16_from_bits(g["pre"]).to(DEV)
    packed = torch.from_numpy(g["packed"]).to(DEV)
    scales = bf16_from_bits(g["scales"]).view(torch.float16).to(DEV)
    q, s = K.quantize_q4(torch.from_numpy(g["table"]).to(DEV))
    assert torch.equal(q, packed) and torch.equal(s, scales)
    for kind, t, sc in (("fp32", torch.from_numpy(g["table"]).to(DEV), None),
                        ("bf16", torch.from_numpy(g["table"]).bfloat16().to(DEV), None), ("q4", packed, scales)):
        close(K.bag_infer(idx, w, t, sc).cpu(), g[f"{kind}_plain"], msg=kind)
        close(K.bag_infer(idx, w, t, sc, pre=pre).cpu(), g[f"{kind}_swilu"], msg=kind)
        ob = K.bag_infer(idx, w, t, sc, pre=pre, out_bf16=True).cpu().float()
        ref = torch.from_numpy(g[f"{kind}_swilu"])
        torch.testing.assert_close(ob, bf16_from_bits(g[f"{kind}_swilu_bf16"]).float(), rtol=2 ** -7,
                                   atol=2 ** -8 * float(ref.abs().max()))


def test_large_table_offsets():
    """6M x 384 table (2.3 G elements > 2^31), lookups of rows beyond 5.6M (row * 384 > 2^31): bag forward,
    backward and lazy Adam against PyTorch on the touched rows (the reference's test_large_table_offsets)."""
    rows, D, N, K_ = 6_000_000, 384, 1024, 128
    gen = torch.Generator(device=DEV).manual_seed(0)
    table = torch.randn(rows, D, device=DEV, generator=gen) * D ** -0.5
    idx = torch.randint(rows - 400_000, rows, (N, K_), device=DEV, generator=gen)
    idx[:, :8] = torch.randint(0, rows, (N, 8), device=DEV, generator=gen)
    w = torch.softmax(torch.randn(N, K_, device=DEV, generator=gen), -1)
    g = torch.randn(N, D, device=DEV, generator=gen)
    rows_read = table[idx.reshape(-1)].view(N, K_, D)
    close(K.bag_forward(idx, w, table), (w[..., None] * rows_read).sum(1))
    acc = torch.zeros_like(table)
    touched = torch.zeros(rows, dtype=torch.bool, device=DEV)
    gw = K.bag_backward_rows(g, idx, w, table, acc, touched)
    close(gw, (rows_read * g[:, None, :]).sum(-1))
    uniq, inv = torch.unique(idx.reshape(-1), return_inverse=True)
    ref_acc = torch.zeros(uniq.numel(), D, device=DEV).index_add_(0, inv, (w[..., None] * g[:, None, :]).view(-1, D))
    close(acc[uniq], ref_acc)
    assert int(touched.sum()) == uniq.numel() and bool(touched[uniq].all())
    del rows_read
    m, v = torch.zeros_like(table), torch.zeros_like(table)
    p0 = table[uniq].clone()
    g_used = acc[uniq].clone()
    probe = torch.tensor([0, rows // 2, rows - 1], device=DEV)
    probe = probe[~touched[probe]]
    before = table[probe].clone()
    K.lazy_adam_step(table, m, v, acc, touched, 1.0, 1, 2.4e-3, 0.9, 0.95, 1e-8)
    m_ref, v_ref = 0.1 * g_used, 0.05 * g_used * g_used
    p_ref = p0 - (2.4e-3 / 0.1) * m_ref / (v_ref.sqrt() / 0.05 ** 0.5 + 1e-8)
    close(table[uniq], p_ref)
    assert torch.equal(table[probe], before)
    assert not touched.any() and torch.count_nonzero(acc[uniq]) == 0
