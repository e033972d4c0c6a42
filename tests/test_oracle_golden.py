"""Pins the CPU oracle (oracle/pkm_oracle.c, oracle/torch_path.py) to the reference's own outputs, the golden
fixtures made by tests/golden/make_golden.py from re133/sparse-memory-lm. CPU only."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import torch_path as TP
from util import bf16_from_bits, close, golden, tie_free_rows


def canonical_ok(s1, s2, knn, sc, idx, bf16):
    """Every returned index carries its returned score, the list is sorted by (score desc, index asc), no index
    twice, and the scores are the knn best pair scores of the half top-k lists."""
    s1f = torch.as_tensor(s1).float()
    s2f = torch.as_tensor(s2).float()
    N, H, NK = s1f.shape
    idx = torch.as_tensor(idx)
    own = s1f.gather(-1, idx // NK) + s2f.gather(-1, idx % NK)
    if bf16:
        own = own.bfloat16().float()
    sc = torch.as_tensor(sc).float()
    assert torch.equal(own, sc)
    flat_s = sc.view(-1, knn)
    flat_i = idx.view(-1, knn)
    ok_order = (flat_s[:, :-1] > flat_s[:, 1:]) | ((flat_s[:, :-1] == flat_s[:, 1:]) & (flat_i[:, :-1] < flat_i[:, 1:]))
    assert bool(ok_order.all())


def test_select_bf16_matches_reference():
    g = golden("select_bf16.npz")
    ties_seen = 0
    for c in range(int(g["n_cases"])):
        N, H, NK, knn = (int(x) for x in g[f"c{c}_shape"])
        s1, s2 = g[f"c{c}_s1"], g[f"c{c}_s2"]
        sc, idx, w = O.select(s1, s2, knn, bf16=True)
        sc_t = bf16_from_bits(sc).float()
        # selected scores exactly the reference's (torch.topk path and Triton kernel)
        assert np.array_equal(sc, g[f"c{c}_torch_scores"])
        assert np.array_equal(sc, g[f"c{c}_triton_scores"])
        canonical_ok(bf16_from_bits(s1), bf16_from_bits(s2), knn, sc_t, idx, bf16=True)
        # index sets equal to the reference wherever no tie makes the set ambiguous
        free = tie_free_rows(bf16_from_bits(s1), bf16_from_bits(s2), knn, bf16=True)
        ti = np.sort(g[f"c{c}_triton_idx"].reshape(-1, knn), -1)
        ri = np.sort(g[f"c{c}_torch_idx"].reshape(-1, knn), -1)
        oi = np.sort(idx.reshape(-1, knn), -1)
        assert np.array_equal(oi[free], ti[free]) and np.array_equal(oi[free], ri[free])
        ties_seen += int((~free).sum())
        np.testing.assert_allclose(w, g[f"c{c}_triton_w"], rtol=0, atol=1e-6)
        np.testing.assert_allclose(w, g[f"c{c}_torch_w"], rtol=0, atol=1e-6)
    assert ties_seen > 0          # the coarse-grid case really exercises ties


def test_select_f32_matches_reference_on_reference_scores():
    g = golden("select_f32.npz")
    for c in range(int(g["n_cases"])):
        N, H, NK, knn, kd = (int(x) for x in g[f"c{c}_shape"])
        s1, s2 = g[f"c{c}_s1"], g[f"c{c}_s2"]
        sc, idx, w = O.select(s1, s2, knn, bf16=False)
        free = tie_free_rows(torch.from_numpy(s1), torch.from_numpy(s2), knn, bf16=False)
        assert free.all()                                   # continuous scores: no ties
        assert np.array_equal(sc, g[f"c{c}_scores"])         # bit-exact scores
        # bit-exact index sets; within equal scores torch.topk's order is unspecified, ours is index ascending
        assert np.array_equal(np.sort(idx, -1), np.sort(g[f"c{c}_idx"], -1))
        canonical_ok(s1, s2, knn, sc, idx, bf16=False)
        np.testing.assert_allclose(w, g[f"c{c}_w"], rtol=0, atol=1e-6)


def test_fmaf_scores_close_to_reference_einsum():
    """The oracle's fixed-order fmaf scores agree with the reference's einsum to fp32 rounding."""
    g = golden("select_f32.npz")
    for c in range(int(g["n_cases"])):
        s1, s2 = O.subkey_scores_f32(g[f"c{c}_q"], g[f"c{c}_keys"])
        np.testing.assert_allclose(s1, g[f"c{c}_s1"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(s2, g[f"c{c}_s2"], rtol=1e-5, atol=1e-6)


def test_select_backward_matches_reference():
    g = golden("select_backward.npz")
    N, H, NK, knn = (int(x) for x in g["shape"])
    ds1, ds2 = O.select_backward(g["idx"], g["w"], g["g"], None, NK, bf16=True)
    d1, e1 = bf16_from_bits(ds1).float(), bf16_from_bits(g["ds1"]).float()
    d2, e2 = bf16_from_bits(ds2).float(), bf16_from_bits(g["ds2"]).float()
    scale = float(e1.abs().max())
    torch.testing.assert_close(d1, e1, rtol=2 ** -7, atol=2 ** -8 * scale)
    torch.testing.assert_close(d2, e2, rtol=2 ** -7, atol=2 ** -8 * scale)
    assert torch.equal(d1 != 0, e1 != 0) and torch.equal(d2 != 0, e2 != 0)


def test_bag_forward_backward_match_reference():
    g = golden("bag.npz")
    out, bad = O.bag_forward(g["idx"], g["w"], g["table"])
    assert bad == 0
    close(out, g["out"])
    acc = np.ones_like(g["table"])
    touched = np.zeros(g["table"].shape[0], np.uint8)
    gw = O.bag_backward(g["g"], g["idx"], g["w"], g["table"], acc, touched)
    close(gw, g["gw"])
    close(acc, g["acc"])
    assert np.array_equal(touched.astype(bool), g["touched"])
    # bf16 table: weights rounded to bf16 as the reference's forward does (sparse_values.py:71)
    wb = O.bf16_bits_to_f32(O.f32_to_bf16_bits(g["w"]))
    out_b, _ = O.bag_forward(g["idx"], wb, g["table_bf16"], bf16=True)
    close(out_b, g["out_bf16_table"])


def test_bag_backward_chunked_schedule_only_changes_rounding():
    g = golden("bag.npz")
    accs = []
    for chunk in (0, 64, 7):
        acc = np.zeros_like(g["table"])
        touched = np.zeros(g["table"].shape[0], np.uint8)
        O.bag_backward(g["g"], g["idx"], g["w"], g["table"], acc, touched, chunk=chunk)
        accs.append(acc)
    close(accs[1], accs[0])
    close(accs[2], accs[0])


def test_lazy_adam_matches_reference_three_steps():
    g = golden("lazy_adam.npz")
    p = g["base"].copy()
    m, v = np.zeros_like(p), np.zeros_like(p)
    pr, mr, vr = p.copy(), m.copy(), v.copy()
    for step in range(3):
        acc, touched = g[f"acc{step}"].copy(), g[f"touched{step}"].astype(np.uint8)
        prev = p.copy()
        O.lazy_adam(p, m, v, acc, touched.copy(), float(g[f"scale{step}"]), step + 1, float(g["lr"]),
                    float(g["beta1"]), float(g["beta2"]), float(g["eps"]))
        close(p, g[f"p{step}"], msg="values")
        close(m, g[f"m{step}"], msg="exp_avg")
        close(v, g[f"v{step}"], msg="exp_avg_sq")
        unread = ~g[f"touched{step}"]
        assert np.array_equal(p[unread], prev[unread])       # unread rows bit-identical
        if O.ref_lib() is not None:
            acc_r = g[f"acc{step}"].copy()
            O.ref_lazy_adam(pr, mr, vr, acc_r, touched.copy(), float(g[f"scale{step}"]), step + 1, float(g["lr"]),
                            float(g["beta1"]), float(g["beta2"]), float(g["eps"]))
            assert np.array_equal(p, pr) and np.array_equal(m, mr) and np.array_equal(v, vr)


def lowmem_replay(g, mode, dim, on_step=None):
    """Replays the fixture's 12 steps through the oracle; returns the final state."""
    key = f"{mode}_{dim}"
    p = g[f"{key}_initial"].astype(np.float32).copy()
    R = p.shape[0]
    i8 = mode == "int8"
    m = np.zeros((R, dim), np.int8 if i8 else np.uint16)
    v = np.zeros((R, dim), np.uint8 if i8 else np.uint16)
    ms, vs = np.zeros(R, np.float32), np.zeros(R, np.float32)
    for step in range(12):
        acc = np.zeros((R, dim), np.float32)
        touched = np.zeros(R, np.uint8)
        rows = g[f"{key}_rows{step}"]
        acc[rows] = g[f"{key}_grads{step}"]
        touched[rows] = 1
        prev = (p.copy(), m.copy(), v.copy(), ms.copy(), vs.copy())
        O.lazy_adam_lowmem(p, m, v, ms, vs, acc, touched, float(g[f"{key}_scale{step}"]), step + 1, float(g["lr"]),
                           float(g["beta1"]), float(g["beta2"]), float(g["eps"]), i8)
        unread = np.ones(R, bool)
        unread[rows] = False
        for a, b in zip((p, m, v, ms, vs), prev):                 # unread rows and their state bit-identical
            assert np.array_equal(a[unread], b[unread])
        assert not touched.any() and not acc.any()
        if on_step:
            on_step(step, p, m, v, ms, vs)
    return p, m, v, ms, vs


@pytest.mark.parametrize("mode", ["bf16", "int8"])
@pytest.mark.parametrize("dim", [23, 384])
def test_lazy_adam_lowmem_matches_reference(mode, dim):
    """Compact-moment lazy Adam: bit-exact against the reference's Triton kernel (kernels.py:445-495, run in the
    interpreter) after 12 steps; within fp32 ulps of its PyTorch path (sparse_values.py:206-255, whose divisions
    by Python scalars round differently) at steps 0, 3, 7, 11."""
    g = golden("lazy_adam_lowmem.npz")
    key = f"{mode}_{dim}"
    dec = lambda m, v, ms, vs: ((np.sign(m) * (m / 127.0) ** 2 * ms[:, None], (v / 255.0 * vs[:, None]) ** 4)
                                if mode == "int8" else (bf16_from_bits(m).float().numpy(),
                                                        bf16_from_bits(v).float().numpy()))

    def check_torch(step, p, m, v, ms, vs):
        t = f"{key}_torch"
        if f"{t}_p{step}" not in g:
            return
        close(p, g[f"{t}_p{step}"], msg="values vs torch path")
        ref = dec(g[f"{t}_m{step}"], g[f"{t}_v{step}"], g.get(f"{t}_ms{step}"), g.get(f"{t}_vs{step}"))
        for a, b in zip(dec(m, v, ms, vs), ref):
            scale = np.maximum(np.abs(b).max(axis=1, keepdims=True), 1e-30)
            # a stored code may sit on the other side of a rounding boundary: one code step of the row's scale
            assert np.all(np.abs(a - b) <= scale * (2.0 ** -7 if mode == "bf16" else 2.0 / 127)), "moments"

    p, m, v, ms, vs = lowmem_replay(g, mode, dim, check_torch)
    t = f"{key}_triton"
    assert np.array_equal(p, g[f"{t}_p11"])
    assert np.array_equal(m, g[f"{t}_m11"]) and np.array_equal(v, g[f"{t}_v11"])
    if mode == "int8":
        assert np.array_equal(ms, g[f"{t}_ms11"]) and np.array_equal(vs, g[f"{t}_vs11"])


@pytest.mark.parametrize("kind", ["rowrms", "rowadagrad"])
def test_rowwise_matches_reference(kind):
    g = golden("rowwise.npz")
    p = g["initial"].copy()
    v = np.zeros(p.shape[0], np.float32)
    n = np.zeros(p.shape[0], np.int32)
    for s in range(4):
        acc = g[f"{kind}_acc{s}"].copy()
        touched = g[f"{kind}_touched{s}"].astype(np.uint8)
        O.rowwise(p, acc, touched, v, n, 1.0, kind, float(g["beta2"]), float(g["eps"]), float(g["lr"]))
        assert not touched.any() and not acc.any()
    for c in ("0", "1"):
        np.testing.assert_allclose(p, g[f"{kind}_c{c}_p"], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(v, g[f"{kind}_c{c}_v"], rtol=1e-5, atol=1e-9)
        if kind == "rowrms":
            assert np.array_equal(n, g[f"{kind}_c{c}_n"])
    np.testing.assert_array_equal(p, g[f"{kind}_c1_p"])       # the reference's C loop: bit for bit


def test_q4_and_inference_bag_match_reference():
    g = golden("infer.npz")
    packed, scales = O.quantize_q4(g["table"])
    assert np.array_equal(packed, g["packed"]) and np.array_equal(scales, g["scales"])
    pre = g["pre"]
    for kind, tab, tt in (("fp32", g["table"], "f32"), ("bf16", O.f32_to_bf16_bits(g["table"]), "bf16"),
                          ("q4", g["packed"], "q4")):
        sc = g["scales"] if kind == "q4" else None
        close(O.bag_infer(g["idx"], g["w"], tab, tt, scales=sc), g[f"{kind}_plain"], msg=kind)
        ref = g[f"{kind}_swilu"]
        close(O.bag_infer(g["idx"], g["w"], tab, tt, scales=sc, pre=pre), ref, msg=kind)
        ob = O.bag_infer(g["idx"], g["w"], tab, tt, scales=sc, pre=pre, out_bf16=True)
        rb = O.bf16_bits_to_f32(g[f"{kind}_swilu_bf16"])
        scale = float(np.abs(ref).max())
        np.testing.assert_allclose(ob, rb, rtol=2 ** -7, atol=2 ** -8 * scale)


def _load_layer(g, v):
    n_keys, heads, knn, k_dim, d, N, bn, swilu = (int(x) for x in g[f"v{v}_cfg"])
    mem = TP.TorchPKM(d, d, n_keys=n_keys, heads=heads, knn=knn, k_dim=k_dim,
                      query_norm="batchnorm" if bn else "none", swilu=bool(swilu), canonical=False)
    pre = f"v{v}_param_"
    sd = {k[len(pre):]: torch.from_numpy(g[k]) for k in g.files if k.startswith(pre)}
    mem.load_state_dict(sd, strict=False)
    return mem


@pytest.mark.parametrize("v", [0, 1])
def test_torch_path_restatement_equals_reference_layer(v):
    """The torch restatement (the layer-level oracle) reproduces the reference layer: the same index selection
    exactly, floats to the rounding that torch's CPU GEMMs / index_put_ vary with the thread count."""
    g = golden("layer.npz")
    mem = _load_layer(g, v)
    x = torch.from_numpy(g[f"v{v}_x"])
    out = mem(x)
    out.backward(torch.from_numpy(g[f"v{v}_gout"]))
    st = TP.row_store(mem.values.weight)
    close(out.detach(), g[f"v{v}_out"], rtol=1e-6, atol=1e-6)
    assert torch.equal(mem.last_indices, torch.from_numpy(g[f"v{v}_idx"]))
    # torch's CPU index_put_(accumulate=True) sums in a thread-count dependent order: fp32 rounding only
    close(st.acc, g[f"v{v}_acc"], rtol=1e-6, atol=1e-6)
    assert torch.equal(st.touched, torch.from_numpy(g[f"v{v}_touched"]))
    close(mem.keys.grad, g[f"v{v}_keys_grad"], rtol=1e-6, atol=1e-6)
    close(mem.query_proj.weight.grad, g[f"v{v}_qw_grad"], rtol=1e-6, atol=1e-6)
    opt = TP.TorchLazyRowAdam([mem.values.weight], lr=1e-3, betas=(0.9, 0.98), eps=1e-8)
    opt.step()
    close(mem.values.weight.detach(), g[f"v{v}_values_after"], rtol=1e-6, atol=1e-6)
    # canonical tie rule: same selection on these (tie-free) inputs
    mem2 = _load_layer(g, v)
    mem2.canonical = True
    mem2(x)
    assert torch.equal(mem2.last_indices, mem.last_indices)


def test_oracle_select_equals_bruteforce_product_search():
    """The product-key search returns exactly the top-k of a brute-force search over all n_keys^2 keys
    (the reference's tests/test_pkm.py:16-37), here on the oracle with fp32 scores."""
    gen = torch.Generator().manual_seed(1)
    for n_keys, knn in ((16, 8), (16, 16), (32, 5), (8, 1)):
        H, half = 3, 8
        keys = torch.randn(H, 2, n_keys, half, generator=gen)
        q = torch.randn(50, H, 2 * half, generator=gen)
        s1, s2 = O.subkey_scores_f32(q.numpy(), keys.numpy())
        sc, idx, _ = O.select(s1, s2, knn, bf16=False)
        full = torch.from_numpy(s1)[..., :, None] + torch.from_numpy(s2)[..., None, :]
        bf, bi = full.reshape(50, H, -1).topk(knn, dim=-1)
        assert np.array_equal(sc, bf.numpy())
        assert np.array_equal(np.sort(idx, -1), np.sort(bi.numpy(), -1))


def test_engram_hash_oracle_and_multipliers_match_reference():
    """Engram: the oracle's n-gram hash gives the reference NgramHash's rows, and this build's NgramHash draws the
    reference's multipliers (same seed -> same rows -> checkpoints and tables stay compatible)."""
    import smlm_b200.engram as E
    g = golden("engram.npz")
    real = E.canonical_ids
    E.canonical_ids = lambda vocab: (torch.arange(vocab, dtype=torch.int64), vocab)   # GPT-2 vocabulary offline
    try:
        for v in (0, 1):
            ng = E.NgramHash(512, orders=(2, 3), heads=2, rows=101, seed=v)
            assert np.array_equal(ng.mult.numpy(), g[f"v{v}_mult"])
            rows = O.ngram_rows(g[f"v{v}_c"], ng.history, g[f"v{v}_mult"], [2, 3], 2, 101)
            assert np.array_equal(rows, g[f"v{v}_rows"])
    finally:
        E.canonical_ids = real


def test_bag_rows_subset_equals_full_backward():
    """oracle.bag_rows_subset (the sums of sampled rows only, for steps whose table does not fit host memory)
    equals the rows bag_backward leaves in a zeroed accumulator, for every chunk schedule, with padding lookups
    and hot rows whose runs cross chunks."""
    rng = np.random.default_rng(3)
    rows, d, n, k = 700, 24, 400, 48
    idx = rng.integers(0, rows, (n, k))
    idx[rng.random((n, k)) < 0.2] = 11                    # one hot row spanning many chunks
    idx[0, :7] = -1
    w = rng.standard_normal((n, k)).astype(np.float32)
    g = rng.standard_normal((n, d)).astype(np.float32)
    table = rng.standard_normal((rows, d)).astype(np.float32)
    sample = np.array([11, 0, 699, 350, 5])
    for chunk in (0, 64, 256):
        acc = np.zeros((rows, d), np.float32)
        O.bag_backward(g, idx, w, table, acc, np.zeros(rows, np.uint8), chunk=chunk)
        assert np.array_equal(O.bag_rows_subset(g, idx, w, rows, sample, chunk=chunk), acc[sample])
