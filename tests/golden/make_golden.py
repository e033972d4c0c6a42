"""Generates the golden fixtures in this directory by running the REFERENCE implementation
(re133/sparse-memory-lm, imported read-only from a local checkout) on seeded inputs.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/reference [fixture names ...]

(or with the reference checkout's path in SMLM_REFERENCE and "-" as the first argument)

The Triton kernels of the reference run in Triton's CPU interpreter (TRITON_INTERPRET=1), its PyTorch path on the
CPU. Each .npz holds the inputs and the reference's outputs; the tests pin the CPU oracle (oracle/) to them and
check the CUDA kernels against both. Nothing at test time needs the reference checkout.
"""
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"            # before triton is imported
if len(sys.argv) < 2:
    sys.exit("usage: make_golden.py /path/to/reference|- [fixture names ...]")
REF = os.environ.get("SMLM_REFERENCE", "") if sys.argv[1] == "-" else sys.argv[1]
if not os.path.isdir(os.path.join(REF, "smlm")):
    sys.exit(f"make_golden.py: no reference checkout (smlm/) at {REF!r}")
sys.path.insert(0, REF)
OUT = os.path.dirname(os.path.abspath(__file__))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from smlm import kernels as RK  # noqa: E402
from smlm.pkm import ProductKeyMemory  # noqa: E402
from smlm.row_optim import RowWiseOptimizer  # noqa: E402
from smlm.sparse_values import LazyRowAdam, RowStore, _RowSparseBag, row_store  # noqa: E402


def bits(t):
    """bf16 tensor -> uint16 bit patterns (a copy: later in-place updates of t do not show through)."""
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def save(name, **arrays):
    path = os.path.join(OUT, name)
    np.savez_compressed(path, **{k: (v.detach().numpy() if torch.is_tensor(v) else np.asarray(v))
                                 for k, v in arrays.items()})
    print(f"{name}: {os.path.getsize(path)} bytes")


def skewed_indices(rows, N, K, gen):
    """tests/test_kernels.py:55-61 of the reference: 20% of the reads on 8 hot rows."""
    idx = torch.randint(0, rows, (N, K), generator=gen)
    hot = torch.randint(0, rows, (8,), generator=gen)
    mask = torch.rand(N, K, generator=gen) < 0.2
    idx[mask] = hot[torch.randint(0, 8, (int(mask.sum()),), generator=gen)]
    return idx


def reference_select(s1, s2, knn):
    """tests/test_kernels.py:128-135 of the reference (torch.topk path)."""
    N, H, NK = s1.shape
    a1, i1 = s1.topk(knn, -1)
    a2, i2 = s2.topk(knn, -1)
    alls = (a1.unsqueeze(-1) + a2.unsqueeze(-2)).view(N, H, -1)
    alli = (i1.unsqueeze(-1) * NK + i2.unsqueeze(-2)).view(N, H, -1)
    sc, best = alls.topk(knn, -1)
    return sc, alli.gather(-1, best), torch.softmax(sc.float(), -1)


def gen_select_bf16():
    cases = [(64, 2, 16, 4), (96, 4, 64, 8), (4, 2, 4096, 32), (64, 4, 256, 32), (16, 4, 1024, 32), (8, 3, 32, 5)]
    out = {}
    for c, (N, H, NK, knn) in enumerate(cases):
        gen = torch.Generator().manual_seed(N + NK)
        s1 = torch.randn(N, H, NK, generator=gen).bfloat16()
        s2 = torch.randn(N, H, NK, generator=gen).bfloat16()
        if c == len(cases) - 1:        # coarse grid: many exactly equal scores
            s1 = (torch.randint(-4, 5, (N, H, NK), generator=gen).float() / 4).bfloat16()
            s2 = (torch.randint(-4, 5, (N, H, NK), generator=gen).float() / 4).bfloat16()
        rs, ri, rw = reference_select(s1, s2, knn)
        ts, ti, tw = RK.pk_select(s1, s2, knn) if (NK & (NK - 1)) == 0 and (knn & (knn - 1)) == 0 else (rs, ri, rw)
        out.update({f"c{c}_shape": np.array([N, H, NK, knn]), f"c{c}_s1": bits(s1), f"c{c}_s2": bits(s2),
                    f"c{c}_torch_scores": bits(rs), f"c{c}_torch_idx": ri, f"c{c}_torch_w": rw,
                    f"c{c}_triton_scores": bits(ts), f"c{c}_triton_idx": ti, f"c{c}_triton_w": tw})
    save("select_bf16.npz", n_cases=len(cases), **out)


def gen_select_f32():
    """fp32 scores through the reference's own module: ProductKeyMemory.subkey_scores / get_indices."""
    cases = [(64, 3, 16, 8, 16), (200, 3, 32, 5, 16), (32, 4, 128, 32, 64), (8, 2, 8, 1, 16)]
    out = {}
    for c, (N, H, NK, knn, kdim) in enumerate(cases):
        torch.manual_seed(c)
        mem = ProductKeyMemory(24, 24, n_keys=NK, heads=H, knn=knn, k_dim=kdim, query_norm="none", swilu=False)
        with torch.no_grad():
            mem.keys.normal_(0, (kdim // 2) ** -0.5)
        q = torch.randn(N, H, kdim, generator=torch.Generator().manual_seed(100 + c))
        with torch.no_grad():
            s1, s2 = mem.subkey_scores(q)
            sc, idx = mem.get_indices(q)
            w = torch.softmax(sc.float(), -1)
        out.update({f"c{c}_shape": np.array([N, H, NK, knn, kdim]), f"c{c}_q": q, f"c{c}_keys": mem.keys.detach(),
                    f"c{c}_s1": s1, f"c{c}_s2": s2, f"c{c}_scores": sc, f"c{c}_idx": idx, f"c{c}_w": w})
    save("select_f32.npz", n_cases=len(cases), **out)


def gen_select_backward():
    N, H, NK, knn = 16, 2, 64, 8
    gen = torch.Generator().manual_seed(7)
    s1 = torch.randn(N, H, NK, generator=gen).bfloat16().requires_grad_()
    s2 = torch.randn(N, H, NK, generator=gen).bfloat16().requires_grad_()
    g = torch.randn(N, H, knn, generator=gen)
    sc, idx, w = RK.PKSelect.apply(s1, s2, knn)
    (w * g).sum().backward()
    save("select_backward.npz", s1=bits(s1.detach()), s2=bits(s2.detach()), g=g, idx=idx, w=w.detach(),
         ds1=bits(s1.grad), ds2=bits(s2.grad), shape=np.array([N, H, NK, knn]))


def gen_bag():
    """sparse_values._RowSparseBag (torch branch) as in the reference's test_bag_backward_rows_matches_reference
    at its interpreter size, with a pre-filled accumulator; plus bf16-table forwards."""
    rows, D, N, K = 512, 32, 16, 128
    gen = torch.Generator().manual_seed(rows)
    table = torch.randn(rows, D, generator=gen) * D ** -0.5
    idx = skewed_indices(rows, N, K, gen)
    w = torch.softmax(torch.randn(N, K, generator=gen), -1)
    g = torch.randn(N, D, generator=gen)
    st = RowStore(table)
    st.acc.add_(1.0)
    wr = w.clone().requires_grad_()
    y = _RowSparseBag.apply(wr, idx, table, st, "torch")
    y.backward(g)
    tb = table.bfloat16()
    y_bf16 = torch.nn.functional.embedding_bag(idx, tb.float(), per_sample_weights=w.bfloat16().float(), mode="sum")
    save("bag.npz", table=table, idx=idx, w=w, g=g, out=y.detach(), gw=wr.grad, acc=st.acc, touched=st.touched,
         table_bf16=bits(tb), out_bf16_table=y_bf16)


def gen_lazy_adam():
    """LazyRowAdam (torch fp32 path), three steps with a clip factor of 0.5 at the second, as the reference's
    test_lazy_adam_kernel_matches_reference at its interpreter size."""
    rows, D, N = 512, 16, 8
    gen = torch.Generator().manual_seed(11)
    base = torch.randn(rows, D, generator=gen) * D ** -0.5
    p = torch.nn.Parameter(base.clone())
    opt = LazyRowAdam([p], lr=2.4e-3, betas=(0.9, 0.95), eps=1e-8, impl="torch")
    arrays = {"base": base}
    for step in range(3):
        idx = skewed_indices(rows, N, 128, gen)
        grad_rows = torch.randn(idx.numel(), D, generator=gen)
        scale = 0.5 if step == 1 else 1.0
        st = row_store(p)
        st.acc.index_put_((idx.reshape(-1),), grad_rows, accumulate=True)
        st.touched[idx.reshape(-1)] = True
        arrays[f"acc{step}"] = st.acc.clone()
        arrays[f"touched{step}"] = st.touched.clone()
        st.grad_scale = scale
        opt.step()
        s = opt.state[p]
        arrays[f"p{step}"] = p.detach().clone()
        arrays[f"m{step}"] = s["exp_avg"].clone()
        arrays[f"v{step}"] = s["exp_avg_sq"].clone()
        arrays[f"scale{step}"] = np.float32(scale)
    save("lazy_adam.npz", lr=np.float64(2.4e-3), beta1=np.float64(0.9), beta2=np.float64(0.95),
         eps=np.float64(1e-8), **arrays)


def gen_lazy_adam_lowmem():
    """LazyRowAdam with bf16 / int8 moments: the reference's torch path (after steps 0, 3, 7, 11) and its Triton
    kernel (interpreter; final state) on the scenario of its test_triton_matches_torch_in_each_state_mode (17 rows,
    per-row gradient scales 1e-7 .. 1e3, 7 rows per step, clip factor 0.25 every third step), 12 steps, widths 23
    and 384."""
    arrays = {}
    for mode in ("bf16", "int8"):
        for dim in (23, 384):
            for impl in ("torch", "triton"):
                gen = torch.Generator().manual_seed(13)
                initial = torch.randn(17, dim, generator=gen) * 0.05
                p = torch.nn.Parameter(initial.clone())
                opt = LazyRowAdam([p], lr=0.002, state_dtype=mode, impl=impl)
                row_scales = torch.logspace(-7, 3, 17)[:, None]
                key = f"{mode}_{dim}_{impl}"
                arrays[f"{mode}_{dim}_initial"] = initial
                for step in range(12):
                    rows = torch.randperm(17, generator=gen)[:7]
                    grads = torch.randn(7, dim, generator=gen) * row_scales[rows]
                    scale = 0.25 if step % 3 == 0 else 1.0
                    st = row_store(p)
                    st.acc[rows] = grads
                    st.touched[rows] = True
                    st.grad_scale = scale
                    opt.step()
                    s = opt.state[p]
                    arrays[f"{mode}_{dim}_rows{step}"] = rows
                    arrays[f"{mode}_{dim}_grads{step}"] = grads
                    arrays[f"{mode}_{dim}_scale{step}"] = np.float32(scale)
                    if step not in ((11,) if impl == "triton" else (0, 3, 7, 11)):
                        continue                    # checkpoints of the trajectory (the kernel: final state)
                    arrays[f"{key}_p{step}"] = p.detach().clone()
                    m, v = s["exp_avg"], s["exp_avg_sq"]
                    arrays[f"{key}_m{step}"] = bits(m) if mode == "bf16" else m.clone()
                    arrays[f"{key}_v{step}"] = bits(v) if mode == "bf16" else v.clone()
                    if mode == "int8":
                        arrays[f"{key}_ms{step}"] = s["exp_avg_scale"].clone()
                        arrays[f"{key}_vs{step}"] = s["exp_avg_sq_scale"].clone()
    save("lazy_adam_lowmem.npz", lr=np.float64(0.002), beta1=np.float64(0.9), beta2=np.float64(0.95),
         eps=np.float64(1e-8), **arrays)


def gen_rowwise():
    """RowWiseOptimizer on a host table, torch formulas (SMLM_HOST_C=0) and the C loop (=1); the visits of the
    reference's test_host_path_matches_formula_and_keeps_unread_rows."""
    arrays = {}
    for kind in ("rowrms", "rowadagrad"):
        for c in ("0", "1"):
            os.environ["SMLM_HOST_C"] = c
            gen = torch.Generator().manual_seed(1)
            initial = torch.randn(300, 24, generator=gen)
            p = torch.nn.Parameter(initial.clone())
            p.host_values = True
            p.pk_value_param = True
            opt = RowWiseOptimizer([p], lr=0.01, kind=kind)
            visits = [torch.arange(300), torch.tensor([1, 2, 7]), torch.tensor([4, 8, 299]), torch.tensor([1, 7, 150])]
            for s, rows in enumerate(visits):
                st = row_store(p)
                for mb in range(2):
                    gr = torch.randn(rows.numel(), 24, generator=gen)
                    st.acc.index_add_(0, rows, gr)
                    st.touched[rows] = True
                if c == "0":
                    arrays[f"{kind}_acc{s}"] = st.acc.clone()
                    arrays[f"{kind}_touched{s}"] = st.touched.clone()
                opt.step()
            arrays[f"{kind}_c{c}_p"] = p.detach().clone()
            arrays[f"{kind}_c{c}_v"] = opt.state[p]["v"].clone()
            if kind == "rowrms":
                arrays[f"{kind}_c{c}_n"] = opt.state[p]["n"].clone()
            arrays["initial"] = initial
    os.environ.pop("SMLM_HOST_C", None)
    save("rowwise.npz", lr=np.float64(0.01), beta2=np.float64(0.95), eps=np.float64(1e-8), **arrays)


def gen_infer():
    """quantize_q4 / dequantize_q4 and bag_infer (Triton interpreter) for fp32 / bf16 / q4 tables, with the swilu
    product and the bf16 output; K=40 leaves the last lookup block partly used."""
    rows, D, N, K = 64, 32, 8, 40
    gen = torch.Generator().manual_seed(5)
    table = torch.randn(rows, D, generator=gen) * D ** -0.5
    idx = torch.randint(0, rows, (N, K), generator=gen)
    w = torch.softmax(torch.randn(N, K, generator=gen), -1)
    pre = torch.randn(N, D, generator=gen).bfloat16()
    packed, scales = RK.quantize_q4(table)
    arrays = dict(table=table, idx=idx, w=w, pre=bits(pre), packed=packed, scales=scales.view(torch.int16).numpy().view(np.uint16),
                  deq=RK.dequantize_q4(packed, scales))
    for kind in ("fp32", "bf16", "q4"):
        if kind == "fp32":
            t, sc = table, None
        elif kind == "bf16":
            t, sc = table.bfloat16(), None
        else:
            t, sc = packed, scales
        arrays[f"{kind}_plain"] = RK.bag_infer(idx, w, t, sc)
        arrays[f"{kind}_swilu"] = RK.bag_infer(idx, w, t, sc, pre=pre)
        arrays[f"{kind}_swilu_bf16"] = bits(RK.bag_infer(idx, w, t, sc, pre=pre, out_bf16=True))
    save("infer.npz", **arrays)


def gen_layer():
    """One PKM layer (reference ProductKeyMemory, impl="torch", value_grad="row_sparse", fp32): forward, backward
    and one LazyRowAdam step; a config-1-like shape scaled down, and one with BatchNorm + swilu."""
    arrays = {}
    variants = [dict(query_norm="none", swilu=False, n_keys=16, heads=4, knn=8, k_dim=32, d=32, N=48),
                dict(query_norm="batchnorm", swilu=True, n_keys=32, heads=2, knn=4, k_dim=16, d=24, N=40)]
    for v, cfg in enumerate(variants):
        torch.manual_seed(v)
        mem = ProductKeyMemory(cfg["d"], cfg["d"], n_keys=cfg["n_keys"], heads=cfg["heads"], knn=cfg["knn"],
                               k_dim=cfg["k_dim"], query_norm=cfg["query_norm"], swilu=cfg["swilu"],
                               value_grad="row_sparse", impl="torch")
        gen = torch.Generator().manual_seed(10 + v)
        x = torch.randn(cfg["N"], cfg["d"], generator=gen)
        gout = torch.randn(cfg["N"], cfg["d"], generator=gen)
        state0 = {k: t.detach().clone() for k, t in mem.state_dict().items()}
        mem.record = True
        out = mem(x)
        out.backward(gout)
        st = row_store(mem.values.weight)
        pre = f"v{v}_"
        for k, t in state0.items():
            arrays[pre + "param_" + k] = t
        arrays.update({pre + "x": x, pre + "gout": gout, pre + "out": out.detach(), pre + "idx": mem.last_indices,
                       pre + "scores": mem.last_scores, pre + "w": mem.last_weights, pre + "acc": st.acc.clone(),
                       pre + "touched": st.touched.clone(), pre + "keys_grad": mem.keys.grad,
                       pre + "qw_grad": mem.query_proj.weight.grad, pre + "qb_grad": mem.query_proj.bias.grad,
                       pre + "cfg": np.array([cfg["n_keys"], cfg["heads"], cfg["knn"], cfg["k_dim"], cfg["d"],
                                              cfg["N"], int(cfg["query_norm"] == "batchnorm"), int(cfg["swilu"])])})
        opt = LazyRowAdam([mem.values.weight], lr=1e-3, betas=(0.9, 0.98), eps=1e-8, impl="torch")
        opt.step()
        s = opt.state[mem.values.weight]
        arrays.update({pre + "values_after": mem.values.weight.detach().clone(), pre + "m_after": s["exp_avg"],
                       pre + "v_after": s["exp_avg_sq"]})
    save("layer.npz", **arrays)


def gen_engram():
    """Engram (reference smlm/engram.py, impl="torch", value_grad="row_sparse", fp32 on the CPU): NgramHash's
    multipliers and rows, one EngramMemory forward / backward (head_dim 8 and 24, a non-zero convolution) and one
    LazyRowAdam step of its table. Token compression needs the GPT-2 vocabulary through tiktoken, which is not
    reachable offline, so the fixture replaces canonical_ids by the identity map (the hash, the module and the
    training step take the compressed ids as given)."""
    import smlm.engram as RE
    RE.canonical_ids = lambda vocab: (torch.arange(vocab, dtype=torch.int64), vocab)
    arrays = {}
    for v, head_dim in enumerate((8, 24)):
        ng = RE.NgramHash(512, orders=(2, 3), heads=2, rows=101, seed=v)
        gen = torch.Generator().manual_seed(20 + v)
        B, T, d = 2, 17, 32
        c = torch.randint(0, 512, (B, ng.history + T), generator=gen)
        c[:, :ng.history] = ng.pad
        rows = ng(c)
        torch.manual_seed(30 + v)
        e = RE.EngramMemory(d, ng.n_lookups, head_dim, 101, conv_kernel=4, dilation=max(ng.orders), impl="torch",
                            value_grad="row_sparse")
        with torch.no_grad():
            e.conv.weight.normal_(std=0.3)
        x = torch.randn(B, T, d, generator=gen).requires_grad_()
        g = torch.randn(B, T, d, generator=gen)
        state0 = {k: t.detach().clone() for k, t in e.state_dict().items()}
        y = e(x, rows)
        y.backward(g)
        st = row_store(e.values.weight)
        pre = f"v{v}_"
        for k, t in state0.items():
            arrays[pre + "param_" + k] = t
        arrays.update({pre + "c": c, pre + "mult": ng.mult, pre + "rows": rows, pre + "x": x.detach(), pre + "g": g,
                       pre + "y": y.detach(), pre + "x_grad": x.grad, pre + "wk_grad": e.w_k.weight.grad,
                       pre + "wv_grad": e.w_v.weight.grad, pre + "conv_grad": e.conv.weight.grad,
                       pre + "hnorm_grad": e.h_norm.weight.grad, pre + "acc": st.acc.clone(),
                       pre + "touched": st.touched.clone(), pre + "head_dim": np.array(head_dim)})
        opt = LazyRowAdam([e.values.weight], lr=1e-3, betas=(0.9, 0.98), eps=1e-8, impl="torch")
        opt.step()
        arrays[pre + "values_after"] = e.values.weight.detach().clone()
    save("engram.npz", **arrays)


def gen_budget():
    """Host arithmetic of the optimizer module (reference smlm/optim.py): value_table_memory of small models (one
    row-sparse memory layer; two layers sharing one table; a dense-gradient table) for every value_state /
    value_optim, and lr_multiplier over a warmup + cosine schedule. Written as JSON (errors as their type name)."""
    import json
    from smlm import optim as RO
    from smlm.model import ModelConfig, Transformer
    base = dict(vocab_size=256, d_model=64, n_layers=3, n_heads=4, ffn_hidden=128, mem_n_keys=64, max_seq_len=64)
    models = {"one_sparse": dict(base, mem_layers=[1], mem_value_grad="row_sparse"),
              "shared_sparse": dict(base, mem_layers=[0, 2], mem_share_values=True, mem_value_grad="row_sparse"),
              "dense": dict(base, mem_layers=[1], mem_value_grad="dense")}
    out = {"models": models, "memory": {}, "lr": []}
    for name, kw in models.items():
        torch.manual_seed(0)
        m = Transformer(ModelConfig(**kw))
        for vs in ("fp32", "bf16", "int8"):
            for vo in ("adam", "rowrms", "rowadagrad"):
                try:
                    r = RO.value_table_memory(m, vs, value_optim=vo)
                except ValueError as e:
                    r = {"error": type(e).__name__}
                out["memory"][f"{name}/{vs}/{vo}"] = r
    for total, warm, mn in ((100, 10, 0.1), (1000, 0, 0.0), (7, 3, 0.5)):
        out["lr"].append({"total": total, "warmup": warm, "min_ratio": mn,
                          "mult": [RO.lr_multiplier(s, total, warm, mn) for s in range(total + 2)]})
    path = os.path.join(OUT, "budget.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print(f"budget.json: {os.path.getsize(path)} bytes")


def gen_model_structure():
    """The reference model's checkpoint layout (smlm/model.py): state_dict keys, shapes and dtypes, param_counts()
    and macs_per_token() of small Transformers (one memory layer; two sharing a table; Engram layers; no BatchNorm /
    swilu; learned score scale). Engram's token compression uses the identity map (tiktoken's vocabulary is not
    reachable offline). Written as JSON."""
    import json
    import smlm.engram as RE
    from smlm.model import ModelConfig, Transformer
    RE.canonical_ids = lambda vocab: (torch.arange(vocab, dtype=torch.int64), vocab)
    base = dict(vocab_size=256, d_model=64, n_layers=4, n_heads=4, ffn_hidden=128, mem_n_keys=64, max_seq_len=64)
    models = {"sparse": dict(base, mem_layers=[1], mem_value_grad="row_sparse"),
              "shared": dict(base, mem_layers=[0, 2], mem_share_values=True, mem_value_grad="row_sparse"),
              "engram": dict(base, mem_layers=[1], eng_layers=[0, 3], eng_rows=31, eng_heads=2, eng_head_dim=8),
              "no_bn_swilu": dict(base, mem_layers=[2], mem_query_norm="none", mem_swilu=False),
              "score_scale": dict(base, mem_layers=[2], mem_score_scale="learned")}
    out = {}
    for name, kw in models.items():
        torch.manual_seed(0)
        m = Transformer(ModelConfig(**kw))
        out[name] = {"config": kw, "state_dict": [[k, list(v.shape), str(v.dtype)] for k, v in m.state_dict().items()],
                     "param_counts": m.param_counts(), "macs_per_token": m.macs_per_token(),
                     "macs_per_token_64": m.macs_per_token(64)}
    path = os.path.join(OUT, "model_structure.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print(f"model_structure.json: {os.path.getsize(path)} bytes")


GENERATORS = {"select_bf16": gen_select_bf16, "select_f32": gen_select_f32, "select_backward": gen_select_backward,
              "bag": gen_bag, "lazy_adam": gen_lazy_adam, "lazy_adam_lowmem": gen_lazy_adam_lowmem,
              "rowwise": gen_rowwise, "infer": gen_infer, "layer": gen_layer, "engram": gen_engram,
              "budget": gen_budget, "model_structure": gen_model_structure}

if __name__ == "__main__":
    # python make_golden.py [reference path] [fixture names ...]: all fixtures by default
    torch.set_num_threads(4)
    for name in (sys.argv[2:] or list(GENERATORS)):
        GENERATORS[name]()
