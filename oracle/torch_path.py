"""TEST INFRASTRUCTURE ONLY: the reference's PyTorch path for the product-key memory layer, restated with the same
torch operations (re133/sparse-memory-lm; file:line per function). It is the layer-level floating-point oracle of
the tests and the CPU baseline that bench.py times on the host cores; the product never imports it.

  TorchPKM          smlm/pkm.py:33-228 with impl="torch" (einsum scores, torch.topk selection, fp32 softmax,
                    row-sparse value bag); parameter names match, so state_dicts load both ways.
  row_sparse_bag    smlm/sparse_values.py:66-123, the aten _embedding_bag forward and the per-sample-weight
                    backward + index_put_(accumulate=True) into RowStore.acc, touched[flat] = True.
  TorchLazyRowAdam  smlm/sparse_values.py:270-305: one torch Adam over the whole table with the unread rows'
                    values and moments saved before and written back after.
  clip_row_sparse   smlm/sparse_values.py:137-151.

canonical=True re-selects with the order (score descending, index ascending) at both stages (a stable sort
instead of torch.topk, whose tie order is unspecified); it equals the reference whenever no two candidates tie
at a selection boundary.
"""
import math

import torch
import torch.nn.functional as F
from torch import nn

CHUNK = 1 << 18


class RowStore:
    def __init__(self, table):
        self.acc = torch.zeros_like(table, dtype=torch.promote_types(table.dtype, torch.float32))
        self.touched = torch.zeros(table.shape[0], dtype=torch.bool, device=table.device)
        self.grad_scale = 1.0

    def reset(self):
        self.acc.zero_()
        self.touched.zero_()
        self.grad_scale = 1.0


def row_store(table):
    st = getattr(table, "row_store_ref", None)
    if st is None or st.acc.shape != table.shape:
        st = table.row_store_ref = RowStore(table)
    return st


class _Bag(torch.autograd.Function):
    """sparse_values.py:66-107, torch branch."""

    @staticmethod
    def forward(ctx, weights, indices, table, store):
        n, j = indices.shape
        flat = indices.reshape(-1).contiguous()
        w = weights.reshape(-1).to(table.dtype).contiguous()
        offsets = torch.arange(0, n * j, j, device=indices.device)
        out, offset2bag, _, _ = torch.ops.aten._embedding_bag(table, flat, offsets, False, 0, False, w, False, -1)
        if offset2bag.numel() != flat.numel():
            offset2bag = torch.arange(n, device=indices.device).repeat_interleave(j)
        ctx.save_for_backward(w, flat, offsets, offset2bag)
        ctx.table, ctx.store, ctx.wshape, ctx.wdtype = table, store, weights.shape, weights.dtype
        return out

    @staticmethod
    def backward(ctx, grad_out):
        table, store = ctx.table, ctx.store
        g = grad_out.contiguous().to(store.acc.dtype)
        w, flat, offsets, offset2bag = ctx.saved_tensors
        gw = torch.ops.aten._embedding_bag_per_sample_weights_backward(g.to(table.dtype), table, flat, offsets,
                                                                       offset2bag, 0, -1)
        for a in range(0, flat.numel(), CHUNK):
            contrib = g.index_select(0, offset2bag[a:a + CHUNK]).mul_(w[a:a + CHUNK, None].to(g.dtype))
            store.acc.index_put_((flat[a:a + CHUNK],), contrib, accumulate=True)
        store.touched[flat] = True
        ctx.table = ctx.store = None
        return gw.view(ctx.wshape).to(ctx.wdtype), None, None, None


def row_sparse_bag(indices, weights, table):
    """sparse_values.py:110-123 (torch)."""
    if not torch.is_grad_enabled():
        return F.embedding_bag(indices, table, per_sample_weights=weights.to(table.dtype), mode="sum")
    return _Bag.apply(weights, indices, table, row_store(table))


def canonical_topk(s, k, index=None):
    """Top-k along the last dim by (value descending, index ascending). index: the index each entry carries
    (defaults to its position)."""
    if index is None:
        vals, order = s.sort(dim=-1, descending=True, stable=True)
        return vals[..., :k], order[..., :k]
    by_index = index.argsort(dim=-1)
    s2 = s.gather(-1, by_index)
    vals, order = s2.sort(dim=-1, descending=True, stable=True)
    pos = by_index.gather(-1, order[..., :k])
    return vals[..., :k], pos


class TorchPKM(nn.Module):
    """pkm.py:33-228 with impl="torch" and value_grad="row_sparse" (dense grads with value_grad="dense")."""

    def __init__(self, d_in, d_out, n_keys=512, heads=4, knn=32, k_dim=256, v_dim=-1, query_norm="batchnorm",
                 swilu=True, value_grad="row_sparse", canonical=True):
        super().__init__()
        self.d_in, self.d_out = d_in, d_out
        self.n_keys, self.heads, self.knn, self.k_dim = n_keys, heads, knn, k_dim
        self.v_dim = v_dim if v_dim > 0 else d_out
        self.swilu, self.value_grad, self.canonical = swilu, value_grad, canonical
        self.keys = nn.Parameter(torch.empty(heads, 2, n_keys, k_dim // 2))
        self.log_score_scale = None
        self.query_proj = nn.Linear(d_in, heads * k_dim, bias=True)
        self.query_norm = nn.BatchNorm1d(heads * k_dim) if query_norm == "batchnorm" else None
        self.values = nn.Embedding(n_keys ** 2, self.v_dim)
        if swilu:
            self.swilu_proj = nn.Linear(d_in, self.v_dim)
            self.value_proj = nn.Linear(self.v_dim, d_out)
        self.values.weight.pk_value_param = True

    def subkey_scores(self, query):
        """pkm.py:117-123"""
        half = self.k_dim // 2
        s1 = torch.einsum("nhd,hkd->nhk", query[..., :half], self.keys[:, 0])
        s2 = torch.einsum("nhd,hkd->nhk", query[..., half:], self.keys[:, 1])
        return s1, s2

    def get_indices(self, query):
        """pkm.py:125-136. With `forced_indices` set (N, heads, knn), the selection is taken from there and the
        scores are gathered from this path's own sub-key scores (same gradient flow as the top-k gather), so
        everything downstream can be compared for a given selection."""
        N = query.shape[0]
        knn, n = self.knn, self.n_keys
        s1, s2 = self.subkey_scores(query)
        forced = getattr(self, "forced_indices", None)
        if forced is not None:
            scores = s1.gather(-1, forced // n) + s2.gather(-1, forced % n)
            return scores, forced
        if self.canonical:
            s1, i1 = canonical_topk(s1, knn)
            s2, i2 = canonical_topk(s2, knn)
        else:
            s1, i1 = s1.topk(knn, dim=-1)
            s2, i2 = s2.topk(knn, dim=-1)
        all_s = (s1.unsqueeze(-1) + s2.unsqueeze(-2)).view(N, self.heads, knn * knn)
        all_i = (i1.unsqueeze(-1) * n + i2.unsqueeze(-2)).view(N, self.heads, knn * knn)
        if self.canonical:
            scores, best = canonical_topk(all_s, knn, all_i)
        else:
            scores, best = all_s.topk(knn, dim=-1)
        return scores, all_i.gather(-1, best)

    def forward(self, x):
        """pkm.py:150-157, 186-228 (training / no-autocast branch)."""
        shape = x.shape
        x = x.reshape(-1, self.d_in)
        N = x.shape[0]
        q = self.query_proj(x)
        if self.query_norm is not None:
            q = self.query_norm(q.to(self.query_norm.weight.dtype))
        q = q.view(N, self.heads, self.k_dim)
        scores, indices = self.get_indices(q)
        weights = F.softmax(scores.float(), dim=-1)
        self.last_indices, self.last_scores, self.last_weights = indices.detach(), scores.detach(), weights.detach()
        idx, w = indices.view(N, -1), weights.view(N, -1)
        if self.value_grad == "row_sparse":
            out = row_sparse_bag(idx, w, self.values.weight)
        else:
            out = F.embedding_bag(idx, self.values.weight, per_sample_weights=w.to(self.values.weight.dtype),
                                  mode="sum")
        if self.swilu:
            out = self.value_proj(out * F.silu(self.swilu_proj(x)).to(out.dtype))
        return out.view(*shape[:-1], self.d_out)


def clip_row_sparse(tables, max_norm):
    """sparse_values.py:137-151"""
    norms = [row_store(t).acc.norm() for t in tables]
    total = torch.linalg.vector_norm(torch.stack(norms))
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    for t in tables:
        row_store(t).grad_scale = coef
    return total


class TorchLazyRowAdam:
    """sparse_values.py:270-305, fp32 torch path."""

    def __init__(self, params, lr, betas=(0.9, 0.95), eps=1e-8):
        self.params = list(params)
        self.lr, self.betas, self.eps = lr, betas, eps
        self.adam = {p: torch.optim.Adam([p], lr=lr, betas=betas, eps=eps) for p in self.params}

    @torch.no_grad()
    def step(self):
        for p in self.params:
            st = row_store(p)
            if not bool(st.touched.any()):
                continue
            adam = self.adam[p]
            state = adam.state[p]
            unread = (~st.touched).nonzero().squeeze(1)
            keep = [p.index_select(0, unread)]
            if state:
                keep += [state["exp_avg"].index_select(0, unread), state["exp_avg_sq"].index_select(0, unread)]
            scale = st.grad_scale
            if not (isinstance(scale, float) and scale == 1.0):
                st.acc.mul_(scale)
            p.grad = st.acc
            adam.step()
            p.grad = None
            p.index_put_((unread,), keep[0])
            if len(keep) == 3:
                state["exp_avg"].index_put_((unread,), keep[1])
                state["exp_avg_sq"].index_put_((unread,), keep[2])
            else:
                state["exp_avg"].index_fill_(0, unread, 0.0)
                state["exp_avg_sq"].index_fill_(0, unread, 0.0)
            st.reset()

    def state(self, p):
        return self.adam[p].state[p]


def init_like_reference(mem, seed=0):
    """Config-1 initialisation: query N(0, 0.02), bias 0, sub-keys N(0, 1/128)
    (variance 1/(k_dim/2)), values N(0, v_dim^-0.5)."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        mem.query_proj.weight.copy_(torch.randn(mem.query_proj.weight.shape, generator=g) * 0.02)
        mem.query_proj.bias.zero_()
        mem.keys.copy_(torch.randn(mem.keys.shape, generator=g) * math.sqrt(1.0 / (mem.k_dim // 2)))
        mem.values.weight.copy_(torch.randn(mem.values.weight.shape, generator=g) * mem.v_dim ** -0.5)
