"""sm_100a kernels of the product-key memory, with the Python signatures of the reference's kernel layer.

Each function below stands in for the function of the same name in re133/sparse-memory-lm smlm/kernels.py
(file:line given per function) and calls libsmlm_b200.so through its C ABI (include/smlm_b200.h). All tensors
must be CUDA tensors; nothing here has a CPU path. Kernels run on the current CUDA stream without host
synchronisation, so every function can be captured in a CUDA graph. The reference's Triton launch-shape arguments
(ch, num_warps, block_j, block_d, P, rows_per_program) are accepted by the same names and have no effect: the
CUDA kernels choose their own launch shapes.
"""
import math

import torch

from . import _lib as L


def _contig(t):
    return t if t.is_contiguous() else t.contiguous()


# ------------------------------------------------------------------------------------------ selection
def pk_select(s1, s2, knn, ch=None, num_warps=None):
    """s1, s2 (N, H, n_keys) bf16 or fp32 sub-key scores -> scores (N, H, knn) (same dtype), indices (N, H, knn)
    int64 into the n_keys^2 table, softmax weights (N, H, knn) fp32 (reference: kernels.py:214-226).

    Both half top-k, the knn x knn pair sums rounded to the score dtype, the final top-k and the softmax.
    Order: score descending, ties to the lower index (i1 * n_keys + i2 for the final list)."""
    if s1.shape != s2.shape or s1.dim() != 3 or s1.dtype != s2.dtype:
        raise ValueError("pk_select: s1 and s2 must be (N, H, n_keys) tensors of one dtype")
    dev = L.require_cuda(s1, s2)
    N, H, NK = s1.shape
    s1, s2 = _contig(s1), _contig(s2)
    scores = torch.empty(N, H, knn, dtype=s1.dtype, device=dev)
    idx = torch.empty(N, H, knn, dtype=torch.int64, device=dev)
    w = torch.empty(N, H, knn, dtype=torch.float32, device=dev)
    with L.timed("pk_select", 1):
        rc = L.lib().smlm_pk_select(L.ptr(s1), L.ptr(s2), L.dtype_code(s1.dtype), N, H, NK, knn, L.ptr(scores),
                                        L.ptr(idx), L.ptr(w), L.stream(dev))
    L.check(rc, "pk_select")
    L.after(dev, "pk_select")
    return scores, idx, w


def select_backward(idx, w, g_w, g_scores, n_keys, dtype):
    """Dense gradients (ds1, ds2) (N, H, n_keys) of the selection (reference: kernels.py:253-266)."""
    dev = L.require_cuda(idx, w, g_w, g_scores)
    N, H, knn = idx.shape
    ds1 = torch.empty(N, H, n_keys, dtype=dtype, device=dev)
    ds2 = torch.empty(N, H, n_keys, dtype=dtype, device=dev)
    g_w = None if g_w is None else _contig(g_w.float())
    g_scores = None if g_scores is None else _contig(g_scores.to(dtype))
    with L.timed("select_backward", 1):
        rc = L.lib().smlm_select_backward(L.ptr(_contig(idx)), L.ptr(_contig(w)), L.ptr(g_w), L.ptr(g_scores),
                                          L.dtype_code(dtype), N, H, n_keys, knn, L.ptr(ds1), L.ptr(ds2),
                                          L.stream(dev))
    L.check(rc, "select_backward")
    return ds1, ds2


def select_grad_entries(idx, w, g_w, g_scores, n_keys, dtype):
    """Sparse selection gradient (N * H * 2, knn) lookups into the keys viewed as (H * 2 * n_keys, half): rows
    (int64) and weights (score dtype), ds1 / ds2 of select_backward at each sub-key's first occurrence; later
    occurrences are row -1, weight 0."""
    dev = L.require_cuda(idx, w, g_w, g_scores)
    N, H, knn = idx.shape
    rows = torch.empty(N * H * 2, knn, dtype=torch.int64, device=dev)
    ew = torch.empty(N * H * 2, knn, dtype=dtype, device=dev)
    g_w = None if g_w is None else _contig(g_w.float())
    g_scores = None if g_scores is None else _contig(g_scores.to(dtype))
    with L.timed("select_grad_entries", 1):
        rc = L.lib().smlm_select_grad_entries(L.ptr(_contig(idx)), L.ptr(_contig(w)), L.ptr(g_w), L.ptr(g_scores),
                                              L.dtype_code(dtype), N, H, n_keys, knn, L.ptr(rows), L.ptr(ew),
                                              L.stream(dev))
    L.check(rc, "select_grad_entries")
    return rows, ew


def scoring_backward_sparse(q, keys, idx, w, g_w, g_scores, need_dq=True, need_dkeys=True):
    """Gradients of q (N, H, 2 half) and keys (H, 2, n_keys, half) through the selection and the sub-key scoring
    contraction, from the nonzero score gradients only: dq is a value bag over the keys, dkeys the row-sparse
    bag backward with the query halves; both accumulate in fp32 and round once to the keys' dtype, as the
    reference's autocast einsum backward does with its dense, mostly-zero (N, H, n_keys) gradients."""
    H, _, NK, half = keys.shape
    N = q.shape[0]
    rows, ew = select_grad_entries(idx, w, g_w, g_scores, NK, keys.dtype)
    table = _contig(keys).view(H * 2 * NK, half)
    dq = dk = None
    if need_dq:
        dq = shard_bag_forward(rows, ew, table, 0, out_dtype=q.dtype, name="select_dq").view(N, H, 2 * half)
    if need_dkeys:
        acc = torch.zeros(H * 2 * NK, half, dtype=torch.float32, device=keys.device)
        shard_bag_backward_rows(_contig(q).view(N * H * 2, half), rows, ew, table, 0, acc, None, want_gw=False,
                                name="select_dkeys")
        dk = acc.to(keys.dtype).view(H, 2, NK, half)
    return dq, dk


class PKSelect(torch.autograd.Function):
    """Differentiable pk_select (reference: kernels.py:240-266). Backward: softmax backward, the score gradient
    rounded to the score dtype, summed per sub-key in fp32 (selection order) and rounded once; dense
    (N, H, n_keys) gradients for the scoring contraction's backward."""

    @staticmethod
    def forward(ctx, s1, s2, knn):
        scores, idx, w = pk_select(s1, s2, knn)
        ctx.save_for_backward(idx, w)
        ctx.nk, ctx.dtype = s1.shape[-1], s1.dtype
        ctx.mark_non_differentiable(idx)
        return scores, idx, w

    @staticmethod
    def backward(ctx, g_scores, g_idx, g_w):
        idx, w = ctx.saved_tensors
        ds1, ds2 = select_backward(idx, w, g_w, g_scores, ctx.nk, ctx.dtype)
        return ds1, ds2, None


def subkey_scores_f32(q, keys):
    """Exact fp32 sub-key scores (reference: pkm.py:117-123 in fp32): q (N, H, k_dim), keys (H, 2, n_keys, k_dim/2)
    -> s1, s2 (N, H, n_keys), each score a sequential fmaf chain over the half dimension."""
    if q.dtype != torch.float32 or keys.dtype != torch.float32:
        raise ValueError("subkey_scores_f32 needs fp32 queries and keys")
    dev = L.require_cuda(q, keys)
    N, H, KD = q.shape
    Hk, two, NK, half = keys.shape
    if Hk != H or two != 2 or KD != 2 * half:
        raise ValueError(f"subkey_scores_f32: query {tuple(q.shape)} does not match keys {tuple(keys.shape)}")
    q, keys = _contig(q), _contig(keys)
    s1 = torch.empty(N, H, NK, dtype=torch.float32, device=dev)
    s2 = torch.empty(N, H, NK, dtype=torch.float32, device=dev)
    step = 65535 * 64
    for a in range(0, max(N, 1), step):
        b = min(N, a + step)
        if b <= a:
            break
        with L.timed("subkey_scores_f32", 1):
            rc = L.lib().smlm_subkey_scores_f32(L.ptr(q[a:b]), L.ptr(keys), b - a, H, NK, half, L.ptr(s1[a:b]),
                                                L.ptr(s2[a:b]), L.stream(dev))
        L.check(rc, "subkey_scores_f32")
    return s1, s2


class SubkeyScoresF32(torch.autograd.Function):
    """Exact fp32 scoring with autograd: forward the fmaf-chain kernel, backward the two contractions
    (dq = ds K, dK = ds^T q) of the reference's einsum backward."""

    @staticmethod
    def forward(ctx, q, keys):
        ctx.save_for_backward(q, keys)
        return subkey_scores_f32(q, keys)

    @staticmethod
    def backward(ctx, ds1, ds2):
        q, keys = ctx.saved_tensors
        half = keys.shape[-1]
        dq = dk = None
        if ctx.needs_input_grad[0]:
            dq = torch.cat([torch.einsum("nhk,hkd->nhd", ds1, keys[:, 0]),
                            torch.einsum("nhk,hkd->nhd", ds2, keys[:, 1])], dim=-1)
        if ctx.needs_input_grad[1]:
            dk = torch.stack([torch.einsum("nhk,nhd->hkd", ds1, q[..., :half]),
                              torch.einsum("nhk,nhd->hkd", ds2, q[..., half:])], dim=1)
        return dq, dk


def fused_scoring_ok(half, n_keys, knn):
    """Shapes the tensor-core scoring kernel takes (the half dimension is one or two 64-wide swizzle atoms)."""
    return half in (64, 128) and n_keys % 8 == 0 and 1 <= knn <= 32 and knn <= n_keys <= 65536


def score_select(q, keys, knn, dump=False):
    """Fused bf16 scoring + selection on the tensor cores (reference: pkm.py:117-136 under bf16 autocast and
    kernels.py:214 pk_select): q (N, H, k_dim) bf16, keys (H, 2, n_keys, k_dim/2) bf16 -> scores (N, H, knn) bf16,
    indices int64, weights fp32. The sub-key scores are never materialised; dump=True also returns them
    (s1, s2 bf16 (N, H, n_keys)) for checking."""
    if q.dtype != torch.bfloat16 or keys.dtype != torch.bfloat16:
        raise ValueError("score_select needs bf16 queries and keys")
    dev = L.require_cuda(q, keys)
    N, H, KD = q.shape
    Hk, two, NK, half = keys.shape
    if Hk != H or two != 2 or KD != 2 * half or not fused_scoring_ok(half, NK, knn):
        raise ValueError(f"score_select: unsupported shapes q {tuple(q.shape)}, keys {tuple(keys.shape)}, knn {knn}")
    q, keys = _contig(q), _contig(keys)
    scores = torch.empty(N, H, knn, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(N, H, knn, dtype=torch.int64, device=dev)
    w = torch.empty(N, H, knn, dtype=torch.float32, device=dev)
    s1 = s2 = None
    if dump:
        s1 = torch.empty(N, H, NK, dtype=torch.bfloat16, device=dev)
        s2 = torch.empty(N, H, NK, dtype=torch.bfloat16, device=dev)
    ws = L.workspace(L.lib().smlm_score_select_workspace(N, H), dev)
    with L.timed("score_select", 2):
        rc = L.lib().smlm_score_select(L.ptr(q), L.ptr(keys), N, H, NK, half, knn, L.ptr(scores), L.ptr(idx),
                                       L.ptr(w), L.ptr(s1), L.ptr(s2), L.ptr(ws), ws.numel(), L.status_ptr(dev),
                                       L.stream(dev))
    L.check(rc, "score_select")
    L.after(dev, "score_select")
    if dump:
        return scores, idx, w, s1, s2
    return scores, idx, w


class ScoreSelect(torch.autograd.Function):
    """Differentiable fused scoring + selection (bf16). Backward: the selection backward of PKSelect restricted to
    its nonzero sub-key gradients (scoring_backward_sparse), with the rounding of the reference's autocast
    einsum backward (bf16 operands, fp32 accumulation, bf16 results)."""

    @staticmethod
    def forward(ctx, q, keys, knn):
        scores, idx, w = score_select(q, keys, knn)
        ctx.save_for_backward(q, keys, idx, w)
        ctx.mark_non_differentiable(idx)
        return scores, idx, w

    @staticmethod
    def backward(ctx, g_scores, g_idx, g_w):
        q, keys, idx, w = ctx.saved_tensors
        dq, dk = scoring_backward_sparse(q, keys, idx, w, g_w, g_scores, ctx.needs_input_grad[0],
                                         ctx.needs_input_grad[1])
        return dq, dk, None


# ------------------------------------------------------------------------------------------ value bag
def bag_forward(indices, weights, table, out_dtype=torch.float32, name="bag_forward", *, block_j=None, block_d=None):
    """out[n] = sum_k weights[n, k] * table[indices[n, k]] (fp32 accumulation); table fp32 / bf16
    (reference: kernels.py:229-237)."""
    dev = L.require_cuda(indices, weights, table)
    N, K = indices.shape
    D = table.shape[1]
    out = torch.empty(N, D, dtype=out_dtype, device=dev)
    idx = _contig(indices.long())
    w = _contig(weights if weights.dtype in (torch.float32, torch.bfloat16) else weights.float())
    table = _contig(table)
    with L.timed(name, 1):
        rc = L.lib().smlm_bag_forward(L.ptr(idx), L.ptr(w), L.dtype_code(w.dtype), L.ptr(table),
                                      L.dtype_code(table.dtype), N, K, table.shape[0], D, L.ptr(out),
                                      L.dtype_code(out_dtype), L.status_ptr(dev), L.stream(dev))
    L.check(rc, "bag_forward")
    L.after(dev, "bag_forward")
    return out


def bag_backward_rows(grad_out, indices, weights, table, acc, touched, row_sqnorm=None, first_touch_writes=False,
                      want_gw=True, *, P=None, block_d=None, num_warps=None):
    """grad_out (N, D) fp32 / bf16, indices / weights (N, K) -> per-sample-weight gradient (N, K) fp32;
    acc[indices[n, k]] += weights[n, k] * grad_out[n] and touched[indices] = True, in place
    (reference: kernels.py:73-88). Deterministic: sorted rows, no float atomics.
    acc / touched may be None (frozen table: only the weight gradient); want_gw=False skips the weight gradient
    (returns None; table may then be None). row_sqnorm: optional fp32 (rows,) that receives the squared norm of
    every accumulator row written. first_touch_writes: rows not yet touched are written instead of accumulated
    (for accumulators whose untouched rows count as zero)."""
    dev = L.require_cuda(grad_out, indices, weights, table, acc, touched)
    N, K = indices.shape
    D = grad_out.shape[1]
    rows = acc.shape[0] if acc is not None else table.shape[0]
    if acc is not None and (acc.dtype != torch.float32 or not acc.is_contiguous() or acc.shape[1] != D or
                            (table is not None and acc.shape != table.shape)):
        raise ValueError("bag_backward_rows: acc must be a contiguous fp32 tensor shaped like the table")
    if touched is not None and (touched.dtype not in (torch.bool, torch.uint8) or not touched.is_contiguous()):
        raise ValueError("bag_backward_rows: touched must be a contiguous bool mask")
    if table is None and want_gw:
        raise ValueError("bag_backward_rows: the weight gradient needs the table")
    g = _contig(grad_out if grad_out.dtype in (torch.float32, torch.bfloat16) else grad_out.float())
    idx = _contig(indices.long())
    w = _contig(weights if weights.dtype in (torch.float32, torch.bfloat16) else weights.float())
    table = _contig(table) if table is not None else None
    gw = torch.empty(N, K, dtype=torch.float32, device=dev) if want_gw else None
    flags = L.BWD_FIRST_TOUCH_WRITES if first_touch_writes else 0
    ws = L.workspace(L.lib().smlm_bag_backward_workspace(N, K, rows, D), dev)
    t_code = L.dtype_code(table.dtype) if table is not None else L.F32
    gw_only = acc is None and touched is None and want_gw
    with L.timed("bag_weight_grad" if gw_only else "bag_backward_rows", 1 if gw_only else L.backward_launches(rows)):
        rc = L.lib().smlm_bag_backward_rows(L.ptr(g), L.dtype_code(g.dtype), L.ptr(idx), L.ptr(w),
                                            L.dtype_code(w.dtype), L.ptr(table), t_code, L.ptr(acc), L.ptr(touched),
                                            L.ptr(row_sqnorm), flags, L.ptr(gw), N, K, rows, D, L.ptr(ws),
                                            ws.numel(), L.status_ptr(dev), L.stream(dev))
    L.check(rc, "bag_backward_rows")
    L.after(dev, "bag_backward_rows")
    return gw


# --------------------------------------------------------------------------------- row-sharded value table
def _index_code(idx):
    if idx.dtype == torch.int32:
        return L.I32
    if idx.dtype == torch.int64:
        return L.I64
    raise ValueError(f"row indices must be int32 or int64, got {idx.dtype}")


def shard_bag_forward(indices, weights, table_shard, row_base, out_dtype=torch.float32, name="shard_bag_forward"):
    """Partial value bag (N, D) (fp32 accumulation, out_dtype fp32 / bf16) of the lookups whose global row lies in
    [row_base, row_base + rows of table_shard); other lookups are skipped (they belong to other ranks' shards)."""
    dev = L.require_cuda(indices, weights, table_shard)
    N, Kk = indices.shape
    rows, D = table_shard.shape
    out = torch.empty(N, D, dtype=out_dtype, device=dev)
    idx = _contig(indices)
    w = _contig(weights if weights.dtype in (torch.float32, torch.bfloat16) else weights.float())
    t = _contig(table_shard)
    with L.timed(name, 1):
        rc = L.lib().smlm_shard_bag_forward(L.ptr(idx), _index_code(idx), int(row_base), L.ptr(w),
                                            L.dtype_code(w.dtype), L.ptr(t) if rows else None,
                                            L.dtype_code(t.dtype), N, Kk, rows, D, L.ptr(out),
                                            L.dtype_code(out_dtype), L.stream(dev))
    L.check(rc, "shard_bag_forward")
    return out


def shard_bag_backward_rows(grad_out, indices, weights, table_shard, row_base, acc, touched, row_sqnorm=None,
                            first_touch_writes=False, want_gw=True, name="shard_bag_backward_rows"):
    """bag_backward_rows restricted to the lookups in this shard's rows: acc / touched / row_sqnorm hold the
    shard's local rows; returns the weight gradient (N, K) fp32, 0 for other shards' lookups (None when
    want_gw=False)."""
    dev = L.require_cuda(grad_out, indices, weights, table_shard, acc, touched)
    N, Kk = indices.shape
    rows, D = table_shard.shape
    if acc is not None and (acc.dtype != torch.float32 or not acc.is_contiguous() or acc.shape != table_shard.shape):
        raise ValueError("shard_bag_backward_rows: acc must be a contiguous fp32 tensor shaped like the shard")
    g = _contig(grad_out if grad_out.dtype in (torch.float32, torch.bfloat16) else grad_out.float())
    idx = _contig(indices)
    w = _contig(weights if weights.dtype in (torch.float32, torch.bfloat16) else weights.float())
    t = _contig(table_shard)
    gw = torch.empty(N, Kk, dtype=torch.float32, device=dev) if want_gw else None
    ws = L.workspace(L.lib().smlm_bag_backward_workspace(N, Kk, rows, D), dev)
    flags = L.BWD_FIRST_TOUCH_WRITES if first_touch_writes else 0
    with L.timed(name, L.backward_launches(rows)):
        rc = L.lib().smlm_shard_bag_backward_rows(L.ptr(g), L.dtype_code(g.dtype), L.ptr(idx), _index_code(idx),
                                                  int(row_base), L.ptr(w), L.dtype_code(w.dtype),
                                                  L.ptr(t) if rows else None, L.dtype_code(t.dtype), L.ptr(acc),
                                                  L.ptr(touched), L.ptr(row_sqnorm), flags, L.ptr(gw), N, Kk, rows, D,
                                                  L.ptr(ws), ws.numel(), L.status_ptr(dev), L.stream(dev))
    L.check(rc, "shard_bag_backward_rows")
    L.after(dev, "shard_bag_backward_rows")
    return gw


def slot_sum(x):
    """x (S, M) fp32 -> (M,) the sum over slots in slot order."""
    dev = L.require_cuda(x)
    x = _contig(x.float())
    out = torch.empty(x.shape[1:], dtype=torch.float32, device=dev)
    with L.timed("slot_sum", 1):
        rc = L.lib().smlm_slot_sum(L.ptr(x), x.shape[0], out.numel(), L.ptr(out), L.stream(dev))
    L.check(rc, "slot_sum")
    return out


class DeferredRows:
    """The sorted lookups of a backward whose row sums were deferred (SMLM_BWD_DEFER_ROWS), with the tensors that
    finish them: the workspace, grad_out and the weights (kept alive until the rows are written or stepped)."""

    def __init__(self, ws, g, w, n, k, rows, d):
        self.ws, self.g, self.w = ws, g, w
        self.n, self.k, self.rows, self.d = n, k, rows, d
        self.ready = None                   # event of a side stream still writing them (overlap=True)


def deferrable(table, acc):
    """Whether bag_backward_deferred applies: float4 rows at most 512 wide, 16-byte aligned."""
    D = table.shape[1]
    return (D % 4 == 0 and D <= 512 and table.dtype in (torch.float32, torch.bfloat16) and acc.is_contiguous()
            and table.data_ptr() % 16 == 0)


_SIDE = {}


def side_stream(dev):
    """A second stream per device for work that may overlap the caller's stream (created on first use)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _SIDE.get(idx)
    if st is None:
        st = _SIDE[idx] = torch.cuda.Stream(device=dev)
    return st


def bag_backward_deferred(grad_out, indices, weights, table, touched, row_sqnorm, want_gw=True, overlap=False):
    """bag_backward_rows into a clean accumulator with the row sums deferred: returns the weight gradient (None
    with want_gw=False) and a DeferredRows; the rows' squared norms and touched marks are written now, the rows
    themselves by bag_rows_materialize or lazy_adam_deferred_step later. overlap=True (with want_gw=False): the
    key build, sort and norm pass run on a side stream, overlapping the caller's next kernels; the DeferredRows
    then carries the event (`ready`) that readers of touched, the norms or the rows wait for (RowStore does)."""
    dev = L.require_cuda(grad_out, indices, weights, table, touched, row_sqnorm)
    N, Kk = indices.shape
    rows, D = table.shape
    g = _contig(grad_out if grad_out.dtype in (torch.float32, torch.bfloat16) else grad_out.float())
    if g.data_ptr() % 16:
        g = g.clone()                       # the deferred passes read grad_out rows as aligned vectors
    idx = _contig(indices.long())
    w = _contig(weights if weights.dtype in (torch.float32, torch.bfloat16) else weights.float())
    t = _contig(table)
    gw = torch.empty(N, Kk, dtype=torch.float32, device=dev) if want_gw else None
    ws = L.workspace(L.lib().smlm_bag_backward_workspace(N, Kk, rows, D), dev)
    main = torch.cuda.current_stream(dev)
    side = side_stream(dev) if overlap and not want_gw else main
    if side is not main:
        side.wait_stream(main)
        if not torch.cuda.is_current_stream_capturing():  # (a captured graph's memory lives as long as the graph)
            for x in (g, idx, w, t, ws, touched, row_sqnorm):
                x.record_stream(side)       # the caching allocator keeps them until the side stream is done
    with torch.cuda.stream(side):
        with L.timed("bag_backward_rows", L.backward_launches(rows) + (1 if want_gw else 0)):
            rc = L.lib().smlm_bag_backward_rows(L.ptr(g), L.dtype_code(g.dtype), L.ptr(idx), L.ptr(w),
                                                L.dtype_code(w.dtype), L.ptr(t), L.dtype_code(t.dtype), None,
                                                L.ptr(touched), L.ptr(row_sqnorm),
                                                L.BWD_FIRST_TOUCH_WRITES | L.BWD_DEFER_ROWS, L.ptr(gw), N, Kk, rows,
                                                D, L.ptr(ws), ws.numel(), L.status_ptr(dev), L.stream(dev))
        L.check(rc, "bag_backward_rows (deferred)")
        L.after(dev, "bag_backward_rows")
    rows_ = DeferredRows(ws, g, w, N, Kk, rows, D)
    if side is not main:
        rows_.ready = torch.cuda.Event()
        rows_.ready.record(side)
    return gw, rows_


def shard_bag_backward_deferred(grad_out, indices, weights, table_shard, row_base, touched, row_sqnorm):
    """shard_bag_backward_rows with the row sums deferred (no weight gradient): the shard's row norms and touched
    marks now, a DeferredRows for the optimizer step (or bag_rows_materialize)."""
    dev = L.require_cuda(grad_out, indices, weights, table_shard, touched, row_sqnorm)
    N, Kk = indices.shape
    rows, D = table_shard.shape
    g = _contig(grad_out if grad_out.dtype in (torch.float32, torch.bfloat16) else grad_out.float())
    if g.data_ptr() % 16:
        g = g.clone()
    idx = _contig(indices)
    w = _contig(weights if weights.dtype in (torch.float32, torch.bfloat16) else weights.float())
    t = _contig(table_shard)
    ws = L.workspace(L.lib().smlm_bag_backward_workspace(N, Kk, rows, D), dev)
    with L.timed("shard_bag_backward_rows", L.backward_launches(rows)):
        rc = L.lib().smlm_shard_bag_backward_rows(L.ptr(g), L.dtype_code(g.dtype), L.ptr(idx), _index_code(idx),
                                                  int(row_base), L.ptr(w), L.dtype_code(w.dtype),
                                                  L.ptr(t) if rows else None, L.dtype_code(t.dtype), None,
                                                  L.ptr(touched), L.ptr(row_sqnorm),
                                                  L.BWD_FIRST_TOUCH_WRITES | L.BWD_DEFER_ROWS, None, N, Kk, rows, D,
                                                  L.ptr(ws), ws.numel(), L.status_ptr(dev), L.stream(dev))
    L.check(rc, "shard_bag_backward_rows (deferred)")
    L.after(dev, "shard_bag_backward_rows")
    return DeferredRows(ws, g, w, N, Kk, rows, D)


def bag_rows_materialize(pending, acc):
    """Writes the deferred rows into acc (rows untouched before the deferred backward)."""
    dev = L.require_cuda(acc)
    p = pending
    with L.timed("bag_rows_materialize", 2):
        rc = L.lib().smlm_bag_rows_materialize(L.ptr(p.g), L.dtype_code(p.g.dtype), L.ptr(p.w), L.dtype_code(p.w.dtype),
                                               L.ptr(acc), p.n, p.k, p.rows, p.d, L.ptr(p.ws), p.ws.numel(),
                                               L.stream(dev))
    L.check(rc, "bag_rows_materialize")


def lazy_adam_deferred_step(param, exp_avg, exp_avg_sq, touched, pending, grad_scale, step, lr, beta1, beta2, eps,
                            value_copy=None, scalars_dev=None):
    """lazy_adam_step fused with the deferred row sums: bit-identical to bag_rows_materialize + lazy_adam_step,
    without writing or reading the accumulator. scalars_dev: a (6,) fp32 device buffer holding the step's scalars
    (1 - beta1, beta2, 1 - beta2, sqrt(1 - beta2^step), eps, -lr / (1 - beta1^step)), read when the kernels run
    (for a step captured in a CUDA graph); step / lr / betas / eps are then not used."""
    dev = L.require_cuda(param, exp_avg, exp_avg_sq, touched, value_copy, scalars_dev)
    p = pending
    sp, sf, keep = _scale_args(grad_scale, dev)
    cp = L.dtype_code(value_copy.dtype) if value_copy is not None else L.F32
    with L.timed("lazy_adam_step", 2):
        if scalars_dev is not None:
            rc = L.lib().smlm_lazy_adam_deferred_step_dev(
                L.ptr(param), L.ptr(exp_avg), L.ptr(exp_avg_sq), L.ptr(touched), L.ptr(p.g),
                L.dtype_code(p.g.dtype), L.ptr(p.w), L.dtype_code(p.w.dtype), sp, sf, p.n, p.k, p.rows, p.d,
                L.ptr(scalars_dev), L.ptr(value_copy), cp, L.ptr(p.ws), p.ws.numel(), L.stream(dev))
        else:
            bc1 = 1 - beta1 ** step
            bc2 = 1 - beta2 ** step
            rc = L.lib().smlm_lazy_adam_deferred_step(
                L.ptr(param), L.ptr(exp_avg), L.ptr(exp_avg_sq), L.ptr(touched), L.ptr(p.g), L.dtype_code(p.g.dtype),
                L.ptr(p.w), L.dtype_code(p.w.dtype), sp, sf, p.n, p.k, p.rows, p.d, 1 - beta1, beta2, 1 - beta2,
                math.sqrt(bc2), eps, -(lr / bc1), L.ptr(value_copy), cp, L.ptr(p.ws), p.ws.numel(), L.stream(dev))
    L.check(rc, "lazy_adam_deferred_step")
    del keep


def quantize_q4(table, chunk=None):
    """table (rows, D) fp32 -> packed (rows, D/2) uint8, scales (rows,) fp16 (reference: kernels.py:280-294):
    per row d = half(w[argmax |w|] / -8) (1 if that is 0), codes clamp(round(w / d), -8, 7) + 8; byte i holds
    column i (low nibble) and column i + D/2 (high nibble)."""
    dev = L.require_cuda(table)
    rows, D = table.shape
    if D % 2:
        raise ValueError("quantize_q4 needs an even row width")
    t = _contig(table.float())
    packed = torch.empty(rows, D // 2, dtype=torch.uint8, device=dev)
    scales = torch.empty(rows, dtype=torch.float16, device=dev)
    L.check(L.lib().smlm_quantize_q4(L.ptr(t), rows, D, L.ptr(packed), L.ptr(scales), L.stream(dev)),
            "quantize_q4")
    return packed, scales


def dequantize_q4(packed, scales):
    """Inverse of quantize_q4 (reference: kernels.py:297-300); a format helper for checks, not on the hot path."""
    lo = (packed & 15).float() - 8
    hi = (packed >> 4).float() - 8
    return torch.cat([lo, hi], dim=1) * scales.float()[:, None]


def bag_infer(indices, weights, table, scales=None, pre=None, out_bf16=False, block_j=None, block_d=None):
    """Inference value bag (reference: kernels.py:364-378). table fp32 / bf16 (scales None) or q4-packed uint8
    (rows, D/2) with fp16 scales. pre: optional (N, D) swilu pre-activation -> out = bag * bf16(silu(pre)).
    Returns (N, D) fp32, or bf16 with out_bf16."""
    dev = L.require_cuda(indices, weights, table, scales, pre)
    N, K = indices.shape
    q4 = scales is not None
    D = table.shape[1] * (2 if q4 else 1)
    out = torch.empty(N, D, dtype=torch.bfloat16 if out_bf16 else torch.float32, device=dev)
    idx = _contig(indices.long())
    w = _contig(weights if weights.dtype in (torch.float32, torch.bfloat16) else weights.float())
    table = _contig(table)
    if q4:
        if table.dtype != torch.uint8 or scales.dtype != torch.float16:
            raise ValueError("bag_infer: q4 tables are uint8 with fp16 scales")
        tcode = L.Q4
    else:
        tcode = L.dtype_code(table.dtype)
    if pre is not None:
        pre = _contig(pre if pre.dtype in (torch.float32, torch.bfloat16) else pre.float())
    with L.timed("bag_infer", 1):
        rc = L.lib().smlm_bag_infer(L.ptr(idx), L.ptr(w), L.dtype_code(w.dtype), L.ptr(table), tcode,
                                   L.ptr(_contig(scales) if q4 else None), L.ptr(pre),
                                   L.dtype_code(pre.dtype) if pre is not None else L.F32, N, K, table.shape[0], D,
                                   L.ptr(out), L.BF16 if out_bf16 else L.F32, L.status_ptr(dev), L.stream(dev))
    L.check(rc, "bag_infer")
    L.after(dev, "bag_infer")
    return out


# ------------------------------------------------------------------------------------------ optimizers
def _scale_args(grad_scale, device):
    """(device pointer or None, host float, keep-alive tensor) for a float or 0-d tensor clip factor."""
    if torch.is_tensor(grad_scale):
        t = grad_scale.detach().to(device=device, dtype=torch.float32).reshape(1)
        t = _contig(t)
        return L.ptr(t), 1.0, t
    return None, float(grad_scale), None


def lazy_adam_step(param, exp_avg, exp_avg_sq, acc, touched, grad_scale, step, lr, beta1, beta2, eps,
                   value_copy=None, keep_acc=False, *, rows_per_program=None, block_d=None, scalars_dev=None):
    """In-place lazy Adam step over the touched rows (reference: kernels.py:417-433): torch's Adam formula, global
    step for the bias correction, no weight decay; the touched accumulator rows are zeroed and the mask cleared.
    grad_scale: 0-d tensor (clip factor) or float; step: the step number after this update (1 for the first).
    value_copy: optional (rows, D) bf16 / fp32 tensor that receives the updated rows too. keep_acc: leave the
    consumed accumulator rows as they are (for accumulators whose untouched rows count as zero). scalars_dev: a
    device fp32 tensor of the six step scalars (LazyRowAdam(capturable=True)); step, lr, betas and eps are then not
    used."""
    dev = L.require_cuda(param, exp_avg, exp_avg_sq, acc, touched, value_copy)
    for t in (param, exp_avg, exp_avg_sq, acc):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.shape != param.shape:
            raise ValueError("lazy_adam_step: param, moments and acc must be contiguous fp32 of one shape")
    rows, D = param.shape
    sp, sf, keep = _scale_args(grad_scale, dev)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    ws = L.workspace(L.lib().smlm_touched_workspace(rows), dev)
    copy_code = L.dtype_code(value_copy.dtype) if value_copy is not None else L.F32
    flags = L.STEP_KEEP_ACC if keep_acc else 0
    with L.timed("lazy_adam_step", L.COMPACT_LAUNCHES + 1):
        if scalars_dev is not None:
            rc = L.lib().smlm_lazy_adam_step_dev(L.ptr(param), L.ptr(exp_avg), L.ptr(exp_avg_sq), L.ptr(acc),
                                                 L.ptr(touched), sp, sf, rows, D, L.ptr(scalars_dev),
                                                 L.ptr(value_copy), copy_code, flags, L.ptr(ws), ws.numel(),
                                                 L.stream(dev))
        else:
            rc = L.lib().smlm_lazy_adam_step(L.ptr(param), L.ptr(exp_avg), L.ptr(exp_avg_sq), L.ptr(acc),
                                             L.ptr(touched), sp, sf, rows, D, 1 - beta1, beta2, 1 - beta2,
                                             math.sqrt(bc2), eps, -(lr / bc1), L.ptr(value_copy), copy_code, flags,
                                             L.ptr(ws), ws.numel(), L.stream(dev))
    L.check(rc, "lazy_adam_step")
    del keep


def lazy_adam_lowmem_step(param, exp_avg, exp_avg_sq, exp_avg_scale, exp_avg_sq_scale, acc, touched, grad_scale,
                          step, lr, beta1, beta2, eps, value_copy=None, keep_acc=False):
    """In-place lazy Adam over the touched rows with compact moments (reference: kernels.py:498-515): bf16
    exp_avg / exp_avg_sq, or int8 / uint8 codes with fp32 row scales (exp_avg_scale, exp_avg_sq_scale given).
    Same arguments and effects as lazy_adam_step otherwise."""
    dev = L.require_cuda(param, exp_avg, exp_avg_sq, exp_avg_scale, exp_avg_sq_scale, acc, touched, value_copy)
    rows, D = param.shape
    for t in (param, acc):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.shape != param.shape:
            raise ValueError("lazy_adam_lowmem_step: param and acc must be contiguous fp32 of one shape")
    if exp_avg.dtype == torch.int8 and exp_avg_sq.dtype == torch.uint8:
        code = L.I8
        for t in (exp_avg_scale, exp_avg_sq_scale):
            if t is None or t.dtype != torch.float32 or t.shape != (rows,) or not t.is_contiguous():
                raise ValueError("lazy_adam_lowmem_step: int8 moments need fp32 (rows,) scales")
    elif exp_avg.dtype == torch.bfloat16 and exp_avg_sq.dtype == torch.bfloat16:
        code = L.BF16
    else:
        raise ValueError("lazy_adam_lowmem_step: moments must be bf16 / bf16 or int8 / uint8")
    for t in (exp_avg, exp_avg_sq):
        if not t.is_contiguous() or t.shape != param.shape:
            raise ValueError("lazy_adam_lowmem_step: moments must be contiguous and shaped like the table")
    sp, sf, keep = _scale_args(grad_scale, dev)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    ws = L.workspace(L.lib().smlm_touched_workspace(rows), dev)
    with L.timed("lazy_adam_lowmem_step", L.COMPACT_LAUNCHES + 1):
        rc = L.lib().smlm_lazy_adam_lowmem_step(
            L.ptr(param), L.ptr(exp_avg), L.ptr(exp_avg_sq), L.ptr(exp_avg_scale), L.ptr(exp_avg_sq_scale), code,
            L.ptr(acc), L.ptr(touched), sp, sf, rows, D, beta1, beta2, 1 - beta1, 1 - beta2, eps, lr / bc1,
            math.sqrt(bc2), L.ptr(value_copy), L.dtype_code(value_copy.dtype) if value_copy is not None else L.F32,
            L.STEP_KEEP_ACC if keep_acc else 0, L.ptr(ws), ws.numel(), L.stream(dev))
    L.check(rc, "lazy_adam_lowmem_step")
    del keep


def lazy_adam_step_lowmem(param, exp_avg, exp_avg_sq, acc, touched, grad_scale, step, lr, beta1, beta2, eps,
                          state_dtype, exp_avg_scale=None, exp_avg_sq_scale=None):
    """The reference's name and argument order for the compact-moment step (kernels.py:493-515): state_dtype
    "bf16" (bf16 exp_avg / exp_avg_sq) or "int8" (int8 / uint8 codes with their fp32 row scales). Same effects as
    lazy_adam_lowmem_step: touched rows updated, their accumulator rows zeroed, touched cleared."""
    if state_dtype not in ("bf16", "int8"):
        raise ValueError("low-memory Adam state_dtype must be 'bf16' or 'int8'")
    int8 = state_dtype == "int8"
    if int8 and (exp_avg_scale is None or exp_avg_sq_scale is None):
        raise ValueError("int8 Adam needs exp_avg_scale and exp_avg_sq_scale")
    want = (torch.int8, torch.uint8) if int8 else (torch.bfloat16, torch.bfloat16)
    if (exp_avg.dtype, exp_avg_sq.dtype) != want:
        raise ValueError(f"state_dtype {state_dtype!r} needs moments of {want[0]} / {want[1]}, got "
                         f"{exp_avg.dtype} / {exp_avg_sq.dtype}")
    lazy_adam_lowmem_step(param, exp_avg, exp_avg_sq, exp_avg_scale if int8 else None,
                          exp_avg_sq_scale if int8 else None, acc, touched, grad_scale, step, lr, beta1, beta2, eps)


def rowwise_step(param, acc, touched, v, n, grad_scale, lr, beta2, eps, kind, keep_acc=False):
    """Row-wise rowrms / rowadagrad step over the touched rows, in place; accumulator rows zeroed, mask cleared
    (reference: row_optim.py:168-201, formulas of host_rows.c:84-117)."""
    dev = L.require_cuda(param, acc, touched, v, n)
    rows, D = param.shape
    code = {"rowrms": L.ROWRMS, "rowadagrad": L.ROWADAGRAD}[kind]
    sp, sf, keep = _scale_args(grad_scale, dev)
    ws = L.workspace(L.lib().smlm_touched_workspace(rows), dev)
    with L.timed("rowwise_step", L.COMPACT_LAUNCHES + 1):
        rc = L.lib().smlm_rowwise_step(L.ptr(param), L.ptr(acc), L.ptr(touched), L.ptr(v), L.ptr(n), sp, sf, rows,
                                       D, code, beta2, eps, lr, L.STEP_KEEP_ACC if keep_acc else 0, L.ptr(ws),
                                       ws.numel(), L.stream(dev))
    L.check(rc, "rowwise_step")
    del keep


def rowwise_deferred_step(param, touched, v, n, pending, grad_scale, lr, beta2, eps, kind):
    """rowwise_step fused with the deferred row sums: bit-identical to bag_rows_materialize + rowwise_step, without
    writing or reading the accumulator."""
    dev = L.require_cuda(param, touched, v, n)
    p = pending
    code = {"rowrms": L.ROWRMS, "rowadagrad": L.ROWADAGRAD}[kind]
    sp, sf, keep = _scale_args(grad_scale, dev)
    with L.timed("rowwise_step", 2):
        rc = L.lib().smlm_rowwise_deferred_step(
            L.ptr(param), L.ptr(touched), L.ptr(v), L.ptr(n), L.ptr(p.g), L.dtype_code(p.g.dtype), L.ptr(p.w),
            L.dtype_code(p.w.dtype), sp, sf, p.n, p.k, p.rows, p.d, code, beta2, eps, lr, L.ptr(p.ws), p.ws.numel(),
            L.stream(dev))
    L.check(rc, "rowwise_deferred_step")
    del keep


def touched_norm(acc, touched, row_sqnorm=None):
    """L2 norm (0-d fp32 tensor on the device) of the accumulator rows marked in `touched`; equals acc.norm()
    for an accumulator whose untouched rows count as zero (reference: sparse_values.py:143). With row_sqnorm (as
    written by bag_backward_rows) only 4 bytes per touched row are read."""
    dev = L.require_cuda(acc, touched, row_sqnorm)
    rows = acc.shape[0]
    D = acc.shape[1] if acc.dim() > 1 else 1
    out = torch.empty((), dtype=torch.float32, device=dev)
    ws = L.workspace(L.lib().smlm_touched_workspace(rows), dev)
    with L.timed("touched_norm", L.COMPACT_LAUNCHES + 2):
        rc = L.lib().smlm_touched_norm(L.ptr(_contig(acc)), L.ptr(row_sqnorm), L.ptr(touched), rows, D, L.ptr(out),
                                       L.ptr(ws), ws.numel(), L.stream(dev))
    L.check(rc, "touched_norm")
    return out


def zero_untouched(acc, touched):
    """acc rows whose touched flag is clear <- 0, in place (makes an accumulator whose untouched rows count as
    zero an ordinary dense tensor again)."""
    dev = L.require_cuda(acc, touched)
    rows = acc.shape[0]
    D = acc.shape[1] if acc.dim() > 1 else 1
    with L.timed("zero_untouched", 1):
        rc = L.lib().smlm_zero_untouched(L.ptr(acc), L.ptr(touched), rows, D, L.stream(dev))
    L.check(rc, "zero_untouched")


# ------------------------------------------------------------------------------------------ Engram rows
def ngram_rows(c, history, mult, orders, heads, rows):
    """Row indices of an Engram module's lookups (reference: engram.py:63-75 NgramHash.forward): c (B, history + T)
    int64 compressed ids, mult (n_orders, heads, max_order) int64 -> (B, T, n_orders * heads) int64, lookup
    (order o, head h) in rows [(o * heads + h) * rows, ... + rows)."""
    import ctypes
    dev = L.require_cuda(c, mult)
    if c.dtype != torch.long or mult.dtype != torch.long:
        raise ValueError("ngram_rows: c and mult must be int64")
    B, W = c.shape
    T = W - history
    if T < 0:
        raise ValueError(f"ngram_rows: {W} ids for a history of {history}")
    n_orders, h, max_order = mult.shape
    if h != heads or len(orders) != n_orders:
        raise ValueError("ngram_rows: mult does not match orders / heads")
    out = torch.empty(B, T, n_orders * heads, dtype=torch.long, device=dev)
    c, mult = _contig(c), _contig(mult)
    arr = (ctypes.c_int * n_orders)(*[int(o) for o in orders])
    with L.timed("ngram_rows", 1):
        rc = L.lib().smlm_ngram_rows(L.ptr(c), B, T, int(history), L.ptr(mult), ctypes.cast(arr, ctypes.c_void_p),
                                     n_orders, heads, max_order, int(rows), L.ptr(out), L.stream(dev))
    L.check(rc, "ngram_rows")
    return out

