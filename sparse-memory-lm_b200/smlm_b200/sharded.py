"""Row-sharded value table over the GPUs of one process group (one process per GPU, NCCL).

The reference runs the product-key memory on one device. Here the value table, its row-sparse gradient store and
its lazy-Adam state are split into contiguous row ranges, one per rank (owner = row // ceil(rows / world)); the
keys, the query projection and everything else stay replicated and data-parallel. Tokens stay on their rank:

  forward   every rank scores and selects its own tokens; the lookups (int32 global row, weight) are all-gathered;
            each owner computes, for every rank's tokens, the partial bag over the lookups in its rows
            (smlm_shard_bag_forward); an all-to-all returns each rank the partial bags of its tokens, which are
            summed in owner order (smlm_slot_sum).
  backward  the output gradients are all-gathered; each owner runs the deterministic row-sparse backward over
            the lookups in its rows (its accumulator, touched mask and squared row norms; the weight gradient
            of its lookups, 0 for the others); an all-to-all returns the weight gradients, summed in owner order
            (each lookup has exactly one nonzero term, so the sum is exact).
  clip      the squared norm of every rank's accumulator rows is all-gathered and summed in rank order.
  step      each rank's LazyRowAdam updates its own rows only.

That is the NCCL exchange (shard_exchange="nccl"). The default, shard_exchange="p2p" (PeerExchange), fuses the
exchange into the kernels through peer memory over NVLink: each rank buckets its lookups by owner (a counting sort
in its own exchange block), each owner reads only its bucket of every rank, gathers its rows and stores the
partial bags straight into the requesting ranks' memory, which sum them in owner order (for inference with the
swilu product fused); in the backward the owner stores each lookup's weight gradient straight into its
requester's memory, and only the output gradients are all-gathered over NCCL. Its epochs live on the device, so
a whole row-sharded step can be captured in one CUDA graph and replayed.

A P-rank step over batches x_0 .. x_{P-1} is the one-rank step over their concatenation (row gradients summed over
all tokens; the replicated parameters' gradients summed with allreduce_replicated_grads); only the fp32 summation
order of the bag (owner partials) and of the row sums differ. Every rank must pass the same number of tokens.
Data-path exchange volume per rank and step (N tokens, K lookups, D columns, P ranks), NCCL exchange: lookups
8 N K P, partial bags and output gradients 2 x 4 N D P, weight gradients 4 N K P bytes received; peer exchange:
lookups about 12 N K read by each owner (its buckets), partial bags and output gradients 2 x 4 N D P, weight
gradients 4 N K.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib as L
from . import kernels as K


class RowShard:
    """Rank `rank`'s contiguous row range of a `rows`-row table split over `world` ranks: rows
    [base, base + count), ceil(rows / world) per rank (the last ranks may hold fewer, or none)."""

    def __init__(self, rows, world, rank):
        if world < 1 or not 0 <= rank < world or rows < 0:
            raise ValueError(f"bad shard: rows={rows}, world={world}, rank={rank}")
        if rows >= 2 ** 31:
            raise ValueError("row-sharded tables exchange int32 row indices: rows must be below 2^31")
        self.rows, self.world, self.rank = rows, world, rank
        self.per = -(-rows // world) if rows else 0
        self.base = min(rows, rank * self.per)
        self.count = max(0, min(rows, self.base + self.per) - self.base)

    def owner(self, row):
        return row // self.per

    def take(self, full):
        """This rank's rows of a full-table tensor."""
        return full[self.base:self.base + self.count]

    def __repr__(self):
        return f"RowShard(rows={self.rows}, world={self.world}, rank={self.rank}, base={self.base}, count={self.count})"


class CudaShardOps:
    """The owner-side kernels (libsmlm_b200.so)."""

    def bag_forward(self, idx, w, table, base):
        return K.shard_bag_forward(idx, w, table, base)

    def bag_backward(self, g, idx, w, table, base, store):
        if store is None:
            return K.shard_bag_backward_rows(g, idx, w, table, base, None, None)
        store.materialize()
        store.live = True
        return K.shard_bag_backward_rows(g, idx, w, table, base, store._acc, store._touched,
                                         row_sqnorm=store._sqnorm if store.clean else None,
                                         first_touch_writes=store.clean)

    def slot_sum(self, x):
        return K.slot_sum(x)


CUDA_OPS = CudaShardOps()


def _all_gather(x, group, world):
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _all_to_all(x, group):
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x.contiguous(), group=group)
    return out


class _ShardedBag(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weights, indices, table, store, shard, group, ops):
        P = shard.world
        N, Kk = indices.shape
        w = weights.reshape(N, Kk).to(table.dtype)
        all_idx = _all_gather(indices.to(torch.int32), group, P)
        all_w = _all_gather(w, group, P)
        part = ops.bag_forward(all_idx, all_w, table, shard.base)            # (P N, D): this owner's partials
        D = part.shape[1]
        out = ops.slot_sum(_all_to_all(part, group).view(P, N * D)).view(N, D)
        ctx.save_for_backward(all_idx, all_w)
        ctx.table, ctx.store, ctx.shard, ctx.group, ctx.ops = table, store, shard, group, ops
        ctx.wshape, ctx.wdtype = weights.shape, weights.dtype
        return out.to(table.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        all_idx, all_w = ctx.saved_tensors
        shard, group, ops = ctx.shard, ctx.group, ctx.ops
        P = shard.world
        N, Kk = all_idx.shape[0] // P, all_idx.shape[1]
        g = grad_out.contiguous()
        if g.dtype not in (torch.float32, torch.bfloat16):
            g = g.float()
        all_g = _all_gather(g, group, P)
        gw_part = ops.bag_backward(all_g, all_idx, all_w, ctx.table, shard.base, ctx.store)   # (P N, K)
        gw = ops.slot_sum(_all_to_all(gw_part, group).view(P, N * Kk)).view(N, Kk)
        ctx.table = ctx.store = ctx.ops = None
        return gw.view(ctx.wshape).to(ctx.wdtype), None, None, None, None, None, None


class PeerExchange:
    """The exchange blocks of every rank mapped into this process (CUDA IPC over NVLink) for the fused exchange:
    each rank buckets its lookups by owner in its own block, the owners' kernels read their buckets and write
    partial bags and weight gradients through peer pointers, with epoch flags and bounded waits (smlm_xchg_* in
    the C ABI). The epochs live on the device (advanced by every forward), so exchanges can be captured in a CUDA
    graph and replayed. Collective to build and to close; sized for up to n_cap tokens per rank."""

    def __init__(self, shard, group, n_cap, k, d, device):
        lib = L.lib()
        self.shard, self.group, self.n_cap, self.k, self.d = shard, group, int(n_cap), int(k), int(d)
        self.device = device
        nbytes = lib.smlm_xchg_bytes(shard.world, self.n_cap, self.k, self.d)
        base = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        with torch.cuda.device(device):
            L.check(lib.smlm_xchg_alloc(nbytes, ctypes.byref(base), handle), "xchg_alloc")
        self.block = base.value
        handles = [None] * shard.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        with torch.cuda.device(device):
            for r, h in enumerate(handles):
                if r == shard.rank:
                    ptrs.append(self.block)
                    continue
                peer = ctypes.c_void_p()
                L.check(lib.smlm_xchg_open(ctypes.create_string_buffer(h, 64), ctypes.byref(peer)), "xchg_open")
                self.opened.append(peer.value)
                ptrs.append(peer.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)

    def forward(self, idx, w, table, n, pre=None, out_dtype=torch.float32, dense=True):
        """One exchange forward (smlm_xchg_forward, device epoch): this rank's tokens' bags (n, d) over the whole
        table, times silu(pre) with `pre`; with dense, also the lookups this shard served, stacked over the ranks
        ((world n, k) int32 global rows, -1 for other shards' lookups, and fp32 weights) for the backward."""
        shard, dev = self.shard, self.device
        P, Kk = shard.world, self.k
        all_idx = torch.empty(P * n, Kk, dtype=torch.int32, device=dev) if dense else None
        all_w = torch.empty(P * n, Kk, dtype=torch.float32, device=dev) if dense else None
        out = torch.empty(n, self.d, dtype=out_dtype, device=dev)
        t = table.detach()
        pre_c = pre.contiguous() if pre is not None else None
        with L.timed("xchg_forward", 6):
            rc = L.lib().smlm_xchg_forward(
                L.ptr(self.peers), ctypes.c_void_p(self.block), shard.rank, P, L.ptr(idx), L.ptr(w), n, Kk,
                self.n_cap, shard.per, L.ptr(t) if shard.count else None, L.dtype_code(t.dtype), shard.base,
                shard.count, self.d, L.ptr(all_idx), L.ptr(all_w), L.ptr(pre_c),
                L.dtype_code(pre_c.dtype) if pre_c is not None else L.F32, L.ptr(out), L.dtype_code(out_dtype), 0,
                L.status_ptr(dev), L.stream(dev))
        L.check(rc, "xchg_forward")
        L.after(dev, "xchg_forward")
        return out, all_idx, all_w

    def close(self):
        """Unmaps the peers' blocks and frees this rank's (collective: no rank may touch a block after)."""
        if self.block is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = L.lib()
        with torch.cuda.device(self.device):
            for p in self.opened:
                lib.smlm_xchg_close(ctypes.c_void_p(p))
            dist.barrier(group=self.group)
            lib.smlm_xchg_free(ctypes.c_void_p(self.block))
        self.block, self.opened = None, []


def peer_exchange(table, shard, group, n, k):
    """The table's PeerExchange, built on first use or rebuilt (collectively) when n outgrows its capacity."""
    x = getattr(table, "peer_exchange", None)
    if x is None or x.n_cap < n or x.k != k or x.d != table.shape[1]:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the row-sharded exchange must be set up (one eager step of this shape) before capture")
        if x is not None:
            x.close()
        x = PeerExchange(shard, group, n, k, table.shape[1], table.device)
        table.peer_exchange = x
    return x


class _PeerBag(torch.autograd.Function):
    """The sharded bag with the exchange fused into the owner's kernels (peer memory) instead of NCCL
    collectives for the lookups, partial bags and weight gradients; the output gradients are all-gathered."""

    @staticmethod
    def forward(ctx, weights, indices, table, store, shard, group):
        from .sparse_values import read_table
        N, Kk = indices.shape
        x = peer_exchange(table, shard, group, N, Kk)
        idx = indices.to(torch.int32).contiguous()
        w = weights.reshape(N, Kk).float().contiguous()
        src = read_table(table)
        out, all_idx, all_w = x.forward(idx, w, src, N)
        ctx.save_for_backward(all_idx, all_w)
        ctx.table, ctx.src, ctx.store, ctx.shard, ctx.group, ctx.x = table, src, store, shard, group, x
        ctx.wshape, ctx.wdtype = weights.shape, weights.dtype
        return out.to(table.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        all_idx, all_w = ctx.saved_tensors
        shard, x, store = ctx.shard, ctx.x, ctx.store
        P = shard.world
        N, Kk = all_idx.shape[0] // P, all_idx.shape[1]
        dev = all_idx.device
        g = grad_out.contiguous()
        if g.dtype not in (torch.float32, torch.bfloat16):
            g = g.float()
        all_g = _all_gather(g, ctx.group, P)
        t, src = ctx.table.detach(), ctx.src.detach()
        status = L.status_ptr(dev)
        with L.timed("xchg_backward_gw", 1):
            rc = L.lib().smlm_xchg_backward_gw(
                L.ptr(x.peers), shard.rank, P, L.ptr(all_g), L.dtype_code(all_g.dtype), L.ptr(all_idx), N, Kk,
                x.n_cap, L.ptr(src) if shard.count else None, L.dtype_code(src.dtype), shard.base, shard.count,
                src.shape[1], 0, status, L.stream(dev))
        L.check(rc, "xchg_backward_gw")
        if store is not None and shard.count:
            if store.can_defer(t):
                # the shard's row sums go straight into the optimizer step (see RowStore)
                store.pending = K.shard_bag_backward_deferred(all_g, all_idx, all_w, t, shard.base, store._touched,
                                                              store._sqnorm)
            else:
                store.materialize()
                store.live = True
                K.shard_bag_backward_rows(all_g, all_idx, all_w, t, shard.base, store._acc, store._touched,
                                          row_sqnorm=store._sqnorm if store.clean else None,
                                          first_touch_writes=store.clean, want_gw=False)
        gw = torch.empty(N, Kk, dtype=torch.float32, device=dev)
        with L.timed("xchg_collect_gw", 1):
            rc = L.lib().smlm_xchg_collect_gw(L.ptr(x.peers), shard.rank, P, N, Kk, x.n_cap, t.shape[1],
                                              L.ptr(gw), 0, status, L.stream(dev))
        L.check(rc, "xchg_collect_gw")
        L.after(dev, "xchg_collect_gw")
        ctx.table = ctx.src = ctx.store = ctx.x = None
        return gw.view(ctx.wshape).to(ctx.wdtype), None, None, None, None, None


def sharded_bag_infer(indices, weights, table, shard, group, pre=None, out_bf16=False):
    """No-grad sharded value bag over the peer exchange for inference (prefill, decoding): the bags of this rank's
    tokens over the whole row-sharded table, with the swilu product silu(pre) and the bf16 cast fused into the
    exchange's final sum (reference: the inference bag of pkm.py:213-224 on one device). Collective: every rank
    calls it with the same token count. Reads the table's bf16 copy when it has one."""
    from .sparse_values import read_table
    if indices.ndim != 2 or table.shape[0] != shard.count:
        raise ValueError("sharded_bag_infer: indices (N, K) and this rank's table shard expected")
    N, Kk = indices.shape
    with torch.no_grad():
        x = peer_exchange(table, shard, group, N, Kk)
        out, _, _ = x.forward(indices.to(torch.int32).contiguous(), weights.reshape(N, Kk).float().contiguous(),
                              read_table(table), N, pre=pre, out_dtype=torch.bfloat16 if out_bf16 else torch.float32,
                              dense=False)
    return out


def sharded_embedding_bag(indices, weights, table, shard, group, ops=None, store=None, exchange="nccl"):
    """sum_j weights[:, j] * V[indices[:, j]] for a table V whose rows [shard.base, shard.base + shard.count) are
    `table` on this rank; row gradients go into the shard's RowStore (`store`, default table.row_store).
    Collective: every rank of `group` calls it with the same token count. exchange="nccl": NCCL collectives
    around the owner kernels (any owner ops); "p2p": the exchange fused into the owner's kernels through peer
    memory (CUDA kernels only; the backward of a forward runs before the next forward)."""
    from .sparse_values import row_store
    if exchange not in ("nccl", "p2p"):
        raise ValueError(f"unknown exchange {exchange!r}")
    if exchange == "p2p" and ops is None:
        if indices.ndim != 2 or table.shape[0] != shard.count:
            raise ValueError("sharded_embedding_bag: indices (N, K) and this rank's table shard expected")
        if store is None and torch.is_grad_enabled() and table.requires_grad:
            store = row_store(table)
        if not torch.is_grad_enabled():
            return sharded_bag_infer(indices, weights, table, shard, group).to(table.dtype)
        return _PeerBag.apply(weights, indices, table, store, shard, group)
    ops = ops or CUDA_OPS
    if indices.ndim != 2 or weights.shape[:1] != indices.shape[:1]:
        raise ValueError("sharded_embedding_bag: indices (N, K) and weights (N, K) expected")
    if table.shape[0] != shard.count:
        raise ValueError(f"table has {table.shape[0]} rows but the shard holds {shard.count}")
    if store is None and torch.is_grad_enabled() and table.requires_grad:
        store = row_store(table)
    if not torch.is_grad_enabled():
        with torch.no_grad():
            return _ShardedBag.forward(_NoCtx(), weights, indices, table, None, shard, group, ops)
    return _ShardedBag.apply(weights, indices, table, store, shard, group, ops)


class _NoCtx:
    """Stand-in autograd context for the no-grad forward."""

    def save_for_backward(self, *t):
        pass


def replicated_params(module):
    """Parameters that every rank holds in full (everything but row-sharded value tables)."""
    return [p for p in module.parameters() if getattr(p, "row_shard", None) is None]


def allreduce_replicated_grads(module, group=None):
    """Sum the replicated parameters' gradients over the ranks (one flat NCCL all-reduce)."""
    grads = [p.grad for p in replicated_params(module) if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=group)
    off = 0
    for g in grads:
        g.copy_(flat[off:off + g.numel()].view_as(g))
        off += g.numel()


def sharded_sq_norm(local_sq, group, world):
    """Sum over ranks, in rank order, of a 0-d fp32 device tensor (deterministic on every rank)."""
    parts = _all_gather(local_sq.reshape(1).float(), group, world)
    total = parts[0]
    for i in range(1, world):
        total = total + parts[i]
    return total.reshape(())


def broadcast_replicated(module, group=None, src=0):
    """Give every rank rank `src`'s copy of the replicated parameters and buffers (one flat broadcast)."""
    ts = [p.data for p in replicated_params(module)] + [b for b in module.buffers() if b.is_floating_point()]
    if not ts:
        return
    flat = torch.cat([t.reshape(-1).float() for t in ts])
    dist.broadcast(flat, src=dist.get_global_rank(group, src) if group is not None else src, group=group)
    off = 0
    for t in ts:
        t.copy_(flat[off:off + t.numel()].view_as(t))
        off += t.numel()
