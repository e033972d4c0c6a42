"""Row-sparse gradients and the lazy Adam of the product-key value table, on the sm_100a kernels.

Same API and semantics as re133/sparse-memory-lm smlm/sparse_values.py:
  * RowStore (sparse_values.py:26-41): one persistent fp32 accumulator shaped like the table, a bool `touched`
    mask and a deferred clip factor `grad_scale` (float or 0-d device tensor).
  * row_sparse_embedding_bag (110-123): forward = value bag; backward adds w * grad_out into the read rows of
    the accumulator and returns the per-sample-weight gradient; the table never gets a .grad.
  * clip_row_sparse (137-151): global norm over the accumulated rows, clip factor stored in the RowStore.
  * LazyRowAdam (154-362): Adam (no weight decay) on the rows read since the last step only; unread rows keep
    values and state bit for bit; global step count for the bias correction; state format
    smlm.lazy_row_adam.v1.
The only implementation is "cuda" (libsmlm_b200.so); the reference's "torch" / "triton" values are accepted
as aliases so that configurations carry over, and CPU tables raise.
"""
import math

import torch

from . import kernels as K

IMPLS = ("cuda", "triton", "torch")        # every value selects the CUDA kernels


def _check_impl(impl):
    if impl not in IMPLS:
        raise ValueError(f"unknown impl {impl!r}")


class RowStore:
    """The row-sparse gradient store of one table (reference: sparse_values.py:26-41): `acc` (fp32, shaped like
    the table), `touched` (bool per row) and the deferred clip factor `grad_scale`.

    While a store is clean (no one has read `acc` or `touched` since its last reset), rows whose touched flag is
    clear count as zero whatever the buffer holds there. That lets the backward write a row it meets for the
    first time instead of reading it back, and the optimizer step leave the rows it consumed as they are (about
    3 KB of traffic saved per touched row and step), and the backward records each written row's squared norm,
    so the clip norm reads 4 bytes per touched row. Reading `acc` or `touched` first turns the stale rows into
    zeros and keeps the store exact, with the reference's semantics, until its next reset()."""

    def __init__(self, table):
        if table.dtype not in (torch.float32, torch.bfloat16):
            raise ValueError(f"row-sparse tables must be fp32 or bf16, got {table.dtype}")
        self._acc = torch.zeros(table.shape, dtype=torch.float32, device=table.device)
        self._touched = torch.zeros(table.shape[0], dtype=torch.bool, device=table.device)
        self._sqnorm = torch.zeros(table.shape[0], dtype=torch.float32, device=table.device)
        self.grad_scale = 1.0           # set by clipping, applied in the optimizer step
        self.clean = True
        self.live = False               # acc holds rows written since the last reset / step
        self.pending = None             # a backward's deferred row sums (kernels.DeferredRows), not yet in acc

    @property
    def acc(self):
        self.expose()
        return self._acc

    @property
    def touched(self):
        self.expose()
        return self._touched

    def sync(self):
        """Order the current stream after a backward whose norm pass still runs on a side stream (overlap)."""
        p = self.pending
        if p is not None and p.ready is not None:
            torch.cuda.current_stream(self._touched.device).wait_event(p.ready)
            p.ready = None

    def expose(self):
        """Make `acc` an exact dense accumulator (stale untouched rows <- 0) before outside code reads it."""
        self.materialize()
        if self.clean:
            K.zero_untouched(self._acc, self._touched)
            self.clean = False

    def materialize(self):
        """Write the deferred row sums of the last backward into acc (where that backward would have)."""
        self.sync()
        if self.pending is not None:
            K.bag_rows_materialize(self.pending, self._acc)
            self.pending = None
            self.live = True

    def can_defer(self, table):
        """A backward may leave its row sums to the optimizer step: nothing else is in the store yet."""
        return self.clean and not self.live and self.pending is None and K.deferrable(table, self._acc)

    def touched_rows(self):
        """Number of touched rows (synchronises; does not expose the store)."""
        self.sync()
        return int(self._touched.sum())

    def reset(self, rows=None):
        self.sync()
        if rows is None:
            if not self.clean:
                self._acc.zero_()
            self._touched.zero_()
            self.clean = True           # every row is untouched and counts as zero
            self.live = False
            self.pending = None
        else:
            self.materialize()
            if not self.clean:
                self._acc.index_fill_(0, rows, 0.0)
            self._touched.index_fill_(0, rows, False)
        self.grad_scale = 1.0

    def stepped(self):
        """The optimizer consumed every touched row (touched cleared, acc rows zeroed or left stale)."""
        self.live = False
        self.pending = None
        self.grad_scale = 1.0

    def norm(self):
        """acc.norm() (reference: sparse_values.py:143): from the per-row squared norms of the touched rows when
        clean, over the whole exposed accumulator otherwise."""
        self.sync()
        if self.clean:
            return K.touched_norm(self._acc, self._touched, row_sqnorm=self._sqnorm)
        return self._acc.norm()


def row_store(table):
    """The RowStore attached to a (possibly shared) table parameter; created on first use. A table in host RAM
    (smlm_b200.host_values) gets a HostRowStore, or keeps the StepStore of its GACC step accumulator."""
    if getattr(table, "host_values", False):
        st = getattr(table, "row_store", None)
        if st is None or (getattr(st, "steprows", None) is None and tuple(st._acc.shape) != tuple(table.shape)):
            from .host_optim import HostRowStore
            st = table.row_store = HostRowStore(table)
        return st
    st = getattr(table, "row_store", None)
    if st is None or st._acc.device != table.device or st._acc.shape != table.shape:
        st = RowStore(table)
        table.row_store = st
    return st


def read_table(table):
    """The tensor a value bag reads for `table`: its bf16 copy when LazyRowAdam(value_copy_dtype=bf16) keeps one
    (half the gather bytes; the fp32 table stays the master that the optimizer updates), else the table itself.
    The optimizer's kernels refresh the copy's rows as they update them; a change made to the table through
    torch (load_state_dict, an in-place op) shows in the table's version counter, and then the whole copy is
    refreshed here before it is read."""
    copy = getattr(table, "value_copy", None)
    if copy is None or copy.shape != table.shape or copy.device != table.device:
        return table
    if getattr(table, "value_copy_version", None) != table._version:
        with torch.no_grad():
            copy.copy_(table)
        table.value_copy_version = table._version
    return copy


class _RowSparseBag(torch.autograd.Function):
    @staticmethod
    def forward(ctx, weights, indices, table, store, impl="cuda"):
        n, j = indices.shape
        w = weights.reshape(n, j).to(table.dtype)
        src = read_table(table)
        out = K.bag_forward(indices, w, src, out_dtype=table.dtype)
        ctx.save_for_backward(w, indices)
        ctx.table, ctx.src, ctx.store, ctx.wshape, ctx.wdtype = table, src, store, weights.shape, weights.dtype
        return out

    @staticmethod
    def backward(ctx, grad_out):
        table, src, store = ctx.table, ctx.src, ctx.store
        w, indices = ctx.saved_tensors
        # the per-sample-weight gradient only when the weights need one (constant weights, e.g. the one-lookup
        # bags of an Engram table, skip its kernel; the row sums are the same either way)
        want_gw = ctx.needs_input_grad[0]
        gw = None
        # the weight gradient reads the rows the forward read (the bf16 copy when there is one)
        if store is None:
            if want_gw:
                gw = K.bag_backward_rows(grad_out, indices, w, src, None, None)
        elif store.can_defer(table):
            # the first backward into an empty store: its row sums go straight into the optimizer step. The weight
            # gradient (which the scoring backward needs next) comes first; the sort and the norm pass (which only
            # the clip and the step need) run on a side stream meanwhile
            if want_gw:
                gw = K.bag_backward_rows(grad_out, indices, w, src, None, None)
            _, store.pending = K.bag_backward_deferred(grad_out, indices, w, table, store._touched, store._sqnorm,
                                                       want_gw=False, overlap=True)
        else:
            store.materialize()
            gw = K.bag_backward_rows(grad_out, indices, w, src, store._acc, store._touched,
                                     row_sqnorm=store._sqnorm if store.clean else None,
                                     first_touch_writes=store.clean, want_gw=want_gw)
            store.live = True
        # drop the RowStore reference so that `del table.row_store` after training frees the accumulator
        ctx.table = ctx.src = ctx.store = None
        return (gw.view(ctx.wshape).to(ctx.wdtype) if gw is not None else None), None, None, None, None


def row_sparse_embedding_bag(indices, weights, table, impl="cuda"):
    """sum_j weights[:, j] * table[indices[:, j]] with row-sparse gradient accumulation into table.row_store
    (reference: sparse_values.py:110-123)."""
    _check_impl(impl)
    if not torch.is_grad_enabled():
        return K.bag_forward(indices, weights.to(table.dtype), read_table(table), out_dtype=table.dtype)
    if not table.requires_grad:
        # frozen table: gradient for the weights only, no row accumulator
        return _RowSparseBag.apply(weights, indices, table, None, impl)
    # the table goes in as an input so that the output needs a gradient even when only the table is trained;
    # its backward returns None for it, the gradient goes into table.row_store instead
    return _RowSparseBag.apply(weights, indices, table, row_store(table), impl)


def row_sparse_tables(model):
    """Distinct value-table parameters that use row-sparse gradients (reference: sparse_values.py:126-134)."""
    seen, out = set(), []
    for m in model.modules():
        if (getattr(m, "value_grad", "dense") == "row_sparse" and m.values.weight.requires_grad
                and id(m.values.weight) not in seen):
            seen.add(id(m.values.weight))
            out.append(m.values.weight)
    return out


def clip_row_sparse(tables, max_norm):
    """Global norm over the accumulated row gradients of all row-sparse tables; the clip factor (0-d device
    tensor, no host sync) is stored and applied in the optimizer step. Returns the pre-clip norm
    (reference: sparse_values.py:137-151)."""
    if not tables:
        return None
    norms = [row_store(t).norm() for t in tables]
    sharded = [i for i, t in enumerate(tables) if getattr(t, "row_shard", None) is not None]
    if sharded:
        # row-sharded tables: each rank holds part of the rows; their squared norms are summed over the ranks
        from .sharded import sharded_sq_norm
        t0 = tables[sharded[0]]
        sq = torch.stack([norms[i].float() for i in sharded]).square().sum()
        total_sq = sharded_sq_norm(sq, t0.shard_group, t0.row_shard.world)
        rest = [norms[i].float() for i in range(len(tables)) if i not in sharded]
        if rest:
            total_sq = total_sq + torch.stack(rest).square().sum()
        total = total_sq.sqrt()
    else:
        total = torch.linalg.vector_norm(torch.stack(norms))
    coef = torch.clamp(max_norm / (total + 1e-6), max=1.0)
    for t in tables:
        row_store(t).grad_scale = coef
    return total


class LazyRowAdam(torch.optim.Optimizer):
    """Adam (no weight decay) on the rows read since the last step; rows that were not read keep their values and
    their Adam state bit-for-bit (global step count for bias correction, as torch SparseAdam / TF LazyAdam).
    One fused kernel per table reads only the touched rows (reference: sparse_values.py:154-362).

    state_dtype="bf16" / "int8" keeps compact moments (reference: sparse_values.py:163-168, kernels.py:445-515):
    bf16 exp_avg / exp_avg_sq, or int8 signed-square-root exp_avg and uint8 fourth-root exp_avg_sq codes with one
    fp32 scale per row each (exp_avg_scale, exp_avg_sq_scale); the update runs in fp32 on the decoded moments.

    value_copy_dtype=torch.bfloat16 keeps a bf16 copy of each table (`table.value_copy`) that the step refreshes
    for the updated rows: the value bag and its weight gradient read the copy (half the gather bytes; read_table)
    while the fp32 table stays the master that the step updates ("values bf16 with fp32 master").

    capturable=True (no counterpart in the reference) lets a training step that ends in this optimizer be captured
    in a CUDA graph (smlm_b200.graph_step): the step's bias-correction scalars are read from a small device buffer,
    which prepare_replay() advances and fills (computed as the eager step computes them, so the same bits) before
    every replay. Captured steps need fp32 moments: one backward per step takes the fused deferred step, several
    (memory layers sharing the table, accumulated micro-batches) the plain step over the written accumulator."""

    def __init__(self, params, lr, betas=(0.9, 0.95), eps=1e-8, name="memory_values", impl="cuda",
                 state_dtype="fp32", value_copy_dtype=None, capturable=False):
        params = list(params)
        _check_impl(impl)
        if state_dtype not in ("fp32", "bf16", "int8"):
            raise ValueError(f"unknown state_dtype: {state_dtype}")
        if any(p.dtype != torch.float32 or p.ndim != 2 or not p.is_contiguous() or p.shape[1] == 0 for p in params):
            raise ValueError("LazyRowAdam needs contiguous fp32 tables with nonzero width (2-D, float32)")
        if not 0 <= lr or not 0 <= eps or not all(0 <= b < 1 for b in betas):
            raise ValueError("invalid LazyRowAdam learning rate, epsilon or betas")
        if any(not p.is_cuda for p in params):
            raise ValueError("LazyRowAdam of this build runs on CUDA tables only (no CPU fallback)")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=0.0))
        for g in self.param_groups:
            g["name"] = name
            g["base_lr"] = lr
        self.impl = "cuda"
        self.state_dtype = state_dtype
        self.value_copy_dtype = value_copy_dtype
        if capturable and state_dtype != "fp32":
            raise ValueError("capturable=True needs fp32 moments")
        self.capturable = capturable
        self._scal = {}                 # capturable: per table, its step scalars on the device, (6,) fp32
        if value_copy_dtype is not None:
            if value_copy_dtype != torch.bfloat16:
                raise ValueError(f"value_copy_dtype must be torch.bfloat16, got {value_copy_dtype}")
            for p in params:
                p.value_copy = p.detach().to(value_copy_dtype)
                p.value_copy_version = p._version

    def _state(self, p):
        state = self.state[p]
        if not state:
            state["step"] = torch.zeros((), dtype=torch.float32)
            int8 = self.state_dtype == "int8"
            mdt = {"fp32": torch.float32, "bf16": torch.bfloat16, "int8": torch.int8}[self.state_dtype]
            vdt = torch.uint8 if int8 else mdt
            state["exp_avg"] = torch.zeros_like(p, dtype=mdt, memory_format=torch.contiguous_format)
            state["exp_avg_sq"] = torch.zeros_like(p, dtype=vdt, memory_format=torch.contiguous_format)
            if int8:
                state["exp_avg_scale"] = torch.zeros(p.shape[0], dtype=torch.float32, device=p.device)
                state["exp_avg_sq_scale"] = torch.zeros(p.shape[0], dtype=torch.float32, device=p.device)
        return state

    @staticmethod
    def _scalars(step, lr, b1, b2, eps):
        """The fused step's six scalars for `step`, as smlm_lazy_adam_deferred_step takes them."""
        bc1 = 1 - b1 ** step
        bc2 = 1 - b2 ** step
        return [1 - b1, b2, 1 - b2, math.sqrt(bc2), eps, -(lr / bc1)]

    def _write_scalars(self, p, group):
        """capturable: this table's scalars for its current step count, copied to the device buffer on the
        current stream."""
        b1, b2 = group["betas"]
        dev_buf = self._scal.get(p)
        if dev_buf is None:
            dev_buf = self._scal[p] = torch.zeros(6, dtype=torch.float32, device=p.device)
        # a fresh pinned staging tensor per write: the host allocator keeps it until its copy has run, so a host
        # that runs steps ahead never overwrites scalars a queued step still has to read
        host = torch.tensor(self._scalars(int(self.state[p]["step"]), group["lr"], b1, b2, group["eps"]),
                            dtype=torch.float32).pin_memory()
        dev_buf.copy_(host, non_blocking=True)
        return dev_buf

    def prepare_replay(self):
        """capturable: advance every table's step count and write its scalars, before replaying a captured step."""
        for group in self.param_groups:
            for p in group["params"]:
                state = self._state(p)
                state["step"] += 1
                self._write_scalars(p, group)

    @torch.no_grad()
    def step(self):
        capturing = torch.cuda.is_current_stream_capturing()
        if capturing and not self.capturable:
            raise RuntimeError("LazyRowAdam: capturing a step needs LazyRowAdam(capturable=True)")
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                st = row_store(p)
                st.sync()
                state = self._state(p)
                if self.capturable and self.state_dtype == "fp32" and st.pending is not None and not st.live:
                    # the scalars come from the device buffer: written now for an eager step, by prepare_replay()
                    # before every replay of a captured one
                    if not capturing:
                        state["step"] += 1
                        self._write_scalars(p, group)
                    elif p not in self._scal:
                        raise RuntimeError("LazyRowAdam(capturable=True): run one eager step before capturing")
                    K.lazy_adam_deferred_step(p, state["exp_avg"], state["exp_avg_sq"], st._touched, st.pending,
                                              st.grad_scale, 1, group["lr"], b1, b2, group["eps"],
                                              value_copy=getattr(p, "value_copy", None),
                                              scalars_dev=self._scal[p])
                    st.stepped()
                    continue
                if self.capturable and self.state_dtype == "fp32":
                    # several backward passes wrote the accumulator: the plain step, scalars from the device buffer
                    if not capturing:
                        state["step"] += 1
                        self._write_scalars(p, group)
                    elif p not in self._scal:
                        raise RuntimeError("LazyRowAdam(capturable=True): run one eager step before capturing")
                    st.materialize()
                    K.lazy_adam_step(p, state["exp_avg"], state["exp_avg_sq"], st._acc, st._touched,
                                     st.grad_scale, 1, group["lr"], b1, b2, group["eps"],
                                     value_copy=getattr(p, "value_copy", None), keep_acc=st.clean,
                                     scalars_dev=self._scal[p])
                    st.stepped()
                    continue
                if capturing:
                    raise RuntimeError("LazyRowAdam: a captured step needs capturable=True and fp32 moments")
                state["step"] += 1
                if self.state_dtype == "fp32" and st.pending is not None and not st.live:
                    # rows of one deferred backward: summed and stepped in one pass, acc never written
                    K.lazy_adam_deferred_step(p, state["exp_avg"], state["exp_avg_sq"], st._touched, st.pending,
                                              st.grad_scale, int(state["step"]), group["lr"], b1, b2, group["eps"],
                                              value_copy=getattr(p, "value_copy", None))
                elif self.state_dtype == "fp32":
                    st.materialize()
                    K.lazy_adam_step(p, state["exp_avg"], state["exp_avg_sq"], st._acc, st._touched,
                                     st.grad_scale, int(state["step"]), group["lr"], b1, b2, group["eps"],
                                     value_copy=getattr(p, "value_copy", None), keep_acc=st.clean)
                else:
                    st.materialize()
                    K.lazy_adam_lowmem_step(p, state["exp_avg"], state["exp_avg_sq"], state.get("exp_avg_scale"),
                                            state.get("exp_avg_sq_scale"), st._acc, st._touched, st.grad_scale,
                                            int(state["step"]), group["lr"], b1, b2, group["eps"],
                                            value_copy=getattr(p, "value_copy", None), keep_acc=st.clean)
                st.stepped()                # touched rows consumed; grad_scale back to 1

    def zero_grad(self, set_to_none=True):
        # the accumulator is cleared in step(); rows accumulated by a backward without a following step stay in
        # table.row_store (row_store(table).reset() drops them)
        pass

    def _params(self):
        return [p for g in self.param_groups for p in g["params"]]

    def _group_positions(self, params):
        pos = {id(p): i for i, p in enumerate(params)}
        return [[pos[id(p)] for p in g["params"]] for g in self.param_groups]

    def state_dict(self):
        """Moments and step count per table, in parameter order (format smlm.lazy_row_adam.v1)."""
        params = self._params()
        return {"format": "smlm.lazy_row_adam.v1", "state_dtype": self.state_dtype,
                "shapes": [list(p.shape) for p in params],
                "param_groups": [{**{k: v for k, v in g.items() if k != "params"}, "params": idx}
                                 for g, idx in zip(self.param_groups, self._group_positions(params))],
                "state": [dict(self.state[p]) for p in params]}

    def load_state_dict(self, state_dict):
        if state_dict.get("format") != "smlm.lazy_row_adam.v1":
            raise ValueError("not a LazyRowAdam state dict (smlm.lazy_row_adam.v1)")
        params = self._params()
        if state_dict["state_dtype"] != self.state_dtype:
            raise ValueError(f"LazyRowAdam state is {state_dict['state_dtype']}, this optimizer keeps "
                             f"{self.state_dtype}")
        if state_dict["shapes"] != [list(p.shape) for p in params]:
            raise ValueError("LazyRowAdam state was saved for other tables (shapes differ)")
        groups = state_dict["param_groups"]
        if [g["params"] for g in groups] != self._group_positions(params):
            raise ValueError("LazyRowAdam state has other parameter groups")
        for g, saved in zip(self.param_groups, groups):
            g.update({k: (tuple(v) if k == "betas" else v) for k, v in saved.items() if k != "params"})
        for p, saved in zip(params, state_dict["state"]):
            if not saved:
                continue
            self.state[p] = {k: (v.detach().clone().cpu() if k == "step" else v.to(device=p.device, copy=True))
                             for k, v in saved.items()}


class OptimizerSet:
    """Several optimizers driven as one (reference: sparse_values.py:365-395)."""

    def __init__(self, *opts):
        self.opts = [o for o in opts if o is not None]

    @property
    def param_groups(self):
        return [g for o in self.opts for g in o.param_groups]

    def step(self):
        for o in self.opts:
            o.step()

    def zero_grad(self, set_to_none=True):
        for o in self.opts:
            o.zero_grad(set_to_none=set_to_none)

    def state_dict(self):
        return {"format": "smlm.optimizer_set.v1",
                "optimizers": [{"type": type(o).__name__, "state_dict": o.state_dict()} for o in self.opts]}

    def load_state_dict(self, state_dict):
        if state_dict.get("format") != "smlm.optimizer_set.v1":
            raise ValueError("not an OptimizerSet state dict (smlm.optimizer_set.v1)")
        saved = state_dict["optimizers"]
        if [s["type"] for s in saved] != [type(o).__name__ for o in self.opts]:
            raise ValueError("OptimizerSet state holds other optimizers: "
                             f"{[s['type'] for s in saved]} vs {[type(o).__name__ for o in self.opts]}")
        for o, s in zip(self.opts, saved):
            o.load_state_dict(s["state_dict"])
