"""Product-key value tables in host RAM, for tables larger than the GPUs' memory (reference: re133/sparse-memory-lm
smlm/host_values.py; same entry points: enable_host_values, HostEmbedding, HotRows, StepRows, StepStore,
enable_step_rows, enable_hot_rows, host_timings).

The reference stages the rows a step reads through the CPU: it copies the distinct row indices to the host,
gathers the rows with a C loop into pinned memory, copies them to the GPU, and on the way back copies the row
gradients to the host and scatter-adds them there with a C loop. Here the host tensors (the table, its gradient
accumulator, the optimizer state) are page-locked and mapped into the GPU's address space once (`mapped`), and
the library's kernels move the rows over the host link themselves:

  forward   the distinct rows of the lookups (torch.unique on the GPU) are gathered by one kernel straight from the
            mapped table (HOT rows from their device copies) into a device tensor; the value bag runs over it with
            the remapped indices (the bag kernel, same order of sums as the device path);
  backward  the row-sparse backward over the gathered rows gives each distinct row's gradient sum on the GPU
            (the deterministic sorted segment sums); one kernel adds them into the mapped accumulator rows and
            sets their touched marks (HOT rows into their device accumulator; with GACC into the step's slots on
            the GPU instead of the host accumulator);
  step      the optimizers' kernels update the touched rows in place in the mapped table and state
            (smlm_b200.host_optim.HostLazyRowAdam, RowWiseOptimizer); nothing is copied back. With GACC the step's
            slots also keep the rows as the forward gathered them, so the row-wise step reads them on the GPU and
            only writes the host table.

So per step only the rows read cross the host link (in for the forward, then once each way for the optimizer,
or only out with GACC), with 16-byte accesses, and no CPU thread touches them; the add kernel also keeps each
row's squared norm on the GPU, so clipping reads no accumulator rows back. The calls that write host memory
synchronise the stream before returning (CPU code may read that memory next), which also makes this path, like
the reference's, not capturable in a CUDA graph. Rows need a width that is a multiple of 4 values. Host tensors
stay registered (and alive) until release() unmaps them.
"""
import ctypes
import time
from contextlib import contextmanager

import torch
from torch import nn

from . import _lib as L
from . import kernels as K

# the reference's staging phases (host_timings keys); the host-link transfers of this build happen inside the
# gather and scatter kernels, so indices_d2h, rows_h2d and gradients_d2h stay 0
PHASES = ("unique", "indices_d2h", "gather", "rows_h2d", "gradients_d2h", "scatter")

_MAPPED = {}        # host storage address -> (bytes, device address, storage kept alive)


def mapped(t):
    """The device address of a CPU tensor's data: its storage is page-locked and mapped into the device's address
    space on first use (smlm_host_register) and stays so, and alive, until release() (or the end of the process)."""
    if t.device.type != "cpu":
        raise ValueError("mapped() takes host (CPU) tensors")
    storage = t.untyped_storage()
    base, nbytes = storage.data_ptr(), storage.nbytes()
    hit = _MAPPED.get(base)
    if hit is None or hit[0] < nbytes:
        if hit is not None:
            L.lib().smlm_host_unregister(ctypes.c_void_p(base))
        dev = ctypes.c_void_p()
        L.check(L.lib().smlm_host_register(ctypes.c_void_p(base), max(nbytes, 1), ctypes.byref(dev)),
                "host_register")
        hit = _MAPPED[base] = (nbytes, dev.value, storage)
    return ctypes.c_void_p(hit[1] + (t.data_ptr() - base))


def release(*tensors):
    """Unmaps the storages of host tensors mapped by mapped() and drops the references that kept them alive, so
    that they are freed with their last owner. No kernel may still use them: call after the stream that last
    touched them has been synchronised."""
    for t in tensors:
        if t is None or not torch.is_tensor(t) or t.device.type != "cpu":
            continue
        hit = _MAPPED.pop(t.untyped_storage().data_ptr(), None)
        if hit is not None:
            L.check(L.lib().smlm_host_unregister(ctypes.c_void_p(t.untyped_storage().data_ptr())), "host_unregister")


def _sync(device):
    torch.cuda.current_stream(device).synchronize()


ROW_GRANULE = 1 << 16     # per-step row buffers are allocated in multiples of this many rows


def _row_buffer(n, d, device, zero=False):
    """An (n, d) fp32 device tensor whose allocation is rounded up to ROW_GRANULE rows: the distinct rows of a step
    vary by a few thousand from step to step, and multi-GB requests of ever new sizes make the caching allocator
    map new memory (a slow cudaMalloc) instead of reusing its blocks."""
    cap = max(1, -(-n // ROW_GRANULE)) * ROW_GRANULE
    t = torch.empty(cap, d, dtype=torch.float32, device=device)[:n]
    return t.zero_() if zero else t


class HostEmbedding(nn.Embedding):
    """A value table that stays fp32 in host RAM when its model moves to the GPU (reference:
    host_values.py:29-161); a normal parameter for checkpoints. `hot`: its HOT rows (enable_hot_rows), `step_rows`:
    its step accumulator on the GPU (enable_step_rows)."""

    def __init__(self, source, profile=False):
        super().__init__(source.num_embeddings, source.embedding_dim, _weight=source.weight)
        self.weight = source.weight
        self.weight.host_values = True
        self.profile = profile
        self.timings = dict.fromkeys(PHASES, 0.0)
        self.hot = None
        self.step_rows = None
        self.register_state_dict_pre_hook(lambda module, *_: module.flush())
        self._register_load_state_dict_pre_hook(lambda *_: self.flush())
        self.register_load_state_dict_post_hook(lambda module, _keys: module.reload_hot())

    def reload_hot(self):
        """After the table was loaded: the HOT rows' device copies from the new table, their gradients dropped
        (the row-wise optimizer takes their state from its own loaded state at the next step)."""
        if self.hot is not None:
            self.hot.values.copy_(self.weight.detach().index_select(0, self.hot.rows.cpu()))
            self.hot.acc.zero_()
            self.hot.touched.zero_()

    def flush(self):
        """Write the GPU copies of the hot rows back into the host table (after any write-back of a GACC step still
        running, so the host table is complete for CPU code)."""
        if self.step_rows is not None:
            self.step_rows.sync()
        if self.hot is not None:
            _sync(self.hot.values.device)
            self.weight.detach().index_copy_(0, self.hot.rows.cpu(), self.hot.values.detach().cpu())

    def _apply(self, fn, recurse=True):
        return self                        # the table never moves: a device copy would not fit

    @contextmanager
    def phase(self, name, device=None):
        if not self.profile:
            yield
            return
        if device is not None and device.type == "cuda":
            torch.cuda.synchronize(device)
        start = time.perf_counter()
        try:
            yield
        finally:
            if device is not None and device.type == "cuda":
                torch.cuda.synchronize(device)
            self.timings[name] += time.perf_counter() - start

    def gather(self, indices):
        """(distinct rows (device int64, sorted), the lookups remapped onto them, their values gathered onto the
        device (fp32; HOT rows and the previous GACC step's rows from their device copies), and their HOT slots
        (device int32, -1 for rows in host RAM) or None)."""
        dev = indices.device
        with self.phase("unique", dev):
            rows, remapped = torch.unique(indices.reshape(-1), sorted=True, return_inverse=True)
        slot = self.hot.slot.index_select(0, rows) if self.hot is not None else None
        prev_slot, cache = self.step_rows.cache() if self.step_rows is not None else (None, None)
        slot2 = prev_slot.index_select(0, rows) if prev_slot is not None else None
        values = _row_buffer(rows.numel(), self.embedding_dim, dev)
        with self.phase("gather", dev):
            t = self.weight.detach()
            rc = L.lib().smlm_host_rows_gather(mapped(t), t.shape[0], L.ptr(rows), L.ptr(slot),
                                               L.ptr(self.hot.values) if slot is not None else None, L.ptr(slot2),
                                               L.ptr(cache), rows.numel(), t.shape[1], L.ptr(values),
                                               L.status_ptr(dev), L.stream(dev))
            L.check(rc, "host_rows_gather")
            L.after(dev, "host_rows_gather")
        return rows, remapped.view_as(indices), values, slot

    def accumulate(self, rows, gradient, slot=None, values=None):
        """Adds each distinct row's gradient sum (device (U, d)) into its accumulator: the step's slots on the GPU
        (GACC; `values`, the rows as the forward gathered them, go into the slots too), the HOT accumulator on the
        GPU, or the mapped host accumulator."""
        dev = gradient.device
        hot = slot is not None
        if hot:
            at_hot = (slot >= 0).nonzero().squeeze(1)
            if at_hot.numel():
                s = slot.index_select(0, at_hot).long()
                self.hot.acc.index_add_(0, s, gradient.index_select(0, at_hot))
                self.hot.touched.index_fill_(0, s, True)
        if self.step_rows is not None:
            with self.phase("scatter", dev):
                if hot:
                    cold = (slot < 0).nonzero().squeeze(1)
                    self.step_rows.add(rows.index_select(0, cold), gradient.index_select(0, cold),
                                       values.index_select(0, cold) if values is not None else None)
                else:
                    self.step_rows.add(rows, gradient, values)
            return
        from .sparse_values import row_store
        st = row_store(self.weight)
        with self.phase("scatter", dev):
            rc = L.lib().smlm_host_rows_add(mapped(st._acc), mapped(st.touched), L.ptr(st.sq_buffer(dev)),
                                            st._acc.shape[0], L.ptr(rows), L.ptr(gradient.contiguous()), L.ptr(slot),
                                            rows.numel(), gradient.shape[1], L.status_ptr(dev), L.stream(dev))
            L.check(rc, "host_rows_add")
            _sync(dev)                     # the host accumulator is complete before CPU code reads it
        L.after(dev, "host_rows_add")

    def bag(self, indices, weights, impl="cuda"):
        """sum_j weights[:, j] * table[indices[:, j]] for CUDA indices (reference: host_values.py:152-161)."""
        if self.weight.device.type != "cpu" or self.weight.dtype != torch.float32:
            raise ValueError("host values must remain fp32 on CPU")
        if not indices.is_cuda:
            raise ValueError("host value tables of this build are read by the GPU: pass CUDA indices")
        rows, remapped, values, slot = self.gather(indices)
        n, j = remapped.shape
        if not torch.is_grad_enabled():
            return K.bag_forward(remapped, weights.reshape(n, j).float(), values)
        return _HostBag.apply(weights, remapped, values, self.weight, rows, self, slot)


class _HostBag(torch.autograd.Function):
    """The value bag over the gathered rows; backward: the weight gradient and each distinct row's gradient sum
    (smlm_bag_backward_rows over the gathered rows, the device path's sorted summation order), the sums handed to
    HostEmbedding.accumulate (reference: host_values.py:164-206)."""

    @staticmethod
    def forward(ctx, weights, indices, values, table, rows, owner, slot):
        n, j = indices.shape
        w = weights.reshape(n, j).float().contiguous()
        out = K.bag_forward(indices, w, values)
        ctx.save_for_backward(w, indices, values, rows, slot)
        ctx.owner, ctx.train_table = owner, table.requires_grad
        ctx.wshape, ctx.wdtype = weights.shape, weights.dtype
        return out

    @staticmethod
    def backward(ctx, grad_out):
        w, indices, values, rows, slot = ctx.saved_tensors
        g = grad_out.contiguous()
        if g.dtype not in (torch.float32, torch.bfloat16):
            g = g.float()
        if ctx.train_table:
            acc = _row_buffer(values.shape[0], values.shape[1], values.device, zero=True)
            touched = torch.zeros(values.shape[0], dtype=torch.bool, device=values.device)
            gw = K.bag_backward_rows(g, indices, w, values, acc, touched)
            ctx.owner.accumulate(rows, acc, slot, values)
        else:
            gw = K.bag_backward_rows(g, indices, w, values, None, None)
        ctx.owner = None
        return gw.view(ctx.wshape).to(ctx.wdtype), None, None, None, None, None, None


def enable_host_values(model, profile=False):
    """Moves the model's product-key value tables to host RAM (HostEmbedding; call on the CPU fp32 model, before
    moving it to the GPU; reference: host_values.py:209-236). Row-sparse gradients only, no Engram tables; the
    one-token decode graphs are switched off (the host path synchronises)."""
    from .pkm import ProductKeyMemory
    memories = [m for m in model.modules() if isinstance(m, ProductKeyMemory)]
    if not memories or any(getattr(m, "is_engram", False) for m in model.modules()):
        raise ValueError("value_device=host requires a PKM model without Engram tables")
    for m in memories:
        if m.value_grad != "row_sparse":
            raise ValueError("value_device=host requires row_sparse PKM gradients")
        if m.values.weight.device.type != "cpu" or m.values.weight.dtype != torch.float32:
            raise ValueError("enable host values on a CPU fp32 model before moving it to the GPU")
        if not m.values.weight.is_contiguous() or m.values.weight.shape[1] == 0:
            raise ValueError("host values require contiguous tables with nonzero width")
        if m.values.weight.shape[1] % 4:
            raise ValueError("host value tables of this build need rows of a multiple of 4 values")
        if m.shard is not None:
            raise ValueError("a row-sharded table cannot also live in host RAM")
    shared = {}
    for m in memories:
        key = id(m.values.weight)
        if key not in shared:
            shared[key] = m.values if isinstance(m.values, HostEmbedding) else HostEmbedding(m.values, profile)
        m.values = shared[key]
        m.values.profile = profile
        m.decode_graph = False
        m._graph = None
    return model


class HotRows:
    """Rows of a host table kept on the GPU (HOT): their values, gradient accumulator, touched mask and the map
    row -> slot (-1 for rows in host RAM); the row-wise optimizer keeps their state in slot order on the GPU too
    (reference: host_values.py:239-250)."""

    def __init__(self, table, rows, device):
        rows = torch.as_tensor(rows, dtype=torch.int64).sort().values
        self.rows = rows.to(device)
        self.slot = torch.full((table.shape[0],), -1, dtype=torch.int32, device=device)
        self.slot[self.rows] = torch.arange(rows.numel(), dtype=torch.int32, device=device)
        self.values = table.detach().index_select(0, rows).to(device)
        self.acc = torch.zeros_like(self.values)
        self.touched = torch.zeros(rows.numel(), dtype=torch.bool, device=device)


class StepRows:
    """GACC: the gradient sums of the host-table rows read in the current step, on the GPU, in up to `capacity`
    slots (a row takes the next free slot when it is first read in the step; later reads add into it). Rows read
    after every slot is taken (overflow) keep their gradients on the host, summed per row before the step, so a
    step that reads more rows than the capacity is slower, not wrong (reference: host_values.py:253-316).

    keep_values (no counterpart; needs `table`): each slot also keeps the row's values as the forward gathered
    them (the table does not change within a step). The row-wise step then updates the slots' rows on the GPU
    (update(), the state too) and writes them back into the host table with one scatter kernel (finish()), and the
    step's rows stay on the GPU as the previous step's cache: the next step's gather reads them there instead of
    over the host link. overlap: that write-back runs on a side stream while the next step computes and gathers the
    other rows (the two directions of the host link at once); it only has to end before the step after next
    touches the host table, and CPU code reads the table after flush() (HostEmbedding.flush, state_dict)."""

    def __init__(self, num_rows, dim, capacity, device, keep_values=True, table=None, overlap=False):
        keep_values = keep_values and table is not None
        if overlap and not keep_values:
            raise ValueError("overlapped write-back needs keep_values and the table")
        self.slot = torch.full((num_rows,), -1, dtype=torch.int32, device=device)
        self.rows = torch.empty(capacity, dtype=torch.int64, device=device)
        self.acc = torch.zeros(capacity, dim, dtype=torch.float32, device=device)
        self.values = torch.empty(capacity, dim, dtype=torch.float32, device=device) if keep_values else None
        self._values_ok = True
        self.n = 0
        self.peak = 0                      # most distinct rows read in one step so far, overflow included
        self.spilled_steps = 0             # steps with an overflow
        self._spill = []                   # (rows, gradients) on the host; a row may appear in several parts
        self._summed = None
        self.table = table
        # the previous step's rows as its step left them: slot map, rows, values (keep_values only)
        if keep_values:
            self.prev_slot = torch.full((num_rows,), -1, dtype=torch.int32, device=device)
            self.prev_rows = torch.empty(capacity, dtype=torch.int64, device=device)
            self.prev_values = torch.empty(capacity, dim, dtype=torch.float32, device=device)
        else:
            self.prev_slot = self.prev_rows = self.prev_values = None
        self.prev_n = 0
        self._prev_version = None
        self.stream = torch.cuda.Stream(device) if overlap else None
        self._written = None               # event: the last write-back has ended (overlap)

    def add(self, rows, gradient, values=None):
        """rows: distinct row ids on the device, gradient: one row each; values: the rows' current values (device),
        or None (then the step reads the rows from the host table)."""
        slots = self.slot[rows]
        new = (slots < 0).nonzero().squeeze(1)
        free = self.rows.numel() - self.n
        keep = None
        if new.numel() > free:
            out = new[free:]
            self._spill.append((rows.index_select(0, out).cpu(), gradient.index_select(0, out).cpu()))
            self._summed = None
            new = new[:free]
            keep = torch.ones_like(slots, dtype=torch.bool).index_fill_(0, out, False)
        k = new.numel()
        if k:
            ids = torch.arange(self.n, self.n + k, dtype=torch.int32, device=rows.device)
            fresh = rows.index_select(0, new)
            self.slot[fresh] = ids
            self.rows[self.n:self.n + k] = fresh
            slots[new] = ids
            if self.values is not None:
                if values is None:
                    self._values_ok = False
                else:
                    self.values[self.n:self.n + k] = values.index_select(0, new)
            self.n += k
            self.peak = max(self.peak, self.n)
        if keep is not None:
            slots, gradient = slots[keep], gradient[keep]
        if self.acc.is_cuda and self.acc.shape[1] % 4 == 0:
            # the slots of one add are distinct: the host-add kernel (acc[slot] + g, 16-byte rows) on device memory
            dev = self.acc.device
            g, idx = gradient.contiguous(), slots.long()
            rc = L.lib().smlm_host_rows_add(L.ptr(self.acc), None, None, self.acc.shape[0], L.ptr(idx), L.ptr(g),
                                            None, idx.numel(), self.acc.shape[1], L.status_ptr(dev), L.stream(dev))
            L.check(rc, "host_rows_add (step slots)")
        else:
            self.acc.index_add_(0, slots.long(), gradient)

    def current(self):
        """The slots' row values (device (n, d)) when every slot's values were given, else None."""
        return self.values[:self.n] if self.values is not None and self._values_ok else None

    def cache(self):
        """(slot map, values) of the previous step's rows for the gather, or (None, None). The cache is dropped
        when the table was changed by anything but these steps (its version counter moved)."""
        if not self.prev_n:
            return None, None
        if self.table._version != self._prev_version:
            self._drop_cache()
            return None, None
        return self.prev_slot, self.prev_values

    def _drop_cache(self):
        self.wait_written()
        self.prev_slot.index_fill_(0, self.prev_rows[:self.prev_n], -1)
        self.prev_n = 0

    def wait_written(self):
        """Orders the current stream after the last write-back (overlap)."""
        if self._written is not None:
            torch.cuda.current_stream(self.acc.device).wait_event(self._written)

    def sync(self):
        """Waits on the host until the last write-back has reached the host table."""
        if self._written is not None:
            self._written.synchronize()

    def spilled(self):
        """(rows, gradient sums) of the overflow on the host, each row once; None without an overflow."""
        if not self._spill:
            return None
        if self._summed is None:
            rows = torch.cat([r for r, _ in self._spill])
            unique, inverse = torch.unique(rows, sorted=True, return_inverse=True)
            sums = torch.zeros(unique.numel(), self.acc.shape[1], dtype=torch.float32)
            sums.index_add_(0, inverse, torch.cat([g for _, g in self._spill]))
            self._summed = (unique, sums)
            self.peak = max(self.peak, self.n + unique.numel())
        return self._summed

    def reset(self):
        """Drops the step's gradients (the table is unchanged; the previous step's cache stays)."""
        if self._spill:
            self.spilled()                 # counts the step's overflow rows in peak
            self.spilled_steps += 1
            self._spill, self._summed = [], None
        self.slot.index_fill_(0, self.rows[:self.n], -1)
        self.acc[:self.n].zero_()
        self.n = 0
        self._values_ok = True

    def finish(self):
        """After update() wrote the step's rows into the slots: the slots become the previous step's cache, their
        rows are written back into the host table (on the side stream with overlap, else here, synchronously),
        and the gradients are dropped."""
        dev = self.acc.device
        self.wait_written()                # the older write-back read the buffers that are reused next
        self.prev_slot.index_fill_(0, self.prev_rows[:self.prev_n], -1)
        self.slot, self.prev_slot = self.prev_slot, self.slot
        self.rows, self.prev_rows = self.prev_rows, self.rows
        self.values, self.prev_values = self.prev_values, self.values
        self.prev_n, n = self.n, self.n
        self.n = 0
        self.acc[:n].zero_()
        self._values_ok = True
        if self._spill:
            self.spilled()
            self.spilled_steps += 1
            self._spill, self._summed = [], None
        table = self.table.detach()
        self._prev_version = self.table._version
        main = torch.cuda.current_stream(dev)
        if self.stream is not None:
            self.stream.wait_stream(main)
            ctx = torch.cuda.stream(self.stream)
        else:
            ctx = torch.cuda.stream(main)
        with ctx:
            rc = L.lib().smlm_host_rows_scatter(mapped(table), table.shape[0], L.ptr(self.prev_rows),
                                                L.ptr(self.prev_values), n, table.shape[1], L.status_ptr(dev),
                                                L.stream(dev))
            L.check(rc, "host_rows_scatter")
        if self.stream is not None:
            self._written = self.stream.record_event()
        else:
            main.synchronize()             # the host table is complete before CPU code reads it


class StepStore:
    """row_store() of a host table with GACC: no table-sized accumulator; the gradients sit in `steprows` (and in
    `hot` for hot rows); grad_scale is set by clipping as for a RowStore (reference: host_values.py:319-340)."""

    def __init__(self, steprows, hot=None):
        self.steprows, self.hot, self.grad_scale = steprows, hot, 1.0

    def norm(self):
        parts = [self.steprows.acc[:self.steprows.n].norm()]
        if self.hot is not None:
            parts.append(self.hot.acc.norm())
        spilled = self.steprows.spilled()
        if spilled is not None:
            parts.append(spilled[1].norm().to(parts[0].device))
        return torch.linalg.vector_norm(torch.stack(parts))

    def reset(self, rows=None):
        self.steprows.reset()
        if self.hot is not None:
            self.hot.acc.zero_()
            self.hot.touched.zero_()
        self.grad_scale = 1.0

    def sync(self):
        pass


def enable_step_rows(model, capacity, device, keep_values=True, overlap=False):
    """GACC for every host table: sum each step's row gradients on `device` in up to `capacity` rows (rows read in
    one step, hot rows not counted). Needs a row-wise table optimizer. Call after enable_hot_rows, if both
    (reference: host_values.py:343-350). keep_values and overlap (no counterpart; StepRows): the step's rows are
    updated on the GPU and kept there as the next step's cache (2 x capacity x width x 4 more bytes on the device),
    and with overlap written back to the host table while the next step runs."""
    for module in model.modules():
        if isinstance(module, HostEmbedding) and module.step_rows is None:
            module.step_rows = StepRows(module.num_embeddings, module.embedding_dim, capacity, device, keep_values,
                                        module.weight, overlap)
            module.weight.row_store = StepStore(module.step_rows, module.hot)
    return model


def enable_hot_rows(model, reads, fraction, device):
    """Keeps the `fraction` most-read rows of each host table on `device`, ranked by `reads` (read counts per row
    from an earlier run). Needs a row-wise table optimizer; call after moving the model to the device and before
    the first step (reference: host_values.py:353-371)."""
    reads = torch.as_tensor(reads)
    for module in model.modules():
        if isinstance(module, HostEmbedding) and module.hot is None:
            if reads.shape != (module.num_embeddings,):
                raise ValueError(f"read counts for {reads.shape[0]} rows, the table has {module.num_embeddings}")
            if module.step_rows is not None:
                raise ValueError("enable hot rows before the step accumulator")
            n = int(round(fraction * module.num_embeddings))
            module.hot = HotRows(module.weight, torch.argsort(reads, descending=True, stable=True)[:n], device)
            module.weight.hot_rows = module.hot
            if getattr(module.weight, "row_store", None) is not None:
                module.weight.row_store.hot = module.hot
    return model


def host_timings(model, reset=False):
    """Cumulative staging wall seconds (synchronised when profiling), shared tables counted once (reference:
    host_values.py:374-383)."""
    totals = dict.fromkeys(PHASES, 0.0)
    seen = set()
    for module in model.modules():
        if isinstance(module, HostEmbedding) and id(module) not in seen:
            seen.add(id(module))
            for phase, elapsed in module.timings.items():
                totals[phase] += elapsed
            if reset:
                module.timings = dict.fromkeys(PHASES, 0.0)
    return totals
