"""Row-wise optimizers for row-sparse value tables: one state number per row instead of Adam's two moments per
value, on the sm_100a kernels (reference: re133/sparse-memory-lm smlm/row_optim.py), for tables on the GPU or in
host RAM (smlm_b200.host_values: mapped host memory, HOT rows, GACC).

Only the rows read since the last step change; rows that were not read keep their values and their state
exactly. g = a row's accumulated gradient times the clip factor, q = the mean of g^2 over the row.
  rowrms      v_r = b2 v_r + (1 - b2) q,  n_r += 1,  p_r -= lr g / (sqrt(v_r / (1 - b2^n_r)) + eps)
  rowadagrad  v_r += q,  p_r -= lr g / (sqrt(v_r) + eps)
State per row: fp32 v plus an int32 n (rowrms). One fused kernel per table visits the touched rows only (the
reference's GPU path runs masked chunks over the whole table, row_optim.py:179-201).
"""
import torch

from . import kernels as K
from .sparse_values import row_store

KINDS = ("rowrms", "rowadagrad")


class RowWiseOptimizer(torch.optim.Optimizer):
    """rowrms / rowadagrad on row-sparse CUDA tables (reference: row_optim.py:25-239)."""

    def __init__(self, params, lr, kind="rowrms", beta2=0.95, eps=1e-8, name="memory_values"):
        params = list(params)
        if kind not in KINDS:
            raise ValueError(f"unknown row-wise optimizer: {kind}")
        if any(p.dtype != torch.float32 or p.ndim != 2 or not p.is_contiguous() or p.shape[1] == 0 for p in params):
            raise ValueError("row-wise optimizers require contiguous fp32 tables with nonzero width")
        if any(not p.is_cuda and not getattr(p, "host_values", False) for p in params):
            raise ValueError("row-wise optimizers of this build run on CUDA tables or host-RAM tables only")
        if not 0 <= lr or not 0 <= eps or not 0 <= beta2 < 1:
            raise ValueError("invalid learning rate, epsilon or beta2")
        super().__init__(params, dict(lr=lr, beta2=beta2, eps=eps, weight_decay=0.0))
        for g in self.param_groups:
            g["name"] = name
            g["base_lr"] = lr
        self.kind = kind

    def _state(self, p):
        state = self.state[p]
        if not state:
            state["step"] = torch.zeros((), dtype=torch.float32)
            state["v"] = torch.zeros(p.shape[0], dtype=torch.float32, device=p.device)
            if self.kind == "rowrms":
                state["n"] = torch.zeros(p.shape[0], dtype=torch.int32, device=p.device)
        return state

    @torch.no_grad()
    def step(self):
        for group in self.param_groups:
            for p in group["params"]:
                st = row_store(p)
                st.sync()
                state = self._state(p)
                state["step"] += 1
                if getattr(p, "host_values", False):
                    self._step_host(group, p, st, state)
                    continue
                if st.pending is not None and not st.live:
                    # rows of one deferred backward: summed and stepped in one pass, acc never written
                    K.rowwise_deferred_step(p, st._touched, state["v"], state.get("n"), st.pending, st.grad_scale,
                                            group["lr"], group["beta2"], group["eps"], self.kind)
                else:
                    st.materialize()
                    K.rowwise_step(p, st._acc, st._touched, state["v"], state.get("n"), st.grad_scale, group["lr"],
                                   group["beta2"], group["eps"], self.kind, keep_acc=st.clean)
                st.stepped()

    @torch.no_grad()
    def _step_host(self, group, p, st, state):
        """A table in host RAM (smlm_b200.host_values; reference: row_optim.py:58-157): the per-row state moves to
        the GPU (8 bytes a row; the reference keeps it in RAM); the HOT rows' state is kept in slot order there and
        they step there; the other rows step in place in host RAM through the mapped table and accumulator
        (smlm_rowwise_step), or, with GACC, from the step's row sums on the GPU (smlm_rows_rowwise_step), overflow
        rows included."""
        from . import _lib as L
        from .host_values import mapped
        hot = getattr(st, "hot", None)
        sr = getattr(st, "steprows", None)
        if hot is not None:
            dev = hot.values.device
        elif sr is not None:
            dev = sr.acc.device
        else:
            dev = torch.device("cuda", torch.cuda.current_device())
        kind = L.ROWRMS if self.kind == "rowrms" else L.ROWADAGRAD
        scale = st.grad_scale
        # the per-row state (8 bytes a row) lives on the GPU, so the steps read no state over the host link
        for key in ("v", "n"):
            if key in state and state[key].device != dev:
                state[key] = state[key].to(dev)
        if hot is not None:
            if "hot_v" not in state:
                state["hot_v"] = state["v"].index_select(0, hot.rows)
                if "n" in state:
                    state["hot_n"] = state["n"].index_select(0, hot.rows)
            K.rowwise_step(hot.values, hot.acc, hot.touched, state["hot_v"], state.get("hot_n"), scale, group["lr"],
                           group["beta2"], group["eps"], self.kind)
        sp, sf, keep = None, 1.0, None
        if torch.is_tensor(scale):
            keep = scale.detach().to(device=dev, dtype=torch.float32).reshape(1).contiguous()
            sp = L.ptr(keep)
        else:
            sf = float(scale)
        count = state.get("n")
        with torch.cuda.device(dev):
            if sr is not None:
                cur = sr.current()
                on_device = cur is not None and sr.prev_slot is not None
                if not on_device and sr.prev_slot is not None:
                    sr._drop_cache()      # rows are about to change in the host table only
                parts = []
                if sr.n:                  # with the rows' values from the forward's gather when the slots keep them
                    parts.append((sr.rows[:sr.n], sr.acc[:sr.n], cur, L.ROWS_TO_CURRENT if on_device else 0))
                spilled = sr.spilled()
                if spilled is not None:   # rows read after every slot was taken: summed on the host, never in a slot
                    sr.wait_written()     # such a row may be in the write-back still running
                    parts.append((spilled[0].to(dev), spilled[1].to(dev), None, 0))
                for rows, g, c, flags in parts:
                    rc = L.lib().smlm_rows_rowwise_step(
                        mapped(p.detach()), p.shape[0], L.ptr(rows), L.ptr(g.contiguous()), L.ptr(c), rows.numel(),
                        p.shape[1], L.ptr(state["v"]), L.ptr(count), kind, group["beta2"], group["eps"],
                        group["lr"], sp, sf, flags, L.status_ptr(dev), L.stream(dev))
                    L.check(rc, "rows_rowwise_step")
                if on_device:
                    sr.finish()           # the updated rows: back into the host table, kept as the next cache
                else:
                    torch.cuda.current_stream(dev).synchronize()
                    sr.reset()
            elif bool(st.touched.any()):
                ws = L.workspace(L.lib().smlm_touched_workspace(p.shape[0]), dev)
                rc = L.lib().smlm_rowwise_step(
                    mapped(p.detach()), mapped(st._acc), mapped(st.touched), L.ptr(state["v"]), L.ptr(count), sp, sf,
                    p.shape[0], p.shape[1], kind,
                    group["beta2"], group["eps"], group["lr"], L.STEP_KEEP_ACC, L.ptr(ws), ws.numel(), L.stream(dev))
                L.check(rc, "rowwise_step (host table)")
                torch.cuda.current_stream(dev).synchronize()
                st.stale = True           # the rows' accumulator values stay; the next add overwrites them
        del keep
        st.grad_scale = 1.0

    def zero_grad(self, set_to_none=True):
        pass                                   # the accumulator is cleared in step(), as in LazyRowAdam

    def _params(self):
        return [p for g in self.param_groups for p in g["params"]]

    def flush(self):
        """Writes the state of the HOT rows of host-RAM tables (on the GPU, in slot order) back into the per-row
        state of the whole table (reference: row_optim.py:209-217); tables on the GPU have nothing to write back."""
        for p in self._params():
            state, hot = self.state[p], getattr(row_store(p), "hot", None)
            if hot is not None and "hot_v" in state:
                rows = hot.rows.to(state["v"].device)
                state["v"].index_copy_(0, rows, state["hot_v"].to(state["v"].device))
                if "hot_n" in state:
                    state["n"].index_copy_(0, rows, state["hot_n"].to(state["n"].device))

    def state_dict(self):
        """Every row's state in table order (HOT rows written back first), so it loads with or without HOT."""
        self.flush()
        params = self._params()
        return {"format": "smlm.row_wise.v1", "kind": self.kind, "shapes": [list(p.shape) for p in params],
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups],
                "state": [{k: v for k, v in self.state[p].items() if not k.startswith("hot_")} for p in params]}

    def load_state_dict(self, state_dict):
        if state_dict.get("format") != "smlm.row_wise.v1" or state_dict.get("kind") != self.kind:
            raise ValueError(f"not a {self.kind} state dict (smlm.row_wise.v1)")
        params = self._params()
        if state_dict["shapes"] != [list(p.shape) for p in params]:
            raise ValueError("row-wise optimizer state was saved for other tables (shapes differ)")
        for g, saved in zip(self.param_groups, state_dict["param_groups"]):
            g.update(saved)
        for p, saved in zip(params, state_dict["state"]):
            if saved:
                self.state[p] = {k: (v.detach().clone() if k == "step" else v.to(device=p.device, copy=True))
                                 for k, v in saved.items()}


def state_bytes(kind, rows):
    """Persistent optimizer state of one table (reference: row_optim.py:241-243)."""
    return rows * (8 if kind == "rowrms" else 4) + 4
