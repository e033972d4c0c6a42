"""Row-wise optimizers for row-sparse value tables: one state number per row instead of Adam's two moments per
value, on the sm_100a kernels (reference: re133/sparse-memory-lm smlm/row_optim.py).

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
        if any(not p.is_cuda for p in params):
            raise ValueError("row-wise optimizers of this build run on CUDA tables only")
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
                if st.pending is not None and not st.live:
                    # rows of one deferred backward: summed and stepped in one pass, acc never written
                    K.rowwise_deferred_step(p, st._touched, state["v"], state.get("n"), st.pending, st.grad_scale,
                                            group["lr"], group["beta2"], group["eps"], self.kind)
                else:
                    st.materialize()
                    K.rowwise_step(p, st._acc, st._touched, state["v"], state.get("n"), st.grad_scale, group["lr"],
                                   group["beta2"], group["eps"], self.kind, keep_acc=st.clean)
                st.stepped()

    def zero_grad(self, set_to_none=True):
        pass                                   # the accumulator is cleared in step(), as in LazyRowAdam

    def _params(self):
        return [p for g in self.param_groups for p in g["params"]]

    def flush(self):
        """The reference writes the state of GPU-cached hot rows of a host-RAM table back into the per-row state
        (row_optim.py:209-217); tables here live on the GPU whole and their state is always in the per-row tensors,
        so there is nothing to write back."""

    def state_dict(self):
        params = self._params()
        return {"format": "smlm.row_wise.v1", "kind": self.kind, "shapes": [list(p.shape) for p in params],
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups],
                "state": [dict(self.state[p]) for p in params]}

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
