"""Row store and lazy Adam of value tables in host RAM (reference: re133/sparse-memory-lm smlm/host_optim.py; same
entry points: HostRowStore, HostLazyRowAdam, value_table_memory_by_device).

The reference updates the touched rows with a multithreaded C loop on the host (smlm/host_rows.c). Here the
accumulator, the touched mask, the table and the moments are mapped host memory (host_values.mapped) and the
library's own optimizer kernels update the touched rows in place over the host link: smlm_lazy_adam_step (the
reference's C loop's operation order, bit for bit) and smlm_lazy_adam_lowmem_step for bf16 / int8 moments. Each step
synchronises its stream before returning, so CPU code sees the updated rows.
"""
import math

import torch

from . import _lib as L
from .host_values import mapped
from .sparse_values import LazyRowAdam, row_store


class HostRowStore:
    """The gradient store of a host table (reference: host_optim.py:78-107): `acc` (fp32, shaped like the table)
    and `touched` in host RAM, the deferred clip factor `grad_scale`, and `hot` (the table's HOT rows, which keep
    their own accumulator on the GPU). The optimizer steps leave the stepped rows' accumulator values in place (a
    step's first add overwrites them, `smlm_host_rows_add`), so the array itself (`_acc`) holds stale rows wherever
    `touched` is 0; reading `acc` zeroes those first, as the reference's store always has them. `row_sq` (no
    counterpart): the touched rows' squared norms on the GPU, written by HostEmbedding.accumulate's add kernel, so
    norm() does not read the accumulator rows back over the host link; code that writes the accumulator by other
    means sets it to None (norm() then reads the rows)."""

    def __init__(self, table):
        if table.device.type != "cpu":
            raise ValueError("host value tables must stay on the CPU")
        self._acc = torch.zeros(table.shape, dtype=torch.float32)
        self.touched = torch.zeros(table.shape[0], dtype=torch.bool)
        self.stale = False                 # rows with touched == 0 may hold old values in _acc
        self.grad_scale = 1.0
        self.hot = getattr(table, "hot_rows", None)
        self.row_sq = None

    @property
    def acc(self):
        if self.stale:
            self._acc[~self.touched] = 0.0
            self.stale = False
        return self._acc

    def sq_buffer(self, device):
        """The device array of per-row squared norms (created on first use)."""
        if self.row_sq is None or self.row_sq.device != device:
            self.row_sq = torch.empty(self._acc.shape[0], dtype=torch.float32, device=device)
        return self.row_sq

    def sync(self):
        pass

    def reset(self, rows=None):
        """Drops the touched rows' gradients (their values stay in `_acc`, stale)."""
        if rows is None:
            rows = self.touched.nonzero().squeeze(1)
            if self.hot is not None:
                self.hot.acc.zero_()
                self.hot.touched.zero_()
        self.touched.index_fill_(0, rows, False)
        self.stale = True
        self.grad_scale = 1.0

    def norm(self, device=None):
        """The accumulator's L2 norm over the touched rows (and the HOT rows'), as a device fp32 scalar, computed
        by the touched-norm kernel from the rows' squared norms on the GPU (or over the mapped accumulator)."""
        if device is None:
            if self.row_sq is not None:
                device = self.row_sq.device
            elif self.hot is not None:
                device = self.hot.acc.device
            else:
                device = torch.device("cuda", torch.cuda.current_device())
        rows, d = self._acc.shape
        sq = self.row_sq if self.row_sq is not None and self.row_sq.device == device else None
        out = torch.empty((), dtype=torch.float32, device=device)
        ws = L.workspace(L.lib().smlm_touched_workspace(rows), device)
        with torch.cuda.device(device):
            rc = L.lib().smlm_touched_norm(mapped(self._acc) if sq is None else None, L.ptr(sq), mapped(self.touched),
                                           rows, d, L.ptr(out), L.ptr(ws), ws.numel(), L.stream(device))
        L.check(rc, "touched_norm")
        if self.hot is not None:
            out = torch.linalg.vector_norm(torch.stack([out, self.hot.acc.norm()]))
        return out


def _scale_args(scale, device):
    """(device pointer or None, float, tensor kept alive) of a clip factor given as a float or a 0-d tensor."""
    if torch.is_tensor(scale):
        t = scale.detach().to(device=device, dtype=torch.float32).reshape(1).contiguous()
        return L.ptr(t), 1.0, t
    return None, float(scale), None


class HostLazyRowAdam(LazyRowAdam):
    """LazyRowAdam on host tables (reference: host_optim.py:110-169): the touched rows' Adam in place in host RAM,
    by the library's kernels over mapped memory; fp32, bf16 or int8 moments (state on the host, like the table).
    Hot rows and GACC need a row-wise optimizer, as in the reference."""

    def __init__(self, params, lr, betas=(0.9, 0.95), eps=1e-8, name="memory_values", impl="cuda",
                 state_dtype="fp32", device=None):
        params = list(params)
        if any(p.device.type != "cpu" or p.dtype != torch.float32 or p.ndim != 2 or not p.is_contiguous()
               or p.shape[1] == 0 for p in params):
            raise ValueError("HostLazyRowAdam requires contiguous CPU fp32 tables with nonzero width")
        if state_dtype not in ("fp32", "bf16", "int8"):
            raise ValueError(f"unknown state_dtype: {state_dtype}")
        if not 0 <= lr or not 0 <= eps or not all(0 <= b < 1 for b in betas):
            raise ValueError("invalid LazyRowAdam learning rate, epsilon or betas")
        torch.optim.Optimizer.__init__(self, params, dict(lr=lr, betas=betas, eps=eps, weight_decay=0.0))
        for g in self.param_groups:
            g["name"] = name
            g["base_lr"] = lr
        self.impl = "cuda"
        self.state_dtype = state_dtype
        self.value_copy_dtype = None
        self.capturable = False
        self._scal = {}
        self.device = device

    def _device(self):
        return self.device if self.device is not None else torch.device("cuda", torch.cuda.current_device())

    @torch.no_grad()
    def step(self):
        dev = self._device()
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                st = row_store(p)
                if getattr(st, "hot", None) is not None or getattr(st, "steprows", None) is not None:
                    raise ValueError("hot rows and GACC need a row-wise table optimizer (value_optim)")
                if not bool(st.touched.any()):
                    continue
                state = self._state(p)
                state["step"] += 1
                step = int(state["step"])
                sp, sf, keep = _scale_args(st.grad_scale, dev)
                rows, d = p.shape
                ws = L.workspace(L.lib().smlm_touched_workspace(rows), dev)
                with torch.cuda.device(dev):
                    if self.state_dtype == "fp32":
                        bc1 = 1 - b1 ** step
                        rc = L.lib().smlm_lazy_adam_step(
                            mapped(p.detach()), mapped(state["exp_avg"]), mapped(state["exp_avg_sq"]), mapped(st._acc),
                            mapped(st.touched), sp, sf, rows, d, 1 - b1, b2, 1 - b2, math.sqrt(1 - b2 ** step),
                            group["eps"], -(group["lr"] / bc1), None, L.F32, L.STEP_KEEP_ACC, L.ptr(ws), ws.numel(),
                            L.stream(dev))
                    else:
                        int8 = self.state_dtype == "int8"
                        rc = L.lib().smlm_lazy_adam_lowmem_step(
                            mapped(p.detach()), mapped(state["exp_avg"]), mapped(state["exp_avg_sq"]),
                            mapped(state["exp_avg_scale"]) if int8 else None,
                            mapped(state["exp_avg_sq_scale"]) if int8 else None, L.I8 if int8 else L.BF16,
                            mapped(st._acc), mapped(st.touched), sp, sf, rows, d, b1, b2, 1 - b1, 1 - b2, group["eps"],
                            group["lr"] / (1 - b1 ** step), math.sqrt(1 - b2 ** step), None, L.F32, L.STEP_KEEP_ACC,
                            L.ptr(ws), ws.numel(), L.stream(dev))
                    L.check(rc, "host lazy Adam step")
                    torch.cuda.current_stream(dev).synchronize()
                del keep
                st.grad_scale = 1.0         # the kernel cleared the marks and left the rows' values (stale now)
                st.stale = True


def value_table_memory_by_device(model, value_state="fp32", value_optim="adam"):
    """Persistent table bytes split by where the tables live (reference: host_optim.py:172-176)."""
    from .optim import value_table_memory
    return {"host": value_table_memory(model, value_state, host=True, value_optim=value_optim),
            "device": value_table_memory(model, value_state, host=False, value_optim=value_optim)}
