"""Optimizer set-up for models that carry product-key (and Engram) value tables.

Interface of re133/sparse-memory-lm smlm/optim.py (build_optimizer, value_table_memory, lr_multiplier, set_lr,
clip_grads: same names, arguments, parameter-group names and order, state-dict layout), designed here around two
tables:

  * GROUPS (with _route) decides, for every trainable parameter, which optimizer and which named group it joins;
  * STATE_BYTES gives the persistent optimizer state a value table costs, per element and per row, for each
    (gradient kind, table optimizer, moment storage).

Dense parameters go to one fused AdamW; row-sparse value tables go to a table optimizer on the sm_100a kernels
(LazyRowAdam, or RowWiseOptimizer for value_optim "rowrms" / "rowadagrad"), one for the product-key tables and
one for the Engram tables (host-RAM tables under Adam get a HostLazyRowAdam of their own), returned together as
one OptimizerSet. Muon (optimizer="muon") is not part of this build and is refused.
"""
import math

import torch

from .sparse_values import LazyRowAdam, OptimizerSet, clip_row_sparse, row_sparse_tables

VALUE_STATES = ("fp32", "bf16", "int8")
VALUE_OPTIMS = ("adam", "rowrms", "rowadagrad")

# AdamW parameter groups, in the order the optimizer holds them (reference: optim.py:48-57):
# name -> (weight decay applies, learning rate source)
GROUPS = {
    "decay": (True, "lr"),
    "no_decay": (False, "lr"),
    "memory_values": (False, "value_lr"),          # product-key tables with dense gradients
    "engram_values": (False, "eng_value_lr"),      # Engram tables with dense gradients
}


def _route(p, row_sparse, engram):
    """The AdamW group of a trainable parameter, or None for a row-sparse table (it gets a table optimizer).
    row_sparse / engram: the ids of the row-sparse tables and of the Engram tables."""
    if id(p) in row_sparse:
        return None
    if getattr(p, "pk_value_param", False):
        return "engram_values" if id(p) in engram else "memory_values"
    if p.dim() >= 2 and not getattr(p, "no_weight_decay", False):
        return "decay"
    return "no_decay"


def _check_choices(value_state, value_optim, optimizer="adamw"):
    if value_state not in VALUE_STATES:
        raise ValueError(f"unknown value_state: {value_state}")
    if value_optim not in VALUE_OPTIMS:
        raise ValueError(f"unknown value_optim: {value_optim}")
    if value_optim != "adam" and value_state != "fp32":
        raise ValueError("value_state only applies to LazyRowAdam (value_optim=adam)")
    if optimizer != "adamw":
        raise ValueError(f"Unknown optimizer: {optimizer!r} (this build routes AdamW only)")


def build_optimizer(model, lr, value_lr, weight_decay, betas=(0.9, 0.95), eps=1e-8, eng_value_lr=None,
                    value_state="fp32", optimizer="adamw", value_optim="adam", value_copy_dtype=None,
                    capturable=False):
    """AdamW over the dense parameters (groups GROUPS, empty value groups left out) plus, when the model has
    row-sparse value tables, their table optimizers; returns the AdamW alone or an OptimizerSet
    (reference: optim.py:17-94). No counterpart in the reference: value_copy_dtype=torch.bfloat16 gives the
    product-key tables under LazyRowAdam a bf16 copy that the forward reads (values bf16 with an fp32 master);
    capturable=True builds both optimizers for a step captured in a CUDA graph (smlm_b200.graph_step)."""
    _check_choices(value_state, value_optim, optimizer)
    if (value_copy_dtype is not None or capturable) and value_optim != "adam":
        raise ValueError("value_copy_dtype / capturable need the LazyRowAdam table optimizer (value_optim='adam')")
    lrs = {"lr": lr, "value_lr": value_lr, "eng_value_lr": eng_value_lr or value_lr}
    tables = row_sparse_tables(model)
    row_sparse = {id(t) for t in tables}
    engram = {id(m.values.weight) for m in model.modules() if getattr(m, "is_engram", False)}
    members = {name: [] for name in GROUPS}
    for _, p in model.named_parameters():
        if p.requires_grad:
            name = _route(p, row_sparse, engram)
            if name is not None:
                members[name].append(p)
    if (members["memory_values"] or members["engram_values"]) and value_state != "fp32":
        raise ValueError("value_state requires row_sparse gradients for every trainable value table")
    groups = []
    for name, (decays, lr_key) in GROUPS.items():
        if name in ("decay", "no_decay") or members[name]:
            groups.append({"params": members[name], "weight_decay": weight_decay if decays else 0.0,
                           "base_lr": lrs[lr_key], "lr": lrs[lr_key], "name": name})
    on_gpu = all(p.is_cuda for g in groups for p in g["params"])
    dense = torch.optim.AdamW(groups, betas=betas, eps=eps, fused=on_gpu or None, capturable=capturable)
    if not tables:
        return dense
    table_opts = []
    for name, lr_key in (("memory_values", "value_lr"), ("engram_values", "eng_value_lr")):
        mine = [t for t in tables if (id(t) in engram) == (name == "engram_values")]
        if mine:
            copy = value_copy_dtype if name == "memory_values" else None
            table_opts += _table_optimizers(mine, lrs[lr_key], betas, eps, value_state, value_optim, name, copy,
                                            capturable)
    return OptimizerSet(dense, *table_opts)


def _table_optimizer(tables, lr, betas, eps, value_state, value_optim, name, value_copy_dtype=None,
                     capturable=False):
    if value_optim == "adam":
        return LazyRowAdam(tables, lr=lr, betas=betas, eps=eps, state_dtype=value_state, name=name,
                           value_copy_dtype=value_copy_dtype, capturable=capturable)
    from .row_optim import RowWiseOptimizer
    return RowWiseOptimizer(tables, lr=lr, kind=value_optim, beta2=betas[1], eps=eps, name=name)


def _table_optimizers(tables, lr, betas, eps, value_state, value_optim, name, value_copy_dtype, capturable):
    """The table optimizer(s) of one group of row-sparse tables: host-RAM tables under Adam get a HostLazyRowAdam
    of their own, the rest (and every table under a row-wise optimizer) one optimizer (reference: optim.py:66-90)."""
    host = [t for t in tables if getattr(t, "host_values", False)]
    rest = [t for t in tables if not getattr(t, "host_values", False)]
    out = []
    if host and value_optim == "adam":
        if value_copy_dtype is not None or capturable:
            raise ValueError("value_copy_dtype / capturable do not apply to host-RAM tables")
        from .host_optim import HostLazyRowAdam
        out.append(HostLazyRowAdam(host, lr=lr, betas=betas, eps=eps, state_dtype=value_state, name=name))
    else:
        rest = tables
    if rest:
        out.append(_table_optimizer(rest, lr, betas, eps, value_state, value_optim, name, value_copy_dtype,
                                    capturable))
    return out


# Persistent optimizer state of one trainable value table, by (gradient kind, table optimizer, moment storage):
# (moment bytes per element, moment bytes per row, scale bytes per row); `size` is the table's element size.
# Dense-gradient tables live in AdamW whatever value_optim says; the row-wise optimizers keep one (rowadagrad) or
# two (rowrms) fp32 numbers per row and ignore value_state. Step counters (4 bytes per table) are counted apart.
STATE_BYTES = {
    ("dense", "adamw", "fp32"): lambda size: (2 * size, 0, 0),
    ("row_sparse", "adam", "fp32"): lambda size: (2 * size, 0, 0),
    ("row_sparse", "adam", "bf16"): lambda size: (4, 0, 0),
    ("row_sparse", "adam", "int8"): lambda size: (2, 0, 8),
    ("row_sparse", "rowrms", "fp32"): lambda size: (0, 8, 0),
    ("row_sparse", "rowadagrad", "fp32"): lambda size: (0, 4, 0),
}


def _state_key(sparse, value_optim, value_state):
    if not sparse:
        return "dense", "adamw", "fp32"
    return "row_sparse", value_optim, value_state if value_optim == "adam" else "fp32"


def value_table_memory(model, value_state="fp32", *, host=None, value_optim="adam"):
    """Persistent bytes of the value tables once their optimizers are set up: the tables, their gradients (the
    fp32 row-sparse accumulator, or .grad), optimizer moments and row scales, touched masks and step counters,
    and the total (reference: optim.py:97-137). host selects host-RAM (True) or device (False) tables only."""
    if value_state not in VALUE_STATES:
        raise ValueError(f"unknown value_state: {value_state}")
    row_sparse = {id(t) for t in row_sparse_tables(model)}
    parts = ("table_bytes", "gradient_bytes", "moment_bytes", "scale_bytes", "touched_bytes", "step_bytes")
    out = dict.fromkeys(parts, 0)
    for p in model.parameters():
        if not getattr(p, "pk_value_param", False):
            continue
        if host is not None and bool(getattr(p, "host_values", False)) != host:
            continue
        n, size, rows = p.numel(), p.element_size(), p.shape[0]
        out["table_bytes"] += n * size
        if not p.requires_grad:
            continue
        sparse = id(p) in row_sparse
        if value_state != "fp32" and not sparse:
            raise ValueError(f"value_state {value_state!r} needs row-sparse gradients on every trainable value table")
        if value_state != "fp32" and p.dtype != torch.float32:
            raise ValueError(f"value_state {value_state!r} needs fp32 value tables")
        per_element, per_row, scales_per_row = STATE_BYTES[_state_key(sparse, value_optim, value_state)](size)
        out["gradient_bytes"] += n * (max(4, size) if sparse else size)
        out["moment_bytes"] += n * per_element + rows * per_row
        out["scale_bytes"] += rows * scales_per_row
        out["touched_bytes"] += rows if sparse else 0
        out["step_bytes"] += 4
    out["total_bytes"] = sum(out[k] for k in parts)
    return out


def lr_multiplier(step, total_steps, warmup_steps, min_ratio):
    """Learning-rate factor at `step`: a linear ramp over the warmup steps, then a half cosine from 1 down to
    min_ratio at total_steps, held there after (reference: optim.py:140-145)."""
    if step < warmup_steps:
        return (step + 1) / warmup_steps
    progress = min(1.0, (step - warmup_steps) / max(1, total_steps - warmup_steps))
    half_cosine = 0.5 * (1 + math.cos(math.pi * progress))      # 1 -> 0; the halving is exact
    return min_ratio + (1 - min_ratio) * half_cosine


def set_lr(opt, mult):
    """Every group at its base learning rate times mult."""
    for g in opt.param_groups:
        g["lr"] = g["base_lr"] * mult


def clip_grads(model, max_norm):
    """Two separate clips, each to max_norm: the value tables (dense .grad by torch's clip, row-sparse tables by
    their accumulated rows' global norm, applied in their optimizer step) and everything else. Returns the
    pre-clip norms (rest, values); values is None without a trainable table (reference: optim.py:153-162)."""
    with_grad = [p for p in model.parameters() if p.grad is not None]
    dense_tables = [p for p in with_grad if getattr(p, "pk_value_param", False)]
    others = [p for p in with_grad if not getattr(p, "pk_value_param", False)]
    values_norm = None
    if dense_tables:
        values_norm = torch.nn.utils.clip_grad_norm_(dense_tables, max_norm, foreach=True)
    sparse_tables = row_sparse_tables(model)
    if sparse_tables:
        values_norm = clip_row_sparse(sparse_tables, max_norm)
    return torch.nn.utils.clip_grad_norm_(others, max_norm, foreach=True), values_norm
