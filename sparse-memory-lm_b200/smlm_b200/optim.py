"""Optimizer routing for models with product-key value tables (reference: re133/sparse-memory-lm smlm/optim.py).

AdamW (fused) for the dense parameters; row-sparse value tables get a LazyRowAdam (or a RowWiseOptimizer with
value_optim="rowrms" / "rowadagrad") on the sm_100a kernels; both are returned as one OptimizerSet. Clipping is
split: the tables by their own global norm (deferred into the table step), the rest by torch's clip.
"""
import math

import torch

from .sparse_values import LazyRowAdam, OptimizerSet, clip_row_sparse, row_sparse_tables


def build_optimizer(model, lr, value_lr, weight_decay, betas=(0.9, 0.95), eps=1e-8, eng_value_lr=None,
                    value_state="fp32", optimizer="adamw", value_optim="adam"):
    """Same routing as the reference (optim.py:17-94)."""
    if value_state not in ("fp32", "bf16", "int8"):
        raise ValueError(f"unknown value_state: {value_state}")
    if value_optim not in ("adam", "rowrms", "rowadagrad"):
        raise ValueError(f"unknown value_optim: {value_optim}")
    if value_optim != "adam" and value_state != "fp32":
        raise ValueError("value_state only applies to LazyRowAdam (value_optim=adam)")
    if optimizer != "adamw":
        raise ValueError(f"Unknown optimizer: {optimizer!r} (this build routes AdamW only)")
    sparse_tables = row_sparse_tables(model)
    sparse_ids = {id(t) for t in sparse_tables}
    engram_ids = {id(m.values.weight) for m in model.modules() if getattr(m, "is_engram", False)}
    decay, no_decay, values, eng_values = [], [], [], []
    for n, p in model.named_parameters():
        if not p.requires_grad or id(p) in sparse_ids:
            continue
        if getattr(p, "pk_value_param", False):
            (eng_values if id(p) in engram_ids else values).append(p)
        elif p.dim() >= 2 and not getattr(p, "no_weight_decay", False):
            decay.append(p)
        else:
            no_decay.append(p)
    if (values or eng_values) and value_state != "fp32":
        raise ValueError("value_state requires row_sparse gradients for every trainable value table")
    groups = [
        {"params": decay, "weight_decay": weight_decay, "base_lr": lr, "name": "decay"},
        {"params": no_decay, "weight_decay": 0.0, "base_lr": lr, "name": "no_decay"},
    ]
    if values:
        groups.append({"params": values, "weight_decay": 0.0, "base_lr": value_lr, "name": "memory_values"})
    if eng_values:                  # dense Engram tables (eng_value_grad="dense"): their own learning rate
        groups.append({"params": eng_values, "weight_decay": 0.0, "base_lr": eng_value_lr or value_lr,
                       "name": "engram_values"})
    for g in groups:
        g["lr"] = g["base_lr"]
    fused = all(p.is_cuda for g in groups for p in g["params"]) or None
    opt = torch.optim.AdamW(groups, betas=betas, eps=eps, fused=fused)
    if sparse_tables:
        # one table optimizer for the product-key table(s), one for the Engram tables (learning rate
        # eng_value_lr, default value_lr); clipping stays one global norm over all of them (clip_grads)
        owners = {id(m.values.weight): m for m in model.modules() if getattr(m, "value_grad", None) == "row_sparse"}
        lazy = []
        for engram in (False, True):
            tabs = [t for t in sparse_tables if getattr(owners[id(t)], "is_engram", False) == engram]
            if not tabs:
                continue
            tlr = (eng_value_lr or value_lr) if engram else value_lr
            name = "engram_values" if engram else "memory_values"
            if value_optim != "adam":
                from .row_optim import RowWiseOptimizer
                lazy.append(RowWiseOptimizer(tabs, lr=tlr, kind=value_optim, beta2=betas[1], eps=eps, name=name))
            else:
                lazy.append(LazyRowAdam(tabs, lr=tlr, betas=betas, eps=eps, state_dtype=value_state, name=name))
        return OptimizerSet(opt, *lazy)
    return opt


def value_table_memory(model, value_state="fp32", *, host=None, value_optim="adam"):
    """Persistent table tensors after optimizer initialisation (reference: optim.py:97-137)."""
    if value_state not in ("fp32", "bf16", "int8"):
        raise ValueError(f"unknown value_state: {value_state}")
    sparse_ids = {id(t) for t in row_sparse_tables(model)}
    out = dict(table_bytes=0, gradient_bytes=0, moment_bytes=0, scale_bytes=0, touched_bytes=0, step_bytes=0)
    for p in model.parameters():
        if not getattr(p, "pk_value_param", False):
            continue
        if host is not None and bool(getattr(p, "host_values", False)) != host:
            continue
        n, size = p.numel(), p.element_size()
        out["table_bytes"] += n * size
        if not p.requires_grad:
            continue
        sparse = id(p) in sparse_ids
        # compact moments exist only for row-sparse fp32 tables (LazyRowAdam(state_dtype=...)): refused otherwise
        if value_state != "fp32" and not sparse:
            raise ValueError(f"value_state {value_state!r} needs row-sparse gradients on every trainable value table")
        if value_state != "fp32" and p.dtype != torch.float32:
            raise ValueError(f"value_state {value_state!r} needs fp32 value tables")
        out["gradient_bytes"] += n * (max(4, size) if sparse else size)
        if sparse and value_optim != "adam":
            from .row_optim import state_bytes
            out["moment_bytes"] += state_bytes(value_optim, p.shape[0]) - 4
        elif sparse and value_state == "bf16":
            out["moment_bytes"] += n * 4
        elif sparse and value_state == "int8":
            out["moment_bytes"] += n * 2
            out["scale_bytes"] += p.shape[0] * 8
        else:
            out["moment_bytes"] += n * 2 * size
        out["touched_bytes"] += p.shape[0] if sparse else 0
        out["step_bytes"] += 4
    out["total_bytes"] = sum(out.values())
    return out


def lr_multiplier(step, total_steps, warmup_steps, min_ratio):
    """Linear warmup, then cosine decay to min_ratio (reference: optim.py:140-145)."""
    if step < warmup_steps:
        return (step + 1) / warmup_steps
    s = min(1.0, (step - warmup_steps) / max(1, total_steps - warmup_steps))
    return min_ratio + 0.5 * (1 - min_ratio) * (1 + math.cos(math.pi * s))


def set_lr(opt, mult):
    for g in opt.param_groups:
        g["lr"] = g["base_lr"] * mult


def clip_grads(model, max_norm):
    """Clip memory values and the rest separately; return the (pre-clip) norm of the rest and of the values
    (reference: optim.py:153-162)."""
    values = [p for p in model.parameters() if getattr(p, "pk_value_param", False) and p.grad is not None]
    rest = [p for p in model.parameters() if not getattr(p, "pk_value_param", False) and p.grad is not None]
    vnorm = torch.nn.utils.clip_grad_norm_(values, max_norm, foreach=True) if values else None
    sparse_tables = row_sparse_tables(model)
    if sparse_tables:
        vnorm = clip_row_sparse(sparse_tables, max_norm)
    norm = torch.nn.utils.clip_grad_norm_(rest, max_norm, foreach=True)
    return norm, vnorm
