"""Checkpoints of a model whose value table is row-sharded, in the unsharded layout.

With ProductKeyMemory(shard_group=...) each rank holds its contiguous rows of the value table and of that table's
optimizer state (smlm_b200.sharded.RowShard). The reference trains on one process and checkpoints
model.state_dict() and opt.state_dict() (smlm/train.py:580-596, format smlm.train_ckpt.v1; table optimizer formats
smlm.lazy_row_adam.v1, smlm/sparse_values.py:324-332, and smlm.row_wise.v1, smlm/row_optim.py:219-226). This module
keeps those files interchangeable:

  save  unsharded_model_state / unsharded_optimizer_state gather every rank's rows onto one rank of the shard group
        (`dst`), in row order, into CPU tensors shaped as the unsharded model's: exactly the state dicts a
        one-process run writes, so one GPU (or the reference) loads them.
  load  load_unsharded_model_state / load_unsharded_optimizer_state cut a full state dict down to this rank's rows.
        No collective: every rank may read the same file memory-mapped (torch.load(..., mmap=True)), as the
        reference resumes (smlm/train.py:441-442), and only its own rows are ever copied.

Per-row optimizer state: in a table's state every tensor entry other than "step" with at least one dimension holds
one entry per table row along dimension 0 (Adam moments; the int8 form's row scales; the row-wise v and n). The
gather moves rows as raw bytes, so every dtype (fp32, bf16, int8, uint8, int32) passes unchanged, through NCCL or
gloo alike. Saving is collective over the shard group: every rank calls it with the same model and optimizer
structure (checked first, so a mismatch raises on every rank instead of leaving some waiting). Call it between
steps: rows a backward accumulated since the last optimizer step are not part of any checkpoint (as in the
reference).
"""
import math

import torch
import torch.distributed as dist

from .sharded import RowShard

LAZY_ADAM, ROW_WISE, OPT_SET = "smlm.lazy_row_adam.v1", "smlm.row_wise.v1", "smlm.optimizer_set.v1"
CHUNK_BYTES = 64 << 20            # rows moved per rank and gather round, at most


def _global(group, rank):
    return dist.get_global_rank(group, rank) if group is not None else rank


def gather_rows(local, shard, group=None, dst=0, chunk_bytes=CHUNK_BYTES):
    """The full (shard.rows, ...) tensor on the CPU of rank `dst` of `group`, assembled in row order from every
    rank's rows `local` (shard.count rows; trailing shape and dtype the same on every rank); None on the other
    ranks. Collective over `group`; moves at most about `chunk_bytes` per rank per round, so the device holds one
    round's rows of every rank at a time."""
    if local.shape[0] != shard.count:
        raise ValueError(f"gather_rows: {local.shape[0]} local rows, the shard holds {shard.count}")
    tail = tuple(local.shape[1:])
    row_bytes = local.element_size() * math.prod(tail)
    is_dst = shard.rank == dst
    if row_bytes == 0:
        return torch.empty((shard.rows,) + tail, dtype=local.dtype) if is_dst else None
    flat = local.detach().contiguous().reshape(shard.count, math.prod(tail)).view(torch.uint8)  # (count, row_bytes)
    full = torch.empty(shard.rows, row_bytes, dtype=torch.uint8) if is_dst else None
    owners = [RowShard(shard.rows, shard.world, r) for r in range(shard.world)]
    step = max(1, chunk_bytes // row_bytes)
    for c0 in range(0, shard.per, step):
        m = min(step, shard.per - c0)
        buf = torch.zeros(m, row_bytes, dtype=torch.uint8, device=local.device)
        n = max(0, min(m, shard.count - c0))
        if n:
            buf[:n].copy_(flat[c0:c0 + n])
        parts = [torch.empty_like(buf) for _ in range(shard.world)] if is_dst else None
        dist.gather(buf, parts, dst=_global(group, dst), group=group)
        if is_dst:
            for o, part in zip(owners, parts):
                n_o = max(0, min(m, o.count - c0))
                if n_o:
                    full[o.base + c0:o.base + c0 + n_o].copy_(part[:n_o])
    if not is_dst:
        return None
    return full.view(local.dtype).reshape((shard.rows,) + tail)


def _sharded_of(tensors):
    """(shard, group) shared by the row-sharded tensors among `tensors` (None, None when there are none)."""
    found = None
    for t in tensors:
        shard = getattr(t, "row_shard", None)
        if shard is None:
            continue
        key = (shard.world, shard.rank, id(getattr(t, "shard_group", None)))
        if found is not None and found[2] != key:
            raise ValueError("row-sharded tables of one model must share one shard group")
        found = (shard, getattr(t, "shard_group", None), key)
    return (None, None) if found is None else found[:2]


def _check_same(struct, group, what):
    """Every rank of `group` holds the same structure (one small all-gather); raises ValueError on all ranks
    otherwise."""
    world = dist.get_world_size(group)
    every = [None] * world
    dist.all_gather_object(every, struct, group=group)
    if any(s != every[0] for s in every):
        bad = [r for r, s in enumerate(every) if s != every[0]]
        raise ValueError(f"{what} differs between the ranks of the shard group (ranks {bad} vs rank 0)")


def _row_entry(key, value):
    return key != "step" and torch.is_tensor(value) and value.ndim >= 1


# ---------------------------------------------------------------------------------------------------- model state


def unsharded_model_state(model, dst=0, chunk_bytes=CHUNK_BYTES):
    """model.state_dict() as the unsharded model's, on rank `dst` of the tables' shard group (CPU tensors; every
    row-sharded table gathered in full); None on the other ranks. Collective over the shard group. A model
    without row-sharded tables returns its own state dict (on the CPU) on every rank."""
    sd = model.state_dict(keep_vars=True)
    shard, group = _sharded_of(sd.values())
    if shard is None:
        return {k: v.detach().cpu() for k, v in sd.items()}
    _check_same([(k, tuple(v.shape[1:]) if getattr(v, "row_shard", None) is not None else tuple(v.shape),
                  str(v.dtype)) for k, v in sd.items()], group, "model structure")
    is_dst = shard.rank == dst
    out, done = ({} if is_dst else None), {}
    for k, v in sd.items():
        if getattr(v, "row_shard", None) is not None:
            if id(v) not in done:                    # a table under several keys (tied) is gathered once
                done[id(v)] = gather_rows(v.detach(), v.row_shard, group, dst, chunk_bytes)
            full = done[id(v)]
        else:
            full = v.detach().cpu() if is_dst else None
        if is_dst:
            out[k] = full
    return out


def shard_model_state(model, full_state):
    """A full (unsharded) state dict cut down to this rank's rows of every row-sharded table (views; no copy, no
    collective)."""
    own = model.state_dict(keep_vars=True)
    local = {}
    for k, v in full_state.items():
        p = own.get(k)
        shard = getattr(p, "row_shard", None) if p is not None else None
        if shard is not None:
            if v.shape[0] != shard.rows or tuple(v.shape[1:]) != tuple(p.shape[1:]):
                raise ValueError(f"{k}: saved shape {tuple(v.shape)}, the unsharded table is "
                                 f"{(shard.rows,) + tuple(p.shape[1:])}")
            v = shard.take(v)
        local[k] = v
    return local


def load_unsharded_model_state(model, full_state, strict=True):
    """model.load_state_dict of a full (unsharded) state dict: each rank copies its own rows only."""
    return model.load_state_dict(shard_model_state(model, full_state), strict=strict)


# ------------------------------------------------------------------------------------------------ optimizer state


def _params(opt):
    return [p for g in opt.param_groups for p in g["params"]]


def _table_entries(sd, params):
    """[(param, state dict of that param or None, saved-state key)] of an optimizer state dict in any of the
    three layouts: smlm.lazy_row_adam.v1 / smlm.row_wise.v1 (state: a list in parameter order) or torch's (state:
    a dict keyed by parameter position)."""
    st = sd["state"]
    if isinstance(st, list):
        return [(p, st[i] if i < len(st) else None, i) for i, p in enumerate(params)]
    return [(p, st.get(i), i) for i, p in enumerate(params)]


def _structure(sd, params):
    out = []
    for p, st, i in _table_entries(sd, params):
        sharded = getattr(p, "row_shard", None) is not None
        ent = sorted((k, str(v.dtype) if torch.is_tensor(v) else type(v).__name__,
                      tuple(v.shape[1:]) if sharded and _row_entry(k, v) else
                      (tuple(v.shape) if torch.is_tensor(v) else None))
                     for k, v in (st or {}).items())
        out.append((i, sharded, ent))
    return out


def unshard_optimizer_state(sd, params, dst=0, chunk_bytes=CHUNK_BYTES):
    """An optimizer state dict `sd` over `params` (the optimizer's parameters in param_groups order) as the
    unsharded optimizer's: every row-sharded table's per-row state gathered in full and its saved shape made the
    full table's (smlm.lazy_row_adam.v1 / smlm.row_wise.v1 "shapes"), on rank `dst` of the shard group (CPU
    tensors); None on the other ranks. Collective over the shard group. Replicated state is rank dst's own."""
    if sd.get("format") == OPT_SET:
        raise ValueError("unshard_optimizer_state takes one optimizer's state; use unsharded_optimizer_state for an "
                         "OptimizerSet")
    shard, group = _sharded_of(params)
    if shard is None:
        return sd
    _check_same(_structure(sd, params), group, "optimizer state")
    is_dst = shard.rank == dst
    entries = _table_entries(sd, params)
    states = []
    for p, st, i in entries:
        pshard = getattr(p, "row_shard", None)
        new = None if st is None else {}
        for k, v in (st or {}).items():
            if pshard is not None and _row_entry(k, v):
                if v.shape[0] != pshard.count:
                    raise ValueError(f"optimizer state {k!r} of a row-sharded table has {v.shape[0]} rows, the "
                                     f"shard holds {pshard.count}")
                v = gather_rows(v, pshard, group, dst, chunk_bytes)
            elif torch.is_tensor(v):
                v = v.detach().cpu() if is_dst else None
            if is_dst:
                new[k] = v
        states.append(new)
    if not is_dst:
        return None
    out = dict(sd)
    if isinstance(sd["state"], list):
        out["state"] = states
    else:
        out["state"] = {i: s for (_, _, i), s in zip(entries, states) if s is not None}
    if "shapes" in sd:
        out["shapes"] = [[p.row_shard.rows] + list(p.shape[1:]) if getattr(p, "row_shard", None) is not None
                         else list(s) for p, s in zip(params, sd["shapes"])]
    return out


def shard_optimizer_state(sd, params):
    """A full (unsharded) optimizer state dict over `params` cut down to this rank's rows (views; no collective);
    the inverse of unshard_optimizer_state."""
    if sd.get("format") == OPT_SET:
        raise ValueError("shard_optimizer_state takes one optimizer's state; use load_unsharded_optimizer_state "
                         "for an OptimizerSet")
    if _sharded_of(params)[0] is None:
        return sd
    entries = _table_entries(sd, params)
    if "shapes" in sd:
        for p, s in zip(params, sd["shapes"]):
            shard = getattr(p, "row_shard", None)
            want = [shard.rows if shard is not None else p.shape[0]] + list(p.shape[1:])
            if list(s) != want:
                raise ValueError(f"optimizer state saved for a table of shape {list(s)}, the unsharded table is "
                                 f"{want}")
    states = []
    for p, st, i in entries:
        shard = getattr(p, "row_shard", None)
        if st is None or shard is None:
            states.append(st)
            continue
        new = {}
        for k, v in st.items():
            if _row_entry(k, v):
                if v.shape[0] != shard.rows:
                    raise ValueError(f"optimizer state {k!r} has {v.shape[0]} rows, the unsharded table {shard.rows}")
                v = shard.take(v)
            new[k] = v
        states.append(new)
    out = dict(sd)
    if isinstance(sd["state"], list):
        out["state"] = states
    else:
        out["state"] = {i: s for (_, _, i), s in zip(entries, states) if s is not None}
    if "shapes" in sd:
        out["shapes"] = [list(p.shape) for p in params]
    return out


def unsharded_optimizer_state(opt, dst=0, chunk_bytes=CHUNK_BYTES):
    """opt.state_dict() as the unsharded optimizer's (LazyRowAdam, RowWiseOptimizer, torch optimizers, or an
    OptimizerSet of them), on rank `dst` of the shard group; None on the other ranks. Collective."""
    sd = opt.state_dict()
    if sd.get("format") == OPT_SET:
        parts = [unshard_optimizer_state(s["state_dict"], _params(o), dst, chunk_bytes)
                 for o, s in zip(opt.opts, sd["optimizers"])]
        shard, _ = _sharded_of(p for o in opt.opts for p in _params(o))
        if shard is not None and shard.rank != dst:
            return None
        return {"format": OPT_SET, "optimizers": [{"type": s["type"], "state_dict": part}
                                                  for s, part in zip(sd["optimizers"], parts)]}
    return unshard_optimizer_state(sd, _params(opt), dst, chunk_bytes)


def load_unsharded_optimizer_state(opt, full_state):
    """opt.load_state_dict of a full (unsharded) optimizer state dict: each rank takes its own rows only."""
    if full_state.get("format") == OPT_SET:
        if not hasattr(opt, "opts") or len(opt.opts) != len(full_state["optimizers"]):
            raise ValueError("the saved OptimizerSet holds another number of optimizers")
        local = {"format": OPT_SET, "optimizers": [
            {"type": s["type"], "state_dict": shard_optimizer_state(s["state_dict"], _params(o))}
            for o, s in zip(opt.opts, full_state["optimizers"])]}
        return opt.load_state_dict(local)
    return opt.load_state_dict(shard_optimizer_state(full_state, _params(opt)))
