"""Engram-style n-gram memory (reference: re133/sparse-memory-lm smlm/engram.py) on the sm_100a kernels.

Same constructor arguments, buffers, parameters, initialisation and forward as the reference's NgramHash and
EngramMemory (after Cheng et al. 2026, "Conditional Memory via Scalable Lookup", section 2): each position looks
up n_lookups = len(orders) x heads rows of head_dim, one per hash head of every n-gram order (the hash of its last
n compressed tokens), gates them with the hidden state and adds a short depthwise causal convolution. On this build
  * the hash is one CUDA kernel (kernels.ngram_rows), with the integer results of the reference's tensor chain;
  * the row lookups are the value bag with one lookup per bag, so their row-sparse gradients and the table's lazy
    Adam are the product-key table's kernels (row_sparse_embedding_bag, LazyRowAdam) for value_grad="row_sparse";
  * the gating, norms and convolution stay PyTorch modules (dense host code).
Token compression (canonical_ids) needs the GPT-2 vocabulary, read through tiktoken as in the reference.
"""
import math
import unicodedata

import torch
import torch.nn.functional as F
from torch import nn

from . import kernels as K
from .sparse_values import row_sparse_embedding_bag

IMPLS = ("cuda", "triton", "torch")


def canonical_ids(vocab_size):
    """GPT-2 token id -> id of its NFKC-normalised, lower-cased string (reference: engram.py:23-41). A token whose
    bytes are not valid UTF-8 alone keeps its bytes as its key; ids past the tokenizer (vocabulary padding) keep
    their own. Returns (int64 tensor of vocab_size ids, number of distinct ids)."""
    import tiktoken
    enc = tiktoken.get_encoding("gpt2")
    index, ids = {}, []
    for i in range(vocab_size):
        if i >= enc.n_vocab:
            key = ("pad", i)
        else:
            raw = enc.decode_single_token_bytes(i)
            try:
                key = ("s", unicodedata.normalize("NFKC", raw.decode("utf-8")).lower())
            except UnicodeDecodeError:
                key = ("b", raw)
        if key not in index:
            index[key] = len(index)
        ids.append(index[key])
    return torch.tensor(ids, dtype=torch.int64), len(index)


class NgramHash(nn.Module):
    """Row indices of all hash heads for every position (reference: engram.py:44-75). One set of indices serves
    every Engram module of a model; each module has its own tables."""

    def __init__(self, vocab_size, orders=(2, 3), heads=8, rows=524287, seed=0, canon=None):
        """canon (no counterpart in the reference): the token compression as (int64 ids of vocab_size entries,
        number of distinct ids), for callers that bring their own table or feed already-compressed ids (the
        identity map); by default it is computed from the GPT-2 vocabulary as the reference does."""
        super().__init__()
        canon, n_canon = canonical_ids(vocab_size) if canon is None else canon
        canon = torch.as_tensor(canon, dtype=torch.int64)
        if canon.shape != (vocab_size,) or not 0 < int(n_canon) < 2 ** 16:
            raise ValueError(f"canon must map {vocab_size} token ids to fewer than 65,536 compressed ids")
        self.register_buffer("canon", canon, persistent=False)
        self.pad = n_canon                                   # compressed id of the positions before a sequence
        self.orders, self.heads, self.rows = list(orders), heads, rows
        self.history = max(orders) - 1
        # the reference's multipliers (same generator, shape and draw): odd, below 2^31, so that an id (< 2^16)
        # times a multiplier stays below 2^47 and nothing overflows int64
        g = torch.Generator().manual_seed(seed)
        mult = torch.randint(0, 2 ** 30, (len(self.orders), heads, max(orders)), generator=g) * 2 + 1
        self.register_buffer("mult", mult, persistent=False)

    @property
    def n_lookups(self):
        return len(self.orders) * self.heads

    def forward(self, c):
        """c: (B, history + T) compressed ids, the first `history` from before the chunk (or pad) -> (B, T,
        n_lookups) row indices; head h of order o in rows [(o * heads + h) * rows, ... + rows)."""
        if not c.is_cuda:
            raise ValueError("NgramHash of smlm_b200 runs on CUDA only (no CPU fallback)")
        return K.ngram_rows(c, self.history, self.mult, self.orders, self.heads, self.rows)


class EngramMemory(nn.Module):
    """One Engram module (reference: engram.py:78-134): n_lookups rows of head_dim per position, gated by the
    hidden state, then a depthwise causal convolution (zero-initialised, so the module starts as the gate)."""

    def __init__(self, d_model, n_lookups, head_dim, rows_per_head, conv_kernel=4, dilation=3, eps=1e-5,
                 impl="cuda", value_grad="row_sparse"):
        super().__init__()
        self.d_model, self.n_lookups, self.head_dim = d_model, n_lookups, head_dim
        self.d_mem = n_lookups * head_dim
        self.values = nn.Embedding(n_lookups * rows_per_head, head_dim)
        self.values.weight.pk_value_param = True             # own learning rate, no weight decay (optim.py)
        if value_grad not in ("row_sparse", "dense"):
            raise ValueError(value_grad)
        self.value_grad = value_grad
        self.is_engram = True
        if impl not in IMPLS:
            raise ValueError(f"unknown impl {impl!r}")
        self.impl = "cuda"
        self.w_k = nn.Linear(self.d_mem, d_model, bias=False)
        self.w_v = nn.Linear(self.d_mem, d_model, bias=False)
        self.h_norm = nn.RMSNorm(d_model, eps=eps)
        self.k_norm = nn.RMSNorm(d_model, eps=eps)
        self.v_norm = nn.RMSNorm(d_model, eps=eps)
        self.conv = nn.Conv1d(d_model, d_model, conv_kernel, dilation=dilation, groups=d_model, bias=False)
        self.past = (conv_kernel - 1) * dilation              # earlier positions the convolution sees
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self, std=0.02):
        nn.init.normal_(self.values.weight, std=self.d_mem ** -0.5)
        nn.init.normal_(self.w_k.weight, std=std)
        nn.init.normal_(self.w_v.weight, std=std)
        nn.init.zeros_(self.conv.weight)

    def read_rows(self, rows):
        """rows (B, T, n_lookups) -> (B, T, d_mem): the rows side by side (one-lookup value bags)."""
        B, T, _ = rows.shape
        flat = rows.reshape(-1, 1)
        if self.value_grad == "dense":
            e = F.embedding(flat.squeeze(1), self.values.weight)
        else:
            ones = torch.ones(flat.shape, device=rows.device, dtype=torch.float32)
            e = row_sparse_embedding_bag(flat, ones, self.values.weight, self.impl)
        return e.view(B, T, self.d_mem)

    def forward(self, h, rows, cache=None):
        """h: (B, T, d) residual stream, rows: (B, T, n_lookups) from NgramHash -> Y (B, T, d) to add to h."""
        B, T, _ = h.shape
        e = self.read_rows(rows)
        k, v = self.w_k(e), self.w_v(e)
        alpha = torch.sigmoid((self.h_norm(h) * self.k_norm(k)).sum(-1, keepdim=True) / math.sqrt(self.d_model))
        vt = alpha * v
        u = self.v_norm(vt)
        past = cache.get("eng_u") if cache is not None else None
        if past is None:
            past = torch.zeros(B, self.past, self.d_model, device=u.device, dtype=u.dtype)
        full = torch.cat([past.to(u.dtype), u], 1)
        if cache is not None:
            cache["eng_u"] = full[:, -self.past:]
        y = self.conv(full.transpose(1, 2)).transpose(1, 2)  # no padding: output j sees full[j .. j + past]
        return F.silu(y) + vt

    def macs_per_token(self):
        return 2 * self.d_mem * self.d_model + 2 * self.d_model + self.conv.kernel_size[0] * self.d_model
