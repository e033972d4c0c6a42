"""Product-key memory layer on the sm_100a kernels (reference: re133/sparse-memory-lm smlm/pkm.py).

Same constructor, parameters, initialisation, state_dict keys and forward contract as the reference's
ProductKeyMemory; the lookup runs on libsmlm_b200.so:
  * scoring + selection: under bf16 autocast one fused tensor-core kernel computes the bf16 sub-key scores
    (pkm.py:197, the reference's einsum) and keeps each half's top-k in its epilogue, then the pairs / final
    top-k / softmax kernel; without autocast the scores are computed exactly in fp32 by the fmaf-chain kernel
    and selected by the selection kernel (both half top-k, pair sums, final top-k, softmax);
  * value bag: row_sparse_embedding_bag (row-sparse accumulation + lazy optimizer), or the inference bag with
    the swilu product fused when there is no grad under bf16 autocast (pkm.py:213-224);
  * decoding (one token, no grad, decode_graph): a captured CUDA graph of the same kernels (pkm.py:159-184).
Ties in the selection go to the lower index. The query projection, BatchNorm and swilu projections stay
PyTorch modules (dense host code).
"""
import math

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from . import kernels as K
from .sharded import RowShard, sharded_bag_infer, sharded_embedding_bag
from .sparse_values import read_table, row_sparse_embedding_bag

IMPLS = ("cuda", "triton", "torch")
MAX_ROW_WIDTH = 512        # SMLM_MAX_ROW_WIDTH: widest value row of the row-sparse backward


class _DecodeGraph:
    """A captured forward with a static input and output. Warmed up twice on a side stream before capture (the
    autocast cache off, so no cast is captured from a stale cache)."""

    def __init__(self, fn, x, key):
        self.key = key
        self.x = x.clone()
        dtype = key[2]
        mode = (torch.autocast("cuda", dtype=dtype, cache_enabled=False) if dtype is not None
                else torch.autocast("cuda", enabled=False))
        here = torch.cuda.current_stream()
        side = torch.cuda.Stream()
        side.wait_stream(here)
        with torch.cuda.stream(side), mode:
            fn(self.x)
            fn(self.x)
        here.wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), mode:
            self.out = fn(self.x)

    def run(self, x):
        self.x.copy_(x)
        self.graph.replay()
        return self.out.clone()


class ProductKeyMemory(nn.Module):
    def __init__(self, d_in, d_out, n_keys=512, heads=4, knn=32, k_dim=256, v_dim=-1,
                 query_norm="batchnorm", swilu=True, value_impl="embedding_bag",
                 keys_weight_decay=True, score_scale="none", score_scale_init=1.0, shared_values=None,
                 value_grad="dense", impl="cuda", shard_group=None, shard_exchange="p2p"):
        """shard_group (no counterpart in the reference): a torch.distributed process group over which the value
        table is row-sharded (one process per GPU; values.weight then holds this rank's rows only, and the
        lookups are exchanged with the other ranks). Needs value_grad="row_sparse". shard_exchange: "p2p" (the
        exchange fused into the kernels through peer memory over NVLink) or "nccl" (NCCL collectives)."""
        super().__init__()
        assert k_dim % 2 == 0 and knn <= n_keys
        self.d_in, self.d_out = d_in, d_out
        self.n_keys, self.heads, self.knn, self.k_dim = n_keys, heads, knn, k_dim
        self.size = n_keys ** 2
        self.v_dim = v_dim if v_dim > 0 else d_out
        self.swilu = swilu
        self.value_impl = value_impl
        assert value_grad in ("dense", "row_sparse")
        self.value_grad = value_grad
        if impl not in IMPLS:
            raise ValueError(f"unknown impl {impl!r}")
        if not (1 <= knn <= 32 and n_keys <= 65536):
            # the selection kernel keeps one selected entry per lane of a warp and packs (i1, i2) into 32 bits
            raise ValueError(f"the CUDA selection needs 1 <= knn <= 32 and n_keys <= 65536, got n_keys={n_keys}, "
                             f"knn={knn}")
        self.impl = "cuda"
        if value_grad == "row_sparse" and (v_dim if v_dim > 0 else d_out) > MAX_ROW_WIDTH:
            raise ValueError(f"row-sparse value gradients support rows of at most {MAX_ROW_WIDTH} values, got "
                             f"{v_dim if v_dim > 0 else d_out}")
        self.score_scale_init = score_scale_init

        self.keys = nn.Parameter(torch.empty(heads, 2, n_keys, k_dim // 2))
        if not keys_weight_decay:
            self.keys.no_weight_decay = True
        if score_scale == "learned":
            assert score_scale_init > 0
            self.log_score_scale = nn.Parameter(torch.empty(heads))
        elif score_scale == "none":
            self.log_score_scale = None
        else:
            raise ValueError(score_scale)
        self.query_proj = nn.Linear(d_in, heads * k_dim, bias=True)
        if query_norm == "batchnorm":
            self.query_norm = nn.BatchNorm1d(heads * k_dim)
        elif query_norm == "none":
            self.query_norm = None
        else:
            raise ValueError(query_norm)
        self.shard = self.shard_group = None
        if shard_group is not None and dist.get_world_size(shard_group) > 1:
            if value_grad != "row_sparse":
                raise ValueError("a row-sharded value table needs value_grad='row_sparse'")
            if shard_exchange not in ("p2p", "nccl"):
                raise ValueError(f"unknown shard_exchange {shard_exchange!r}")
            self.shard = RowShard(self.size, dist.get_world_size(shard_group), dist.get_rank(shard_group))
            self.shard_group = shard_group
            self.shard_exchange = shard_exchange
        if shared_values is not None:
            # a table shared by several layers (this rank's rows of it when row-sharded)
            rows = self.shard.count if self.shard is not None else self.size
            if tuple(shared_values.weight.shape) != (rows, self.v_dim):
                raise ValueError(f"shared value table of shape {tuple(shared_values.weight.shape)}, expected "
                                 f"{(rows, self.v_dim)}")
            self.values = shared_values
        else:
            self.values = nn.Embedding(self.shard.count if self.shard else self.size, self.v_dim)
        if self.shard is not None:
            self.values.weight.row_shard = self.shard
            self.values.weight.shard_group = shard_group
        if swilu:
            self.swilu_proj = nn.Linear(d_in, self.v_dim)
            self.value_proj = nn.Linear(self.v_dim, d_out)
        else:
            assert self.v_dim == d_out
        self.record = False
        self.last_indices = None
        self.last_scores = None
        self.last_weights = None
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self):
        """Initialisation of the reference (pkm.py:94-109)."""
        bound = 1 / math.sqrt(self.k_dim)
        nn.init.uniform_(self.keys, -bound, bound)
        nn.init.normal_(self.values.weight, mean=0.0, std=self.v_dim ** -0.5)
        nn.init.xavier_uniform_(self.query_proj.weight)
        nn.init.zeros_(self.query_proj.bias)
        if self.swilu:
            nn.init.normal_(self.swilu_proj.weight, mean=0.0, std=self.d_out ** -0.5)
            nn.init.normal_(self.value_proj.weight, mean=0.0, std=self.d_out ** -0.5)
            nn.init.zeros_(self.swilu_proj.bias)
            nn.init.zeros_(self.value_proj.bias)
        if self.log_score_scale is not None:
            nn.init.constant_(self.log_score_scale, math.log(self.score_scale_init))
        self.values.weight.pk_value_param = True

    def score_scale(self):
        if self.log_score_scale is None:
            return torch.ones(self.heads, device=self.keys.device)
        return self.log_score_scale.exp()

    def subkey_scores(self, query):
        """query (N, heads, k_dim) -> sub-key scores s1, s2 (N, heads, n_keys) (reference: pkm.py:117-123).
        fp32 queries: the exact fmaf-chain kernel; bf16 queries: the bf16 contraction (fp32 accumulation)."""
        if query.dtype == torch.float32:
            return K.SubkeyScoresF32.apply(query, self.keys)
        half = self.k_dim // 2
        k1, k2 = self.keys[:, 0].to(query.dtype), self.keys[:, 1].to(query.dtype)
        s1 = torch.einsum("nhd,hkd->nhk", query[..., :half], k1)
        s2 = torch.einsum("nhd,hkd->nhk", query[..., half:], k2)
        return s1, s2

    def get_indices(self, query):
        """query (N, heads, k_dim) -> scores, indices (N, heads, knn): the product-key top-k
        (reference: pkm.py:125-136), ties to the lower index."""
        s1, s2 = self.subkey_scores(query)
        scores, indices, _ = K.PKSelect.apply(s1, s2, self.knn)
        return scores, indices

    def read_values(self, indices, weights):
        """indices, weights (N, heads*knn) -> (N, v_dim) (reference: pkm.py:138-148)."""
        w = self.values.weight
        if getattr(w, "host_values", False):
            return self.values.bag(indices, weights, self.impl)        # table in host RAM (host_values.py)
        if self.shard is not None:
            return sharded_embedding_bag(indices, weights, w, self.shard, self.shard_group,
                                         exchange=self.shard_exchange)
        if self.value_grad == "row_sparse":
            return row_sparse_embedding_bag(indices, weights, w, self.impl)
        if self.value_impl == "embedding_bag":
            return F.embedding_bag(indices, w, per_sample_weights=weights.to(w.dtype), mode="sum")
        return torch.einsum("nj,njd->nd", weights.to(w.dtype), F.embedding(indices, w))

    def forward(self, x):
        shape = x.shape
        x = x.reshape(-1, self.d_in)
        if not x.is_cuda:
            raise ValueError("ProductKeyMemory of smlm_b200 runs on CUDA only (no CPU fallback)")
        if (getattr(self, "decode_graph", False) and x.shape[0] == 1 and not self.record
                and not torch.is_grad_enabled() and (self.shard is None or self.shard_exchange == "p2p")
                and not getattr(self.values.weight, "host_values", False)):
            return self._graph_forward(x).view(*shape[:-1], self.d_out)
        return self._forward(x).view(*shape[:-1], self.d_out)

    def _graph_forward(self, x):
        """One-token no-grad forward as a CUDA-graph replay (reference: pkm.py:159-184): the graph of _forward
        for this input's shape, dtype, autocast state and inference table is captured on first use (and again
        when any of them changes), then replayed with the token copied into its static input. Same kernels as
        the eager path, so the same bits, without the per-launch host work."""
        ac = torch.is_autocast_enabled("cuda")
        key = (tuple(x.shape), x.dtype, torch.get_autocast_dtype("cuda") if ac else None,
               id(getattr(self.values, "infer_table", None)))
        dg = getattr(self, "_graph", None)
        if dg is None or dg.key != key:
            dg = self._graph = _DecodeGraph(self._forward, x, key)
        return dg.run(x)

    def _select(self, q, autocast_bf16):
        """q (N, heads, k_dim) -> scores, indices, weights (N, heads, knn). Under bf16 autocast the fused
        tensor-core scoring + selection (no (N, heads, n_keys) score tensors); in fp32 the exact fmaf-chain scores
        and the selection kernel."""
        if autocast_bf16 and K.fused_scoring_ok(self.k_dim // 2, self.n_keys, self.knn):
            scores, indices, weights = K.ScoreSelect.apply(q.to(torch.bfloat16), self.keys.to(torch.bfloat16),
                                                           self.knn)
        else:
            s1, s2 = self.subkey_scores(q.to(torch.bfloat16) if autocast_bf16 else q.float())
            scores, indices, weights = K.PKSelect.apply(s1, s2, self.knn)
        if self.log_score_scale is not None:
            logits = scores.float() * self.log_score_scale.float().exp().view(1, self.heads, 1)
            weights = F.softmax(logits, dim=-1)
        return scores, indices, weights

    def _forward(self, x):
        N = x.shape[0]
        q = self.query_proj(x)
        if self.query_norm is not None:
            q = self.query_norm(q.to(self.query_norm.weight.dtype))     # BN in fp32 under autocast
        q = q.view(N, self.heads, self.k_dim)
        autocast_bf16 = (torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16)
        with torch.autocast("cuda", enabled=False):
            scores, indices, weights = self._select(q, autocast_bf16)
        if self.record:
            self.last_indices = indices.detach()
            self.last_scores = scores.detach()
            self.last_weights = weights.detach()
        if (not torch.is_grad_enabled() and self.swilu and autocast_bf16 and self.shard is not None
                and self.shard_exchange == "p2p"):
            # inference over a row-sharded table: the swilu product and the bf16 cast fused into the peer
            # exchange's final sum of the owners' partial bags
            K_ = self.heads * self.knn
            out = sharded_bag_infer(indices.view(N, K_), weights.view(N, K_), self.values.weight, self.shard,
                                    self.shard_group, pre=self.swilu_proj(x), out_bf16=True)
            return self.value_proj(out)
        if (not torch.is_grad_enabled() and self.swilu and autocast_bf16 and self.shard is None
                and not getattr(self.values.weight, "host_values", False)):
            # inference: value bag on the inference table (fp32 / bf16 / q4) with the swilu product and the
            # bf16 cast fused (reference: pkm.py:213-224)
            pre = self.swilu_proj(x)
            t = getattr(self.values, "infer_table", None) or (read_table(self.values.weight), None)
            K_ = self.heads * self.knn
            out = K.bag_infer(indices.view(N, K_), weights.view(N, K_), t[0], t[1], pre=pre, out_bf16=True)
            return self.value_proj(out)
        K_ = self.heads * self.knn
        out = self.read_values(indices.view(N, K_), weights.view(N, K_))
        if self.swilu:
            out = self.value_proj(out * F.silu(self.swilu_proj(x)).to(out.dtype))
        return out

    def macs_per_token(self):
        """Multiply-accumulates per token (reference: pkm.py:230-237)."""
        m = self.d_in * self.heads * self.k_dim
        m += self.heads * 2 * self.n_keys * (self.k_dim // 2)
        m += self.heads * self.knn * self.v_dim
        if self.swilu:
            m += self.d_in * self.v_dim + self.v_dim * self.d_out + self.v_dim
        return m
