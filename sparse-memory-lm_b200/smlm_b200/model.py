"""Decoder-only language model that hosts the product-key memory layers (interface of re133/sparse-memory-lm
smlm/model.py: ModelConfig fields and defaults, module and parameter names, forward signature, state_dict keys,
so checkpoints load across; mem_impl / eng_impl default to "cuda").

Architecture (the reference's): token embedding tied with the LM head; pre-norm blocks of RMSNorm -> causal
self-attention with rotary position embedding (half-split rotation) and RMSNorm -> SwiGLU feed-forward; blocks
listed in mem_layers replace the feed-forward by a ProductKeyMemory (smlm_b200.pkm, on the sm_100a kernels), with
one table optionally shared by all of them and an optional second read (mem_round_layers); blocks in eng_layers
first add an Engram n-gram memory (smlm_b200.engram).

Design of this module: the rotary tables are built once per model and sliced once per forward call for every
layer (a _Positions object carries the call's cos / sin, cast once per dtype, and the static cache's visibility
mask); attention has three cache modes, chosen by the cache the caller passes: none (training, prefill without a
cache), a growing cache (the reference's decoding loop: {"k", "v"} concatenated per step) and a static cache
(smlm_b200.decode.GraphDecoder: preallocated {"kbuf", "vbuf"}, positions on the device, fixed shapes).
"""
import math
from dataclasses import asdict, dataclass, field

import torch
import torch.nn.functional as F
from torch import nn
from torch.nn.attention import SDPBackend, sdpa_kernel

from .engram import EngramMemory, NgramHash
from .pkm import ProductKeyMemory


@dataclass
class ModelConfig:
    vocab_size: int = 50304
    d_model: int = 384
    n_layers: int = 12
    n_heads: int = 6
    ffn_hidden: int = 1024
    max_seq_len: int = 1024
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    init_std: float = 0.02
    mem_layers: list = field(default_factory=list)
    mem_n_keys: int = 512
    mem_heads: int = 4
    mem_knn: int = 32
    mem_k_dim: int = 256
    mem_v_dim: int = -1
    mem_query_norm: str = "batchnorm"
    mem_swilu: bool = True
    mem_value_impl: str = "embedding_bag"
    mem_keys_weight_decay: bool = True
    mem_score_scale: str = "none"
    mem_score_scale_init: float = 1.0
    mem_share_values: bool = False
    mem_round_layers: list = field(default_factory=list)
    mem_value_grad: str = "dense"
    mem_impl: str = "cuda"
    eng_layers: list = field(default_factory=list)
    eng_orders: list = field(default_factory=lambda: [2, 3])
    eng_heads: int = 8
    eng_head_dim: int = 24
    eng_rows: int = 524287
    eng_conv_kernel: int = 4
    eng_hash_seed: int = 0
    eng_impl: str = "cuda"
    eng_value_grad: str = "row_sparse"

    def to_dict(self):
        return asdict(self)

    @property
    def head_dim(self):
        return self.d_model // self.n_heads

    @property
    def value_dim(self):
        return self.mem_v_dim if self.mem_v_dim > 0 else self.d_model


# ------------------------------------------------------------------------------------------- positions
def rope_tables(head_dim, max_len, theta):
    """cos / sin of position x frequency, (max_len, head_dim / 2) fp32: frequency i is 1 / theta^(2i / head_dim)
    (the usual rotary embedding)."""
    freq = 1.0 / theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
    angle = torch.arange(max_len, dtype=torch.float32)[:, None] * freq[None, :]
    return angle.cos(), angle.sin()


def rotate(x, cos, sin):
    """Rotary embedding of x (..., T, head_dim) with the half-split pairing: (a, b) -> (a cos - b sin,
    b cos + a sin) where a is the first half of the head dimension and b the second."""
    a, b = x.chunk(2, dim=-1)
    return torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)


class _Positions:
    """The positions of one forward call, shared by every layer: the rotary tables' rows for them (cast once
    per dtype) and, for a static cache, which cache slots each query sees."""

    def __init__(self, cos, sin, index=None, visible=None):
        self.cos, self.sin = cos, sin
        self.index = index            # static cache: the positions as a device tensor (T,)
        self.visible = visible        # static cache: (T, max_len) bool, slot <= position
        self._cast = {}

    def rope(self, dtype):
        t = self._cast.get(dtype)
        if t is None:
            t = self._cast[dtype] = (self.cos.to(dtype), self.sin.to(dtype))
        return t


def _is_static(cache):
    return cache is not None and "kbuf" in cache


# ------------------------------------------------------------------------------------------- attention
# backends that need no per-shape plan, for the growing cache (a new length every step)
_GROWING_BACKENDS = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]
# backends that take a boolean mask, for the static cache
_MASK_BACKENDS = [SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]


class Attention(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.n_heads = cfg.n_heads
        self.head_dim = cfg.head_dim
        self.wqkv = nn.Linear(cfg.d_model, 3 * cfg.d_model, bias=False)
        self.wo = nn.Linear(cfg.d_model, cfg.d_model, bias=False)

    def forward(self, x, pos, cache=None):
        """x (B, T, d) -> (B, T, d). pos: the call's _Positions; cache: None, a growing or a static cache."""
        B, T, d = x.shape
        # (B, T, 3 d) -> q, k, v each (B, heads, T, head_dim)
        q, k, v = self.wqkv(x).unflatten(-1, (3, self.n_heads, self.head_dim)).movedim(1, -2).unbind(1)
        cos, sin = pos.rope(q.dtype)
        q, k = rotate(q, cos, sin), rotate(k, cos, sin)
        if cache is None:
            y = F.scaled_dot_product_attention(q, k, v, is_causal=T > 1)
        elif _is_static(cache):
            y = self._static_cache(q, k, v, cache, pos)
        else:
            y = self._growing_cache(q, k, v, cache)
        return self.wo(y.transpose(1, 2).reshape(B, T, d))

    @staticmethod
    def _growing_cache(q, k, v, cache):
        """The reference's decoding cache: this call's keys / values appended to the earlier ones."""
        if cache.get("k") is not None:
            k = torch.cat((cache["k"], k), dim=2)
            v = torch.cat((cache["v"], v), dim=2)
        cache["k"], cache["v"] = k, v
        T, S = q.shape[2], k.shape[2]
        with sdpa_kernel(_GROWING_BACKENDS):
            if T > 1 and S > T:
                # a chunk after cached positions: query t sees every cached slot and the chunk up to itself
                seen = torch.ones(T, S, dtype=torch.bool, device=q.device).tril(S - T)
                return F.scaled_dot_product_attention(q, k, v, attn_mask=seen)
            return F.scaled_dot_product_attention(q, k, v, is_causal=T > 1)

    @staticmethod
    def _static_cache(q, k, v, cache, pos):
        """Preallocated (B, heads, max_len, head_dim) buffers written at the positions (a device tensor), every
        query masked to the slots up to its own position: fixed shapes, capturable in one CUDA graph."""
        kbuf, vbuf = cache["kbuf"], cache["vbuf"]
        kbuf.index_copy_(2, pos.index, k.to(kbuf.dtype))
        vbuf.index_copy_(2, pos.index, v.to(vbuf.dtype))
        # one query over few (sequence, head) pairs (small-batch decoding): the plain matmul form spreads the
        # cache length over the GPU, where a fused kernel would give each pair one CTA
        few = q.shape[2] == 1 and q.shape[0] * q.shape[1] < 64
        with sdpa_kernel([SDPBackend.MATH] if few else _MASK_BACKENDS):
            return F.scaled_dot_product_attention(q, kbuf.to(q.dtype), vbuf.to(q.dtype), attn_mask=pos.visible)


class SwiGLU(nn.Module):
    """w2(silu(gate) * up) with gate and up from one fused projection w13 (gate first)."""

    def __init__(self, d, hidden):
        super().__init__()
        self.w13 = nn.Linear(d, 2 * hidden, bias=False)
        self.w2 = nn.Linear(hidden, d, bias=False)

    def forward(self, x):
        gate, up = self.w13(x).chunk(2, dim=-1)
        return self.w2(F.silu(gate) * up)


# ----------------------------------------------------------------------------------------------- blocks
def _product_key_memory(cfg, shared_values, shard=None):
    """A memory layer as ModelConfig's mem_* fields describe it; shard: (process group, exchange) to row-shard its
    table over (no counterpart in the reference)."""
    group, exchange = shard if shard is not None else (None, "p2p")
    return ProductKeyMemory(
        cfg.d_model, cfg.d_model, n_keys=cfg.mem_n_keys, heads=cfg.mem_heads, knn=cfg.mem_knn,
        k_dim=cfg.mem_k_dim, v_dim=cfg.mem_v_dim, query_norm=cfg.mem_query_norm, swilu=cfg.mem_swilu,
        value_impl=cfg.mem_value_impl, keys_weight_decay=cfg.mem_keys_weight_decay,
        score_scale=cfg.mem_score_scale, score_scale_init=cfg.mem_score_scale_init, shared_values=shared_values,
        value_grad=cfg.mem_value_grad, impl=cfg.mem_impl, shard_group=group, shard_exchange=exchange)


class Block(nn.Module):
    """Residual branches in order: [Engram memory], attention, feed-forward or memory read, [second read]."""

    def __init__(self, cfg, layer_id, shared_values=None, shard=None):
        super().__init__()
        self.is_memory = layer_id in cfg.mem_layers
        self.dormant = False                  # a block that grows in later (set_dormant / wake): skipped
        self.attn_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.attn = Attention(cfg)
        self.ffn_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.ffn = (_product_key_memory(cfg, shared_values, shard) if self.is_memory
                    else SwiGLU(cfg.d_model, cfg.ffn_hidden))
        self.ffn_r2 = None
        if layer_id in cfg.mem_round_layers:
            if not (self.is_memory and shared_values is not None):
                raise ValueError(f"layer {layer_id}: a second memory read needs a memory layer with a shared table")
            self.ffn_norm_r2 = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
            self.ffn_r2 = _product_key_memory(cfg, shared_values, shard)
        self.engram = None
        if layer_id in cfg.eng_layers:
            self.engram = EngramMemory(cfg.d_model, len(cfg.eng_orders) * cfg.eng_heads, cfg.eng_head_dim,
                                       cfg.eng_rows, conv_kernel=cfg.eng_conv_kernel, dilation=max(cfg.eng_orders),
                                       eps=cfg.norm_eps, impl=cfg.eng_impl, value_grad=cfg.eng_value_grad)

    def reads(self):
        """This block's memory layers (first read, then the second)."""
        if not self.is_memory:
            return []
        return [self.ffn] + ([self.ffn_r2] if self.ffn_r2 is not None else [])

    def forward(self, h, pos, cache=None, eng_rows=None):
        if self.engram is not None:
            h = h + self.engram(h, eng_rows, cache)
        h = h + self.attn(self.attn_norm(h), pos, cache)
        h = h + self.ffn(self.ffn_norm(h))
        if self.ffn_r2 is not None:
            h = h + self.ffn_r2(self.ffn_norm_r2(h))
        return h


# ---------------------------------------------------------------------------------------------- the model
class Transformer(nn.Module):
    def __init__(self, cfg, shard_group=None, shard_exchange="p2p"):
        """shard_group (no counterpart in the reference): a torch.distributed process group over which the
        product-key value tables are row-sharded (one process per GPU, each holding its rows; see
        smlm_b200.sharded), shard_exchange "p2p" or "nccl"; everything else stays replicated. Needs
        mem_value_grad="row_sparse"."""
        super().__init__()
        self.cfg = cfg
        self.tok_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        shard = None
        rows = cfg.mem_n_keys ** 2
        if shard_group is not None and torch.distributed.get_world_size(shard_group) > 1:
            from .sharded import RowShard
            shard = (shard_group, shard_exchange)
            rows = RowShard(rows, torch.distributed.get_world_size(shard_group),
                            torch.distributed.get_rank(shard_group)).count
        shared = nn.Embedding(rows, cfg.value_dim) if cfg.mem_share_values and cfg.mem_layers else None
        self.layers = nn.ModuleList(Block(cfg, i, shared, shard) for i in range(cfg.n_layers))
        self.ngram = (NgramHash(cfg.vocab_size, cfg.eng_orders, cfg.eng_heads, cfg.eng_rows, cfg.eng_hash_seed)
                      if cfg.eng_layers else None)
        self.norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.tok_emb.weight                        # tied
        cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self._init_dense()

    @torch.no_grad()
    def _init_dense(self):
        """N(0, init_std) for the embedding and every projection into a block; projections back onto the
        residual stream (attention output, feed-forward down) get init_std / sqrt(2 n_layers). Memory layers
        initialise themselves."""
        std, out_std = self.cfg.init_std, self.cfg.init_std / math.sqrt(2 * self.cfg.n_layers)
        nn.init.normal_(self.tok_emb.weight, std=std)
        for blk in self.layers:
            nn.init.normal_(blk.attn.wqkv.weight, std=std)
            nn.init.normal_(blk.attn.wo.weight, std=out_std)
            if not blk.is_memory:
                nn.init.normal_(blk.ffn.w13.weight, std=std)
                nn.init.normal_(blk.ffn.w2.weight, std=out_std)

    # -------------------------------------------------------------------------------- growing blocks in
    def set_dormant(self, layers):
        """Skip these plain blocks until wake()."""
        for i in layers:
            blk = self.layers[i]
            if blk.is_memory or blk.engram is not None:
                raise ValueError(f"block {i} reads a table; only plain blocks can grow in")
            blk.dormant = True

    @torch.no_grad()
    def wake(self):
        """Dormant blocks join as identities: their output projections start at zero."""
        for blk in self.layers:
            if blk.dormant:
                blk.attn.wo.weight.zero_()
                blk.ffn.w2.weight.zero_()
                blk.dormant = False

    # ---------------------------------------------------------------------------------------- memories
    def memory_layers(self):
        return [m for blk in self.layers for m in blk.reads()]

    def memory_sites(self):
        """Names of the memory reads: "L<layer>" and "L<layer>r2" for a second read."""
        return [f"L{i}" + ("r2" if r else "") for i, blk in enumerate(self.layers) for r in range(len(blk.reads()))]

    def engram_layers(self):
        return [blk.engram for blk in self.layers if blk.engram is not None]

    def set_memory_decode_graphs(self, enabled=True):
        """One-token forwards of the memory layers replay a CUDA graph each (ProductKeyMemory.decode_graph)."""
        for m in self.memory_layers():
            m.decode_graph = enabled
            m._graph = None

    @torch.no_grad()
    def set_memory_inference_table(self, kind="fp32"):
        """The table copy no-grad bf16 forwards read: "fp32" (the weights), "bf16" or "q4" (4-bit, one fp16
        scale per row); call again after the weights change (reference: model.py:244-264)."""
        from .kernels import quantize_q4
        make = {"fp32": lambda w: None, "bf16": lambda w: (w.to(torch.bfloat16), None), "q4": quantize_q4}
        if kind not in make:
            raise ValueError(kind)
        done = set()
        for m in self.memory_layers():
            m._graph = None
            if id(m.values) not in done:
                done.add(id(m.values))
                m.values.infer_table = make[kind](m.values.weight.detach())

    # ----------------------------------------------------------------------------------------- forward
    def _positions(self, T, pos0, caches):
        first = caches[0] if caches else None
        if _is_static(first):
            index = first["pos"]
            visible = first["arange"].view(1, -1) <= index.view(-1, 1)
            return _Positions(self.rope_cos.index_select(0, index), self.rope_sin.index_select(0, index), index,
                              visible)
        return _Positions(self.rope_cos[pos0:pos0 + T], self.rope_sin[pos0:pos0 + T])

    def _engram_rows(self, idx, caches):
        """Engram row indices of the call's tokens; the n-gram history comes from the cache (decoding) or is
        padding (a sequence start)."""
        ids = self.ngram.canon[idx]
        hist = caches[0].get("eng_hist") if caches is not None else None
        if hist is None:
            hist = torch.full((ids.shape[0], self.ngram.history), self.ngram.pad, dtype=ids.dtype, device=ids.device)
        ids = torch.cat((hist, ids), dim=1)
        if caches is not None:
            caches[0]["eng_hist"] = ids[:, -self.ngram.history:]
        return self.ngram(ids)

    def forward(self, idx, targets=None, kv_caches=None, pos0=0, fused_ce=False, ce_chunk_size=1024):
        """idx (B, T) token ids -> logits (B, T, vocab); with targets, (logits, mean cross entropy), the logits
        None when fused_ce is set. kv_caches: one dict per layer (growing or static caches), pos0: the first
        position for a growing cache. ce_chunk_size is accepted for the reference's signature (the loss here is
        one plain cross entropy)."""
        pos = self._positions(idx.shape[1], pos0, kv_caches)
        rows = self._engram_rows(idx, kv_caches) if self.ngram is not None else None
        h = self.tok_emb(idx)
        for i, blk in enumerate(self.layers):
            if not blk.dormant:
                h = blk(h, pos, None if kv_caches is None else kv_caches[i], rows)
        logits = self.lm_head(self.norm(h))
        if targets is None:
            return logits
        loss = F.cross_entropy(logits.float().flatten(0, -2), targets.reshape(-1))
        return (None if fused_ce else logits), loss

    # ---------------------------------------------------------------------------------------- counting
    def param_counts(self):
        """Parameter counts: total (tied head once), embedding, the rest, value tables (each shared table
        once), the dense body, what one token touches outside the embedding (the body plus the rows it reads),
        and the BatchNorm running statistics."""
        total = sum(p.numel() for p in self.parameters())
        embedding = self.tok_emb.weight.numel()
        reads = self.memory_layers()
        engrams = self.engram_layers()
        tables = {id(m.values.weight): m.values.weight.numel() for m in reads + engrams}
        values = sum(tables.values())
        body = total - embedding - values
        read_per_token = (sum(m.heads * m.knn * m.v_dim for m in reads)
                          + sum(e.n_lookups * e.head_dim for e in engrams))
        running = sum(b.numel() for name, b in self.named_buffers() if "running" in name)
        return {"total": total, "embedding": embedding, "non_embedding": total - embedding,
                "memory_values": values, "dense_body": body, "active_non_embedding_per_token": body + read_per_token,
                "bn_running_stats": running}

    def macs_per_token(self, context_len=None):
        """Multiply-accumulates per token by part, attention scores at an average context of half of
        context_len (default max_seq_len)."""
        c, d = self.cfg, self.cfg.d_model
        ctx = context_len or c.max_seq_len
        n = len(self.layers)
        plain = [blk for blk in self.layers if not blk.is_memory]
        out = {"attn_proj": n * 4 * d * d, "attn_scores": n * 2 * d * (ctx / 2),
               "ffn": len(plain) * 3 * d * c.ffn_hidden,
               "memory": sum(m.macs_per_token() for m in self.memory_layers()),
               "engram": sum(e.macs_per_token() for e in self.engram_layers()),
               "lm_head": d * c.vocab_size}
        out["total"] = sum(out.values())
        return out
