"""Llama-style decoder hosting product-key memory layers (reference: re133/sparse-memory-lm smlm/model.py).

The dense parts (RMSNorm, RoPE attention, SwiGLU, tied LM head) are plain PyTorch; the memory layers are
smlm_b200.pkm.ProductKeyMemory on the sm_100a kernels. ModelConfig keeps the reference's field names and
defaults (mem_impl / eng_impl default to "cuda"); state_dict keys match the reference's, so checkpoints load
across. Engram n-gram memories (eng_layers) are smlm_b200.engram.EngramMemory, as in the reference.
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


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim, max_seq_len, theta):
        super().__init__()
        inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
        freqs = torch.outer(torch.arange(max_seq_len).float(), inv_freq)
        self.register_buffer("cos", freqs.cos(), persistent=False)
        self.register_buffer("sin", freqs.sin(), persistent=False)

    def forward(self, x, pos0=0):
        """pos0: the first position (int), or a device tensor of the T positions (static-cache decoding)."""
        T = x.shape[-2]
        if torch.is_tensor(pos0):
            cos = self.cos.index_select(0, pos0).to(x.dtype)
            sin = self.sin.index_select(0, pos0).to(x.dtype)
        else:
            cos = self.cos[pos0:pos0 + T].to(x.dtype)
            sin = self.sin[pos0:pos0 + T].to(x.dtype)
        x1, x2 = x.chunk(2, dim=-1)
        return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


class Attention(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.n_heads = cfg.n_heads
        self.head_dim = cfg.d_model // cfg.n_heads
        self.wqkv = nn.Linear(cfg.d_model, 3 * cfg.d_model, bias=False)
        self.wo = nn.Linear(cfg.d_model, cfg.d_model, bias=False)
        self.rope = RotaryEmbedding(self.head_dim, cfg.max_seq_len, cfg.rope_theta)

    def forward(self, x, kv_cache=None, pos0=0):
        B, T, C = x.shape
        q, k, v = self.wqkv(x).view(B, T, 3, self.n_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        if kv_cache is not None and "kbuf" in kv_cache:
            return self.wo(self._static(q, k, v, kv_cache).transpose(1, 2).reshape(B, T, C))
        q, k = self.rope(q, pos0), self.rope(k, pos0)
        if kv_cache is not None:
            if kv_cache.get("k") is not None:
                k = torch.cat([kv_cache["k"], k], dim=2)
                v = torch.cat([kv_cache["v"], v], dim=2)
            kv_cache["k"], kv_cache["v"] = k, v
        S = k.shape[2]
        if kv_cache is not None:
            # the cache grows by one position per decoding step: keep to the backends that need no per-shape
            # plan (a backend that builds one per sequence length would re-plan on every step)
            with sdpa_kernel(_CACHED_BACKENDS):
                y = _attend(q, k, v, T, S)
        else:
            y = _attend(q, k, v, T, S)
        return self.wo(y.transpose(1, 2).reshape(B, T, C))


    def _static(self, q, k, v, cache):
        """Static KV cache (smlm_b200.decode.GraphDecoder): preallocated (B, heads, max_len, head_dim) buffers and
        the tokens' positions as a device tensor, so a decoding step has fixed shapes and no host-side position
        (it can be captured in one CUDA graph). The new keys / values are written at their positions; each query
        attends to the cache positions up to its own."""
        pos = cache["pos"]
        # per-step values every layer shares (the rotary tables are the same in all layers): computed once
        shared = cache.get("step")
        if shared is None:
            shared = {}
        rope = shared.get("rope")
        if rope is None or rope[0].dtype != q.dtype:
            rope = shared["rope"] = (self.rope.cos.index_select(0, pos).to(q.dtype),
                                     self.rope.sin.index_select(0, pos).to(q.dtype))
        q, k = _rotate(q, *rope), _rotate(k, *rope)
        kbuf, vbuf = cache["kbuf"], cache["vbuf"]
        kbuf.index_copy_(2, pos, k.to(kbuf.dtype))
        vbuf.index_copy_(2, pos, v.to(vbuf.dtype))
        mask = shared.get("mask")
        if mask is None:
            mask = shared["mask"] = cache["arange"].view(1, -1) <= pos.view(-1, 1)
        # one query for few (sequence, head) pairs (decoding at small batch): the plain matmul form spreads the
        # cache length over the GPU, where a fused kernel would give each pair one CTA
        small = q.shape[2] == 1 and q.shape[0] * q.shape[1] < 64
        with sdpa_kernel([SDPBackend.MATH] if small else _MASKED_BACKENDS):
            return F.scaled_dot_product_attention(q, kbuf.to(q.dtype), vbuf.to(q.dtype), attn_mask=mask)


def _rotate(x, cos, sin):
    """RotaryEmbedding.forward with the position tables already selected."""
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)


_CACHED_BACKENDS = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]
_MASKED_BACKENDS = [SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]


def _attend(q, k, v, T, S):
    if T > 1 and S > T:
        mask = torch.ones(T, S, dtype=torch.bool, device=q.device).tril(S - T)
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    return F.scaled_dot_product_attention(q, k, v, is_causal=T > 1)


class SwiGLU(nn.Module):
    def __init__(self, d, hidden):
        super().__init__()
        self.w13 = nn.Linear(d, 2 * hidden, bias=False)
        self.w2 = nn.Linear(hidden, d, bias=False)

    def forward(self, x):
        a, b = self.w13(x).chunk(2, dim=-1)
        return self.w2(F.silu(a) * b)


def _memory(cfg, shared_values):
    return ProductKeyMemory(
        cfg.d_model, cfg.d_model, n_keys=cfg.mem_n_keys, heads=cfg.mem_heads, knn=cfg.mem_knn,
        k_dim=cfg.mem_k_dim, v_dim=cfg.mem_v_dim, query_norm=cfg.mem_query_norm, swilu=cfg.mem_swilu,
        value_impl=cfg.mem_value_impl, keys_weight_decay=cfg.mem_keys_weight_decay,
        score_scale=cfg.mem_score_scale, score_scale_init=cfg.mem_score_scale_init, shared_values=shared_values,
        value_grad=cfg.mem_value_grad, impl=cfg.mem_impl)


class Block(nn.Module):
    def __init__(self, cfg, layer_id, shared_values=None):
        super().__init__()
        self.attn_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.attn = Attention(cfg)
        self.ffn_norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.is_memory = layer_id in cfg.mem_layers
        self.dormant = False
        self.ffn = _memory(cfg, shared_values) if self.is_memory else SwiGLU(cfg.d_model, cfg.ffn_hidden)
        self.ffn_r2 = None
        if layer_id in cfg.mem_round_layers:
            assert self.is_memory and shared_values is not None, "a second read needs a shared value table"
            self.ffn_norm_r2 = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
            self.ffn_r2 = _memory(cfg, shared_values)
        self.engram = None
        if layer_id in cfg.eng_layers:
            self.engram = EngramMemory(cfg.d_model, len(cfg.eng_orders) * cfg.eng_heads, cfg.eng_head_dim,
                                       cfg.eng_rows, conv_kernel=cfg.eng_conv_kernel, dilation=max(cfg.eng_orders),
                                       eps=cfg.norm_eps, impl=cfg.eng_impl, value_grad=cfg.eng_value_grad)

    def forward(self, x, kv_cache=None, pos0=0, eng_rows=None):
        if self.engram is not None:
            x = x + self.engram(x, eng_rows, kv_cache)
        x = x + self.attn(self.attn_norm(x), kv_cache, pos0)
        x = x + self.ffn(self.ffn_norm(x))
        if self.ffn_r2 is not None:
            x = x + self.ffn_r2(self.ffn_norm_r2(x))
        return x


class Transformer(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        self.tok_emb = nn.Embedding(cfg.vocab_size, cfg.d_model)
        shared = None
        if cfg.mem_share_values and cfg.mem_layers:
            v_dim = cfg.mem_v_dim if cfg.mem_v_dim > 0 else cfg.d_model
            shared = nn.Embedding(cfg.mem_n_keys ** 2, v_dim)
        self.layers = nn.ModuleList([Block(cfg, i, shared) for i in range(cfg.n_layers)])
        self.ngram = (NgramHash(cfg.vocab_size, cfg.eng_orders, cfg.eng_heads, cfg.eng_rows, cfg.eng_hash_seed)
                      if cfg.eng_layers else None)
        self.norm = nn.RMSNorm(cfg.d_model, eps=cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.tok_emb.weight
        self._init_weights()

    @torch.no_grad()
    def _init_weights(self):
        std = self.cfg.init_std
        nn.init.normal_(self.tok_emb.weight, std=std)
        for blk in self.layers:
            nn.init.normal_(blk.attn.wqkv.weight, std=std)
            nn.init.normal_(blk.attn.wo.weight, std=std / math.sqrt(2 * self.cfg.n_layers))
            if not blk.is_memory:
                nn.init.normal_(blk.ffn.w13.weight, std=std)
                nn.init.normal_(blk.ffn.w2.weight, std=std / math.sqrt(2 * self.cfg.n_layers))

    def set_dormant(self, layers):
        for i in layers:
            blk = self.layers[i]
            if blk.is_memory or blk.engram is not None:
                raise ValueError(f"block {i} reads a table; only plain blocks can grow in")
            blk.dormant = True

    @torch.no_grad()
    def wake(self):
        for blk in self.layers:
            if blk.dormant:
                blk.attn.wo.weight.zero_()
                blk.ffn.w2.weight.zero_()
                blk.dormant = False

    def memory_layers(self):
        out = []
        for b in self.layers:
            if b.is_memory:
                out.append(b.ffn)
                if b.ffn_r2 is not None:
                    out.append(b.ffn_r2)
        return out

    def memory_sites(self):
        out = []
        for i, b in enumerate(self.layers):
            if b.is_memory:
                out.append(f"L{i}")
                if b.ffn_r2 is not None:
                    out.append(f"L{i}r2")
        return out

    def engram_layers(self):
        return [b.engram for b in self.layers if b.engram is not None]

    def set_memory_decode_graphs(self, enabled=True):
        for m in self.memory_layers():
            m.decode_graph = enabled
            m._graph = None

    @torch.no_grad()
    def set_memory_inference_table(self, kind="fp32"):
        """Inference copy of the value table(s): "fp32" (the weights), "bf16" or "q4" (reference: model.py:244-264)."""
        from .kernels import quantize_q4
        seen = set()
        for m in self.memory_layers():
            m._graph = None
            v = m.values
            if id(v) in seen:
                continue
            seen.add(id(v))
            if kind == "fp32":
                v.infer_table = None
            elif kind == "bf16":
                v.infer_table = (v.weight.detach().to(torch.bfloat16), None)
            elif kind == "q4":
                v.infer_table = quantize_q4(v.weight.detach())
            else:
                raise ValueError(kind)

    def forward(self, idx, targets=None, kv_caches=None, pos0=0, fused_ce=False, ce_chunk_size=1024):
        x = self.tok_emb(idx)
        rows = None
        if self.ngram is not None:
            # n-gram rows need the last tokens before this chunk: pad at the start, else from the cache
            c = self.ngram.canon[idx]
            hist = kv_caches[0].get("eng_hist") if kv_caches is not None else None
            if hist is None:
                hist = torch.full((c.shape[0], self.ngram.history), self.ngram.pad, dtype=c.dtype, device=c.device)
            c = torch.cat([hist, c], 1)
            if kv_caches is not None:
                kv_caches[0]["eng_hist"] = c[:, -self.ngram.history:]
            rows = self.ngram(c)
        for i, blk in enumerate(self.layers):
            if blk.dormant:
                continue
            x = blk(x, None if kv_caches is None else kv_caches[i], pos0, rows)
        logits = self.lm_head(self.norm(x))
        if targets is None:
            return logits
        loss = F.cross_entropy(logits.float().view(-1, logits.size(-1)), targets.reshape(-1))
        return (None if fused_ce else logits), loss

    def param_counts(self):
        emb = self.tok_emb.weight.numel()
        tables = {id(m.values.weight): m.values.weight.numel() for m in self.memory_layers() + self.engram_layers()}
        values = sum(tables.values())
        total = sum(p.numel() for p in self.parameters())
        buffers = sum(b.numel() for n, b in self.named_buffers() if "running" in n)
        return {"total": total, "embedding": emb, "non_embedding": total - emb, "memory_values": values,
                "dense_body": total - emb - values,
                "active_non_embedding_per_token": total - emb - values + sum(
                    m.heads * m.knn * m.v_dim for m in self.memory_layers()) + sum(
                    m.n_lookups * m.head_dim for m in self.engram_layers()),
                "bn_running_stats": buffers}

    def macs_per_token(self, context_len=None):
        c = self.cfg
        T = context_len or c.max_seq_len
        d = c.d_model
        out = {"attn_proj": 0, "attn_scores": 0, "ffn": 0, "memory": 0, "engram": 0, "lm_head": d * c.vocab_size}
        for blk in self.layers:
            if blk.engram is not None:
                out["engram"] += blk.engram.macs_per_token()
            out["attn_proj"] += 4 * d * d
            out["attn_scores"] += 2 * d * (T / 2)
            if blk.is_memory:
                out["memory"] += blk.ffn.macs_per_token()
                if blk.ffn_r2 is not None:
                    out["memory"] += blk.ffn_r2.macs_per_token()
            else:
                out["ffn"] += 3 * d * c.ffn_hidden
        out["total"] = sum(out.values())
        return out
