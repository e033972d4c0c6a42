"""Greedy decoding with the whole step in one CUDA graph (no counterpart in the reference).

The reference's decoding loop (smlm/train.py:283-315) runs the dense blocks eagerly and replays CUDA graphs of the
memory layers only (smlm/pkm.py:159-184); with about 30 PyTorch launches per block, a one-token step is bound by
the host. GraphDecoder gives every attention layer a static KV cache (preallocated (B, heads, max_len, head_dim)
buffers) and keeps the position on the device, so that one step (embedding, every block with its memory layers'
scoring + selection + value bag, the final norm, the LM head and the argmax that picks the next token) has fixed
shapes and replays as one captured graph. The model's own modules run inside it, unchanged: the same kernels as
the eager path, except that attention reads the masked static cache.

    dec = GraphDecoder(model, batch=1, max_len=2304)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        dec.prefill(prompt_ids)            # (B, P) -> logits of the prompt; next tokens in dec.tokens
        for _ in range(256):
            nxt = dec.step()                # (B, 1) greedy tokens, device tensor (replays the graph)
"""
import torch

from .model import Transformer


class GraphDecoder:
    def __init__(self, model: Transformer, batch: int, max_len: int = None, dtype=None):
        cfg = model.cfg
        if cfg.eng_layers:
            raise ValueError("GraphDecoder: Engram memories keep growing caches (decode them with the KV-cache loop)")
        if model.training:
            raise ValueError("GraphDecoder: put the model in eval mode first (BatchNorm uses its running statistics)")
        self.model = model
        self.batch = batch
        self.max_len = max_len or cfg.max_seq_len
        if self.max_len > cfg.max_seq_len:
            raise ValueError(f"max_len {self.max_len} exceeds the model's max_seq_len {cfg.max_seq_len}")
        dev = model.tok_emb.weight.device
        if dev.type != "cuda":
            raise ValueError("GraphDecoder runs on CUDA")
        if dtype is None:
            dtype = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else torch.float32
        hd = cfg.d_model // cfg.n_heads
        arange = torch.arange(self.max_len, device=dev)
        self.caches = [{"kbuf": torch.zeros(batch, cfg.n_heads, self.max_len, hd, dtype=dtype, device=dev),
                        "vbuf": torch.zeros(batch, cfg.n_heads, self.max_len, hd, dtype=dtype, device=dev),
                        "arange": arange, "pos": None} for _ in range(cfg.n_layers)]
        self.tokens = torch.zeros(batch, 1, dtype=torch.long, device=dev)   # the next step's input tokens
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)            # their position
        self.logits = None
        self.length = 0
        self._graph = None
        self._key = None

    def _set_pos(self, pos):
        for c in self.caches:
            c["pos"] = pos

    @torch.no_grad()
    def prefill(self, ids):
        """ids (B, P): fills the caches for positions 0 .. P-1 (eager) and sets the next tokens to the greedy
        choice after the prompt. Returns the prompt's logits (B, P, vocab)."""
        B, P = ids.shape
        if B != self.batch or P >= self.max_len:
            raise ValueError(f"prefill: ids {tuple(ids.shape)} for batch {self.batch}, max_len {self.max_len}")
        self._set_pos(torch.arange(P, device=ids.device))
        logits = self.model(ids, kv_caches=self.caches)
        self.tokens.copy_(logits[:, -1:].argmax(-1))
        self.pos.fill_(P)
        self.length = P
        return logits

    def _body(self):
        self._set_pos(self.pos)
        self.logits = self.model(self.tokens, kv_caches=self.caches)
        self.tokens.copy_(self.logits[:, -1:].argmax(-1))
        self.pos.add_(1)

    @torch.no_grad()
    def step(self, tokens=None):
        """One greedy step: feeds self.tokens (or `tokens`, (B, 1)) at the current position and leaves the
        argmax of its logits in self.tokens (returned; self.logits holds the logits). The first call captures
        the graph (with the memory layers' own one-token graphs switched off inside it)."""
        if self.length + 1 > self.max_len:
            raise ValueError("GraphDecoder: the static cache is full")
        if tokens is not None:
            self.tokens.copy_(tokens)
        ac = torch.is_autocast_enabled("cuda")
        key = (ac, torch.get_autocast_dtype("cuda") if ac else None)
        if self._graph is None or self._key != key:
            self._capture(key)
        self._graph.replay()
        self.length += 1
        return self.tokens

    def _capture(self, key):
        mems = self.model.memory_layers()
        flags = [getattr(m, "decode_graph", False) for m in mems]
        for m in mems:
            m.decode_graph = False
        ctx = (torch.autocast("cuda", dtype=key[1], cache_enabled=False) if key[0]
               else torch.autocast("cuda", enabled=False))
        saved_tok, saved_pos = self.tokens.clone(), self.pos.clone()
        try:
            s = torch.cuda.Stream(self.tokens.device)
            s.wait_stream(torch.cuda.current_stream(self.tokens.device))
            with torch.cuda.stream(s), ctx:
                for _ in range(2):              # warm-up: writes cache slots past the position, masked until used
                    self._body()
                    self.pos.copy_(saved_pos)
            torch.cuda.current_stream(self.tokens.device).wait_stream(s)
            self.tokens.copy_(saved_tok)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph), ctx:
                self._body()
            self.tokens.copy_(saved_tok)
            self.pos.copy_(saved_pos)
        finally:
            for m, f in zip(mems, flags):
                m.decode_graph = f
        self._graph, self._key = graph, key
