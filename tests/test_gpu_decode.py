"""Whole-step CUDA-graph decoding (smlm_b200.decode.GraphDecoder): the static-cache step gives the logits of the
reference-style KV-cache loop (smlm/train.py:283-315: model(token, kv_caches, pos0) one token at a time), and the
captured graph replays exactly what the same step computes eagerly."""
import pytest
import torch

from smlm_b200.decode import GraphDecoder
from smlm_b200.model import ModelConfig, Transformer

pytestmark = pytest.mark.gpu
DEV = "cuda"


def small_model():
    # k_dim 256 (halves of 128): the bf16 path takes the fused tensor-core scoring
    cfg = ModelConfig(vocab_size=256, d_model=64, n_layers=4, n_heads=4, ffn_hidden=128, max_seq_len=48,
                      mem_layers=[1, 3], mem_n_keys=64, mem_heads=2, mem_knn=8, mem_k_dim=256,
                      mem_share_values=True, mem_value_grad="row_sparse")
    torch.manual_seed(0)
    return Transformer(cfg).to(DEV).eval()


def eager_loop(m, prompt, tokens):
    caches = [dict() for _ in range(m.cfg.n_layers)]
    out = [m(prompt, kv_caches=caches, pos0=0)[:, -1:]]
    for i, t in enumerate(tokens):
        out.append(m(t, kv_caches=caches, pos0=prompt.shape[1] + i))
    return out


@pytest.mark.parametrize("batch", [1, 3])
def test_graph_decoder_matches_kv_cache_loop_fp32(batch):
    m = small_model()
    prompt = torch.randint(0, 256, (batch, 12), generator=torch.Generator().manual_seed(batch)).to(DEV)
    with torch.no_grad():
        dec = GraphDecoder(m, batch, max_len=40)
        logits = [dec.prefill(prompt)[:, -1:]]
        fed = []
        for _ in range(10):
            fed.append(dec.tokens.clone())
            dec.step()
            logits.append(dec.logits.clone())
        ref = eager_loop(m, prompt, fed)
    for i, (a, b) in enumerate(zip(logits, ref)):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-4, msg=f"step {i}")
    for lg, t in zip(logits[:-1], fed):          # greedy: every fed token is the argmax of the step before
        assert torch.equal(lg.argmax(-1), t)


def test_graph_replay_equals_eager_step_bf16():
    """Under bf16 autocast the captured step is bit-identical to running the same static-cache step eagerly."""
    m = small_model()
    prompt = torch.randint(0, 256, (2, 9), generator=torch.Generator().manual_seed(5)).to(DEV)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        g, e = GraphDecoder(m, 2, max_len=32), GraphDecoder(m, 2, max_len=32)
        torch.testing.assert_close(g.prefill(prompt), e.prefill(prompt), rtol=0, atol=0)
        for i in range(8):
            g.step()
            e._body()
            assert torch.equal(g.logits, e.logits), f"step {i}"
            assert torch.equal(g.tokens, e.tokens)


def test_graph_decoder_rejects_overflow():
    m = small_model()
    with torch.no_grad():
        dec = GraphDecoder(m, 1, max_len=8)
        dec.prefill(torch.zeros(1, 6, dtype=torch.long, device=DEV))
        dec.step()
        dec.step()
        with pytest.raises(ValueError, match="full"):
            dec.step()
