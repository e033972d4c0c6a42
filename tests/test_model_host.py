"""The model's checkpoint layout against the reference's (no GPU): state_dict keys, shapes and dtypes,
param_counts() and macs_per_token() of small Transformers built on the CPU (one memory layer, two layers sharing a
table, Engram layers, no BatchNorm / swilu, learned score scale), equal to tests/golden/model_structure.json (made
by tests/golden/make_golden.py from the reference's smlm/model.py), so that checkpoints load across."""
import json
import os

import pytest
import torch

import smlm_b200.engram as E
from conftest import GOLDEN
from smlm_b200.model import ModelConfig, Transformer

GOLD = json.load(open(os.path.join(GOLDEN, "model_structure.json")))


@pytest.mark.parametrize("name", sorted(GOLD))
def test_checkpoint_layout_matches_reference(name, monkeypatch):
    # token compression needs tiktoken's GPT-2 vocabulary (offline: unavailable); the layout does not depend on it
    monkeypatch.setattr(E, "canonical_ids", lambda vocab: (torch.arange(vocab, dtype=torch.int64), vocab))
    want = GOLD[name]
    torch.manual_seed(0)
    m = Transformer(ModelConfig(**want["config"]))
    assert [[k, list(v.shape), str(v.dtype)] for k, v in m.state_dict().items()] == want["state_dict"]
    assert m.param_counts() == want["param_counts"]
    assert m.macs_per_token() == want["macs_per_token"]
    assert m.macs_per_token(64) == want["macs_per_token_64"]
