"""Host arithmetic of smlm_b200.optim against the reference's (no GPU): value_table_memory of small models for every
value_state / value_optim (one row-sparse memory table, two layers sharing a table, a dense-gradient table; the
refused combinations refused alike) and the warmup + cosine lr_multiplier, bit for bit, against
tests/golden/budget.json (made by tests/golden/make_golden.py from the reference's smlm/optim.py)."""
import json
import os

import pytest
import torch

from conftest import GOLDEN
from smlm_b200 import optim as O
from smlm_b200.model import ModelConfig, Transformer

GOLD = json.load(open(os.path.join(GOLDEN, "budget.json")))


@pytest.mark.parametrize("name", sorted(GOLD["models"]))
def test_value_table_memory_matches_reference(name):
    torch.manual_seed(0)
    m = Transformer(ModelConfig(**GOLD["models"][name]))
    for vs in ("fp32", "bf16", "int8"):
        for vo in ("adam", "rowrms", "rowadagrad"):
            want = GOLD["memory"][f"{name}/{vs}/{vo}"]
            if "error" in want:
                with pytest.raises(ValueError):
                    O.value_table_memory(m, vs, value_optim=vo)
            else:
                assert O.value_table_memory(m, vs, value_optim=vo) == want, (name, vs, vo)


def test_lr_multiplier_matches_reference():
    for case in GOLD["lr"]:
        got = [O.lr_multiplier(s, case["total"], case["warmup"], case["min_ratio"])
               for s in range(case["total"] + 2)]
        assert got == case["mult"]
