"""Host side of the Engram n-gram hash (no GPU): a caller-given token compression table."""
import pytest
import torch

from smlm_b200.engram import NgramHash


def test_given_compression_table():
    ng = NgramHash(100, orders=(2, 3), heads=2, rows=11, seed=0, canon=(torch.arange(100), 100))
    assert ng.pad == 100 and torch.equal(ng.canon, torch.arange(100))
    assert ng.history == 2 and ng.n_lookups == 4
    # the multipliers do not depend on the compression table: odd, below 2^31, the reference's draw
    assert bool((ng.mult % 2 == 1).all()) and int(ng.mult.max()) < 2 ** 31
    with pytest.raises(ValueError):
        NgramHash(100, canon=(torch.arange(99), 99))            # one id per token id
    with pytest.raises(ValueError):
        NgramHash(100, canon=(torch.arange(100), 1 << 16))      # ids must stay below 2^16
    with pytest.raises(ValueError, match="CUDA"):
        ng(torch.zeros(1, 5, dtype=torch.int64))
