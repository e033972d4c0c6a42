"""Host-RAM value tables, the parts that need no GPU: enable_host_values checks the model before changing it and
keeps the table fp32 on the host through device and dtype moves; the GACC step accumulator (StepRows) on the CPU:
slots, overflow summed per row, reset; host_timings; the optimizer memory split (reference:
tests/test_host_values.py, tests/test_hot_rows.py)."""
import pytest
import torch

from smlm_b200.host_optim import HostRowStore, value_table_memory_by_device
from smlm_b200.host_values import HostEmbedding, StepRows, enable_host_values, host_timings
from smlm_b200.model import ModelConfig, Transformer


def tiny(**kw):
    cfg = dict(vocab_size=64, d_model=32, n_layers=4, n_heads=4, ffn_hidden=48, max_seq_len=24, mem_layers=[0, 2, 3],
               mem_n_keys=16, mem_heads=2, mem_knn=4, mem_k_dim=16, mem_share_values=True,
               mem_value_grad="row_sparse")
    cfg.update(kw)
    torch.manual_seed(0)
    return Transformer(ModelConfig(**cfg))


def test_opt_in_keeps_the_table_fp32_on_the_host():
    model = enable_host_values(tiny())
    tables = {id(m.values) for m in model.memory_layers()}
    assert len(tables) == 1                                  # the shared table: one HostEmbedding
    emb = model.memory_layers()[0].values
    assert isinstance(emb, HostEmbedding) and emb.weight.host_values
    model = model.double()
    assert emb.weight.dtype == torch.float32 and emb.weight.device.type == "cpu"
    assert all(m.decode_graph is False for m in model.memory_layers())
    assert set(host_timings(model)) == {"unique", "indices_d2h", "gather", "rows_h2d", "gradients_d2h", "scatter"}
    split = value_table_memory_by_device(model, "fp32")
    assert split["device"]["table_bytes"] == 0 and split["host"]["table_bytes"] == emb.weight.numel() * 4


@pytest.mark.parametrize("invalid", ["dense", "engram", "width"])
def test_unsupported_models_are_refused_before_any_change(invalid, monkeypatch):
    import smlm_b200.engram as E
    # token compression needs tiktoken's GPT-2 vocabulary (offline: unavailable); the check does not depend on it
    monkeypatch.setattr(E, "canonical_ids", lambda vocab: (torch.arange(vocab, dtype=torch.int64), vocab))
    if invalid == "dense":
        model = tiny(mem_value_grad="dense")
    elif invalid == "engram":
        model = tiny(eng_layers=[1])
    else:
        model = tiny(d_model=30, n_heads=3, mem_v_dim=30)
    before = [type(m.values) for m in model.memory_layers()]
    with pytest.raises(ValueError):
        enable_host_values(model)
    assert [type(m.values) for m in model.memory_layers()] == before


def test_step_rows_slots_overflow_and_reset():
    sr = StepRows(num_rows=50, dim=3, capacity=4, device=torch.device("cpu"))
    sr.add(torch.tensor([7, 2, 9]), torch.ones(3, 3))
    sr.add(torch.tensor([2, 11, 30, 40]), torch.full((4, 3), 2.0))    # 11 takes the last slot; 30, 40 overflow
    assert sr.n == 4 and sr.rows[:4].tolist() == [7, 2, 9, 11]
    assert torch.equal(sr.acc[1], torch.full((3,), 3.0))
    sr.add(torch.tensor([30, 7]), torch.full((2, 3), 5.0))
    rows, sums = sr.spilled()
    assert rows.tolist() == [30, 40]
    assert torch.equal(sums[0], torch.full((3,), 7.0)) and torch.equal(sums[1], torch.full((3,), 2.0))
    assert sr.peak == 6
    sr.reset()
    assert sr.n == 0 and sr.spilled() is None and sr.spilled_steps == 1
    assert int((sr.slot >= 0).sum()) == 0 and torch.count_nonzero(sr.acc) == 0


def test_host_row_store_reads_zeros_where_rows_were_stepped():
    """The optimizer steps leave stepped rows' accumulator values in place (the next add overwrites them); reading
    `acc` shows zeros there, as the reference's store, and keeps the touched rows."""
    st = HostRowStore(torch.zeros(6, 4))
    st._acc[:] = torch.arange(24.0).view(6, 4)
    st.touched[[1, 4]] = True
    st.stale = True
    acc = st.acc
    assert torch.equal(acc[[1, 4]], torch.arange(24.0).view(6, 4)[[1, 4]])
    assert torch.count_nonzero(acc[[0, 2, 3, 5]]) == 0 and not st.stale
    st.reset()
    assert st.stale and not st.touched.any() and torch.count_nonzero(st.acc) == 0
