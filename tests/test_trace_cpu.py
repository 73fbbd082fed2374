"""CPU: the router-trace records -- the flattened ExpertSelectionTrace schema
of the reference (expert_selection.py:52-157, context.py:31-95: column
order, types, schema-version metadata), one record per (batch, offset) token
with the recorder's sequence / token / event numbering (recorder.py:160-216),
the record checks of ExpertSelectionTrace.__attrs_post_init__, and a Parquet
round trip.  Captures here are host tensors (no ring); the GPU test covers
the kernel writing into the pinned ring."""

import numpy as np
import pytest
import torch

from preemptlm_b200.trace import (EXPERT_SELECTION_TRACE_SCHEMA_VERSION, ExpertTraceRecorder, ListTraceSink,
                                  ParquetTraceSink, TraceRunContext, TraceStepContext, arrow_schema,
                                  validate_record)

# the reference schema, flattened in attrs field order
REFERENCE_COLUMNS = [
    ("schema_version", "int16"), ("run_id", "string"), ("instrumentation_version", "string"),
    ("model_id", "string"), ("model_architecture", "string"), ("model_revision", "string"),
    ("sequence_id", "int32"), ("token_idx", "int32"), ("token_id", "int64"), ("event_idx", "int64"),
    ("timestamp", "timestamp[us, tz=UTC]"), ("path", "string"), ("module_class", "string"),
    ("transformer_block_idx", "int32"), ("expert_ids", "list<item: int32 not null>"),
    ("softmax_weights", "list<item: float not null>"), ("gate_logits", "list<item: float>"),
]


def test_schema_matches_the_reference_columns():
    sch = arrow_schema()
    assert [(f.name, str(f.type)) for f in sch] == REFERENCE_COLUMNS
    assert sch.metadata[b"preempt.schema_version"] == str(EXPERT_SELECTION_TRACE_SCHEMA_VERSION).encode()
    assert sch.field("model_revision").nullable and sch.field("gate_logits").nullable
    assert not sch.field("expert_ids").nullable


def _recorder():
    rc = TraceRunContext.with_generated_run_id(run_id_prefix="t", model_id="m", model_architecture="qwen3_next")
    rec = ExpertTraceRecorder(rc, top_k=2, num_experts=8, capacity_tokens=16)
    rec._ring = None  # host tensors only
    return rec


def test_records_per_token_with_running_indices(tmp_path):
    rec = _recorder()
    with pytest.raises(RuntimeError):
        rec.capture(layer_path="l", layer_class="c", block_idx=0, expert_ids=torch.zeros(1, 1, 2),
                    softmax_weights=torch.ones(1, 1, 2))
    rec.start_trace(TraceStepContext(sequence_id=3, token_idx=10, token_id=7))
    ids = torch.tensor([[[1, 4], [0, 2], [5, 6]], [[7, 3], [2, 1], [0, 6]]], dtype=torch.int32)  # [B=2, S=3, k]
    w = torch.rand(2, 3, 2) + 0.1
    logits = torch.randn(2, 3, 8)
    rec.capture(layer_path="model.layers.0.mlp", layer_class="Qwen3NextSparseMoeBlock", block_idx=0,
                expert_ids=ids, softmax_weights=w, gate_logits=logits)
    rec.capture(layer_path="model.layers.1.mlp", layer_class="Qwen3NextSparseMoeBlock", block_idx=1,
                expert_ids=ids, softmax_weights=w, gate_logits=None)
    sink = ListTraceSink()
    assert rec.flush(sink) == 12
    r = sink.records
    assert [x["event_idx"] for x in r] == list(range(12))
    assert [(x["sequence_id"], x["token_idx"]) for x in r[:6]] == [(3, 10), (3, 11), (3, 12), (4, 10), (4, 11),
                                                                  (4, 12)]
    assert all(x["token_id"] == 7 for x in r)
    assert r[4]["expert_ids"] == [2, 1] and np.allclose(r[4]["softmax_weights"], w[1, 1].numpy())
    assert np.allclose(r[4]["gate_logits"], logits[1, 1].numpy()) and r[7]["gate_logits"] is None
    assert r[7]["transformer_block_idx"] == 1 and r[7]["path"] == "model.layers.1.mlp"
    # the step is closed by flush; event numbering continues in the next step
    with pytest.raises(RuntimeError):
        rec.flush(ListTraceSink())
    rec.start_trace(TraceStepContext(sequence_id=0, token_idx=13))
    rec.capture(layer_path="l", layer_class="c", block_idx=0, expert_ids=ids[:1, :1], softmax_weights=w[:1, :1])
    pq_path = tmp_path / "t.parquet"
    sink = ParquetTraceSink(pq_path)
    assert rec.flush(sink) == 1
    sink.close()
    import pyarrow.parquet as pq

    t = pq.read_table(pq_path)
    assert t.schema.equals(arrow_schema(), check_metadata=False)
    assert t.column("event_idx").to_pylist() == [12] and t.column("expert_ids").to_pylist() == [[1, 4]]


@pytest.mark.parametrize("bad", [dict(expert_ids=[1, 1], softmax_weights=[0.5, 0.5]),
                                 dict(expert_ids=[1, -2], softmax_weights=[0.5, 0.5]),
                                 dict(expert_ids=[1, 2], softmax_weights=[0.5, -0.1]),
                                 dict(expert_ids=[1, 2], softmax_weights=[0.0, 0.0]),
                                 dict(expert_ids=[1, 2, 3], softmax_weights=[0.5, 0.5])])
def test_record_checks_of_the_reference(bad):
    with pytest.raises(ValueError):
        validate_record(bad)
