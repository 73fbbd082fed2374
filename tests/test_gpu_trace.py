"""GPU: router-trace capture on the device.  The fused routing kernel writes
each token's expert ids, renormalised scores and raw logits into the
recorder's pinned host ring while it routes; the flushed ExpertSelectionTrace
records must equal the oracle's routing of the same tokens bit for bit (ids
exactly, scores and logits as the exact bf16 values), for two layer calls
(blocks) of one step and a second step after the flush reused the ring."""

import numpy as np
import pytest
import torch

from oracle import slotted_glu_oracle as orc
from preemptlm_b200.layer import Qwen3_xMoEWrapper
from preemptlm_b200.synthetic import LayerConfig, make_layer, make_tokens
from preemptlm_b200.trace import ExpertTraceRecorder, ListTraceSink, TraceRunContext, TraceStepContext

from ._util import bits16

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("with_logits", [True, False])
def test_trace_ring_records_match_oracle_routing(with_logits):
    cfg = LayerConfig("trace", 3, 512, 64, 4, 128, 128, 8, 64)
    block, tens = make_layer(cfg, device="cuda")
    rc = TraceRunContext.with_generated_run_id(run_id_prefix="gpu", model_id="synthetic", model_architecture="x")
    rec = ExpertTraceRecorder(rc, top_k=cfg.top_k, num_experts=cfg.num_experts, capacity_tokens=64)
    moes = [Qwen3_xMoEWrapper(block, "fp", f"model.layers.{i}.mlp", i, recorder=rec, capture_gate_logits=with_logits)
            for i in range(2)]
    rb = bits16(tens["router"])
    for step in range(2):
        B, S = 2, 5 + step
        rec.start_trace(TraceStepContext(sequence_id=10 * step, token_idx=3, token_id=11))
        xs = [make_tokens(cfg, B * S, step=20 * step + i).view(B, S, cfg.hidden) for i in range(2)]
        outs = [m(x) for m, x in zip(moes, xs)]
        sink = ListTraceSink()
        assert rec.flush(sink) == 2 * B * S
        recs = sink.records
        for i, x in enumerate(xs):
            lg = orc.router_logits(bits16(x.reshape(B * S, -1)), rb)
            ids, sc, _ = orc.get_routings(lg, cfg.top_k, True)
            for t in range(B * S):
                r = recs[i * B * S + t]
                assert r["path"] == f"model.layers.{i}.mlp" and r["transformer_block_idx"] == i
                assert (r["sequence_id"], r["token_idx"]) == (10 * step + t // S, 3 + t % S)
                assert r["expert_ids"] == ids[t].tolist()
                assert np.array_equal(np.asarray(r["softmax_weights"], np.float32), orc.bf16_bits_to_f32(sc[t]))
                if with_logits:
                    assert np.array_equal(np.asarray(r["gate_logits"], np.float32), orc.bf16_bits_to_f32(lg[t]))
                else:
                    assert r["gate_logits"] is None
        assert [r["event_idx"] for r in recs] == list(range(recs[0]["event_idx"], recs[0]["event_idx"] + len(recs)))
        del outs
