"""GPU: the streaming branch of the wrapper (qwen3_x_moe.py:136-208, 276-280).

Experts live in an expert bank on disk written by ExpertBankWriter; the layer
holds fewer slots than experts, so steps miss, read blobs through
DiskBackedExpertLoader (pread into pinned host buffers), evict, refill slots
with sg_refill_h2d and run the gathered GLU over the slot arena.  Every step's
output must match the oracle computed with all experts resident.
"""

import numpy as np
import pytest
import torch

from oracle import slotted_glu_oracle as orc
from preemptlm_b200 import ops
from preemptlm_b200.bank import (ExpertBankWriter, ModelMoESpec, PreadExpertBank, assemble_expert_blob,
                                 derive_tensor_specs, make_encoding_tag)
from preemptlm_b200.cache_manager import ExpertCacheManager
from preemptlm_b200.layer import Qwen3_xMoEWrapper
from preemptlm_b200.loader import DiskBackedExpertLoader, HostExpertCache
from preemptlm_b200.synthetic import LayerConfig, make_layer, make_tokens

from ._util import LazyExperts, assert_close, bits16, f32

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _write_bank(path, cfg, tens, arena):
    names = arena.tensor_names()
    ex = tens["experts"]
    specs = derive_tensor_specs({n: ex[n][0] for n in names}, names)
    spec = ModelMoESpec(moe_block_idxs=(0,), num_routed_experts=cfg.num_experts, top_k=cfg.top_k)
    enc = make_encoding_tag(None if cfg.bits == 16 else cfg.bits, 64)
    with ExpertBankWriter(path, model_id="synthetic", model_fingerprint="fp", encoding=enc, tensor_specs=specs,
                          model_moe_spec=spec) as w:
        for e in range(cfg.num_experts):
            w.add_expert(0, e, assemble_expert_blob({n: ex[n][e] for n in names}, specs))
    return specs


@pytest.mark.parametrize("bits,policy,path,prefetch", [(8, "lfru", "auto", 0), (4, "lfru", "auto", 0),
                                                       (16, "lfru", "auto", 0), (8, "lfru", "tc", 4),
                                                       (4, "lfru", "gemv", 4)])
def test_streaming_layer_matches_oracle(tmp_path, bits, policy, path, prefetch):
    """Steps that miss run the resident experts' pairs first (missed experts
    skipped), read and refill the missed ones meanwhile, then run the missed
    pairs into the same output rows; with ``prefetch`` the layer also queues
    PREFETCH reads of its most often routed non-resident experts."""
    ops.set_glu_path(path)
    cfg = LayerConfig("stream", 7, 512, 32, 4, 128, 128, bits, 12)
    block, tens = make_layer(cfg, device=DEV)
    _write_bank(tmp_path / "bank", cfg, tens, block.switch_mlp)
    bank = PreadExpertBank(tmp_path / "bank")
    cache = HostExpertCache(ExpertCacheManager(budget_bytes=6 * bank.manifest.expert_num_bytes()))
    loader = DiskBackedExpertLoader(expert_bank=bank, cache=cache)
    try:
        factory = Qwen3_xMoEWrapper.make_wrapper_factory(
            model_fingerprint="fp", expert_loader=loader, expert_cache=cache, num_slots=cfg.num_slots,
            slot_size=bank.manifest.expert_num_bytes(), slot_policy=policy, prefetch_experts=prefetch)

        class Cand:
            layer_path, block_idx = "model.layers.0.mlp", 0

        moe = factory(block, Cand())
        experts = LazyExperts(tens["experts"], cfg.bits)
        shared = LazyExperts(tens["shared"], cfg.bits)[0]
        seen = set()
        for step in range(14):
            T = 1 + step % 3
            x = make_tokens(cfg, T, step=step)
            out = moe(x.reshape(1, T, cfg.hidden)).reshape(T, cfg.hidden)
            ref = orc.layer_forward(bits16(x), bits16(tens["router"]), cfg.top_k, cfg.norm_topk_prob, experts,
                                    shared, bits16(tens["shared_gate"]))
            assert_close(f32(out), ref["out"], what=f"step {step}")
            # slot tables stay a bijection between resident experts and slots
            eid2sid, sid2eid = moe._eid_lookup_table, moe._sid_lookup_table
            res = np.nonzero(eid2sid >= 0)[0]
            assert np.all(sid2eid[eid2sid[res]] == res)
            assert np.array_equal(moe.eid2sid_device.cpu().numpy(), eid2sid)
            seen.update(int(e) for e in np.unique(ref["inds"]))
        assert len(seen) > cfg.num_slots  # the run had to evict
        assert moe.admit_stats["missed"] > 0
        assert ops.device_status(reset=True) == 0
    finally:
        ops.set_glu_path("auto")
        loader.close()
        bank.close()
