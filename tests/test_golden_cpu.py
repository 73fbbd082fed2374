"""CPU: the oracle and the host logic against the reference's golden fixtures
(tests/golden/, generated from the reference's own code by make_golden.py)."""

import json
import shutil
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import slotted_glu_oracle as orc
from preemptlm_b200 import bank as B
from preemptlm_b200.cache_manager import CacheEvictionPolicy, ExpertCacheManager
from preemptlm_b200.quant import dequantize_affine, quantize_affine
from preemptlm_b200.slot_map import SlotCorruptionError, SlotTable

GOLDEN = Path(__file__).resolve().parent / "golden"


def _steps():
    z = np.load(GOLDEN / "admission_steps.npz")
    n = int(z["n_steps"])
    return z, n


def _replay(table, z, i):
    table._eid_lookup_table = z[f"pre_eid_{i}"].copy()
    table._sid_lookup_table = z[f"pre_sid_{i}"].copy()
    table._slot_freq = z[f"pre_freq_{i}"].copy()
    table._slot_recency = z[f"pre_rec_{i}"].copy()
    table._clock = int(z[f"pre_clock_{i}"])


def test_oracle_admission_matches_reference_every_step():
    """The oracle's maybe_admit/choose_slots/touch reproduce the reference's
    tables, unique/inverse and slot choices on every recorded step."""
    z, n = _steps()
    E, S = int(z["num_experts"]), int(z["num_slots"])
    assert n >= 30
    for i in range(n):
        t = orc.SlotTables(E, S)
        t.eid_lookup, t.sid_lookup = z[f"pre_eid_{i}"].copy(), z[f"pre_sid_{i}"].copy()
        t.freq, t.recency, t.clock = z[f"pre_freq_{i}"].copy(), z[f"pre_rec_{i}"].copy(), int(z[f"pre_clock_{i}"])
        unique, inverse, missed, acquired, _ = t.maybe_admit(z[f"routed_{i}"])
        assert np.array_equal(unique, z[f"unique_{i}"]), i
        assert np.array_equal(inverse, z[f"inverse_{i}"].reshape(-1)), i
        assert np.array_equal(np.asarray(acquired), z[f"chosen_{i}"]), i
        t.touch(t.eid_lookup[unique])
        for a, b in (("eid_lookup", "post_eid"), ("sid_lookup", "post_sid"), ("freq", "post_freq"),
                     ("recency", "post_rec")):
            assert np.array_equal(getattr(t, a), z[f"{b}_{i}"]), (i, a)
        assert t.clock == int(z[f"post_clock_{i}"])


def test_product_slot_table_reference_policy():
    """The product's 'reference' policy returns the reference's slot ids on
    every safe step and raises where the reference overwrites a slot in use."""
    z, n = _steps()
    E, S = int(z["num_experts"]), int(z["num_slots"])
    n_safe = n_corrupt = 0
    for i in range(n):
        t = SlotTable(E, S, slot_policy="reference")
        _replay(t, z, i)
        unique = z[f"unique_{i}"]
        missed = unique[t._eid_lookup_table[unique] < 0]
        if missed.size == 0:
            continue
        if bool(z[f"corrupt_{i}"]):
            with pytest.raises(SlotCorruptionError):
                t._choose_slots(missed.size, protected=unique)
            n_corrupt += 1
        else:
            assert np.array_equal(t._choose_slots(missed.size, protected=unique), z[f"chosen_{i}"]), i
            n_safe += 1
    assert n_safe > 0 and n_corrupt > 0


def test_product_lfru_policy_never_evicts_protected():
    z, n = _steps()
    E, S = int(z["num_experts"]), int(z["num_slots"])
    for i in range(n):
        t = SlotTable(E, S, slot_policy="lfru")
        _replay(t, z, i)
        unique = z[f"unique_{i}"]
        missed = unique[t._eid_lookup_table[unique] < 0]
        if missed.size == 0:
            continue
        chosen = t._choose_slots(missed.size, protected=unique)
        prot = t._eid_lookup_table[unique]
        assert np.unique(chosen).size == chosen.size
        assert not np.isin(chosen, prot[prot >= 0]).any()


def test_touch_matches_reference():
    z, n = _steps()
    E, S = int(z["num_experts"]), int(z["num_slots"])
    t = SlotTable(E, S)
    _replay(t, z, 0)
    t._eid_lookup_table = z["post_eid_0"].copy()
    slots = t._eid_lookup_table[z["unique_0"]]
    t._touch(slots)
    assert np.array_equal(t._slot_freq, z["post_freq_0"])
    assert np.array_equal(t._slot_recency, z["post_rec_0"])


# ----------------------------------------------------------------------------- cache manager

def _cm_golden():
    return json.loads((GOLDEN / "cache_manager.json").read_text())


def _scripted(policy):
    m = ExpertCacheManager(budget_bytes=300, policy=policy, sample_size=8)
    m.admit(0, 100)
    for _ in range(3):
        m.touch(0)
    m.admit(1, 100)
    m.admit(2, 100)
    m.touch(2)
    m.touch(1)
    return list(m.admit(9, 100))


def test_cache_manager_lfru_lru_known_answers():
    g = _cm_golden()
    assert _scripted(CacheEvictionPolicy.LFRU) == g["lfru_victims"] == [2]
    assert _scripted(CacheEvictionPolicy.LRU) == g["lru_victims"] == [0]
    m = ExpertCacheManager(budget_bytes=200, sample_size=8)
    m.admit(0, 100)
    m.admit(1, 100)
    m.touch(0)
    m.touch(1)
    assert list(m.admit(2, 100)) == g["lfru_tie_victims"] == [0]


@pytest.mark.parametrize("seed", [0, 1])
def test_cache_manager_sampled_sequence(seed):
    g = _cm_golden()[f"sampled_seed{seed}"]
    m = ExpertCacheManager(budget_bytes=800, sample_size=3, seed=seed)
    ev = []
    for i in range(24):
        c = i % 12
        if not m.touch(c):
            ev.extend(m.admit(c, 100))
    assert ev == g["evicted"]
    assert (m.hits, m.misses, m.evictions, m.bytes_read) == (g["hits"], g["misses"], g["evictions"], g["bytes_read"])


def test_cache_manager_errors():
    with pytest.raises(ValueError):
        ExpertCacheManager(budget_bytes=0)
    with pytest.raises(ValueError):
        ExpertCacheManager(budget_bytes=1, sample_size=0)
    m = ExpertCacheManager(budget_bytes=100)
    with pytest.raises(ValueError):
        m.admit(0, 200)
    m.admit(0, 100, priority=B.ReadPriority.DEMAND)
    with pytest.raises(RuntimeError):
        m.admit(1, 100)


# ----------------------------------------------------------------------------- bank format

def test_reads_reference_written_bank():
    bank = B.PreadExpertBank(GOLDEN / "bank", pinned=False)
    m = bank.manifest
    assert m.encoding == "mlx-affine-q4-g64-bfloat16"
    assert [s.name for s in m.tensor_specs] == [f"{p}.{x}" for p in ("gate_proj", "up_proj", "down_proj")
                                                  for x in ("weight", "scales", "biases")]
    raw = (GOLDEN / "bank" / "experts.bin").read_bytes()
    for i, blob in enumerate(bank.blob_index):
        assert blob.offset % 4096 == 0
        e = bank.read_sync(i)
        assert bytes(e.data.numpy()) == raw[blob.offset: blob.offset + blob.length]
        arrays = B.decode_serialized_expert(e, B.parse_encoding_tag(m.encoding))
        assert arrays["gate_proj.weight"].dtype == np.uint32
    with pytest.raises(KeyError):
        bank.read_sync(len(bank.blob_index))
    bank.close()
    with pytest.raises(RuntimeError):
        bank.read_into(0, torch.empty(10, dtype=torch.uint8))


def test_writer_reproduces_reference_bank(tmp_path):
    src = B.PreadExpertBank(GOLDEN / "bank", pinned=False)
    m = src.manifest
    with B.ExpertBankWriter(tmp_path / "b", model_id=m.model_id, model_fingerprint=m.model_fingerprint,
                            encoding=m.encoding, tensor_specs=m.tensor_specs, model_moe_spec=m.model_moe_spec,
                            alignment=m.alignment) as w:
        for i, blob in enumerate(m.blob_index):
            w.add_expert(blob.block_idx, blob.expert_idx, bytes(src.read_sync(i).data.numpy()))
    assert (tmp_path / "b" / "experts.bin").read_bytes() == (GOLDEN / "bank" / "experts.bin").read_bytes()
    ours = json.loads((tmp_path / "b" / "manifest.json").read_text())
    ref = json.loads((GOLDEN / "bank" / "manifest.json").read_text())
    assert ours == ref


def test_writer_rejects_bad_input(tmp_path):
    specs = (B.TensorSpec("w", "uint8", (3,), 3),)
    topo = B.ModelMoESpec((0,), 2, 1)
    w = B.ExpertBankWriter(tmp_path / "s", model_id="m", model_fingerprint="fp", encoding="mlx-unquantized-uint8",
                           tensor_specs=specs, model_moe_spec=topo, alignment=8)
    with pytest.raises(ValueError):
        w.add_expert(0, 0, b"toolong")
    w.add_expert(0, 0, b"aaa")
    with pytest.raises(ValueError, match="[Dd]uplicate"):
        w.add_expert(0, 0, b"aaa")
    with pytest.raises(RuntimeError):
        w.finalize()
    with pytest.raises(FileExistsError):
        B.ExpertBankWriter(tmp_path / "s", model_id="m", model_fingerprint="fp", encoding="e", tensor_specs=specs,
                           model_moe_spec=topo)


def test_short_read_raises_ioerror(tmp_path):
    shutil.copytree(GOLDEN / "bank", tmp_path / "bank")
    last = B.ExpertBankManifest.load(tmp_path / "bank").blob_index[-1]
    with open(tmp_path / "bank" / "experts.bin", "r+b") as f:
        f.truncate(last.offset + 100)
    bank = B.PreadExpertBank(tmp_path / "bank", pinned=False)
    bank.read_sync(0)
    with pytest.raises(IOError):
        bank.read_sync(len(bank.blob_index) - 1)


def test_encoding_tags_match_reference():
    g = json.loads((GOLDEN / "encoding_tags.json").read_text())
    for tag, want in g["good"].items():
        e = B.parse_encoding_tag(tag)
        assert {"backend": e.backend, "mode": e.mode, "bits": e.bits, "group_size": e.group_size,
                "dtype": e.dtype} == want
    for tag in g["bad"]:
        with pytest.raises(ValueError):
            B.parse_encoding_tag(tag)
    assert B.make_encoding_tag(4, 64) == "mlx-affine-q4-g64-bfloat16"
    assert B.make_encoding_tag(None) == "mlx-unquantized-bfloat16"


# ----------------------------------------------------------------------------- quantisation / numerics

@pytest.mark.parametrize("bits", [4, 8])
def test_torch_quantizer_matches_oracle(bits):
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(48, 256, generator=g) * 0.02).to(torch.bfloat16)
    w[3, :64] = 0.01  # a constant group (scale 0)
    q, s, b = quantize_affine(w, bits, 64)
    wb = w.view(torch.int16).numpy().view(np.uint16)
    q2, s2, b2 = orc.quantize_affine(wb, bits, 64)
    assert np.array_equal(q.numpy().view(np.uint32), q2)
    assert np.array_equal(s.view(torch.int16).numpy().view(np.uint16), s2)
    assert np.array_equal(b.view(torch.int16).numpy().view(np.uint16), b2)
    deq = dequantize_affine(q, s, b, bits).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(orc.f32_to_bf16_bits(orc.dequant_affine(q2, s2, b2, bits)), deq)
    err = np.abs(orc.dequant_affine(q2, s2, b2, bits) - orc.bf16_bits_to_f32(wb)).max()
    step = orc.bf16_bits_to_f32(s2).max()
    assert err <= 0.5 * step + 1e-3


def test_routing_exp_error_bound():
    x = np.linspace(-87.0, 0.0, 400001).astype(np.float32)
    e = orc.sg_exp(x).astype(np.float64)
    r = np.exp(x.astype(np.float64))
    assert (np.abs(e - r) / r).max() < 4 * 2.0 ** -24
    assert orc.sg_exp(np.float32(-200.0)) == 0.0


def test_oracle_topk_tie_order():
    # eight experts share the top gate exactly: lower ids win
    E, k = 64, 4
    logits = np.zeros((1, E), np.float32)
    logits[0, [50, 7, 33, 12, 9, 40, 2, 61]] = 3.0
    inds, sc, _ = orc.get_routings(orc.f32_to_bf16_bits(logits), k, True)
    assert inds.tolist() == [[2, 7, 9, 12]]
    s = orc.bf16_bits_to_f32(sc)[0]
    assert np.all(s == s[0])


def test_bf16_rounding_ties_to_even():
    vals = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -0.0, np.inf, np.nan], np.float32)
    r = orc.bf16_round(vals)
    assert r[0] == 1.0 and r[1] == 1.0 + 2.0 ** -6 and np.isinf(r[3]) and np.isnan(r[4])
    t = torch.tensor(vals[:4]).to(torch.bfloat16).float().numpy()
    assert np.array_equal(r[:4], t)
