"""Generate the golden fixtures in this folder from the reference's own code.

Run here (the reference tree must be importable):

    python tests/golden/make_golden.py <reference tree>

(or set PREEMPTLM_REFERENCE to the reference tree and give no argument).

What it pins, and how:

* ``admission_steps.npz`` -- the reference's slot bookkeeping run as-is:
  ``Qwen3_xMoEWrapper._maybe_admit`` (qwen3_x_moe.py:136-208),
  ``BaseMoEWrapper._choose_slots`` / ``_touch`` (base_moe_wrapper.py:152-172),
  ``decode_serialized_expert`` and ``SlottedGLU`` (expert_cache.py:24-80,
  :199-224).  Those functions do all their work in numpy; the ``mlx`` and
  ``mlx_lm`` modules they import are replaced by a small numpy stand-in
  (``mx.asarray`` -> ``np.asarray``, ``mx.eval`` -> no-op, ``mx.zeros`` ->
  ``np.zeros``), which is enough because no MLX arithmetic is reached on that
  path.  Every step stores the pre-state, the routed ids, and the post-state,
  so a test can replay any single step.
* ``cache_manager.json`` -- victims of the reference ``ExpertCacheManager``
  (cache_manager.py:196-310) on the scripted workloads of
  tests/unit/test_expert_cache_manager.py:115-175, with int keys.
* ``bank/`` -- a tiny expert bank written by the reference ``ExpertBankWriter``
  (writer.py:48-153): ``experts.bin`` + ``manifest.json``.
* ``encoding_tags.json`` -- ``parse_encoding_tag`` (encoding.py:61-120) on tags.

The stand-in never runs at test time and nothing here is imported by the
product; the committed outputs are plain arrays and JSON.
"""

from __future__ import annotations

import json
import shutil
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


# --------------------------------------------------------------------------- numpy stand-in for mlx


def _install_mlx_standin() -> None:
    mx = types.ModuleType("mlx.core")

    class _Dt:
        def __init__(self, name):
            self.name = name

        def __repr__(self):
            return f"mx.{self.name}"

    for n in ("bool_", "int8", "int16", "int32", "uint8", "uint16", "uint32",
              "bfloat16", "float16", "float32", "float64"):
        setattr(mx, n, _Dt(n))
    mx.array = np.ndarray
    mx.Dtype = _Dt
    mx.DeviceType = object
    mx.Stream = object
    mx.Device = object
    mx.gpu = "gpu"
    mx.cpu = "cpu"

    def asarray(a, dtype=None, copy=None):
        if isinstance(dtype, _Dt):
            dtype = np.dtype(dtype.name)
        return np.array(a, dtype=dtype, copy=True) if copy else np.asarray(a, dtype=dtype)

    def zeros(shape, dtype=None):
        if isinstance(dtype, _Dt):
            dtype = np.dtype(dtype.name)
        return np.zeros(shape, dtype=dtype)

    mx.asarray = asarray
    mx.zeros = zeros
    mx.eval = lambda *a, **k: None
    mx.compile = lambda f: f
    mx.default_device = lambda: "cpu"

    nn = types.ModuleType("mlx.nn")

    class Module:
        pass

    nn.Module = Module
    nn.silu = lambda v: v
    nn.layers = types.SimpleNamespace(distributed=types.SimpleNamespace(sum_gradients=None))

    mlx = types.ModuleType("mlx")
    mlx.core, mlx.nn = mx, nn
    utils = types.ModuleType("mlx.utils")
    utils.tree_flatten = lambda t: t
    mlx.utils = utils

    lm = types.ModuleType("mlx_lm")
    lm.load = None
    lm_utils = types.ModuleType("mlx_lm.utils")
    lm_utils._get_classes = None
    models = types.ModuleType("mlx_lm.models")
    sw = types.ModuleType("mlx_lm.models.switch_layers")
    for n in ("QuantizedSwitchLinear", "SwitchGLU", "SwitchLinear"):
        setattr(sw, n, type(n, (), {}))
    sw._gather_sort = sw._scatter_unsort = None
    q3 = types.ModuleType("mlx_lm.models.qwen3_next")
    q3.Qwen3NextSparseMoeBlock = type("Qwen3NextSparseMoeBlock", (), {})

    sys.modules.update({
        "mlx": mlx, "mlx.core": mx, "mlx.nn": nn, "mlx.utils": utils,
        "mlx_lm": lm, "mlx_lm.utils": lm_utils, "mlx_lm.models": models,
        "mlx_lm.models.switch_layers": sw, "mlx_lm.models.qwen3_next": q3,
    })


# --------------------------------------------------------------------------- admission


def make_admission(num_experts=32, num_slots=12, top_k=4, steps=40, seed=7):
    from preempt.backends.mlx_metal.module_wrappers.base_moe_wrapper import BaseMoEWrapper
    from preempt.backends.mlx_metal.module_wrappers.qwen3_x_moe import Qwen3_xMoEWrapper
    from preempt.backends.mlx_metal.expert_cache import SlottedGLU
    from preempt.datamodel.expert_bank.blob import SerializedExpert
    from preempt.datamodel.identity import TensorSpec

    I, H = 4, 6  # tiny uint16 "weights": gate/up [I, H], down [H, I]
    specs = (
        TensorSpec(name="gate_proj.weight", dtype="uint16", shape=(I, H), num_bytes=I * H * 2),
        TensorSpec(name="up_proj.weight", dtype="uint16", shape=(I, H), num_bytes=I * H * 2),
        TensorSpec(name="down_proj.weight", dtype="uint16", shape=(H, I), num_bytes=I * H * 2),
    )

    def blob_for(glob):
        base = np.arange(3 * I * H, dtype=np.uint16) + np.uint16(1000 * (glob + 1) % 60000)
        return base.tobytes()

    class Loader:
        def load_sync(self, idxs):
            return tuple(SerializedExpert(idx=i, data=blob_for(i), encoding="mlx-unquantized-uint16",
                                          tensor_specs=specs) for i in idxs)

    block_idx = 3
    w = Qwen3_xMoEWrapper.__new__(Qwen3_xMoEWrapper)
    BaseMoEWrapper.__init__(
        w, inner=types.SimpleNamespace(num_experts=num_experts, top_k=top_k),
        model_fingerprint="fp", layer_path="model.layers.3.mlp", block_idx=block_idx,
        num_experts=num_experts, recorder=None, capture_gate_logits=False,
        expert_loader=Loader(), expert_cache=object(), num_slots=num_slots,
        slot_size=3 * I * H * 2,
    )
    w._weight_slots = SlottedGLU(num_slots, (I, H), (H, I), np.uint16)

    rng = np.random.default_rng(seed)
    ranks = np.arange(1, num_experts + 1, dtype=np.float64)
    probs = ranks ** -1.1
    probs /= probs.sum()
    perm = rng.permutation(num_experts)

    rec = {k: [] for k in ("T", "routed", "pre_eid", "pre_sid", "pre_freq", "pre_rec", "pre_clock",
                           "unique", "inverse", "chosen", "post_eid", "post_sid", "post_freq",
                           "post_rec", "post_clock", "corrupt", "arena_owner_ok")}
    for step in range(steps):
        T = int(rng.integers(1, 4))
        routed = np.zeros((T, top_k), np.int32)
        for t in range(T):
            routed[t] = perm[rng.choice(num_experts, size=top_k, replace=False, p=probs)]
        pre = (w._eid_lookup_table.copy(), w._sid_lookup_table.copy(), w._slot_freq.copy(),
               w._slot_recency.copy(), w._clock)
        chosen_box = []
        orig = w._choose_slots

        def spy(n, protected, _orig=orig):
            out = _orig(n, protected)
            chosen_box.append(np.asarray(out).copy())
            return out

        w._choose_slots = spy
        uniq_n = np.unique(routed).size
        if uniq_n > num_slots:
            continue
        unique, inverse = w._maybe_admit(routed)
        w._choose_slots = orig
        chosen = chosen_box[0] if chosen_box else np.zeros(0, np.int64)
        # Does the reference overwrite a slot that this step still uses, or
        # write two experts into one slot?  (base_moe_wrapper.py:164-172)
        corrupt = bool(chosen.size and (np.unique(chosen).size != chosen.size or
                       np.isin(chosen, pre[0][unique][pre[0][unique] >= 0]).any()))
        slot_ids = w._eid_lookup_table[unique]
        w._touch(slot_ids)  # qwen3_x_moe.py:277, :290
        owner_ok = True
        for sid in range(num_slots):
            eid = w._sid_lookup_table[sid]
            if eid >= 0:
                ref = np.frombuffer(blob_for(block_idx * num_experts + eid), np.uint16)[I * H: 2 * I * H]
                owner_ok &= bool((w._weight_slots.up_proj[sid].reshape(-1) == ref).all())
        for k, v in (("T", T), ("routed", routed), ("pre_eid", pre[0]), ("pre_sid", pre[1]),
                     ("pre_freq", pre[2]), ("pre_rec", pre[3]), ("pre_clock", pre[4]),
                     ("unique", unique), ("inverse", np.asarray(inverse)), ("chosen", chosen),
                     ("post_eid", w._eid_lookup_table.copy()), ("post_sid", w._sid_lookup_table.copy()),
                     ("post_freq", w._slot_freq.copy()), ("post_rec", w._slot_recency.copy()),
                     ("post_clock", w._clock), ("corrupt", corrupt), ("arena_owner_ok", owner_ok)):
            rec[k].append(v)

    out = {"num_experts": num_experts, "num_slots": num_slots, "top_k": top_k,
           "n_steps": len(rec["T"])}
    for k, v in rec.items():
        for i, item in enumerate(v):
            out[f"{k}_{i}"] = np.asarray(item)
    np.savez_compressed(HERE / "admission_steps.npz", **out)
    n_corrupt = sum(rec["corrupt"])
    print(f"admission: {len(rec['T'])} steps, {n_corrupt} where the reference corrupts a slot")


# --------------------------------------------------------------------------- cache manager


def make_cache_manager():
    from preempt.engine.expert_io.cache_manager import ExpertCacheManager
    from preempt.core.enums import CacheEvictionPolicy, ReadPriority

    UNIT = 100
    P = ReadPriority.PREFETCH
    res = {}

    def scripted(policy):
        m = ExpertCacheManager(budget_bytes=3 * UNIT, policy=policy, sample_size=8)
        m.admit(0, UNIT, P)
        for _ in range(3):
            m.touch(0)
        m.admit(1, UNIT, P)
        m.admit(2, UNIT, P)
        m.touch(2)
        m.touch(1)
        return list(m.admit(9, UNIT, P))

    res["lfru_victims"] = scripted(CacheEvictionPolicy.LFRU)
    res["lru_victims"] = scripted(CacheEvictionPolicy.LRU)
    m = ExpertCacheManager(budget_bytes=2 * UNIT, sample_size=8)
    m.admit(0, UNIT, P)
    m.admit(1, UNIT, P)
    m.touch(0)
    m.touch(1)
    res["lfru_tie_victims"] = list(m.admit(2, UNIT, P))

    def seq(seed):
        m = ExpertCacheManager(budget_bytes=8 * UNIT, sample_size=3, seed=seed)
        ev = []
        for i in range(24):
            c = i % 12
            if not m.touch(c):
                ev.extend(m.admit(c, UNIT, P))
        return ev, m.hits, m.misses, m.evictions, m.bytes_read

    for s in (0, 1):
        ev, h, mi, e, b = seq(s)
        res[f"sampled_seed{s}"] = {"evicted": [int(v) for v in ev], "hits": h, "misses": mi,
                                   "evictions": e, "bytes_read": b}
    (HERE / "cache_manager.json").write_text(json.dumps(res, indent=1))
    print("cache_manager:", res["lfru_victims"], res["lru_victims"], res["sampled_seed0"]["evicted"])


# --------------------------------------------------------------------------- bank


def make_bank():
    sys.path.insert(0, str(HERE.parents[1]))
    from oracle.slotted_glu_oracle import quantize_affine, f32_to_bf16_bits
    from preempt.datamodel.expert_bank.writer import ExpertBankWriter
    from preempt.datamodel.expert_bank.manifest import ModelMoESpec
    from preempt.datamodel.expert_bank.blob import derive_tensor_specs, assemble_expert_blob

    H, I, bits, gs = 128, 64, 4, 64
    blocks, E = (0, 1), 3
    rng = np.random.default_rng(1234)
    order = [f"{p}.{part}" for p in ("gate_proj", "up_proj", "down_proj")
             for part in ("weight", "scales", "biases")]
    dst = HERE / "bank"
    if dst.exists():
        shutil.rmtree(dst)
    blobs = {}
    specs = None
    for b in blocks:
        for e in range(E):
            arrays = {}
            for p, shape in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
                w = f32_to_bf16_bits((rng.standard_normal(shape) * 0.02).astype(np.float32))
                q, s, bb = quantize_affine(w, bits, gs)
                arrays[f"{p}.weight"] = q
                arrays[f"{p}.scales"] = s
                arrays[f"{p}.biases"] = bb
            specs = specs or derive_tensor_specs(arrays, order)
            blobs[(b, e)] = assemble_expert_blob(arrays, specs)
    with ExpertBankWriter(dst, model_id="synthetic/tiny-q4", model_fingerprint="fp-tiny",
                          encoding=f"mlx-affine-q{bits}-g{gs}-bfloat16", tensor_specs=specs,
                          model_moe_spec=ModelMoESpec(moe_block_idxs=blocks, num_routed_experts=E, top_k=2),
                          alignment=4096, verbose=False) as wr:
        for (b, e), data in blobs.items():
            wr.add_expert(b, e, data)
    print("bank:", sorted(p.name for p in dst.iterdir()), (dst / "experts.bin").stat().st_size)


def make_encoding_tags():
    from preempt.datamodel.expert_bank.encoding import parse_encoding_tag

    good = ["mlx-affine-q4-g64-bfloat16", "mlx-affine-q8-g32-float16", "mlx-mxfp4-q4-g32-bfloat16",
            "mlx-unquantized-bfloat16", "mlx-unquantized-float16", "mlx-unquantized-float32",
            "mlx-affine-q8-g64-bfloat16"]
    bad = ["", "mlx", "mlx-affine-q4-g64", "mlx-affine-4-64-bfloat16", "mlx-affine-qx-g64-bfloat16",
           "mlx-affine-q4-g64-bfloat16-extra", "mlx-affine-q0-g64-bfloat16", "mlx-affine-q4-g0-bfloat16",
           "mlx--q4-g64-bfloat16", "MLX-affine-q4-g64-bfloat16", "mlx-unquantized",
           "mlx-unquantized-bfloat16-g64", "torch-affine-q4-g64-bfloat16", "gguf-unquantized-float32",
           "mlx-affine-q4-g64-fp8", "mlx-unquantized-f64", "mlx-affine-q4-g64-int12"]
    res = {"good": {}, "bad": {}}
    for t in good:
        e = parse_encoding_tag(t)
        res["good"][t] = {"backend": e.backend, "mode": e.mode, "bits": e.bits,
                          "group_size": e.group_size, "dtype": e.dtype}
    for t in bad:
        try:
            parse_encoding_tag(t)
            res["bad"][t] = None
        except ValueError as exc:
            res["bad"][t] = str(exc).split(" ")[0]
    (HERE / "encoding_tags.json").write_text(json.dumps(res, indent=1))
    print("encoding tags:", len(res["good"]), "good,", len(res["bad"]), "bad")


if __name__ == "__main__":
    where = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PREEMPTLM_REFERENCE")
    if not where:
        raise SystemExit("usage: make_golden.py <reference tree>  (or set PREEMPTLM_REFERENCE)")
    ref = Path(where)
    sys.path.insert(0, str(ref))
    _install_mlx_standin()
    make_admission()
    make_cache_manager()
    make_bank()
    make_encoding_tags()
