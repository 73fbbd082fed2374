"""Shared helpers of the test suite: bit views and oracle adapters."""

from __future__ import annotations

import numpy as np
import torch

from oracle import slotted_glu_oracle as orc

# bf16 output tolerance of the layer (max-abs and relative L2)
MAX_ABS = 2e-2
REL_L2 = 1e-2


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def bits32(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().numpy().view(np.uint32)


def f32(t: torch.Tensor) -> np.ndarray:
    return orc.bf16_bits_to_f32(bits16(t))


def oracle_expert(tensors: dict, idx: int, bits: int) -> orc.ExpertWeights:
    """Dequantised (exact bf16 values) weights of expert ``idx`` of a synthetic
    tensor dict (``gate_proj.weight`` ... with a leading expert axis)."""
    mats = []
    for p in ("gate_proj", "up_proj", "down_proj"):
        if bits == 16:
            mats.append(orc.bf16_bits_to_f32(bits16(tensors[f"{p}.weight"][idx])))
        else:
            mats.append(orc.dequant_affine(bits32(tensors[f"{p}.weight"][idx]), bits16(tensors[f"{p}.scales"][idx]),
                                           bits16(tensors[f"{p}.biases"][idx]), bits, 64))
    return orc.ExpertWeights(*mats)


class LazyExperts:
    def __init__(self, tensors, bits):
        self.tensors, self.bits, self._cache = tensors, bits, {}

    def __getitem__(self, idx):
        idx = int(idx)
        if idx not in self._cache:
            self._cache[idx] = oracle_expert(self.tensors, idx, self.bits)
        return self._cache[idx]


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_close(dev, ref, max_abs=MAX_ABS, rel=REL_L2, what=""):
    dev = np.asarray(dev, np.float64)
    ref = np.asarray(ref, np.float64)
    assert dev.shape == ref.shape, (what, dev.shape, ref.shape)
    err = float(np.abs(dev - ref).max()) if dev.size else 0.0
    r = rel_l2(dev, ref) if dev.size else 0.0
    assert err <= max_abs and r <= rel, f"{what}: max-abs {err:.3e} (<= {max_abs}), rel-L2 {r:.3e} (<= {rel})"
    return err, r
