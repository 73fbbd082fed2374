"""MLX affine quantisation settings and the per-group min/max quantiser.

Mirrors ``QuantSettings`` / ``MlxQuantMode`` (preempt/backends/mlx_metal/
quantization.py:9-40) and the MLX affine layout consumed by
``mx.gather_qmm(..., transpose=True, group_size, bits, mode="affine")``
(preempt/backends/mlx_metal/ops/fused.py:77-88): a weight [out, in] is stored
as packed uint32 [out, in*bits/32] (weight m of a word at bits
[m*bits, (m+1)*bits)), plus bf16 scales and biases [out, in/group_size]; each
group of ``group_size`` consecutive input weights decodes as scale * q + bias.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum

import torch


class MlxQuantMode(str, Enum):
    AFFINE = "affine"
    MXFP4 = "mxfp4"
    MXFP8 = "mxfp8"
    NVFP4 = "nvfp4"


@dataclass(frozen=True)
class QuantSettings:
    """(mode, bits, group_size) of a quantised projection
    (quantization.py:16-40).  Only affine 4/8-bit with group 64 has kernels."""

    mode: MlxQuantMode
    bits: int
    group_size: int

    def __post_init__(self):
        object.__setattr__(self, "mode", MlxQuantMode(self.mode))

    def check_supported(self) -> None:
        if self.mode is not MlxQuantMode.AFFINE or self.bits not in (4, 8) or self.group_size != 64:
            raise ValueError(f"unsupported quantisation {self!r}: kernels cover affine 4/8-bit, group 64")


def quantize_affine(w: torch.Tensor, bits: int, group_size: int = 64):
    """Quantise bf16 ``w`` [..., out, in] per group of ``group_size`` input
    weights: scale = (max - min) / (2^bits - 1), bias = min (both rounded to
    bf16), q = clip(rint((w - bias) / scale)).  Returns (packed int32 view of
    the uint32 words, scales bf16, biases bf16)."""
    if w.dtype != torch.bfloat16:
        raise TypeError("quantize_affine expects bf16 weights")
    if bits not in (4, 8) or w.shape[-1] % group_size:
        raise ValueError("bits must be 4 or 8 and the input dim a multiple of group_size")
    *lead, out, inn = w.shape
    g = w.float().reshape(*lead, out, inn // group_size, group_size)
    mn = g.amin(-1)
    mx = g.amax(-1)
    nmax = (1 << bits) - 1
    scale = ((mx - mn) / nmax).to(torch.bfloat16)
    bias = mn.to(torch.bfloat16)
    s32 = scale.float()
    safe = torch.where(s32 == 0, torch.ones_like(s32), s32)
    q = torch.round((g - bias.float()[..., None]) / safe[..., None])
    q = torch.where(s32[..., None] == 0, torch.zeros_like(q), q)
    q = q.clamp_(0, nmax).to(torch.int64).reshape(*lead, out, inn)
    per = 32 // bits
    qw = q.reshape(*lead, out, inn // per, per)
    shifts = torch.arange(per, device=w.device, dtype=torch.int64) * bits
    words = (qw << shifts).sum(-1)  # < 2^32, no overlap between fields
    packed = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)
    return packed, scale, bias


def dequantize_affine(packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int,
                      group_size: int = 64) -> torch.Tensor:
    """bf16(scale * q + bias) in fp32 arithmetic: the exact values the
    tensor-core path feeds its MMAs."""
    per = 32 // bits
    words = packed.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, device=packed.device, dtype=torch.int64) * bits
    q = (words[..., None] >> shifts) & ((1 << bits) - 1)
    q = q.reshape(*packed.shape[:-1], packed.shape[-1] * per).float()
    s = scales.float().repeat_interleave(group_size, dim=-1)
    b = biases.float().repeat_interleave(group_size, dim=-1)
    return (s * q + b).to(torch.bfloat16)
