"""``SlottedGLU``: the pre-allocated per-layer expert slot arena in HBM.

Mirrors ``SlottedGLU(num_slots, up_shape, down_shape, dtype)``
(preempt/backends/mlx_metal/expert_cache.py:199-224): ``gate_proj`` and
``up_proj`` are [S, *up_shape] = [S, I, H] and ``down_proj`` is
[S, *down_shape] = [S, H, I], zero-initialised.  The reference arena is bf16
only (expert_cache.py:198); with ``quant=QuantSettings("affine", 4|8, 64)`` the
arena holds the MLX affine layout instead: ``{proj}`` packed uint32 (int32
view) [S, out, in*bits/32] plus ``{proj}_scales`` / ``{proj}_biases`` bf16
[S, out, in/64].
"""

from __future__ import annotations

from collections.abc import Mapping, Sequence

import torch

from . import _abi
from .quant import QuantSettings

GLU_PROJECTION_NAMES = ("gate_proj", "up_proj", "down_proj")  # constants.py:20-34
MLX_QUANTIZED_TENSOR_PARTS = ("weight", "scales", "biases")


class SlottedGLU:
    def __init__(self, num_slots: int, up_shape: Sequence[int], down_shape: Sequence[int],
                 dtype: torch.dtype = torch.bfloat16, quant: QuantSettings | None = None,
                 device: str | torch.device = "cuda"):
        I, H = int(up_shape[0]), int(up_shape[1])
        if tuple(down_shape) != (H, I):
            raise ValueError(f"down_shape {tuple(down_shape)} must be (H, I) = {(H, I)}")
        if dtype != torch.bfloat16:
            raise TypeError("the arena holds bf16 weights (or bf16 scales/biases when quantised)")
        self.num_slots, self.hidden, self.inter = int(num_slots), H, I
        self.quant = quant
        self.device = torch.device(device)
        if quant is None:
            self.bits, self.group_size = 16, 0
            self.gate_proj = torch.zeros((num_slots, I, H), dtype=dtype, device=device)
            self.up_proj = torch.zeros((num_slots, I, H), dtype=dtype, device=device)
            self.down_proj = torch.zeros((num_slots, H, I), dtype=dtype, device=device)
            for n in GLU_PROJECTION_NAMES:
                setattr(self, f"{n}_scales", None)
                setattr(self, f"{n}_biases", None)
        else:
            quant.check_supported()
            self.bits, self.group_size = quant.bits, quant.group_size
            gs, b = quant.group_size, quant.bits
            for n, (o, i) in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
                setattr(self, n, torch.zeros((num_slots, o, i * b // 32), dtype=torch.int32, device=device))
                setattr(self, f"{n}_scales", torch.zeros((num_slots, o, i // gs), dtype=dtype, device=device))
                setattr(self, f"{n}_biases", torch.zeros((num_slots, o, i // gs), dtype=dtype, device=device))
        self._desc = None

    # ------------------------------------------------------------------ info
    @property
    def is_quantized(self) -> bool:
        return self.quant is not None

    def tensor_names(self) -> tuple[str, ...]:
        """Blob order of one expert's tensors (serialisation order of the bank,
        expert_bank/qwen3_x.py:66-77)."""
        parts = MLX_QUANTIZED_TENSOR_PARTS if self.is_quantized else ("weight",)
        return tuple(f"{p}.{part}" for p in GLU_PROJECTION_NAMES for part in parts)

    def _tensor(self, name: str) -> torch.Tensor:
        proj, part = name.split(".")
        return getattr(self, proj if part == "weight" else f"{proj}_{part}")

    def expert_num_bytes(self) -> int:
        return sum(self._tensor(n)[0].numel() * self._tensor(n).element_size() for n in self.tensor_names())

    def nbytes(self) -> int:
        return self.expert_num_bytes() * self.num_slots

    def desc(self) -> _abi.sg_arena:
        """The C-ABI descriptor (device pointers of the arena)."""
        if self._desc is None:
            d = _abi.sg_arena()
            d.num_slots, d.hidden, d.inter = self.num_slots, self.hidden, self.inter
            d.bits, d.group_size = self.bits, self.group_size or 64
            for n in GLU_PROJECTION_NAMES:
                p = n.split("_")[0]
                setattr(d, f"{p}_w", getattr(self, n).data_ptr())
                s = getattr(self, f"{n}_scales")
                b = getattr(self, f"{n}_biases")
                setattr(d, f"{p}_s", s.data_ptr() if s is not None else None)
                setattr(d, f"{p}_b", b.data_ptr() if b is not None else None)
            self._desc = d
        return self._desc

    # ------------------------------------------------------------------ writes
    def write_slot(self, sid: int, weights: Mapping[str, torch.Tensor]) -> None:
        """``arena.{proj}[sid] = weights[...]`` for every tensor of one expert
        (the slot writes of qwen3_x_moe.py:186-195)."""
        for n in self.tensor_names():
            dst = self._tensor(n)[sid]
            src = weights[n]
            if src.dtype != dst.dtype:
                src = src.view(dst.dtype)
            dst.copy_(src.reshape(dst.shape), non_blocking=True)

    def refill_from_blob(self, sid: int, blob: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """Copy one serialised expert (pinned host uint8 tensor, tensors in blob
        order) into slot ``sid`` with cudaMemcpyAsync on ``stream``
        (``sg_refill_h2d``)."""
        if blob.device.type != "cpu" or blob.dtype != torch.uint8:
            raise TypeError("blob must be a host uint8 tensor")
        s = stream or torch.cuda.current_stream(self.device)
        lib = _abi.load()
        _abi.check(lib.sg_refill_h2d(blob.data_ptr(), blob.numel(), ctypes_byref(self.desc()), int(sid),
                                     s.cuda_stream), "sg_refill_h2d")


def ctypes_byref(obj):
    import ctypes

    return ctypes.byref(obj)
