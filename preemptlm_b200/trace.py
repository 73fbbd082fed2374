"""Router-selection telemetry: the expert ids, scores and gate logits of every
routed token as ``ExpertSelectionTrace`` records.

Mirrors the reference's recorder and record schema:

* ``ExpertTraceRecorder`` follows ``MlxTraceRecorder``
  (preempt/backends/mlx_metal/recorder.py:40-238): ``start_trace(step)``,
  ``capture(layer_path=..., layer_class=..., block_idx=..., expert_ids=...,
  softmax_weights=..., gate_logits=...)`` from inside the MoE block, and
  ``flush(sink)``, which writes one record per (batch, sequence-offset) token
  with ``sequence_id = step.sequence_id + b``, ``token_idx = step.token_idx +
  s`` and a running ``event_idx`` (recorder.py:160-216).
* The records are the flattened Arrow rows of ``ExpertSelectionTrace``
  (preempt/datamodel/tracing/expert_selection.py:52-157, context.py:31-95),
  schema version 1, in the same column order and types (``arrow_schema``).

The B200 difference is where the numbers come from.  The reference buffers
lazy MLX arrays and evaluates them at flush.  Here the recorder owns a ring of
pinned host memory mapped into the GPU's address space
(``TraceRing``); before the routing launch the layer reserves the step's rows
in it and the fused routing kernel (``sg_route_dispatch``) writes each
token's ids, renormalised scores and raw logits there as it computes them.
Tracing therefore costs no extra launch and no device-side copy; ``flush``
waits on one event per capture and reads host memory.  Tensors captured
without a reserved span (any other caller) are copied at flush instead.
"""

from __future__ import annotations

import ctypes
import uuid
from dataclasses import dataclass
from datetime import UTC, datetime

import numpy as np
import torch

from . import _abi

EXPERT_SELECTION_TRACE_SCHEMA_VERSION = 1  # preempt/core/constants.py:7


@dataclass(frozen=True)
class TraceRunContext:
    """context.py:31-78 (run id, instrumentation version, model identity)."""

    run_id: str
    model_id: str
    model_architecture: str
    instrumentation_version: str = "0.1.0"
    model_revision: str | None = None

    @classmethod
    def with_generated_run_id(cls, *, run_id_prefix: str, model_id: str, model_architecture: str,
                              model_revision: str | None = None, instrumentation_version: str = "0.1.0"):
        return cls(run_id=f"{run_id_prefix}-{uuid.uuid4().hex[:12]}", model_id=model_id,
                   model_architecture=model_architecture, instrumentation_version=instrumentation_version,
                   model_revision=model_revision)


@dataclass(frozen=True)
class TraceStepContext:
    """context.py:83-95: one forward pass of a generation run."""

    sequence_id: int
    token_idx: int
    token_id: int | None = None


def arrow_schema():
    """The flattened Arrow schema of an ExpertSelectionTrace record
    (expert_selection.py:134-157): nested context fields in declaration order,
    schema version in the metadata."""
    import pyarrow as pa

    fields = [
        pa.field("schema_version", pa.int16(), nullable=False),
        pa.field("run_id", pa.string(), nullable=False),
        pa.field("instrumentation_version", pa.string(), nullable=False),
        pa.field("model_id", pa.string(), nullable=False),
        pa.field("model_architecture", pa.string(), nullable=False),
        pa.field("model_revision", pa.string(), nullable=True),
        pa.field("sequence_id", pa.int32(), nullable=False),
        pa.field("token_idx", pa.int32(), nullable=False),
        pa.field("token_id", pa.int64(), nullable=True),
        pa.field("event_idx", pa.int64(), nullable=False),
        pa.field("timestamp", pa.timestamp("us", tz="UTC"), nullable=False),
        pa.field("path", pa.string(), nullable=False),
        pa.field("module_class", pa.string(), nullable=False),
        pa.field("transformer_block_idx", pa.int32(), nullable=False),
        pa.field("expert_ids", pa.list_(pa.field("item", pa.int32(), nullable=False)), nullable=False),
        pa.field("softmax_weights", pa.list_(pa.field("item", pa.float32(), nullable=False)), nullable=False),
        pa.field("gate_logits", pa.list_(pa.field("item", pa.float32(), nullable=True)), nullable=True),
    ]
    return pa.schema(fields, metadata={b"preempt.schema_version": str(EXPERT_SELECTION_TRACE_SCHEMA_VERSION).encode()})


def validate_record(rec: dict) -> None:
    """The checks of ExpertSelectionTrace.__attrs_post_init__ (expert_selection.py:111-127)."""
    ids, w = rec["expert_ids"], rec["softmax_weights"]
    if len(ids) != len(w):
        raise ValueError("`expert_ids` and `softmax_weights` must contain the same number of values")
    if len(set(ids)) != len(ids):
        raise ValueError("`expert_ids` must only contain unique values.")
    if any(e < 0 for e in ids):
        raise ValueError("`expert_ids` must all be non-negative.")
    if any(x < 0.0 for x in w):
        raise ValueError("`softmax_weights` must all be non-negative.")
    if not any(x > 0.0 for x in w):
        raise ValueError("At least one expert weight must be positive.")


class ListTraceSink:
    """Keeps the records in memory."""

    def __init__(self):
        self.records: list[dict] = []

    def write(self, record: dict) -> None:
        self.records.append(record)


class ParquetTraceSink:
    """Writes records to a Parquet file with ``arrow_schema`` (the role of the
    reference's ParquetTraceSink, engine/sinks.py:49-187), a row group per
    ``flush_rows`` records."""

    def __init__(self, path, flush_rows: int = 4096):
        import pyarrow.parquet as pq

        self._schema = arrow_schema()
        self._writer = pq.ParquetWriter(str(path), self._schema)
        self._rows: list[dict] = []
        self._flush_rows = flush_rows

    def write(self, record: dict) -> None:
        self._rows.append(record)
        if len(self._rows) >= self._flush_rows:
            self._drain()

    def _drain(self) -> None:
        import pyarrow as pa

        if self._rows:
            self._writer.write_table(pa.Table.from_pylist(self._rows, schema=self._schema))
            self._rows = []

    def close(self) -> None:
        self._drain()
        self._writer.close()


class TraceRing:
    """Pinned host arrays mapped into the GPU's address space, which the
    routing kernel fills: ids int32 [capacity, k], scores bf16 bits
    [capacity, k] and (optionally) logits bf16 bits [capacity, E]."""

    def __init__(self, capacity_tokens: int, top_k: int, num_experts: int, with_logits: bool = True):
        self.capacity, self.top_k, self.num_experts = int(capacity_tokens), int(top_k), int(num_experts)
        self.ids = torch.empty((self.capacity, self.top_k), dtype=torch.int32, pin_memory=True)
        self.scores = torch.empty((self.capacity, self.top_k), dtype=torch.int16, pin_memory=True)
        self.logits = (torch.empty((self.capacity, self.num_experts), dtype=torch.int16, pin_memory=True)
                       if with_logits else None)
        lib = _abi.load()
        self._dev = {}
        for name in ("ids", "scores", "logits"):
            t = getattr(self, name)
            if t is None:
                continue
            p = ctypes.c_void_p()
            _abi.check(lib.sg_host_device_ptr(ctypes.c_void_p(t.data_ptr()), ctypes.byref(p)), "sg_host_device_ptr")
            self._dev[name] = p.value
        self.used = 0

    def reserve(self, T: int, with_logits: bool) -> tuple[int, _abi.sg_route_trace]:
        """Rows [start, start + T) for the next routing launch, and the
        device-visible addresses the kernel writes them to."""
        if self.used + T > self.capacity:
            raise RuntimeError(f"trace ring full ({self.used} + {T} > {self.capacity} tokens): flush() first")
        start = self.used
        self.used += T
        tr = _abi.sg_route_trace()
        tr.ids = self._dev["ids"] + start * self.top_k * 4
        tr.scores = self._dev["scores"] + start * self.top_k * 2
        tr.logits = (self._dev["logits"] + start * self.num_experts * 2) if (with_logits and "logits" in self._dev) \
            else None
        return start, tr

    def reset(self) -> None:
        self.used = 0


@dataclass
class _Capture:
    layer_path: str
    layer_class: str
    block_idx: int
    batch_shape: tuple[int, int]
    step: TraceStepContext
    timestamp: datetime
    span: int | None  # first ring row, or None for tensors copied at flush
    has_logits: bool
    event: torch.cuda.Event | None
    tensors: tuple | None


def _bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


class ExpertTraceRecorder:
    """recorder.py:40-238 on B200 (module docstring).  ``capacity_tokens``
    bounds the tokens captured between two flushes."""

    def __init__(self, run_context: TraceRunContext, *, top_k: int, num_experts: int,
                 capacity_tokens: int = 65536, with_logits: bool = True):
        self._run_context = run_context
        self._ring = TraceRing(capacity_tokens, top_k, num_experts, with_logits) if torch.cuda.is_available() else None
        self._step_context: TraceStepContext | None = None
        self._buffer: list[_Capture] = []
        self._pending_span: tuple[int, bool] | None = None
        self._num_captures = 0
        self._num_records = 0

    # ------------------------------------------------------------------ steps
    def start_trace(self, step_context: TraceStepContext) -> None:
        self._step_context = step_context

    def stop_trace(self) -> None:
        self._step_context = None

    # ------------------------------------------------------------------ capture
    def reserve(self, T: int, with_logits: bool):
        """Called by the MoE block before its routing launch: ring rows for T
        tokens, as the kernel's trace argument (None without a ring)."""
        if self._ring is None:
            return None
        start, tr = self._ring.reserve(T, with_logits)
        self._pending_span = (start, with_logits)
        return tr

    def capture(self, *, layer_path: str, layer_class: str, block_idx: int, expert_ids, softmax_weights,
                gate_logits=None) -> None:
        """Buffers one MoE block's routing of a [B, S] batch (recorder.py:57-111)."""
        if self._step_context is None:
            raise RuntimeError("`capture()` called without an active `TraceStepContext`. "
                               "Call `start_trace()` before recording events.")
        B, S = int(expert_ids.shape[0]), int(expert_ids.shape[1])
        span = self._pending_span
        self._pending_span = None
        event = None
        if expert_ids.is_cuda:
            event = torch.cuda.Event()
            event.record()
        tensors = None
        if span is None:  # no ring rows: keep the tensors, copied at flush
            tensors = (expert_ids, softmax_weights, gate_logits)
        self._buffer.append(_Capture(layer_path, layer_class, int(block_idx), (B, S), self._step_context,
                                     datetime.now(UTC), None if span is None else span[0],
                                     gate_logits is not None if span is None else span[1], event, tensors))
        self._num_captures += 1

    # ------------------------------------------------------------------ flush
    def _arrays(self, c: _Capture):
        n = c.batch_shape[0] * c.batch_shape[1]
        if c.span is not None:
            r = self._ring
            ids = r.ids[c.span: c.span + n].numpy()
            w = _bf16_bits_to_f32(r.scores[c.span: c.span + n].numpy())
            lg = _bf16_bits_to_f32(r.logits[c.span: c.span + n].numpy()) if c.has_logits else None
            return ids, w, lg
        e, s, g = c.tensors
        ids = e.reshape(n, -1).to(torch.int32).cpu().numpy()
        w = s.reshape(n, -1).float().cpu().numpy()
        lg = None if g is None else g.reshape(n, -1).float().cpu().numpy()
        return ids, w, lg

    def flush(self, sink) -> int:
        """Materialises the buffered captures as records (one per token) into
        ``sink.write`` and closes the step (recorder.py:113-160)."""
        if self._step_context is None:
            raise RuntimeError("No capture step currently active.")
        try:
            n = 0
            rc = self._run_context
            for c in self._buffer:
                if c.event is not None:
                    c.event.synchronize()
                ids, w, lg = self._arrays(c)
                B, S = c.batch_shape
                for b in range(B):
                    for s in range(S):
                        i = b * S + s
                        rec = {
                            "schema_version": EXPERT_SELECTION_TRACE_SCHEMA_VERSION,
                            "run_id": rc.run_id, "instrumentation_version": rc.instrumentation_version,
                            "model_id": rc.model_id, "model_architecture": rc.model_architecture,
                            "model_revision": rc.model_revision,
                            "sequence_id": c.step.sequence_id + b, "token_idx": c.step.token_idx + s,
                            "token_id": c.step.token_id,
                            "event_idx": self._num_records + n, "timestamp": c.timestamp,
                            "path": c.layer_path, "module_class": c.layer_class,
                            "transformer_block_idx": c.block_idx,
                            "expert_ids": [int(v) for v in ids[i]],
                            "softmax_weights": [float(v) for v in w[i]],
                            "gate_logits": None if lg is None else [float(v) for v in lg[i]],
                        }
                        validate_record(rec)
                        sink.write(rec)
                        n += 1
            self._num_records += n
            self._buffer = []
            if self._ring is not None:
                self._ring.reset()
            return n
        finally:
            self.stop_trace()
