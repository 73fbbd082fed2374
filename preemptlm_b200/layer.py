"""The slotted MoE block: ``Qwen3_xMoEWrapper`` on B200.

Mirrors preempt/backends/mlx_metal/module_wrappers/qwen3_x_moe.py:85-337:
the constructor arguments, ``_maybe_admit``, ``_gather_forward``, ``_touch``,
``_choose_slots``, ``__call__`` and ``make_wrapper_factory`` keep their names
and meaning.  The math runs in the libsg_b200 kernels:

  router GEMV -> routing (softmax/top-k/renorm) -> device dispatch
  (unique, inverse, slot lookup, permutation) -> gate/up + SwiGLU -> down
  -> weighted combine with the sigmoid-gated shared expert.

Differences from the reference, all deliberate:
* the device->host sync of the routed ids (qwen3_x_moe.py:145) is replaced by
  a device-side unique/lookup; the host reads back two counters, and the
  unique ids only when a slot must be refilled;
* ``mx.take`` copies of the arena (qwen3_x_moe.py:225-227) are gone: the
  kernels read slots in place;
* when the non-streaming branch is taken (``expert_cache is None``,
  qwen3_x_moe.py:272-273) the full expert stack ``inner.switch_mlp`` is an
  arena with slot == expert id.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch

from . import _abi, ops
from .arena import SlottedGLU
from .quant import QuantSettings
from .slot_map import EMPTY, SlotTable

BaseMoEWrapper = SlotTable


@dataclass
class SparseMoeBlock:
    """The fields of mlx_lm's ``Qwen3NextSparseMoeBlock`` that the wrapper uses
    (``gate``, ``switch_mlp``, ``shared_expert``, ``shared_expert_gate``,
    ``top_k``, ``norm_topk_prob``, ``num_experts``), as torch tensors.

    gate: router weight [E, H] bf16.  switch_mlp: all routed experts as an
    arena with one slot per expert, or None when the experts are streamed.
    shared_expert: a one-slot arena, or None.  shared_expert_gate: [1, H] bf16.
    """

    gate: torch.Tensor
    top_k: int
    norm_topk_prob: bool
    moe_intermediate_size: int
    quant: QuantSettings | None = None
    switch_mlp: SlottedGLU | None = None
    shared_expert: SlottedGLU | None = None
    shared_expert_gate: torch.Tensor | None = None
    sharding_group: object | None = None

    @property
    def num_experts(self) -> int:
        return int(self.gate.shape[0])

    @property
    def hidden_size(self) -> int:
        return int(self.gate.shape[1])


# --------------------------------------------------------------------------- functional pieces


def _get_routings(logits: torch.Tensor, top_k: int, norm_topk_prob: bool):
    """qwen3_x_moe.py:26-40.  Returns (inds int32 [T, k], scores bf16 [T, k])
    in the order (gate desc, expert id asc)."""
    shape = logits.shape
    inds, scores = ops.route_topk(logits.reshape(-1, shape[-1]), top_k, norm_topk_prob)
    return inds.reshape(*shape[:-1], top_k), scores.reshape(*shape[:-1], top_k)


def _combine_shared(y, scores, shared_y, shared_gate):
    """qwen3_x_moe.py:71-80.  y [..., k, H], scores [..., k] -> [..., H]."""
    H = y.shape[-1]
    k = scores.shape[-1]
    lead = scores.shape[:-1]
    T = int(np.prod(lead)) if len(lead) else 1
    out = ops.combine(y.reshape(T * k, H), scores.reshape(T, k),
                      None if shared_y is None else shared_y.reshape(T, H),
                      None if shared_gate is None else shared_gate.reshape(T))
    return out.reshape(*lead, H)


def shared_expert_forward(arena: SlottedGLU, x2: torch.Tensor) -> torch.Tensor:
    """Dense SwiGLU of the shared expert (mlx_lm Qwen3NextMLP) on every token:
    the dense tensor-core kernel from two tokens on (its B rows are contiguous
    and load by TMA), else the one-group gathered path."""
    if x2.shape[0] >= 2 and ops.glu_path() != "gemv":
        y = ops.dense_glu(arena, x2)
        if y is not None:
            return y
    d = ops.token_dispatch(x2.shape[0], x2.device)
    h = ops.glu_gate_up(arena, x2, d, pair_div=1)
    return ops.glu_down(arena, h, d)


# --------------------------------------------------------------------------- the wrapper


class Qwen3_xMoEWrapper(SlotTable):
    """Slotted MoE block wrapper (qwen3_x_moe.py:85-297) over libsg_b200."""

    def __init__(self, inner: SparseMoeBlock, model_fingerprint: str | None, layer_path: str, block_idx: int,
                 recorder=None, capture_gate_logits: bool = False, expert_loader=None, expert_cache=None,
                 num_slots: int = 0, slot_size: int = 0, slot_policy: str = "reference",
                 device: str | torch.device | None = None, prefetch_experts: int = 0):
        # base_moe_wrapper.py:84-87
        if expert_loader is not None and any(v is None for v in (expert_cache, num_slots, slot_size)):
            raise ValueError("expert_loader requires expert_cache, num_slots and slot_size")
        device = torch.device(device) if device is not None else inner.gate.device
        super().__init__(inner.num_experts, num_slots or 0, slot_policy=slot_policy, device=device)
        self.inner = inner
        self.model_fingerprint = model_fingerprint
        self.layer_path = layer_path
        self.block_idx = int(block_idx)
        self.recorder = recorder
        self._capture_gate_logits = capture_gate_logits
        self.expert_loader = expert_loader
        self.expert_cache = expert_cache
        self.slot_size = slot_size or 0
        self._quants = inner.quant
        self._pending: list = []  # (event, pinned blobs) kept alive until their copies finish
        self._copy_stream: torch.cuda.Stream | None = None  # slot refills, overlapped with compute
        self._refill_event: torch.cuda.Event | None = None  # the last step's refills, for the GLU to wait on
        self.admit_stats = {"steps": 0, "unique": 0, "missed": 0}  # streaming: routed experts seen / refilled
        # streaming: after each step, queue PREFETCH reads of this many of the
        # most often routed experts that are neither in a slot nor in the host
        # blob cache (a frequency predictor; the reference has the hook,
        # loader.py:286-310, but no caller)
        self.prefetch_experts = int(prefetch_experts)
        self._routed_freq = np.zeros(inner.num_experts, np.int64)
        self._side_stream: torch.cuda.Stream | None = None  # the shared expert, beside the routed path
        self._weight_slots: SlottedGLU | None = None
        if expert_loader is not None or expert_cache is not None:
            H, I = inner.hidden_size, inner.moe_intermediate_size
            self._weight_slots = SlottedGLU(self.num_slots, (I, H), (H, I), torch.bfloat16, quant=inner.quant,
                                            device=device)
        # zero int32 [E + 1] buffer of the fused routing + dispatch kernel (left zero by every call)
        self._route_work = torch.zeros(inner.num_experts + 1, dtype=torch.int32, device=device)
        self._identity = None
        if expert_cache is None:
            if inner.switch_mlp is None:
                raise ValueError("non-streaming wrapper needs inner.switch_mlp (all experts resident)")
            self._identity = torch.arange(inner.num_experts, dtype=torch.int32, device=device)

    # ------------------------------------------------------------------ properties
    @property
    def is_quantized(self) -> bool:
        return self._quants is not None

    @property
    def should_capture_traces(self) -> bool:
        return self.recorder is not None

    @property
    def should_stream_experts(self) -> bool:
        return self.expert_loader is not None

    @property
    def arena(self) -> SlottedGLU:
        return self._weight_slots if self._weight_slots is not None else self.inner.switch_mlp

    # ------------------------------------------------------------------ admission
    def _release_finished(self) -> None:
        self._pending = [(ev, keep) for ev, keep in self._pending if not ev.query()]

    def _maybe_admit(self, routed_eids: torch.Tensor, on_miss=None, dispatch: ops.Dispatch | None = None):
        """qwen3_x_moe.py:136-208.  Returns (unique eids on host, inverse_map
        on device, the step's Dispatch with resolved slot ids).

        ``on_miss(d)``, when given, is called once the step is known to miss
        and before any blob is read, with the step's Dispatch (missed experts
        have slot id -1 there): work queued by it runs on the GPU while the
        host reads the missed blobs, and the slot refills do not wait for it
        (they wait only for the compute stream's work queued before it).
        ``dispatch``: the step's dispatch when the routing kernel already
        built it against the current slot table."""
        assert self.expert_loader is not None and self._weight_slots is not None
        self._release_finished()
        d = dispatch if dispatch is not None else ops.dispatch(routed_eids, self.num_experts, self.eid2sid_device)
        counts = d.counts.cpu()  # the one host read of a hit-only step
        n_unique, n_missed = int(counts[0]), int(counts[1])
        self.admit_stats["steps"] += 1
        self.admit_stats["unique"] += n_unique
        self.admit_stats["missed"] += n_missed
        if n_unique > self.num_slots:
            raise RuntimeError(
                f"MoE block {self.block_idx}: total slots available ({self.num_slots}) "
                f" < unique experts routed across the batch ({n_unique}). Either "
                f"decrease batch size or initialize {self.__class__.__name__!r} with more slots."
            )
        unique = d.unique[:n_unique].cpu().numpy()
        if n_missed == 0:
            return unique, d.inverse, d
        missed = unique[self._eid_lookup_table[unique] < 0]
        glob_eids = self.block_idx * self.num_experts + missed
        compute = torch.cuda.current_stream(self._device)
        before = torch.cuda.Event()
        before.record(compute)  # earlier steps' reads of the slots about to be replaced are queued before this
        if on_miss is not None:
            on_miss(d)
        acquired = self._choose_slots(missed.size, protected=unique)
        old = self._sid_lookup_table[acquired]
        evicted = old[old >= 0]
        self._eid_lookup_table[evicted] = EMPTY
        self._sid_lookup_table[acquired] = EMPTY
        blobs = self.expert_loader.load_sync(glob_eids.tolist())
        # refills run on a side stream: they start once earlier work on the
        # compute stream (the previous steps' reads of the replaced slots) is
        # done, while the GLU over the resident experts and the shared expert
        # run; the GLU over the missed experts waits on them
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(self._device)
        copy = self._copy_stream
        copy.wait_event(before)
        for eid, sid, payload in zip(missed, acquired, blobs):
            self._weight_slots.refill_from_blob(int(sid), payload.as_tensor(), copy)
            self._eid_lookup_table[eid] = sid
            self._sid_lookup_table[sid] = eid
        ev = torch.cuda.Event()
        ev.record(copy)
        self._pending.append((ev, blobs))
        self._refill_event = ev
        self.sync_device()
        d.slot_ids[:n_unique] = self.eid2sid_device[d.unique[:n_unique].long()]
        return unique, d.inverse, d

    def _prefetch_predicted(self) -> None:
        """Queue PREFETCH reads (loader.enqueue_prefetch, never blocking) of
        the most often routed experts that are in no slot and not cached on
        the host yet, so that a later miss on them costs only the copy."""
        cand = np.argsort(-self._routed_freq, kind="stable")
        cand = cand[self._eid_lookup_table[cand] < 0]
        cache = self.expert_cache
        picks = []
        for e in cand:
            g = self.block_idx * self.num_experts + int(e)
            if cache is not None and g in cache:
                continue
            picks.append(g)
            if len(picks) == self.prefetch_experts:
                break
        if picks:
            self.expert_loader.enqueue_prefetch(picks, await_free_slot=False)

    # ------------------------------------------------------------------ forward
    def _shared_begin(self, x2: torch.Tensor):
        """Queue the shared expert and its gate on a side stream (they only
        need x); returns the pending (y, gate) for _shared_end."""
        if self.inner.shared_expert is None:
            return None
        main = torch.cuda.current_stream(x2.device)
        if self._side_stream is None:
            self._side_stream = torch.cuda.Stream(x2.device)
        side = self._side_stream
        side.wait_stream(main)
        if not torch.cuda.is_current_stream_capturing():  # a graph's pool keeps its tensors alive
            x2.record_stream(side)  # read on the side stream after the caller may drop it
        with torch.cuda.stream(side):
            sy = shared_expert_forward(self.inner.shared_expert, x2)
            sg = ops.router_linear(x2, self.inner.shared_expert_gate)
        return sy, sg

    def _shared_end(self, pending):
        """Join the side stream; the shared results become usable on the
        current stream."""
        if pending is None:
            return None, None
        sy, sg = pending
        main = torch.cuda.current_stream(sy.device)
        main.wait_stream(self._side_stream)
        if not torch.cuda.is_current_stream_capturing():
            sy.record_stream(main)
            sg.record_stream(main)
        return sy, sg

    def _gather_forward_dispatched(self, x2: torch.Tensor, d: ops.Dispatch, arena: SlottedGLU) -> torch.Tensor:
        return ops.gather_forward(arena, x2, d, self.inner.top_k)

    def _gather_forward(self, x, gate_proj, up_proj, down_proj, slot_idxs, inverse_map):
        """qwen3_x_moe.py:210-248: pair p = t*k + j runs expert slot
        ``slot_idxs[inverse_map[p]]``.  The projections must be this block's
        arena tensors (they are read in place).  Returns [B, S, k, H]."""
        arena = self.arena
        if gate_proj is not arena.gate_proj or up_proj is not arena.up_proj or down_proj is not arena.down_proj:
            raise ValueError("_gather_forward reads this block's arena in place; pass its gate/up/down tensors")
        B, S, H = x.shape
        k = self.inner.top_k
        slot_idxs = torch.as_tensor(slot_idxs, dtype=torch.int32, device=x.device)
        inv = torch.as_tensor(inverse_map, dtype=torch.int32, device=x.device).reshape(-1)
        d = ops.dispatch(inv, int(slot_idxs.numel()), slot_idxs)
        y = self._gather_forward_dispatched(x.reshape(B * S, H), d, arena)
        return y.reshape(B, S, k, H)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """qwen3_x_moe.py:250-297.  x [B, S, H] bf16 -> [B, S, H] bf16."""
        if self.inner.sharding_group is not None:
            raise NotImplementedError("tensor-parallel sharding groups are not supported; use ep.ExpertParallelMoE")
        B, S, H = x.shape
        x2 = x.reshape(B * S, H).contiguous()
        logits = ops.router_linear(x2, self.inner.gate)
        # softmax / top-k / renorm fused with the slot lookup and the pair
        # permutation (sg_route_dispatch; _get_routings + the np.unique of
        # _maybe_admit + the slot lookup of qwen3_x_moe.py:277)
        table = self._identity if self.expert_cache is None else self.eid2sid_device
        trace = None
        if self.should_capture_traces and hasattr(self.recorder, "reserve"):
            # the routing kernel writes the step's ids / scores / logits into
            # the recorder's pinned host ring as it computes them
            trace = self.recorder.reserve(B * S, self._capture_gate_logits)
        inds, scores, d_step = ops.route_dispatch(logits, self.inner.top_k, self.inner.norm_topk_prob, table,
                                                  self._route_work, trace=trace)
        admitted = None
        early: dict = {}
        if self.expert_cache is not None:
            flat = inds.reshape(-1)

            def start_resident(d):
                # missed experts have slot -1 in d: the GLU skips their pairs
                # (zero rows, rewritten below) and runs the rest now
                early["missed_ids"] = torch.where(self.eid2sid_device[flat.long()] < 0, flat, torch.full_like(flat, -1))
                early["y"] = self._gather_forward_dispatched(x2, d, self._weight_slots)

            admitted = self._maybe_admit(inds, on_miss=start_resident, dispatch=d_step)  # refills on the side stream
        pending = self._shared_begin(x2)
        if self.should_capture_traces:
            self.recorder.capture(layer_path=self.layer_path, layer_class="Qwen3NextSparseMoeBlock",
                                  block_idx=self.block_idx, expert_ids=inds.reshape(B, S, -1),
                                  softmax_weights=scores.reshape(B, S, -1),
                                  gate_logits=logits if self._capture_gate_logits else None)
        if self.expert_cache is None:
            y = self._gather_forward_dispatched(x2, d_step, self.inner.switch_mlp)
        else:
            unique, _inverse, d = admitted
            slot_ids = self._eid_lookup_table[unique]
            if early:
                # the resident experts' pairs already ran; now the missed
                # experts' pairs, once their slots are refilled
                y = early["y"]
                torch.cuda.current_stream(self._device).wait_event(self._refill_event)
                self._refill_event = None
                dm = ops.dispatch(early["missed_ids"], self.num_experts, self.eid2sid_device)
                h = ops.glu_gate_up(self._weight_slots, x2, dm, self.inner.top_k, _abi.SG_OUT_DISPATCH_ORDER)
                ops.glu_down(self._weight_slots, h, dm, _abi.SG_IN_DISPATCH_ORDER, out=y)
            else:
                y = self._gather_forward_dispatched(x2, d, self._weight_slots)
            self._touch(slot_ids)
            self._routed_freq[unique] += 1
            if self.prefetch_experts > 0:
                self._prefetch_predicted()
        shared_y, shared_gate = self._shared_end(pending)
        out = _combine_shared(y.reshape(B * S, self.inner.top_k, H), scores, shared_y, shared_gate)
        return out.reshape(B, S, H)

    def capture(self, B: int, S: int, warmup: int = 2, seed: int = 0) -> None:
        """Record the layer call for [B, S, H] inputs in a CUDA graph, so that
        ``replay`` runs it on new tokens for the host cost of one graph
        launch.  Only the non-streaming wrapper (every expert resident, no
        trace recorder): the streaming branch reads slot misses on the host.
        No counterpart in the reference (MLX builds its own graphs)."""
        if self.expert_cache is not None or self._identity is None:
            raise ValueError("only the non-streaming wrapper (all experts resident) can be captured")
        if self.should_capture_traces:
            raise ValueError("a wrapper with a trace recorder cannot be captured")
        dev = self._device
        g = torch.Generator(device=dev).manual_seed(seed)
        H = self.inner.hidden_size
        self.graph_input = torch.randn((B, S, H), generator=g, device=dev).to(torch.bfloat16)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):  # warm-up off the default stream, as capture requires
            for _ in range(warmup):
                self(self.graph_input)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        n0 = ops.LAUNCHES[0]
        with torch.cuda.graph(graph):
            self.graph_output = self(self.graph_input)
        self._graph_launches = ops.LAUNCHES[0] - n0
        self._graph = graph

    def replay(self, x: torch.Tensor | None = None) -> torch.Tensor:
        """One captured layer call; ``x`` (if given) is first copied into the
        graph's input.  Returns the graph's output buffer [B, S, H],
        overwritten by the next replay."""
        if getattr(self, "_graph", None) is None:
            raise RuntimeError("capture() first")
        if x is not None:
            self.graph_input.copy_(x, non_blocking=True)
        self._graph.replay()
        ops.LAUNCHES[0] += self._graph_launches
        return self.graph_output

    def host_pipeline(self) -> "ops.HostPipeline":
        """Replays of the captured call fed from and drained to pinned host
        buffers, with the copies overlapped with the neighbouring steps'
        compute (``ops.HostPipeline``).  ``capture`` first."""
        if getattr(self, "_graph", None) is None:
            raise RuntimeError("capture() first")
        return ops.HostPipeline(self.graph_input, self.graph_output, self.replay)

    def forward_resident(self, x2: torch.Tensor, timing: dict | None = None) -> torch.Tensor:
        """The non-streaming step on [T, H] with no host synchronisation at all
        (capturable in a CUDA graph): every expert is resident.  ``timing``
        (optional) receives CUDA events around the routed gate/up and down
        kernels plus the step's Dispatch, for per-kernel timing."""
        if self._identity is None:
            raise RuntimeError("forward_resident needs the non-streaming (all-resident) wrapper")
        pending = self._shared_begin(x2)
        logits = ops.router_linear(x2, self.inner.gate)
        inds, scores, d = ops.route_dispatch(logits, self.inner.top_k, self.inner.norm_topk_prob, self._identity,
                                             self._route_work)
        arena = self.inner.switch_mlp
        y = ops.gather_forward(arena, x2, d, self.inner.top_k, timing=timing)
        shared_y, shared_gate = self._shared_end(pending)
        return ops.combine(y, scores, shared_y, None if shared_gate is None else shared_gate.reshape(-1))

    # ------------------------------------------------------------------ factory
    @staticmethod
    def make_wrapper_factory(*, model_fingerprint: str | None = None, recorder=None, capture_gate_logits: bool = False,
                             expert_loader=None, expert_cache=None, num_slots: int = 0, slot_size: int = 0,
                             slot_policy: str = "reference", prefetch_experts: int = 0) -> Callable:
        """qwen3_x_moe.py:299-337.  ``candidate`` needs ``layer_path`` and
        ``block_idx`` attributes (LayerCandidate)."""

        def factory(module: SparseMoeBlock, candidate) -> Qwen3_xMoEWrapper:
            if getattr(candidate, "block_idx", None) is None:
                raise ValueError(
                    f"Cannot instrument layer {getattr(candidate, 'layer_path', '?')!r} because the index of its "
                    "parent transformer block could not be determined."
                )
            return Qwen3_xMoEWrapper(module, model_fingerprint, candidate.layer_path, candidate.block_idx,
                                     recorder, capture_gate_logits, expert_loader, expert_cache, num_slots,
                                     slot_size, slot_policy=slot_policy, prefetch_experts=prefetch_experts)

        return factory


SlottedMoE = Qwen3_xMoEWrapper
