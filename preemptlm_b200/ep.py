"""Expert parallelism for the slotted MoE layer: one process per GPU, the
experts of every layer split evenly across ranks, token dispatch and combine
over NVLink -- by the library's own peer-memory exchange kernels on GPUs (the
default), or by NCCL / gloo all-to-alls.

Rank r of R owns experts [r*E/R, (r+1)*E/R) in its arena (slot = expert id -
r*E/R); the router and the shared expert are replicated; every rank routes its
own tokens.  Per layer:

  1. route the local tokens (router GEMV + softmax/top-k) and queue the local
     shared expert;
  2. order the T*k (token, expert) pairs by owning rank; exchange the per-rank
     pair counts (all-to-all of R ints, the one host read of the step);
  3. all-to-all the pairs' hidden rows and their local expert ids;
  4. run the gathered SwiGLU on the received rows against the local arena;
  5. all-to-all the expert outputs back, restore pair order, combine with the
     routing scores and the shared expert's output.

The math of steps 1, 4, 5 goes through a ``backend`` object so that the same
exchange logic runs with the CUDA kernels (``CudaBackend``) on GPUs and with a
CPU implementation in the multi-process CPU tests.

Two transports for steps 2, 3 and 5:
  * ``"p2p"`` (GPUs, the default there): the library's own exchange kernels
    over NVLink peer memory (``sg_ep_*``, ``PeerExchange``).  Every rank owns
    an inbox per source rank sized for the worst case, sources write rows,
    expert ids and pair ids straight into it and raise a per-step flag, and
    outputs go back the same way into the source's pair-order buffer.  There
    is no host read in the step, so the host queues steps ahead of the GPU.
  * ``"collective"``: ``torch.distributed.all_to_all_single`` (NCCL or gloo)
    with the per-rank pair counts read on the host; the CPU tests use it.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, replace

import torch
import torch.distributed as dist

from . import _abi, ops
from .arena import SlottedGLU


class ExchangeTimeoutError(_abi.SlottedGLUError):
    """A bounded wait of the peer-memory exchange expired (a peer did not
    take part in the step in time)."""


def set_wait_limit(seconds: float) -> None:
    """Wait limit of the exchange kernels launched from now on, on the current
    device (default 2 s)."""
    _abi.call("sg_ep_set_wait_limit", int(round(seconds * 1e6)))


@dataclass
class ExpertShard:
    """This rank's slice of a layer: experts [first, first + count)."""

    rank: int
    world: int
    num_experts: int

    @property
    def count(self) -> int:
        return self.num_experts // self.world

    @property
    def first(self) -> int:
        return self.rank * self.count


def check_divisible(num_experts: int, world: int) -> None:
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")


class CudaBackend:
    """Per-rank math on the libsg_b200 kernels."""

    def __init__(self, router: torch.Tensor, top_k: int, norm_topk_prob: bool, arena: SlottedGLU,
                 shared: SlottedGLU | None, shared_gate: torch.Tensor | None):
        self.router, self.top_k, self.norm = router, top_k, norm_topk_prob
        self.arena, self.shared, self.shared_gate = arena, shared, shared_gate
        self.ident = torch.arange(arena.num_slots, dtype=torch.int32, device=router.device)
        self.timing: dict | None = None  # receives events around the expert kernels when set
        self._side: torch.cuda.Stream | None = None  # the shared expert's stream

    def route(self, x: torch.Tensor):
        logits = ops.router_linear(x, self.router)
        return ops.route_topk(logits, self.top_k, self.norm)

    def experts(self, rows: torch.Tensor, local_eids: torch.Tensor) -> torch.Tensor:
        d = ops.dispatch(local_eids, self.arena.num_slots, self.ident)
        y = ops.gather_forward(self.arena, rows, d, 1, timing=self.timing)
        if self.timing is not None:
            self.timing.setdefault("rows", []).append(rows.shape[0])
        return y

    def experts_inbox(self, rows: torch.Tensor, local_eids: torch.Tensor, expected_pairs: int) -> torch.Tensor:
        """The experts over peer-exchange inboxes in place: ``rows`` [N, H]
        with ``local_eids`` [N] (-1: empty entry, skipped by the dispatch).
        Returns y [N, H] with each filled entry's output in its row."""
        N = rows.shape[0]
        d = ops.dispatch(local_eids, self.arena.num_slots, self.ident)
        # the pair-tile width follows the mean pairs per group: count only the
        # entries expected to be filled (a host hint; any bound >= the groups works)
        hint = -(-N * self.arena.num_slots // max(1, expected_pairs))
        d = replace(d, grid_groups=max(d.grid_groups, min(2048, hint)))
        # the fused call: rows permuted into dispatch order first for large
        # groups (TMA row loads), pieces of the filled entries for the
        # integer-operand kernels at decode sizes
        y = ops.gather_forward(self.arena, rows, d, 1, timing=self.timing)
        if self.timing is not None:
            # filled entries (group_off[U]): read after timing
            self.timing.setdefault("rows", []).append((d.counts, d.group_off))
        return y

    def shared_terms(self, x: torch.Tensor):
        """The shared expert and its gate, queued on a side stream beside the
        exchange and the routed experts; joined by ``combine``."""
        if self.shared is None:
            return None, None
        from .layer import shared_expert_forward

        main = torch.cuda.current_stream(x.device)
        if self._side is None:
            self._side = torch.cuda.Stream(x.device)
        self._side.wait_stream(main)
        if not torch.cuda.is_current_stream_capturing():  # a graph's pool keeps its tensors alive
            x.record_stream(self._side)
        with torch.cuda.stream(self._side):
            sy = shared_expert_forward(self.shared, x)
            sg = ops.router_linear(x, self.shared_gate).reshape(-1)
        return sy, sg

    def combine(self, y: torch.Tensor, scores: torch.Tensor, shared_y, shared_gate) -> torch.Tensor:
        if shared_y is not None:
            main = torch.cuda.current_stream(y.device)
            main.wait_stream(self._side)
            if not torch.cuda.is_current_stream_capturing():
                shared_y.record_stream(main)
                shared_gate.record_stream(main)
        return ops.combine(y, scores, shared_y, shared_gate)


class _DeviceArray:
    """A raw device pointer as a tensor source (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "strides": None, "version": 3}


def _view(ptr: int, shape, dtype, device) -> torch.Tensor:
    code = {torch.bfloat16: "<i2", torch.int32: "<i4"}[dtype]
    t = torch.as_tensor(_DeviceArray(ptr, shape, code), device=device)
    return t.view(dtype) if dtype == torch.bfloat16 else t


class PeerExchange:
    """This rank's buffers of the NVLink peer-memory exchange (``sg_ep_*``).

    One region per rank (allocated by the library, every peer's region mapped
    here by CUDA IPC), laid out identically on all ranks for ``max_tokens``
    tokens per rank per step.  Creation and ``close`` are collective."""

    def __init__(self, group, world: int, rank: int, max_tokens: int, top_k: int, hidden: int, device):
        lib = _abi.load()
        self.lib, self.world, self.rank, self.hidden = lib, world, rank, hidden
        self.cap = max_tokens * top_k
        self.device = torch.device(device)
        nbytes = lib.sg_ep_region_bytes(world, self.cap, hidden)
        _abi.check(min(0, nbytes), "sg_ep_region_bytes")
        region = ctypes.c_void_p()
        _abi.check(lib.sg_ep_alloc(nbytes, ctypes.byref(region)), "sg_ep_alloc")
        self.region = region.value
        handle = (ctypes.c_uint8 * 64)()
        _abi.check(lib.sg_ep_ipc_handle(ctypes.c_void_p(self.region), handle), "sg_ep_ipc_handle")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened, bases = [], []
        for r in range(world):
            if r == rank:
                bases.append(self.region)
                continue
            p = ctypes.c_void_p()
            _abi.check(lib.sg_ep_ipc_open((ctypes.c_uint8 * 64).from_buffer_copy(handles[r]), ctypes.byref(p)),
                       "sg_ep_ipc_open")
            self.opened.append(p.value)
            bases.append(p.value)
        self.regions = (ctypes.c_void_p * world)(*bases)
        off = (ctypes.c_longlong * 5)()
        _abi.check(lib.sg_ep_layout(world, self.cap, hidden, off), "sg_ep_layout")
        n = world * self.cap
        self.rows = _view(self.region + off[0], (n, hidden), torch.bfloat16, self.device)
        self.eids = _view(self.region + off[1], (n,), torch.int32, self.device)
        self.ybuf = _view(self.region + off[4], (self.cap, hidden), torch.bfloat16, self.device)
        self.dcnt = torch.zeros(world, dtype=torch.int32, device=self.device)  # inbox slot counters (kept at zero)
        self.group = group

    def close(self) -> None:
        """Collective: every rank stops touching every region before any is freed."""
        if self.region is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self.opened:
            _abi.check(self.lib.sg_ep_ipc_close(ctypes.c_void_p(p)), "sg_ep_ipc_close")
        dist.barrier(group=self.group)
        _abi.check(self.lib.sg_ep_free(ctypes.c_void_p(self.region)), "sg_ep_free")
        self.region, self.opened = None, []


class ExpertParallelMoE:
    """One slotted MoE layer split expert-parallel over the process group."""

    def __init__(self, backend, num_experts: int, hidden: int, top_k: int, group=None, transport: str | None = None,
                 max_tokens: int = 256, exchange: "PeerExchange | None" = None):
        """``exchange``: a peer exchange to use instead of allocating one (p2p
        transport), e.g. one shared by the layers of a stack, which run one
        after another.  It must have this layer's world, hidden size and room
        for ``max_tokens * top_k`` pairs per source; the layer does not close
        it."""
        self.backend = backend
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        check_divisible(num_experts, self.world)
        self.shard = ExpertShard(self.rank, self.world, num_experts)
        self.num_experts, self.hidden, self.top_k = num_experts, hidden, top_k
        self.last_counts = None  # (send, recv) per-rank pair counts of the last collective step
        if transport is None:
            transport = "p2p" if isinstance(backend, CudaBackend) else "collective"
        if transport not in ("p2p", "collective"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport = transport
        self.max_tokens = max_tokens
        self.exchange = None
        self._owns_exchange = False
        if transport == "p2p":
            if exchange is None:
                exchange = PeerExchange(group, self.world, self.rank, max_tokens, top_k, hidden,
                                        backend.router.device)
                self._owns_exchange = True
            elif exchange.world != self.world or exchange.hidden != hidden or exchange.cap < max_tokens * top_k:
                raise ValueError("the shared exchange does not fit this layer (world, hidden or pair capacity)")
            self.exchange = exchange
        self._graph = None
        self.graph_input = self.graph_output = None
        self._graph_launches = 0
        self.broken = False  # set by check() after a timed-out exchange wait

    def capture(self, T: int, warmup: int = 2, seed: int = 0) -> None:
        """Record one peer-exchange step for T tokens in a CUDA graph, so that
        a step costs the host one graph launch (``replay``).  Collective:
        every rank captures with the same arguments (the warm-up steps
        exchange with the peers).  The step number lives on the device, so
        replays synchronise correctly."""
        if self.transport != "p2p":
            raise ValueError("only the p2p transport can be captured")
        dev = self.backend.router.device
        g = torch.Generator(device=dev).manual_seed(seed)
        self.graph_input = torch.randn((T, self.hidden), generator=g, device=dev).to(torch.bfloat16)
        timing, self.backend.timing = self.backend.timing, None
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):  # warm-up off the default stream, as capture requires
            for _ in range(warmup):
                self._forward_p2p(self.graph_input)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        n0 = ops.LAUNCHES[0]
        with torch.cuda.graph(graph):
            self.graph_output = self._forward_p2p(self.graph_input)
        self._graph_launches = ops.LAUNCHES[0] - n0
        self._graph = graph
        self.backend.timing = timing

    def replay(self, x: torch.Tensor | None = None) -> torch.Tensor:
        """One captured step; ``x`` (if given) is first copied into the
        graph's input.  Returns the graph's output buffer, overwritten by
        the next replay."""
        if self.broken:
            raise ExchangeTimeoutError(_abi.SG_ERR_TIMEOUT, "expert-parallel exchange (timed out earlier; rebuild it)")
        if x is not None:
            self.graph_input.copy_(x, non_blocking=True)
        self._graph.replay()
        ops.LAUNCHES[0] += self._graph_launches
        return self.graph_output

    def host_pipeline(self) -> "ops.HostPipeline":
        """Replays of the captured step fed from and drained to pinned host
        buffers, the copies overlapped with the neighbouring steps' compute
        (``ops.HostPipeline``).  ``capture`` first."""
        if self._graph is None:
            raise RuntimeError("capture() first")
        return ops.HostPipeline(self.graph_input, self.graph_output, self.replay)

    def check(self) -> None:
        """Read the device status word (synchronises): raise
        ``ExchangeTimeoutError`` if a bounded wait of an exchange kernel gave
        up since the last check.  The outputs of such a step had the late
        rank's rows zeroed, and the exchange is out of step with its peers (a
        late peer may still write into this rank's region), so it is marked
        broken: later steps raise until it is closed and rebuilt.  Call it
        between steps, outside timed regions and graph replays."""
        st = ops.device_status(reset=True)
        if st == _abi.SG_ERR_TIMEOUT:
            self.broken = True
            raise ExchangeTimeoutError(st, "expert-parallel exchange")
        _abi.check(st, "expert-parallel step")

    def close(self) -> None:
        """Collective: release the captured graph and the peer-exchange
        buffers (p2p transport)."""
        self._graph = None
        self.graph_input = self.graph_output = None
        if self.exchange is not None and self._owns_exchange:
            self.exchange.close()
        self.exchange = None

    def _forward_p2p(self, x: torch.Tensor) -> torch.Tensor:
        if self.broken:
            raise ExchangeTimeoutError(_abi.SG_ERR_TIMEOUT, "expert-parallel exchange (timed out earlier; rebuild it)")
        ex, lib = self.exchange, self.exchange.lib
        T, H = x.shape
        k, R, per = self.top_k, self.world, self.shard.count
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the exchange's {self.max_tokens} per rank")
        x = x.contiguous()
        timing = getattr(self.backend, "timing", None)
        marks = [] if timing is not None else None

        def mark():  # phase boundaries of the step, when timing
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append(ev)

        mark()
        inds, scores = self.backend.route(x)
        shared_y, shared_gate = self.backend.shared_terms(x)
        mark()
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _abi.check(lib.sg_ep_send(ex.regions, R, self.rank, ex.cap, H, x.data_ptr(), inds.data_ptr(), T, k, per,
                                  ex.dcnt.data_ptr(), stream), "sg_ep_send")
        mark()
        _abi.check(lib.sg_ep_wait_inbox(ctypes.c_void_p(ex.region), R, ex.cap, H, stream), "sg_ep_wait_inbox")
        mark()
        y_local = self.backend.experts_inbox(ex.rows, ex.eids, T * k)
        mark()
        _abi.check(lib.sg_ep_send_back(ex.regions, R, self.rank, ex.cap, H, y_local.data_ptr(), stream),
                   "sg_ep_send_back")
        mark()
        _abi.check(lib.sg_ep_wait_back(ctypes.c_void_p(ex.region), R, ex.cap, H, inds.data_ptr(), T, k, per, stream),
                   "sg_ep_wait_back")
        mark()
        ops.LAUNCHES[0] += 6
        out = self.backend.combine(ex.ybuf[: T * k], scores, shared_y, shared_gate)
        mark()
        if marks is not None:
            timing.setdefault("phases", []).append(marks)
        return out

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits) -> None:
        if out.dtype == torch.bfloat16:  # moved as raw bytes (an all-to-all is a copy; gloo has no bf16)
            out, inp = out.view(torch.uint8), inp.contiguous().view(torch.uint8)
        dist.all_to_all_single(out, inp.contiguous(), output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=self.group)

    def begin(self, x: torch.Tensor) -> dict:
        """Everything of a step that does not need the pair counts on the
        host: routing, the shared expert, the send order and rows, and the
        count exchange, whose result is copied to pinned host memory without
        blocking.  ``end`` finishes the step."""
        T, H = x.shape
        k, R, per = self.top_k, self.world, self.shard.count
        inds, scores = self.backend.route(x)
        shared_y, shared_gate = self.backend.shared_terms(x)
        flat = inds.reshape(-1).to(torch.int64)
        dest = torch.div(flat, per, rounding_mode="floor")
        order = torch.argsort(dest, stable=True)            # pair ids in send order
        # scatter-add rather than bincount: bincount sizes its output from the
        # data, a device-to-host wait in the middle of the step
        send_counts = torch.zeros(R, dtype=torch.int64, device=dest.device).scatter_add_(0, dest,
                                                                                      torch.ones_like(dest))
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send_rows = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
        send_eid = (flat.index_select(0, order) - dest.index_select(0, order) * per).to(torch.int32)
        counts = torch.stack([send_counts, recv_counts])
        if counts.is_cuda:
            host = torch.empty(counts.shape, dtype=counts.dtype).pin_memory()
            host.copy_(counts, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record()
        else:
            host, ready = counts, None
        return {"T": T, "H": H, "dtype": x.dtype, "device": x.device, "scores": scores, "shared_y": shared_y,
                "shared_gate": shared_gate, "order": order, "send_rows": send_rows, "send_eid": send_eid,
                "counts": host, "ready": ready}

    def end(self, st: dict) -> torch.Tensor:
        """The exchange, the local experts and the combine of a begun step
        (the one host wait: the pair counts)."""
        if st["ready"] is not None:
            st["ready"].synchronize()
        send, recv = st["counts"][0].tolist(), st["counts"][1].tolist()
        self.last_counts = (send, recv)
        n_recv, T, H, k = sum(recv), st["T"], st["H"], self.top_k
        recv_rows = torch.empty((n_recv, H), dtype=st["dtype"], device=st["device"])
        recv_eid = torch.empty((n_recv,), dtype=torch.int32, device=st["device"])
        self._a2a(recv_rows, st["send_rows"], recv, send)
        self._a2a(recv_eid, st["send_eid"], recv, send)
        y_local = self.backend.experts(recv_rows, recv_eid)
        y_back = torch.empty((T * k, H), dtype=st["dtype"], device=st["device"])
        self._a2a(y_back, y_local, send, recv)
        y = torch.empty_like(y_back)
        y.index_copy_(0, st["order"], y_back)
        return self.backend.combine(y, st["scores"], st["shared_y"], st["shared_gate"])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [T, H] bf16 (this rank's tokens) -> [T, H] bf16."""
        if self.transport == "p2p":
            return self._forward_p2p(x)
        return self.end(self.begin(x))

    def forward_many(self, xs) -> list:
        """Several independent token batches (micro-batches of one step).
        Collective transport: every batch's count exchange is queued before
        the host waits on the first, so the GPU stays busy while the host
        issues the rest."""
        if self.transport == "p2p":
            return [self._forward_p2p(x) for x in xs]
        states = [self.begin(x) for x in xs]
        return [self.end(s) for s in states]

    __call__ = forward


class ExpertParallelStack:
    """The MoE blocks of a decoder stack, each expert-parallel: L layers
    applied in turn to the residual stream, ``x <- x + layer(x)`` (the
    attention blocks between them are outside this library).  The layers may
    share one peer exchange: they run one after another on the stream, so a
    rank's next send into a peer follows its wait for that peer's outputs of
    the layer before, as between two steps of one layer.  ``capture`` records
    the whole stack as one CUDA graph."""

    def __init__(self, layers):
        self.layers = list(layers)
        if not self.layers:
            raise ValueError("a stack needs at least one layer")
        self._graph = None
        self.graph_input = self.graph_output = None
        self._graph_launches = 0

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [T, H] bf16 (this rank's tokens) -> the residual stream after
        every layer, [T, H] bf16."""
        for layer in self.layers:
            x = x + layer.forward(x)
        return x

    __call__ = forward

    def capture(self, T: int, warmup: int = 2, seed: int = 0) -> None:
        """Collective: one CUDA graph of the whole stack for T tokens (p2p
        layers; see ``ExpertParallelMoE.capture``)."""
        if any(layer.transport != "p2p" for layer in self.layers):
            raise ValueError("only p2p layers can be captured")
        dev = self.layers[0].backend.router.device
        g = torch.Generator(device=dev).manual_seed(seed)
        self.graph_input = torch.randn((T, self.layers[0].hidden), generator=g, device=dev).to(torch.bfloat16)
        timings = [layer.backend.timing for layer in self.layers]
        for layer in self.layers:
            layer.backend.timing = None
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.forward(self.graph_input)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        n0 = ops.LAUNCHES[0]
        with torch.cuda.graph(graph):
            self.graph_output = self.forward(self.graph_input)
        self._graph_launches = ops.LAUNCHES[0] - n0
        self._graph = graph
        for layer, t in zip(self.layers, timings):
            layer.backend.timing = t

    def replay(self, x: torch.Tensor | None = None) -> torch.Tensor:
        """One captured pass through the stack (``x`` first copied into the
        graph's input); returns the graph's output buffer."""
        if any(layer.broken for layer in self.layers):
            raise ExchangeTimeoutError(_abi.SG_ERR_TIMEOUT, "expert-parallel exchange (timed out earlier; rebuild it)")
        if x is not None:
            self.graph_input.copy_(x, non_blocking=True)
        self._graph.replay()
        ops.LAUNCHES[0] += self._graph_launches
        return self.graph_output

    def host_pipeline(self) -> "ops.HostPipeline":
        """Replays fed from and drained to pinned host buffers, the copies
        overlapped with the neighbouring steps' compute.  ``capture`` first."""
        if self._graph is None:
            raise RuntimeError("capture() first")
        return ops.HostPipeline(self.graph_input, self.graph_output, self.replay)

    def check(self) -> None:
        """As ``ExpertParallelMoE.check``; a timeout marks every layer broken."""
        st = ops.device_status(reset=True)
        if st == _abi.SG_ERR_TIMEOUT:
            for layer in self.layers:
                layer.broken = True
            raise ExchangeTimeoutError(st, "expert-parallel exchange")
        _abi.check(st, "expert-parallel stack step")

    def close(self) -> None:
        """Collective: release the graph, the layers and every exchange they
        use (a shared one once)."""
        self._graph = None
        self.graph_input = self.graph_output = None
        shared = []
        for layer in self.layers:
            ex = layer.exchange
            if ex is not None and not layer._owns_exchange and all(ex is not o for o in shared):
                shared.append(ex)
            layer.close()
        for ex in shared:
            ex.close()


def shard_layer(cfg, rank: int, world: int, device, seed_offset: int = 0, layer: int = 0):
    """This rank's shard of the seeded synthetic layer ``cfg``: the same global
    weights for any world size (all experts generated, the shard kept).
    ``layer`` > 0 draws another layer of a stack (every tensor from its own
    seeds)."""
    from .synthetic import _gen, _randn, fill_arena, make_expert_tensors

    check_divisible(cfg.num_experts, world)
    sh = ExpertShard(rank, world, cfg.num_experts)
    c = cfg.cfg_id + 1_000_000 * layer
    router = _randn((cfg.num_experts, cfg.hidden), _gen(1000 * c + 1, device), device, 0.02)
    full = make_expert_tensors(cfg, cfg.num_experts, cfg.inter, 1000 * c + 2 + seed_offset, device)
    mine = {k: v[sh.first: sh.first + sh.count].contiguous() for k, v in full.items()}
    del full
    arena = SlottedGLU(sh.count, (cfg.inter, cfg.hidden), (cfg.hidden, cfg.inter), quant=cfg.quant, device=device)
    fill_arena(arena, mine)
    shared = sgate = None
    if cfg.shared_inter is not None:
        st = make_expert_tensors(cfg, 1, cfg.shared_inter, 1000 * c + 3, device)
        shared = SlottedGLU(1, (cfg.shared_inter, cfg.hidden), (cfg.hidden, cfg.shared_inter), quant=cfg.quant,
                            device=device)
        fill_arena(shared, st)
        sgate = _randn((1, cfg.hidden), _gen(1000 * c + 4, device), device, 0.02)
    backend = CudaBackend(router, cfg.top_k, cfg.norm_topk_prob, arena, shared, sgate)
    return backend, mine
