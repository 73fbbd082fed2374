"""Torch-facing wrappers of the C-ABI kernels (one function per entry point).

All tensors must be CUDA tensors on the current device; results are
allocated with torch and written by the kernels on the current stream.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _abi

# number of kernel launches issued through this module (read by the benchmark)
LAUNCHES = [0]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _bf16_2d(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype != torch.bfloat16 or not t.is_cuda or t.dim() != 2:
        raise TypeError(f"{name} must be a 2-D bf16 CUDA tensor")
    return t.contiguous()


def router_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """bf16(x @ w^T), fp32 accumulation in the fixed router order
    (``sg_router_logits``; qwen3_x_moe.py:254, :259)."""
    x = _bf16_2d(x, "x")
    w = _bf16_2d(w, "w")
    T, H = x.shape
    E = w.shape[0]
    out = torch.empty((T, E), dtype=torch.bfloat16, device=x.device)
    LAUNCHES[0] += T > 0
    _abi.call("sg_router_logits", x.data_ptr(), w.data_ptr(), out.data_ptr(), T, H, E, _stream())
    return out


def route_topk(logits: torch.Tensor, top_k: int, norm_topk_prob: bool):
    """``_get_routings`` (qwen3_x_moe.py:26-40): (inds int32 [T, k], scores bf16 [T, k])."""
    logits = _bf16_2d(logits, "logits")
    T, E = logits.shape
    inds = torch.empty((T, top_k), dtype=torch.int32, device=logits.device)
    scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=logits.device)
    LAUNCHES[0] += T > 0
    _abi.call("sg_route_topk", logits.data_ptr(), T, E, int(top_k), int(bool(norm_topk_prob)), inds.data_ptr(),
              scores.data_ptr(), _stream())
    return inds, scores


@dataclass
class Dispatch:
    """Device-side unique/inverse/slot/permutation of one step (sg_dispatch)."""

    unique: torch.Tensor     # [max_unique] int32, first counts[0] valid (ascending)
    inverse: torch.Tensor    # [P] int32
    counts: torch.Tensor     # [2] int32: (U, #missed)
    slot_ids: torch.Tensor   # [max_unique] int32
    miss_eids: torch.Tensor  # [max_unique] int32
    group_off: torch.Tensor  # [max_unique] int32 (U + 1 valid)
    perm: torch.Tensor       # [P] int32
    grid_groups: int         # host upper bound on U


def dispatch(ids: torch.Tensor, num_ids: int, eid2sid: torch.Tensor) -> Dispatch:
    ids = ids.reshape(-1)
    if ids.dtype != torch.int32 or not ids.is_cuda:
        raise TypeError("ids must be int32 CUDA")
    if eid2sid.dtype != torch.int32 or eid2sid.numel() < num_ids:
        raise TypeError("eid2sid must be int32 with num_ids entries")
    P = ids.numel()
    mu = min(P, num_ids) + 1
    dev = ids.device
    d = Dispatch(
        unique=torch.empty(mu, dtype=torch.int32, device=dev),
        inverse=torch.empty(P, dtype=torch.int32, device=dev),
        counts=torch.empty(2, dtype=torch.int32, device=dev),
        slot_ids=torch.empty(mu, dtype=torch.int32, device=dev),
        miss_eids=torch.empty(mu, dtype=torch.int32, device=dev),
        group_off=torch.empty(mu, dtype=torch.int32, device=dev),
        perm=torch.empty(P, dtype=torch.int32, device=dev),
        grid_groups=mu - 1,
    )
    LAUNCHES[0] += 1
    _abi.call("sg_dispatch", ids.contiguous().data_ptr(), P, int(num_ids), eid2sid.data_ptr(), d.unique.data_ptr(),
              d.inverse.data_ptr(), d.counts.data_ptr(), d.slot_ids.data_ptr(), d.miss_eids.data_ptr(),
              d.group_off.data_ptr(), d.perm.data_ptr(), mu, _stream())
    return d


def route_dispatch(logits: torch.Tensor, top_k: int, norm_topk_prob: bool, eid2sid: torch.Tensor,
                   work: torch.Tensor, trace=None):
    """``_get_routings`` plus the dispatch of the routed pairs in one launch
    (``sg_route_dispatch``): (inds int32 [T, k], scores bf16 [T, k],
    Dispatch).  ``work`` is an int32 [E + 1] zero buffer owned by the caller
    (left zero; one call at a time per buffer).  ``trace``: an
    ``_abi.sg_route_trace`` of device-visible addresses the kernel also writes
    the ids, scores and logits to (router telemetry), or None."""
    logits = _bf16_2d(logits, "logits")
    T, E = logits.shape
    if eid2sid.dtype != torch.int32 or eid2sid.numel() < E:
        raise TypeError("eid2sid must be int32 with E entries")
    if work.dtype != torch.int32 or work.numel() < E + 1 or not work.is_cuda:
        raise TypeError("work must be an int32 CUDA tensor of E + 1 zeros")
    dev = logits.device
    P = T * top_k
    mu = min(P, E) + 1
    inds = torch.empty((T, top_k), dtype=torch.int32, device=dev)
    scores = torch.empty((T, top_k), dtype=torch.bfloat16, device=dev)
    d = Dispatch(
        unique=torch.empty(mu, dtype=torch.int32, device=dev),
        inverse=torch.empty(P, dtype=torch.int32, device=dev),
        counts=torch.empty(2, dtype=torch.int32, device=dev),
        slot_ids=torch.empty(mu, dtype=torch.int32, device=dev),
        miss_eids=torch.empty(mu, dtype=torch.int32, device=dev),
        group_off=torch.empty(mu, dtype=torch.int32, device=dev),
        perm=torch.empty(P, dtype=torch.int32, device=dev),
        grid_groups=mu - 1,
    )
    LAUNCHES[0] += 1
    _abi.call("sg_route_dispatch", logits.data_ptr(), T, E, int(top_k), int(bool(norm_topk_prob)), eid2sid.data_ptr(),
              inds.data_ptr(), scores.data_ptr(), d.unique.data_ptr(), d.inverse.data_ptr(), d.counts.data_ptr(),
              d.slot_ids.data_ptr(), d.miss_eids.data_ptr(), d.group_off.data_ptr(), d.perm.data_ptr(), mu,
              work.data_ptr(), None if trace is None else ctypes.byref(trace), _stream())
    return inds, scores, d


_TOKEN_DISPATCH: dict = {}


def token_dispatch(T: int, device) -> Dispatch:
    """A single group holding every token (the shared expert): pairs are
    tokens, slot 0.  Cached per (device, T): building it copies from the host."""
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    key = (str(dev), int(T))
    if key not in _TOKEN_DISPATCH:
        _TOKEN_DISPATCH[key] = _make_token_dispatch(T, dev)
    return _TOKEN_DISPATCH[key]


def _make_token_dispatch(T: int, dev) -> Dispatch:
    return Dispatch(
        unique=torch.zeros(2, dtype=torch.int32, device=dev),
        inverse=torch.zeros(T, dtype=torch.int32, device=dev),
        counts=torch.tensor([1, 0], dtype=torch.int32, device=dev),
        slot_ids=torch.zeros(2, dtype=torch.int32, device=dev),
        miss_eids=torch.zeros(2, dtype=torch.int32, device=dev),
        group_off=torch.tensor([0, T], dtype=torch.int32, device=dev),
        perm=torch.arange(T, dtype=torch.int32, device=dev),
        grid_groups=1,
    )


def glu_gate_up(arena, x: torch.Tensor, d: Dispatch, pair_div: int, flags: int = 0) -> torch.Tensor:
    """h = swiglu over the arena (``sg_glu_gate_up``); rows in pair order
    unless ``flags`` (SG_IN/OUT_DISPATCH_ORDER) say otherwise."""
    x = _bf16_2d(x, "x")
    P = d.perm.numel()
    h = torch.empty((P, arena.inter), dtype=torch.bfloat16, device=x.device)
    if P == 0:
        return h
    lib = _abi.load()
    desc = ctypes.byref(arena.desc())
    nwork = lib.sg_glu_gate_up_work_bytes(desc, P, int(pair_div), d.grid_groups, int(flags))
    if nwork < 0:
        _abi.check(int(nwork), "sg_glu_gate_up_work_bytes")
    LAST_GATE_UP[0] = "sg_glu_gate_up_work (piece split + integer-operand tcgen05)" if nwork > 0 else "sg_glu_gate_up"
    if nwork > 0:  # 8-bit arena at decode sizes: the token rows' pieces, then the integer-operand kernel
        work = torch.empty(int(nwork), dtype=torch.uint8, device=x.device)
        LAUNCHES[0] += 2
        _abi.check(lib.sg_glu_gate_up_work(desc, x.data_ptr(), P, int(pair_div), d.counts.data_ptr(),
                                           d.slot_ids.data_ptr(), d.group_off.data_ptr(), d.perm.data_ptr(),
                                           d.grid_groups, h.data_ptr(), int(flags), work.data_ptr(), int(nwork),
                                           _stream()), "sg_glu_gate_up_work")
        return h
    LAUNCHES[0] += 1
    _abi.check(lib.sg_glu_gate_up(desc, x.data_ptr(), P, int(pair_div), d.counts.data_ptr(),
                                  d.slot_ids.data_ptr(), d.group_off.data_ptr(), d.perm.data_ptr(), d.grid_groups,
                                  h.data_ptr(), int(flags), _stream()), "sg_glu_gate_up")
    return h


# which entry point the last glu_gate_up call took (for reports)
LAST_GATE_UP = ["sg_glu_gate_up"]


def quantize_pieces(x: torch.Tensor, order: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """8-bit pieces of the rows of x (``sg_quantize_pieces``): (pieces int8
    [rows, 2, K], ex fp32 [rows, K // 64, 2])."""
    x = _bf16_2d(x, "x")
    rows, K = x.shape
    pieces = torch.empty((rows, 2, K), dtype=torch.int8, device=x.device)
    ex = torch.empty((rows, K // 64, 2), dtype=torch.float32, device=x.device)
    if rows:
        LAUNCHES[0] += 1
        _abi.call("sg_quantize_pieces", x.data_ptr(), rows, K, int(order), pieces.data_ptr(), ex.data_ptr(),
                  _stream())
    return pieces, ex


def glu_down(arena, h: torch.Tensor, d: Dispatch, flags: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = h @ down^T over the arena (``sg_glu_down``); into ``out`` when
    given (only the rows of the dispatch's pairs are written)."""
    h = _bf16_2d(h, "h")
    P = d.perm.numel()
    if out is not None:
        if out.dtype != torch.bfloat16 or not out.is_contiguous() or tuple(out.shape) != (P, arena.hidden):
            raise TypeError(f"out must be a contiguous bf16 [{P}, {arena.hidden}] tensor")
        y = out
    else:
        y = torch.empty((P, arena.hidden), dtype=torch.bfloat16, device=h.device)
    if P == 0:
        return y
    lib = _abi.load()
    desc = ctypes.byref(arena.desc())
    nwork = lib.sg_glu_down_work_bytes(desc, P, d.grid_groups)
    if nwork < 0:
        _abi.check(int(nwork), "sg_glu_down_work_bytes")
    if nwork > 0:  # 8-bit arena at decode sizes: h's pieces, then the integer-operand kernel
        work = torch.empty(int(nwork), dtype=torch.uint8, device=h.device)
        LAUNCHES[0] += 2
        _abi.check(lib.sg_glu_down_work(desc, h.data_ptr(), P, d.counts.data_ptr(), d.slot_ids.data_ptr(),
                                        d.group_off.data_ptr(), d.perm.data_ptr(), d.grid_groups, y.data_ptr(),
                                        int(flags), work.data_ptr(), int(nwork), _stream()), "sg_glu_down_work")
        return y
    LAUNCHES[0] += 1
    _abi.check(lib.sg_glu_down(desc, h.data_ptr(), P, d.counts.data_ptr(), d.slot_ids.data_ptr(),
                               d.group_off.data_ptr(), d.perm.data_ptr(), d.grid_groups, y.data_ptr(), int(flags),
                               _stream()), "sg_glu_down")
    return y


def permute_rows(x: torch.Tensor, d: Dispatch, pair_div: int) -> torch.Tensor:
    """xs[pos] = x[perm[pos] // pair_div] for the dispatch's filled pair
    positions (``sg_permute_pairs``; rows past them are left unset)."""
    x = _bf16_2d(x, "x")
    P = d.perm.numel()
    xs = torch.empty((P, x.shape[1]), dtype=torch.bfloat16, device=x.device)
    if P:
        LAUNCHES[0] += 1
        _abi.check(_abi.load().sg_permute_pairs(x.data_ptr(), d.perm.data_ptr(), int(pair_div), d.counts.data_ptr(),
                                                d.group_off.data_ptr(), P, x.shape[1], xs.data_ptr(), _stream()),
                   "sg_permute_pairs")
    return xs


def _extra_launches(lib, desc, P: int, pair_div: int, grid_groups: int, scratch: bool) -> int:
    """Launches sg_glu_forward adds to its two GLU kernels: the row
    permutation, or one piece split per integer-operand projection."""
    if not scratch:
        return 0
    if lib.sg_glu_use_permute(desc, P, grid_groups) == 1:
        return 1
    return int(lib.sg_glu_gate_up_work_bytes(desc, P, pair_div, grid_groups, 0) > 0) + int(
        lib.sg_glu_down_work_bytes(desc, P, grid_groups) > 0)


def gather_forward(arena, x: torch.Tensor, d: Dispatch, pair_div: int, timing: dict | None = None) -> torch.Tensor:
    """y[p] = down(swiglu(gate(x[p // pair_div]), up(...))) for every pair, in
    pair order: the reference's ``_gather_forward`` (``sg_glu_forward``).
    With ``timing``, the same kernels run as separate calls with CUDA events
    around the gate/up and down launches (per-kernel timing)."""
    x = _bf16_2d(x, "x")
    P = d.perm.numel()
    lib = _abi.load()
    if timing is None:
        y = torch.empty((P, arena.hidden), dtype=torch.bfloat16, device=x.device)
        if P == 0:
            return y
        h = torch.empty((P, arena.inter), dtype=torch.bfloat16, device=x.device)
        desc = ctypes.byref(arena.desc())
        nscratch = lib.sg_glu_forward_scratch_bytes(desc, P, int(pair_div), d.grid_groups)
        if nscratch < 0:
            _abi.check(int(nscratch), "sg_glu_forward_scratch_bytes")
        # the permuted token rows, or the pieces of the token rows / of h
        xs = torch.empty(int(nscratch), dtype=torch.uint8, device=x.device) if nscratch > 0 else None
        LAUNCHES[0] += 2 + _extra_launches(lib, desc, P, int(pair_div), d.grid_groups, xs is not None)
        _abi.check(lib.sg_glu_forward(desc, x.data_ptr(), P, int(pair_div), d.counts.data_ptr(),
                                      d.slot_ids.data_ptr(), d.group_off.data_ptr(), d.perm.data_ptr(), d.grid_groups,
                                      None if xs is None else xs.data_ptr(), h.data_ptr(), y.data_ptr(), _stream()),
                   "sg_glu_forward")
        return y
    permute = P > 0 and lib.sg_glu_use_permute(ctypes.byref(arena.desc()), P, d.grid_groups) == 1
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    src, fl = (permute_rows(x, d, pair_div), _abi.SG_IN_DISPATCH_ORDER) if permute else (x, 0)
    ev[0].record()
    h = glu_gate_up(arena, src, d, pair_div, fl | _abi.SG_OUT_DISPATCH_ORDER)
    ev[1].record()
    y = glu_down(arena, h, d, _abi.SG_IN_DISPATCH_ORDER)
    ev[2].record()
    timing.setdefault("events", []).append(ev)
    timing.setdefault("dispatch", []).append(d.counts)  # U of the step (the rest is freed and reused)
    return y


def gather_forward_noalloc(arena, x: torch.Tensor, d: Dispatch, pair_div: int) -> torch.Tensor:
    """``gather_forward`` with the intermediate rows in the library's fixed
    device scratch area (``sg_glu_forward_noalloc``): no scratch tensors are
    allocated.  Calls overlapping in time on one device race on that area."""
    x = _bf16_2d(x, "x")
    P = d.perm.numel()
    y = torch.empty((P, arena.hidden), dtype=torch.bfloat16, device=x.device)
    if P == 0:
        return y
    lib = _abi.load()
    nscratch = lib.sg_glu_forward_scratch_bytes(ctypes.byref(arena.desc()), P, int(pair_div), d.grid_groups)
    LAUNCHES[0] += 2 + _extra_launches(lib, ctypes.byref(arena.desc()), P, int(pair_div), d.grid_groups,
                                       nscratch > 0)
    _abi.check(_abi.load().sg_glu_forward_noalloc(ctypes.byref(arena.desc()), x.data_ptr(), P, int(pair_div),
                                                  d.counts.data_ptr(), d.slot_ids.data_ptr(), d.group_off.data_ptr(),
                                                  d.perm.data_ptr(), d.grid_groups, y.data_ptr(), _stream()),
               "sg_glu_forward_noalloc")
    return y


def dense_glu(arena, x: torch.Tensor, sid: int = 0) -> torch.Tensor | None:
    """y = down(swiglu(gate(x), up(x))) of slot ``sid`` over every row of x
    (``sg_dense_glu``, the shared expert).  Returns None for shapes the dense
    tensor-core kernel does not take (the caller then runs the one-group
    gathered path)."""
    x = _bf16_2d(x, "x")
    T = x.shape[0]
    y = torch.empty((T, arena.hidden), dtype=torch.bfloat16, device=x.device)
    if T == 0:
        return y
    h = torch.empty((T, arena.inter), dtype=torch.bfloat16, device=x.device)
    lib = _abi.load()
    st = lib.sg_dense_glu(ctypes.byref(arena.desc()), int(sid), x.data_ptr(), T, h.data_ptr(), y.data_ptr(),
                          _stream())
    if st == _abi.SG_ERR_SHAPE:
        return None
    _abi.check(st, "sg_dense_glu")
    LAUNCHES[0] += 2
    return y


GLU_PATHS = {"auto": 0, "gemv": 1, "tc": 2, "tc-perm": 3, "i8": 4}


_GLU_PATH = ["auto"]


def set_glu_path(mode: str) -> None:
    """Pick the gathered-GLU kernel: "auto", "gemv" (streaming CUDA-core
    GEMV), "tc" (dequantising tcgen05 kernels), "tc-perm" (as "tc" with the
    token rows permuted) or "i8" (the integer-operand tcgen05 gate/up for
    8-bit arenas wherever it applies)."""
    _abi.call("sg_set_glu_path", GLU_PATHS[mode])
    _GLU_PATH[0] = mode


def set_glu_tile(bn: int) -> None:
    """Pair-tile width: 0 (automatic); 8 fixes the integer-operand kernels',
    32/64/128 the dequantising kernels', 16 both."""
    _abi.call("sg_set_glu_tile", int(bn))


def glu_path() -> str:
    return _GLU_PATH[0]


def device_status(reset: bool = True) -> int:
    """First error recorded by a kernel (SG_ERR_TIMEOUT after a bounded wait
    expired), or 0."""
    return int(_abi.load().sg_device_status(int(reset)))


def combine(y: torch.Tensor, scores: torch.Tensor, shared_y: torch.Tensor | None,
            shared_gate: torch.Tensor | None) -> torch.Tensor:
    """``_combine_shared`` (qwen3_x_moe.py:71-80) -> out [T, H] bf16."""
    T, k = scores.shape
    H = y.shape[-1]
    y = y.reshape(T * k, H).contiguous()
    out = torch.empty((T, H), dtype=torch.bfloat16, device=y.device)
    sy = shared_y.contiguous().data_ptr() if shared_y is not None else None
    sg = shared_gate.contiguous().data_ptr() if shared_gate is not None else None
    LAUNCHES[0] += T > 0
    _abi.call("sg_combine", y.data_ptr(), scores.contiguous().data_ptr(), T, k, H, sy, sg, out.data_ptr(), _stream())
    return out


class HostPipeline:
    """Host-buffer steps of a captured layer graph with the PCIe copies taken
    off the critical path: the host->device copy of step i+1 (into a device
    staging buffer, on an upload stream) and the device->host copy of step
    i-1 (from a staging buffer, on a download stream) run while the graph of
    step i computes.  The compute stream only moves the staged rows into and
    out of the graph's own buffers (device copies of a few microseconds).

    ``step(x_host, out_host)`` queues one step; ``out_host`` holds that step's
    output once ``drain()`` (or a synchronisation) has passed.  Steps are
    ordered as issued; ``depth`` staging buffers per direction."""

    def __init__(self, graph_input: torch.Tensor, graph_output: torch.Tensor, replay, depth: int = 2):
        dev = graph_input.device
        self._dev, self._gin, self._gout, self._replay, self._depth = dev, graph_input, graph_output, replay, depth
        self._up, self._down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        self._inb = [torch.empty_like(graph_input) for _ in range(depth)]
        self._outb = [torch.empty_like(graph_output) for _ in range(depth)]
        ev = lambda: [torch.cuda.Event() for _ in range(depth)]  # noqa: E731
        self._in_ready, self._in_free, self._out_ready, self._out_free = ev(), ev(), ev(), ev()
        self._i = 0

    def step(self, x_host: torch.Tensor, out_host: torch.Tensor) -> None:
        j, first = self._i % self._depth, self._i < self._depth
        cur = torch.cuda.current_stream(self._dev)
        with torch.cuda.stream(self._up):
            if not first:  # the compute stream has taken staging buffer j's previous rows
                self._up.wait_event(self._in_free[j])
            self._inb[j].copy_(x_host.view_as(self._inb[j]), non_blocking=True)
            self._in_ready[j].record(self._up)
        cur.wait_event(self._in_ready[j])
        self._gin.copy_(self._inb[j], non_blocking=True)
        self._in_free[j].record(cur)
        self._replay()
        if not first:  # staging buffer j's previous output has reached the host
            cur.wait_event(self._out_free[j])
        self._outb[j].copy_(self._gout, non_blocking=True)
        self._out_ready[j].record(cur)
        with torch.cuda.stream(self._down):
            self._down.wait_event(self._out_ready[j])
            out_host.view_as(self._outb[j]).copy_(self._outb[j], non_blocking=True)
            self._out_free[j].record(self._down)
        self._i += 1

    def drain(self) -> None:
        """Make the current stream wait for every queued copy."""
        cur = torch.cuda.current_stream(self._dev)
        cur.wait_stream(self._up)
        cur.wait_stream(self._down)
