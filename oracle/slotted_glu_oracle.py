"""CPU oracle for the SlottedGLU MoE hot path.

TEST INFRASTRUCTURE ONLY.  This module is the checker: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it.  The product path (``preemptlm_b200``) never imports, calls or links it.

It restates, in numpy, the algorithm of preemptLM's slotted MoE block
(``preempt/backends/mlx_metal/module_wrappers/qwen3_x_moe.py``) and its slot
bookkeeping (``preempt/backends/mlx_metal/module_wrappers/base_moe_wrapper.py``).
The floating-point arithmetic of that block lives in mlx 0.32.2 / mlx-lm 0.31.3
(``uv.lock:1680-1681``, ``uv.lock:1725-1726``), which are not vendored in the
reference and cannot be installed here.  The MLX calls are restated from their
published semantics:

* ``mx.softmax(precise=True)``: fp32 internal, output in the input dtype (bf16).
* ``mx.argpartition(kth=-k)[..., -k:]``: the k largest; MLX leaves the order and
  the tie order unspecified.  The oracle fixes a total order
  (gate value descending, expert id ascending) and the CUDA kernel uses the same.
* ``mx.gather_mm`` / ``mx.gather_qmm(transpose=True, mode="affine")``: per-pair
  matmul against the selected expert, fp32 accumulation, bf16 output; affine
  dequantisation ``w = scale * q + bias`` per group of ``group_size`` input
  weights, q packed little-endian in uint32 words.

PARITY STATUS: the integer bookkeeping (``choose_slots``, ``touch``,
``maybe_admit``, ``decode_serialized_expert``) is pinned against the reference's
own Python run under a numpy stand-in for ``mlx`` (fixtures in
``tests/golden/``, made by ``tests/golden/make_golden.py``).  The floating-point
layer math is **parity unpinned** against MLX itself (no MLX on this machine);
it is pinned only against these restated semantics.

Reduction orders that the CUDA kernels reproduce bit-for-bit (so that routing is
bit-exact):

* Router dot product (``router_logits``): 32 lane partial sums, lane j adding
  ``x[h] * w[h]`` for ``h = 256*i + 8*j + e`` in (i, e) order, then a pairwise
  fold 16, 8, 4, 2, 1.  bf16 x bf16 products are exact in fp32, so fused and
  unfused multiply-add agree.
* Softmax sum (``softmax_bf16``): lane j adds ``exp(l[e] - max)`` for
  ``e = j, j+32, ...`` then the same fold.
* ``sg_exp``: e^x by Cody-Waite reduction (x = n ln2 + r, ln2 split into a
  15-bit head and a tail) and a degree-7 Taylor polynomial of e^r in Horner
  form, every step one IEEE-rounded fp32 multiply or add.
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_ROUTER_CHUNK = 64  # tokens per work item of router_logits (numpy releases the GIL)

# --------------------------------------------------------------------------- bf16


def bf16_round(a) -> np.ndarray:
    """Round fp32 values to the nearest bf16 value (ties to even), kept as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = a.view(np.uint32).astype(np.uint64)
    lsb = (b >> 16) & 1
    r = ((b + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    nan = np.isnan(a)
    if nan.any():
        r = np.where(nan, np.uint32(0x7FC00000), r)
    return r.view(np.float32)


def bf16_bits_to_f32(u16) -> np.ndarray:
    u = np.ascontiguousarray(u16).view(np.uint16).astype(np.uint32) << 16
    return u.view(np.float32)


def f32_to_bf16_bits(a) -> np.ndarray:
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


# --------------------------------------------------------------------------- exp

def _f32(bits: int) -> np.float32:
    return np.array([bits], np.uint32).view(np.float32)[0]


# exact fp32 constants (bit patterns shared with the CUDA routing kernel)
LOG2E = _f32(0x3FB8AA3B)  # log2(e)
LN2_HI = _f32(0x3F317200)  # head of ln2, 15 significant bits
LN2_LO = _f32(0x35BFBE8E)  # ln2 - LN2_HI
# Taylor coefficients 1/7!, 1/6!, 1/5!, 1/4!, 1/3!, 1/2!, 1/1!, 1/0!
_TAYLOR = [_f32(0x39500D01), _f32(0x3AB60B61), _f32(0x3C088889), _f32(0x3D2AAAAB),
           _f32(0x3E2AAAAB), _f32(0x3F000000), _f32(0x3F800000), _f32(0x3F800000)]


def sg_exp(x) -> np.ndarray:
    """e^x for fp32 x <= 0, the routing kernel's exp (see module docstring)."""
    x = np.asarray(x, dtype=np.float32)
    n = np.rint(x * LOG2E).astype(np.float32)
    r = (x - n * LN2_HI).astype(np.float32)
    r = (r - n * LN2_LO).astype(np.float32)
    p = _TAYLOR[0]
    for c in _TAYLOR[1:]:
        p = (p * r).astype(np.float32)
        p = (p + c).astype(np.float32)
    ni = np.clip(n, -126, 127).astype(np.int32)
    scale = ((ni + 127).astype(np.uint32) << 23).view(np.float32)
    out = (p * scale).astype(np.float32)
    return np.where(n < -126, np.float32(0.0), out).astype(np.float32)


def _lane_fold(v: np.ndarray) -> np.ndarray:
    """Pairwise fold of a trailing 32-lane axis: 16, 8, 4, 2, 1."""
    off = 16
    while off >= 1:
        v = (v[..., :off] + v[..., off : 2 * off]).astype(np.float32)
        off //= 2
    return v[..., 0]


# --------------------------------------------------------------------------- router (a1)


def router_logits(x_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """bf16 logits = x @ w^T in the router's lane order.

    Follows ``logits = self.inner.gate(x)`` (``qwen3_x_moe.py:254``), an mlx_lm
    bias-free ``nn.Linear``: bf16 in, fp32 accumulate, bf16 out.  Also used for
    the shared-expert gate ``self.inner.shared_expert_gate(x)`` (``:259``).

    x_bits: [T, H] uint16 (bf16 bits); w_bits: [E, H] uint16.  H % 256 == 0.
    Returns [T, E] uint16 bf16 bits.
    """
    T, H = x_bits.shape
    E = w_bits.shape[0]
    assert H % 256 == 0
    # [i, e, rows, lane]: element h = 256 i + 8 lane + e of every row
    Xt = np.ascontiguousarray(bf16_bits_to_f32(x_bits).reshape(T, H // 256, 32, 8).transpose(1, 3, 0, 2))
    Wt = np.ascontiguousarray(bf16_bits_to_f32(w_bits).reshape(E, H // 256, 32, 8).transpose(1, 3, 0, 2))
    out = np.empty((T, E), np.uint16)

    def tokens(t0: int) -> None:  # one chunk of tokens; the order of adds per lane is (i, e)
        t1 = min(T, t0 + _ROUTER_CHUNK)
        acc = np.zeros((t1 - t0, E, 32), np.float32)
        tmp = np.empty_like(acc)
        for i in range(H // 256):
            for e in range(8):
                np.multiply(Xt[i, e, t0:t1, None, :], Wt[i, e][None], out=tmp)
                np.add(acc, tmp, out=acc)
        out[t0:t1] = f32_to_bf16_bits(_lane_fold(acc))

    starts = range(0, T, _ROUTER_CHUNK)
    if T > _ROUTER_CHUNK:
        with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
            list(ex.map(tokens, starts))
    else:
        for t0 in starts:
            tokens(t0)
    return out


# --------------------------------------------------------------------------- routing (a2)


def softmax_bf16(logit_bits: np.ndarray) -> np.ndarray:
    """``mx.softmax(logits, axis=-1, precise=True)`` (``qwen3_x_moe.py:32``).

    fp32 internally, bf16 out.  E % 32 == 0.  Returns [T, E] uint16 bits.
    """
    T, E = logit_bits.shape
    assert E % 32 == 0
    lg = bf16_bits_to_f32(logit_bits)
    m = lg.max(axis=1, keepdims=True)
    ex = sg_exp((lg - m).astype(np.float32))
    lanes = ex.reshape(T, E // 32, 32)
    acc = np.zeros((T, 32), dtype=np.float32)
    for c in range(E // 32):
        acc += lanes[:, c, :]
    s = _lane_fold(acc)
    return f32_to_bf16_bits((ex / s[:, None]).astype(np.float32))


def get_routings(logit_bits: np.ndarray, top_k: int, norm_topk_prob: bool):
    """``_get_routings`` (``qwen3_x_moe.py:26-40``).

    softmax -> k largest gates -> take -> optional renormalisation.  The k
    indices are returned in the fixed total order (gate desc, expert id asc);
    the renormalising sum adds the k bf16 scores in that order in fp32 and
    rounds to bf16 (the dtype of ``scores.sum``), then ``scores / sum`` is one
    fp32 division rounded to bf16.

    Returns (inds [T, k] int32, scores [T, k] uint16 bf16 bits, gates bits).
    """
    gates = softmax_bf16(logit_bits)
    T, E = gates.shape
    eid = np.arange(E, dtype=np.int64)
    key = (gates.astype(np.int64) << 16) | (0xFFFF - eid)[None, :]
    order = np.argsort(-key, axis=1, kind="stable")[:, :top_k]
    inds = order.astype(np.int32)
    sc_bits = np.take_along_axis(gates, order, axis=1)
    if norm_topk_prob:
        sc = bf16_bits_to_f32(sc_bits)
        acc = np.zeros(T, dtype=np.float32)
        for j in range(top_k):
            acc = (acc + sc[:, j]).astype(np.float32)
        ssum = bf16_bits_to_f32(f32_to_bf16_bits(acc))
        sc_bits = f32_to_bf16_bits((sc / ssum[:, None]).astype(np.float32))
    return inds, sc_bits, gates


# --------------------------------------------------------------------------- slot bookkeeping (a3-a6)

EMPTY = -1  # CacheSlotState.EMPTY, preempt/core/enums.py:42-46


class SlotTables:
    """eid<->sid tables and LFRU counters of ``BaseMoEWrapper``
    (``base_moe_wrapper.py:105-121``)."""

    def __init__(self, num_experts: int, num_slots: int):
        self.num_slots = num_slots
        self.eid_lookup = np.full(num_experts, EMPTY, np.int32)
        self.sid_lookup = np.full(num_slots, EMPTY, np.int32)
        self.clock = 0
        self.freq = np.zeros(num_slots, np.int64)
        self.recency = np.zeros(num_slots, np.int64)

    def touch(self, slots: np.ndarray) -> None:
        """``_touch`` (``base_moe_wrapper.py:152-155``)."""
        self.clock += 1
        np.add.at(self.freq, slots, 1)
        self.recency[slots] = self.clock

    def choose_slots(self, n: int, protected: np.ndarray) -> np.ndarray:
        """``_choose_slots`` (``base_moe_wrapper.py:157-172``), bug for bug:
        ``np.delete`` shortens the score array, so the returned positions index
        the shortened array, and free slots may be picked again by argsort."""
        free = np.nonzero(self.sid_lookup < 0)[0]
        if free.size >= n:
            return free[:n]
        prot = self.eid_lookup[protected]
        prot = prot[prot >= 0]
        score = self.freq * (self.clock + 1) + self.recency
        score = np.delete(score, prot)
        evicted = np.argsort(score, kind="stable")[: n - free.size]
        return np.concatenate([free, evicted])

    def maybe_admit(self, routed_eids: np.ndarray, load_fn=None):
        """``_maybe_admit`` (``qwen3_x_moe.py:136-208``) without the arena
        writes: returns (unique, inverse_map, missed_eids, acquired_slots,
        evicted_eids).  ``load_fn(missed, acquired)`` is called where the
        reference loads and writes the slots (``:184-195``)."""
        flat = np.asarray(routed_eids).reshape(-1)
        unique, inverse = np.unique(flat, return_inverse=True)
        if unique.size > self.num_slots:
            raise RuntimeError(
                f"total slots available ({self.num_slots}) < unique experts routed "
                f"across the batch ({unique.size})"
            )
        missed = unique[self.eid_lookup[unique] < 0]
        if missed.size == 0:
            return unique, inverse.astype(np.int32), missed, np.zeros(0, np.int64), np.zeros(0, np.int32)
        acquired = self.choose_slots(missed.size, protected=unique)
        old = self.sid_lookup[acquired]
        evicted = old[old >= 0]
        self.eid_lookup[evicted] = EMPTY
        self.sid_lookup[acquired] = EMPTY
        if load_fn is not None:
            load_fn(missed, acquired)
        for eid, sid in zip(missed, acquired):
            self.eid_lookup[eid] = sid
            self.sid_lookup[sid] = eid
        return unique, inverse.astype(np.int32), missed, acquired, evicted


# --------------------------------------------------------------------------- MLX affine quantisation (a12)


def quantize_affine(w_bits: np.ndarray, bits: int, group_size: int = 64):
    """Per-group min/max affine quantisation of a bf16 [out, in] matrix into the
    MLX layout: packed uint32 [out, in*bits/32], scales/biases bf16 [out, in/gs].

    scale = (max - min) / (2^bits - 1) and bias = min, both rounded to bf16,
    then q = clip(rint((w - bias) / scale)).  Packing is little-endian within
    each uint32 word (weight m of a word at bits [m*bits, (m+1)*bits)).
    """
    w = bf16_bits_to_f32(w_bits)
    out, inn = w.shape
    assert inn % group_size == 0 and 32 % bits == 0
    g = w.reshape(out, inn // group_size, group_size)
    mn = g.min(axis=2)
    mx = g.max(axis=2)
    nmax = (1 << bits) - 1
    scale = bf16_round((mx - mn) / np.float32(nmax))
    bias = bf16_round(mn)
    safe = np.where(scale == 0, np.float32(1), scale)
    q = np.rint((g - bias[..., None]) / safe[..., None])
    q = np.where(scale[..., None] == 0, 0, q)
    q = np.clip(q, 0, nmax).astype(np.uint32).reshape(out, inn)
    per = 32 // bits
    qw = q.reshape(out, inn // per, per)
    packed = np.zeros((out, inn // per), np.uint32)
    for m in range(per):
        packed |= qw[:, :, m] << np.uint32(m * bits)
    return packed, f32_to_bf16_bits(scale), f32_to_bf16_bits(bias)


def unpack_affine(packed: np.ndarray, bits: int) -> np.ndarray:
    out, words = packed.shape
    per = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    q = np.zeros((out, words, per), np.uint32)
    for m in range(per):
        q[:, :, m] = (packed >> np.uint32(m * bits)) & mask
    return q.reshape(out, words * per)


def dequant_affine(packed, scale_bits, bias_bits, bits: int, group_size: int = 64) -> np.ndarray:
    """w = bf16(scale * q + bias), fp32 arithmetic (one rounding for the add).
    Returns fp32 values that are exactly bf16."""
    q = unpack_affine(np.asarray(packed, dtype=np.uint32), bits).astype(np.float32)
    out, inn = q.shape
    s = np.repeat(bf16_bits_to_f32(scale_bits), group_size, axis=1)
    b = np.repeat(bf16_bits_to_f32(bias_bits), group_size, axis=1)
    return bf16_round((s * q).astype(np.float32) + b)


# --------------------------------------------------------------------------- expert math (a9-a11)


def _sigmoid32(v):
    v = np.asarray(v, np.float32)
    return (np.float32(1) / (np.float32(1) + np.exp(-v))).astype(np.float32)


def swiglu(x_up: np.ndarray, x_gate: np.ndarray) -> np.ndarray:
    """``swiglu_activation = silu(gate) * up`` (``ops/experts.py:26-28``) with
    silu(g) = g * sigmoid(g) and bf16 rounding after each elementwise op."""
    sig = bf16_round(_sigmoid32(x_gate))
    return bf16_round(bf16_round(x_gate * sig) * x_up)


def _mm_bf16(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    """bf16(a @ w^T) with fp32 accumulation."""
    return bf16_round(np.matmul(a.astype(np.float32), w.astype(np.float32).T))


class ExpertWeights:
    """Dequantised (exactly-bf16 fp32) weights of one expert: gate/up [I, H],
    down [H, I]."""

    def __init__(self, gate, up, down):
        self.gate, self.up, self.down = gate, up, down


def expert_forward(x: np.ndarray, ew: ExpertWeights) -> np.ndarray:
    """One expert's SwiGLU on rows x [n, H] (exact bf16 values as fp32)."""
    x_up = _mm_bf16(x, ew.up)
    x_gate = _mm_bf16(x, ew.gate)
    return _mm_bf16(swiglu(x_up, x_gate), ew.down)


def gather_forward(x: np.ndarray, experts_by_slot, slot_ids: np.ndarray, inverse_map: np.ndarray, top_k: int):
    """``_gather_forward`` (``qwen3_x_moe.py:210-248``): pair p = t*k + j uses
    expert slot ``slot_ids[inverse_map[p]]``.  Returns y [T, k, H] (bf16 fp32)."""
    T, H = x.shape
    inv = np.asarray(inverse_map).reshape(T * top_k)
    y = np.zeros((T * top_k, H), np.float32)
    for u in np.unique(inv):
        pairs = np.nonzero(inv == u)[0]
        ew = experts_by_slot[int(slot_ids[u])]
        y[pairs] = expert_forward(x[pairs // top_k], ew)
    return y.reshape(T, top_k, H)


def combine_shared(y, scores, shared_y=None, shared_gate=None):
    """``_combine_shared`` (``qwen3_x_moe.py:71-80``):
    ``sum_k(y * score) + sigmoid(shared_gate) * shared_y``.  Products round to
    bf16, the k-sum adds in fp32 in k order and rounds to bf16, the shared term
    rounds to bf16 after the sigmoid and after the product, the final add rounds
    to bf16."""
    T, k, H = y.shape
    acc = np.zeros((T, H), np.float32)
    for j in range(k):
        acc = (acc + bf16_round(y[:, j, :] * scores[:, j : j + 1])).astype(np.float32)
    out = bf16_round(acc)
    if shared_y is not None:
        sgate = bf16_round(_sigmoid32(shared_gate.reshape(T, 1)))
        out = bf16_round(out + bf16_round(sgate * shared_y))
    return out


# --------------------------------------------------------------------------- whole layer


def layer_forward(x_bits, router_w_bits, top_k, norm_topk_prob, experts_by_eid,
                  shared: ExpertWeights | None = None, shared_gate_w_bits=None):
    """``Qwen3_xMoEWrapper.__call__`` (``qwen3_x_moe.py:250-297``) with every
    routed expert resident (the reference's non-streaming branch ``:272-273``,
    identity slot map).  Returns dict of intermediates, all fp32/uint16 arrays."""
    T, H = x_bits.shape
    x = bf16_bits_to_f32(x_bits)
    logits = router_logits(x_bits, router_w_bits)
    inds, sc_bits, _ = get_routings(logits, top_k, norm_topk_prob)
    unique, inverse = np.unique(inds.reshape(-1), return_inverse=True)
    y = gather_forward(x, experts_by_eid, unique, inverse, top_k)
    shared_y = sg = None
    if shared is not None:
        shared_y = expert_forward(x, shared)
        sg = bf16_bits_to_f32(router_logits(x_bits, shared_gate_w_bits))
    out = combine_shared(y, bf16_bits_to_f32(sc_bits), shared_y, sg)
    return {"logits": logits, "inds": inds, "scores": sc_bits, "unique": unique,
            "inverse": inverse.astype(np.int32), "y": y, "shared_y": shared_y, "out": out}
