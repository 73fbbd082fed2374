"""GPU parity: every kernel through the C-ABI against the CPU oracle.

Routing (logits, top-k ids, scores, unique/inverse, slot ids) is bit-exact;
GLU / layer outputs meet max-abs 2e-2 and rel-L2 1e-2 (bf16 tolerance).
"""

import numpy as np
import pytest
import torch

from oracle import slotted_glu_oracle as orc
from preemptlm_b200 import ops
from preemptlm_b200.synthetic import CONFIGS, LayerConfig, make_layer, make_tokens
from preemptlm_b200.layer import Qwen3_xMoEWrapper

from ._util import LazyExperts, assert_close, bits16, f32

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf16(shape, seed, std=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=DEV) * std).to(torch.bfloat16)


# ----------------------------------------------------------------------------- router / routing

@pytest.mark.parametrize("T,H,E", [(1, 2048, 512), (7, 256, 128), (33, 4096, 64), (9, 2048, 1), (256, 2048, 512),
                                   (256, 2048, 1), (5, 512, 31), (6, 512, 33)])
def test_router_logits_bitexact(T, H, E):
    x = _bf16((T, H), 1)
    w = _bf16((E, H), 2, 0.02)
    dev = bits16(ops.router_linear(x, w))
    ref = orc.router_logits(bits16(x), bits16(w))
    assert np.array_equal(dev, ref)


@pytest.mark.parametrize("E,k,norm", [(32, 1, True), (128, 8, True), (512, 10, True), (512, 10, False),
                                      (1024, 32, True), (96, 5, True)])
def test_route_topk_bitexact(E, k, norm):
    T = 300
    logits = _bf16((T, E), 3, 1.0)
    inds, scores = ops.route_topk(logits, k, norm)
    ri, rs, _ = orc.get_routings(bits16(logits), k, norm)
    assert np.array_equal(inds.cpu().numpy(), ri)
    assert np.array_equal(bits16(scores), rs)


def test_route_topk_ties_bitexact():
    """Logits on a coarse grid: many exact bf16 ties at the k-th gate."""
    T, E, k = 512, 512, 10
    g = torch.Generator(device=DEV).manual_seed(4)
    logits = torch.randint(-3, 4, (T, E), generator=g, device=DEV).float().mul(0.5).to(torch.bfloat16)
    inds, scores = ops.route_topk(logits, k, True)
    ri, rs, gates = orc.get_routings(bits16(logits), k, True)
    assert np.array_equal(inds.cpu().numpy(), ri)
    assert np.array_equal(bits16(scores), rs)
    kth = np.sort(gates, axis=1)[:, -k]
    ties = ((gates == kth[:, None]).sum(1) > 1).sum()
    assert ties > T // 2  # the case is really tie-heavy


def test_routing_from_router_bitexact_cfg3_full_size():
    cfg = CONFIGS["cfg3"]
    T = 256
    x = make_tokens(cfg, T)
    w = _bf16((cfg.num_experts, cfg.hidden), 5, 0.02)
    logits = ops.router_linear(x, w)
    inds, scores = ops.route_topk(logits, cfg.top_k, True)
    rl = orc.router_logits(bits16(x), bits16(w))
    ri, rs, _ = orc.get_routings(rl, cfg.top_k, True)
    assert np.array_equal(bits16(logits), rl)
    assert np.array_equal(inds.cpu().numpy(), ri)
    assert np.array_equal(bits16(scores), rs)


# ----------------------------------------------------------------------------- dispatch

@pytest.mark.parametrize("P,E,resident", [(1, 128, 1.0), (80, 128, 0.5), (2560, 512, 0.25), (65536, 128, 0.9),
                                          (40, 8192, 0.5)])
def test_dispatch_matches_numpy(P, E, resident):
    g = np.random.default_rng(P + E)
    ids = g.integers(0, E, size=P).astype(np.int32)
    eid2sid = np.where(g.random(E) < resident, g.permutation(E), -1).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(ids).to(DEV), E, torch.from_numpy(eid2sid).to(DEV))
    U, nmiss = d.counts.cpu().tolist()
    uq, inv = np.unique(ids, return_inverse=True)
    assert U == uq.size
    assert np.array_equal(d.unique[:U].cpu().numpy(), uq)
    assert np.array_equal(d.inverse.cpu().numpy(), inv)
    assert np.array_equal(d.slot_ids[:U].cpu().numpy(), eid2sid[uq])
    miss = uq[eid2sid[uq] < 0]
    assert nmiss == miss.size and np.array_equal(d.miss_eids[:nmiss].cpu().numpy(), miss)
    off = d.group_off[: U + 1].cpu().numpy()
    perm = d.perm.cpu().numpy()
    assert off[0] == 0 and off[-1] == P
    assert np.array_equal(np.sort(perm), np.arange(P))
    for u in range(U):
        grp = perm[off[u]: off[u + 1]]
        assert np.all(inv[grp] == u)


@pytest.mark.parametrize("T,E,k,resident", [(1, 512, 10, 1.0), (256, 512, 10, 1.0), (37, 128, 8, 0.5),
                                             (300, 1024, 32, 0.7), (2048, 128, 8, 0.5), (8192, 128, 8, 1.0),
                                             (5, 32, 1, 0.0), (64, 96, 5, 0.9)])
def test_route_dispatch_fused_matches_separate_calls(T, E, k, resident):
    """sg_route_dispatch (one launch) gives the ids and scores of
    sg_route_topk bit for bit and the dispatch of sg_dispatch (the order of
    pairs inside a group aside), and leaves its work buffer zero, on two calls
    in a row with one buffer."""
    g = np.random.default_rng(T + E)
    eid2sid = torch.from_numpy(np.where(g.random(E) < resident, g.permutation(E), -1).astype(np.int32)).to(DEV)
    work = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    for call in range(2):
        logits = _bf16((T, E), 30 + call, 1.0)
        inds, scores, d = ops.route_dispatch(logits, k, True, eid2sid, work)
        ri, rs = ops.route_topk(logits, k, True)
        assert torch.equal(inds, ri) and torch.equal(scores, rs)
        ref = ops.dispatch(ri, E, eid2sid)
        U = int(ref.counts[0].item())
        assert torch.equal(d.counts, ref.counts)
        for name in ("unique", "slot_ids", "group_off"):
            assert torch.equal(getattr(d, name)[: U + (name == "group_off")],
                               getattr(ref, name)[: U + (name == "group_off")]), name
        nm = int(ref.counts[1].item())
        assert torch.equal(d.miss_eids[:nm], ref.miss_eids[:nm])
        assert torch.equal(d.inverse, ref.inverse)
        off = d.group_off[: U + 1].cpu().numpy()
        a, b = d.perm.cpu().numpy(), ref.perm.cpu().numpy()
        for u in range(U):
            assert np.array_equal(np.sort(a[off[u]: off[u + 1]]), np.sort(b[off[u]: off[u + 1]]))
        assert int(work.abs().sum().item()) == 0


# ----------------------------------------------------------------------------- gathered GLU

@pytest.fixture
def glu_path(request):
    ops.set_glu_path(request.param)
    yield request.param
    ops.set_glu_path("auto")
    assert ops.device_status(reset=True) == 0  # no kernel gave up on a bounded wait


@pytest.mark.parametrize("glu_path", ["gemv", "tc", "tc-perm"], indirect=True)
@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("H,I,E,T,k", [(256, 128, 8, 5, 2), (2048, 768, 16, 33, 4), (1024, 512, 6, 1, 6),
                                       (512, 256, 4, 300, 2),
                                       # ~25 and ~50 pairs per expert: 32- and 64-wide pair tiles
                                       (512, 256, 8, 100, 2), (512, 256, 4, 100, 2),
                                       # K = 576 / 640: packed and row-gather stages end part-way
                                       (576, 256, 8, 40, 2), (640, 384, 8, 24, 3)])
def test_glu_matches_oracle(glu_path, bits, H, I, E, T, k):
    cfg = LayerConfig("t", 9, H, E, k, I, None, bits, E)
    block, tens = make_layer(cfg, device=DEV)
    x = _bf16((T, H), 11)
    g = np.random.default_rng(T * 7 + E)
    inds = np.stack([g.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(inds).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    h = ops.glu_gate_up(block.switch_mlp, x, d, pair_div=k)
    y = ops.glu_down(block.switch_mlp, h, d)
    ex = LazyExperts(tens["experts"], bits)
    xf = f32(x)
    href = np.zeros((T * k, I), np.float32)
    yref = np.zeros((T * k, H), np.float32)
    for p in range(T * k):
        ew = ex[inds.reshape(-1)[p]]
        xr = xf[p // k: p // k + 1]
        up = orc._mm_bf16(xr, ew.up)
        gate = orc._mm_bf16(xr, ew.gate)
        href[p] = orc.swiglu(up, gate)[0]
        yref[p] = orc._mm_bf16(href[p: p + 1], ew.down)[0]
    # intermediates: the north-star bound scaled by the largest magnitude (a
    # one-ulp bf16 flip of |h| ~ 8 is 0.06; the kernel skips the oracle's bf16
    # rounding of dequantised weights, so flips near rounding ties are expected)
    assert_close(f32(h), href, max_abs=2e-2 * max(1.0, float(np.abs(href).max())), what="h")
    assert_close(f32(y), yref, max_abs=2e-2 * max(1.0, float(np.abs(yref).max())), what="y")
    # the device's own h through the oracle's down projection: isolates down
    hdev = f32(h)
    ydown = np.stack([orc._mm_bf16(hdev[p: p + 1], ex[inds.reshape(-1)[p]].down)[0] for p in range(T * k)])
    assert_close(f32(y), ydown, max_abs=1e-2, rel=4e-3, what="y|h")
    # the fused call (h kept in dispatch order, token rows permuted first under
    # "tc-perm"): the same kernels' arithmetic, so the same bits
    assert torch.equal(ops.gather_forward(block.switch_mlp, x, d, k), y)


@pytest.mark.parametrize("glu_path", ["tc"], indirect=True)
@pytest.mark.parametrize("bits", [16, 8, 4])
def test_glu_forced_tile_widths(glu_path, bits):
    """sg_set_glu_tile fixes the dequantising kernels' pair tile: every width
    gives the oracle's h and y on groups of ~50 pairs (one 64- or 128-wide
    tile, two 32-wide or four 16-wide tiles per group)."""
    H, I, E, T, k = 512, 256, 4, 100, 2
    cfg = LayerConfig("t", 9, H, E, k, I, None, bits, E)
    block, tens = make_layer(cfg, device=DEV)
    x = _bf16((T, H), 5)
    g = np.random.default_rng(3)
    inds = np.stack([g.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(inds).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    ex = LazyExperts(tens["experts"], bits)
    xf = f32(x)
    href = np.stack([orc.swiglu(orc._mm_bf16(xf[p // k: p // k + 1], ex[inds.reshape(-1)[p]].up),
                                orc._mm_bf16(xf[p // k: p // k + 1], ex[inds.reshape(-1)[p]].gate))[0]
                     for p in range(T * k)])
    try:
        for bn in (16, 32, 64, 128):
            ops.set_glu_tile(bn)
            h = ops.glu_gate_up(block.switch_mlp, x, d, pair_div=k)
            assert_close(f32(h), href, max_abs=2e-2 * max(1.0, float(np.abs(href).max())), what=f"h bn={bn}")
            y = ops.glu_down(block.switch_mlp, h, d)
            hdev = f32(h)
            ydown = np.stack([orc._mm_bf16(hdev[p: p + 1], ex[inds.reshape(-1)[p]].down)[0] for p in range(T * k)])
            assert_close(f32(y), ydown, max_abs=1e-2, rel=4e-3, what=f"y|h bn={bn}")
    finally:
        ops.set_glu_tile(0)


@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("H,I,T", [(1024, 512, 2), (1024, 512, 37), (1024, 512, 256), (1024, 512, 1100),
                                   (1024, 512, 2400),  # 4 x 38 tiles of 64 > 148 SMs: 128-wide tiles
                                   (4096, 1024, 4096)])  # the 397B-style shared expert at prefill
def test_dense_glu_matches_oracle(bits, H, I, T):
    """The shared expert's dense path (sg_dense_glu): 16/32/64-wide pair tiles
    with TMA row loads, and 128-wide ones once the tiles overflow one wave.
    Rows are checked on a seeded sample (h and y)."""
    cfg = LayerConfig("t", 9, H, 3, 1, I, None, bits, 3)
    block, tens = make_layer(cfg, device=DEV)
    x = _bf16((T, H), 13)
    arena = block.switch_mlp
    h = torch.empty((T, I), dtype=torch.bfloat16, device=DEV)
    y = torch.empty((T, H), dtype=torch.bfloat16, device=DEV)
    from preemptlm_b200 import _abi
    import ctypes
    _abi.check(_abi.load().sg_dense_glu(ctypes.byref(arena.desc()), 2, x.data_ptr(), T, h.data_ptr(), y.data_ptr(),
                                        torch.cuda.current_stream().cuda_stream), "sg_dense_glu")
    rows = np.sort(np.random.default_rng(T).choice(T, min(T, 48), replace=False))
    ew = LazyExperts(tens["experts"], bits)[2]
    xr = f32(x)[rows]
    href = orc.swiglu(orc._mm_bf16(xr, ew.up), orc._mm_bf16(xr, ew.gate))
    assert_close(f32(h)[rows], href, max_abs=2e-2 * max(1.0, float(np.abs(href).max())), what="dense h")
    # down alone, from the device's own h: isolates the down projection
    ydown = orc._mm_bf16(f32(h)[rows], ew.down)
    # one bf16 ulp of the largest output (accumulation order differs)
    assert_close(f32(y)[rows], ydown, max_abs=1e-2 * max(1.0, float(np.abs(ydown).max())), rel=4e-3,
                 what="dense y|h")
    ref = orc._mm_bf16(href, ew.down)
    assert_close(f32(y)[rows], ref, max_abs=2e-2 * max(1.0, float(np.abs(ref).max())), what="dense y")
    assert torch.equal(ops.dense_glu(arena, x, sid=2), y)
    assert ops.device_status(reset=True) == 0


def test_glu_cfg4_shape_prefill_pairs():
    """Routed gate/up and down at the 397B-style layer shape (H 4096, I 1024,
    q4) with prefill-sized groups (128-wide pair tiles, token rows permuted):
    h and y of a sample of pairs against the oracle, down isolated from h."""
    cfg = CONFIGS["cfg4"]
    block, tens = make_layer(cfg.scaled(shared_inter=None), device=DEV)
    T, k, E = 4096, cfg.top_k, cfg.num_experts
    x = make_tokens(cfg, T)
    g = np.random.default_rng(41)
    inds = np.stack([g.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(inds).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    arena = block.switch_mlp
    xs = ops.permute_rows(x, d, k)
    h = ops.glu_gate_up(arena, xs, d, k, _abi_flags("in|out"))
    y = ops.glu_down(arena, h, d, _abi_flags("in"))
    perm = d.perm.cpu().numpy()
    pos = np.sort(g.choice(T * k, 40, replace=False))  # dispatch positions
    ex = LazyExperts(tens["experts"], cfg.bits)
    xf = f32(x)
    hd, yd = f32(h), f32(y)
    for q in pos:
        p = perm[q]
        ew = ex[inds.reshape(-1)[p]]
        xr = xf[p // k: p // k + 1]
        hr = orc.swiglu(orc._mm_bf16(xr, ew.up), orc._mm_bf16(xr, ew.gate))
        assert_close(hd[q: q + 1], hr, max_abs=2e-2 * max(1.0, float(np.abs(hr).max())), what=f"h pos {q}")
        yr = orc._mm_bf16(hd[q: q + 1], ew.down)
        assert_close(yd[p: p + 1], yr, max_abs=1e-2 * max(1.0, float(np.abs(yr).max())), rel=4e-3, what=f"y|h pair {p}")
    assert torch.equal(ops.gather_forward(arena, x, d, k), y)
    assert ops.device_status(reset=True) == 0


def _abi_flags(which: str) -> int:
    from preemptlm_b200 import _abi

    return {"in|out": _abi.SG_IN_DISPATCH_ORDER | _abi.SG_OUT_DISPATCH_ORDER,
            "in": _abi.SG_IN_DISPATCH_ORDER}[which]


def test_glu_skips_missing_slots():
    cfg = LayerConfig("t", 9, 256, 4, 1, 128, None, 8, 4)
    block, _ = make_layer(cfg, device=DEV)
    x = _bf16((3, 256), 12)
    inds = torch.tensor([[0], [1], [2]], dtype=torch.int32, device=DEV)
    eid2sid = torch.tensor([0, -1, 2, 3], dtype=torch.int32, device=DEV)
    d = ops.dispatch(inds, 4, eid2sid)
    assert d.counts.cpu().tolist() == [3, 1]
    h = ops.glu_gate_up(block.switch_mlp, x, d, pair_div=1)
    assert torch.all(h[1] == 0) and torch.any(h[0] != 0)


# ----------------------------------------------------------------------------- combine

@pytest.mark.parametrize("shared", [False, True])
def test_combine_matches_oracle(shared):
    T, k, H = 37, 10, 2048
    y = _bf16((T * k, H), 20, 0.1)
    sc = torch.rand((T, k), device=DEV).to(torch.bfloat16)
    sy = _bf16((T, H), 21, 0.1) if shared else None
    sg = _bf16((T,), 22) if shared else None
    out = ops.combine(y, sc, sy, sg)
    ref = orc.combine_shared(f32(y).reshape(T, k, H), f32(sc), None if sy is None else f32(sy),
                             None if sg is None else f32(sg))
    assert_close(f32(out), ref, max_abs=1e-6, rel=1e-6, what="combine") if not shared else \
        assert_close(f32(out), ref, max_abs=4e-3, rel=2e-3, what="combine")


# ----------------------------------------------------------------------------- whole layer

@pytest.mark.parametrize("glu_path", ["auto", "tc"], indirect=True)
@pytest.mark.parametrize("cfg_name,T", [("cfg1", 1), ("cfg1", 4), ("cfg1", 16), ("cfg1", 32), ("cfg2", 16),
                                        ("cfg2", 512), ("cfg3", 1), ("cfg3", 8), ("cfg3", 16), ("cfg4", 2)])
def test_layer_matches_oracle(glu_path, cfg_name, T):
    cfg = CONFIGS[cfg_name]
    block, tens = make_layer(cfg, device=DEV)
    moe = Qwen3_xMoEWrapper(block, "fp", "model.layers.0.mlp", 0)
    x = make_tokens(cfg, T)
    out = moe(x.reshape(1, T, cfg.hidden)).reshape(T, cfg.hidden)
    shared = None
    if tens["shared"] is not None:
        shared = LazyExperts(tens["shared"], cfg.bits)[0]
    ref = orc.layer_forward(bits16(x), bits16(tens["router"]), cfg.top_k, cfg.norm_topk_prob,
                            LazyExperts(tens["experts"], cfg.bits), shared,
                            None if tens["shared_gate"] is None else bits16(tens["shared_gate"]))
    assert_close(f32(out), ref["out"], what=f"{cfg_name} T={T}")
    res = moe.forward_resident(x)
    assert torch.equal(res, out)


def _sampled_layer_check(cfg, T, n_sample, what):
    """The whole layer at a benchmark size: router logits, top-k ids and scores
    bit-exact for every token (and the dispatch of every pair against
    np.unique), outputs of a seeded sample of tokens against the oracle (the
    oracle's cost grows with the experts the sample touches, not with T)."""
    block, tens = make_layer(cfg, device=DEV)
    moe = Qwen3_xMoEWrapper(block, "fp", "l", 0)
    x = make_tokens(cfg, T)
    out = f32(moe.forward_resident(x))
    logits = orc.router_logits(bits16(x), bits16(tens["router"]))
    inds, sc, _ = orc.get_routings(logits, cfg.top_k, cfg.norm_topk_prob)
    dl = ops.router_linear(x, block.gate)
    assert np.array_equal(bits16(dl), logits), f"{what}: router logits"
    di, ds = ops.route_topk(dl, cfg.top_k, cfg.norm_topk_prob)
    assert np.array_equal(di.cpu().numpy(), inds), f"{what}: top-k ids"
    assert np.array_equal(bits16(ds), sc), f"{what}: scores"
    d = ops.dispatch(di, cfg.num_experts, torch.arange(cfg.num_experts, dtype=torch.int32, device=DEV))
    uq, inv = np.unique(inds.reshape(-1), return_inverse=True)
    assert int(d.counts[0].item()) == uq.size
    assert np.array_equal(d.unique[: uq.size].cpu().numpy(), uq) and np.array_equal(d.inverse.cpu().numpy(), inv)
    sample = np.sort(np.random.default_rng(T).choice(T, n_sample, replace=False))
    ex = LazyExperts(tens["experts"], cfg.bits)
    xs = f32(x)[sample]
    y = np.stack([np.stack([orc.expert_forward(xs[i: i + 1], ex[inds[t, j]])[0] for j in range(cfg.top_k)])
                  for i, t in enumerate(sample)])
    sy = sg = None
    if tens["shared"] is not None:
        sy = orc.expert_forward(xs, LazyExperts(tens["shared"], cfg.bits)[0])
        sg = orc.bf16_bits_to_f32(orc.router_logits(bits16(x[sample]), bits16(tens["shared_gate"])))
    ref = orc.combine_shared(y, orc.bf16_bits_to_f32(sc[sample]), sy, sg)
    assert_close(out[sample], ref, what=f"{what} sampled")
    assert ops.device_status(reset=True) == 0


@pytest.mark.parametrize("glu_path", ["gemv", "tc"], indirect=True)
def test_layer_full_size_sampled_tokens_cfg3(glu_path):
    """cfg3 at its largest decode batch (T=256) on both GLU kernels."""
    _sampled_layer_check(CONFIGS["cfg3"], 256, 6, f"cfg3 T=256 {glu_path}")


@pytest.mark.parametrize("cfg_name,T,n_sample", [
    ("cfg3", 32, 6), ("cfg3", 64, 6), ("cfg3", 128, 6),   # the decode sweep between 16 and 256
    ("cfg2", 2048, 6), ("cfg2", 8192, 6),                  # prefill: 128-wide pair tiles, permuted rows
    ("cfg4", 64, 3), ("cfg4", 4096, 3),                    # the 397B-style layer: decode and prefill
])
def test_layer_benchmark_sizes_sampled(cfg_name, T, n_sample):
    """Every configuration at the sizes it is benchmarked at, on the
    automatic kernel choice (the path the benchmark times)."""
    ops.set_glu_path("auto")
    _sampled_layer_check(CONFIGS[cfg_name], T, n_sample, f"{cfg_name} T={T}")


def test_layer_ragged_and_empty():
    cfg = LayerConfig("t", 9, 256, 32, 3, 128, 128, 8, 32)
    block, tens = make_layer(cfg, device=DEV)
    moe = Qwen3_xMoEWrapper(block, "fp", "l", 0)
    x = torch.zeros((0, 256), dtype=torch.bfloat16, device=DEV)
    assert moe.forward_resident(x).shape == (0, 256)
    for T in (1, 3, 17):
        x = make_tokens(cfg, T)
        out = moe(x.reshape(1, T, 256)).reshape(T, 256)
        ref = orc.layer_forward(bits16(x), bits16(tens["router"]), cfg.top_k, True,
                                LazyExperts(tens["experts"], 8), LazyExperts(tens["shared"], 8)[0],
                                bits16(tens["shared_gate"]))
        assert_close(f32(out), ref["out"], what=f"T={T}")


@pytest.mark.parametrize("H,I,bits", [(4096, 1024, 4), (2048, 1024, 4), (4096, 1024, 8)])
def test_glu_prefill_tiles_every_element_and_repeatable(H, I, bits):
    """128-wide pair tiles with several tiles per CTA (64 experts x 128 pairs):
    every element of h against a plain fp32 torch reference of the same op
    (dequantised weights, bf16 roundings of x_up, x_gate, sigmoid, silu and
    the product), and four calls bit-identical.  Guards the ordering of the
    dequantising warps' shared-memory reads of a packed stage before the TMA
    that refills it."""
    from preemptlm_b200.quant import dequantize_affine

    torch.backends.cuda.matmul.allow_tf32 = False
    E, T, k = 64, 1024, 8
    cfg = LayerConfig("rep", 9, H, E, k, I, None, bits, E)
    block, tens = make_layer(cfg, device=DEV)
    arena = block.switch_mlp
    x = make_tokens(cfg, T)
    g = np.random.default_rng(5)
    inds = np.stack([g.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(inds).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    xs = ops.permute_rows(x, d, k)
    hs = [ops.glu_gate_up(arena, xs, d, k, _abi_flags("in|out")) for _ in range(4)]
    for h in hs[1:]:
        assert torch.equal(h, hs[0])
    ex = tens["experts"]
    off = d.group_off.cpu().numpy()
    U = int(d.counts[0].item())

    def bf(t):
        return t.to(torch.bfloat16).float()

    worst = 0.0
    for u in range(U):
        e = int(d.unique[u].item())
        a, b = int(off[u]), int(off[u + 1])
        w = {p: dequantize_affine(ex[f"{p}.weight"][e], ex[f"{p}.scales"][e], ex[f"{p}.biases"][e], bits).float()
             for p in ("gate_proj", "up_proj")}
        xr = xs[a:b].float()
        gate, up = bf(xr @ w["gate_proj"].T), bf(xr @ w["up_proj"].T)
        ref = bf(bf(gate * bf(torch.sigmoid(gate))) * up)
        scale = ref.abs().amax(dim=1, keepdim=True).clamp_min(1.0)
        worst = max(worst, float(((hs[0][a:b].float() - ref).abs() / scale).max()))
    assert worst <= 2e-2, f"worst element error {worst:.3e} of its row's scale"
    assert ops.device_status(reset=True) == 0


def test_forward_padded_ids_prefill_groups():
    """Rows per pair with unused entries (id -1, an expert-parallel inbox) and
    prefill-sized groups: the fused call permutes only the filled positions
    (perm's tail is never written) and matches the two halves called apart."""
    from preemptlm_b200 import _abi

    H, I, E, N = 1024, 512, 4, 640
    cfg = LayerConfig("t", 9, H, E, 1, I, None, 4, E)
    block, _ = make_layer(cfg, device=DEV)
    arena = block.switch_mlp
    rows = _bf16((N, H), 31)
    g = np.random.default_rng(9)
    eids = g.integers(0, E, N).astype(np.int32)
    eids[g.random(N) < 0.5] = -1
    d = ops.dispatch(torch.from_numpy(eids).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    import ctypes
    assert _abi.load().sg_glu_use_permute(ctypes.byref(arena.desc()), N, d.grid_groups) == 1
    y = ops.gather_forward(arena, rows, d, 1)
    h = ops.glu_gate_up(arena, rows, d, 1, _abi.SG_OUT_DISPATCH_ORDER)
    y2 = ops.glu_down(arena, h, d, _abi.SG_IN_DISPATCH_ORDER)
    valid = torch.from_numpy(eids >= 0).to(DEV)
    assert torch.equal(y[valid], y2[valid])
    assert ops.device_status(reset=True) == 0
