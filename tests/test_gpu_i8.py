"""GPU: the integer-operand kernels (8- and 4-bit arenas at decode tile widths).

* sg_quantize_pieces against a numpy statement of the piece split (exact);
* h through the integer-operand gate/up against the CPU oracle within the
  bf16 tolerance of the layer, and against the dequantising tcgen05 kernel;
  y through the integer-operand down projection against the oracle's down
  projection of the device's h;
* missing slots, several pair tiles per group, rows in dispatch order.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import slotted_glu_oracle as orc
from preemptlm_b200 import _abi, ops
from preemptlm_b200.synthetic import LayerConfig, make_layer

from ._util import LazyExperts, assert_close, bits16, f32

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _bf16(shape, seed, std=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=DEV) * std).to(torch.bfloat16)


def pieces_numpy(xbits: np.ndarray, order: int = 0):
    """The piece split of sg_quantize_pieces restated: per 64-group, the
    largest biased exponent eM of the nonzero elements; each element's integer
    m8 * 2^(ex - eM + 6) (rounded half away from zero); hi = floor((v + 128) /
    256), lo = v - 256 hi; E = 2^(eM - 140); X = E * sum(v)."""
    rows, K = xbits.shape
    b = xbits.astype(np.int64)
    ex = (b >> 7) & 0xFF
    mant = np.where(ex == 0, b & 0x7F, (b & 0x7F) | 0x80)
    e_eff = np.where(ex == 0, 1, ex)
    nz = (b & 0x7FFF) != 0
    eg = np.where(nz, e_eff, 0).reshape(rows, K // 64, 64).max(axis=2)
    eM = np.repeat(eg, 64, axis=1)
    sh = e_eff - eM + 6
    pos = np.where(sh >= 0, mant << np.clip(sh, 0, 62), 0)
    rs = np.clip(-sh, 1, 62)
    neg = np.where((sh < 0) & (-sh < 31), (mant + (1 << (rs - 1))) >> rs, 0)
    v = np.where(sh >= 0, pos, neg)
    v = np.where((b & 0x8000) != 0, -v, v)
    hi = np.floor_divide(v + 128, 256)
    lo = v - 256 * hi
    if order:
        perm = np.array([0, 2, 4, 6, 1, 3, 5, 7])
        idx = (np.arange(K) // 8) * 8 + perm[np.arange(K) % 8]
        hi, lo = hi[:, idx], lo[:, idx]
    E = np.ldexp(1.0, (eg - 140).astype(np.int32)).astype(np.float32)
    X = (v.reshape(rows, K // 64, 64).sum(axis=2) * E.astype(np.float64)).astype(np.float32)
    return hi.astype(np.int8), lo.astype(np.int8), E, X, v


@pytest.mark.parametrize("order", [0, 1])
def test_quantize_pieces_exact(order):
    rows, K = 37, 1024
    x = _bf16((rows, K), 5)
    # a spread of magnitudes inside groups, exact zeros, an all-zero group, subnormals
    x[0, :64] = 0
    x[1, :64] *= torch.logspace(-12, 3, 64, device=DEV).to(torch.bfloat16)
    x[2, 5] = 0
    x[3, 64:128] = torch.tensor(1e-39, device=DEV).to(torch.bfloat16)
    pieces, ex = ops.quantize_pieces(x, order)
    hi, lo, E, X, v = pieces_numpy(bits16(x), order)
    p = pieces.cpu().numpy()
    assert np.array_equal(p[:, 0], hi)
    assert np.array_equal(p[:, 1], lo)
    e = ex.cpu().numpy()
    assert np.array_equal(e[..., 0], E)
    assert np.array_equal(e[..., 1], X)
    assert hi.min() >= -64 and hi.max() <= 64
    # the pieces reproduce x to 2^-14 of each group's largest magnitude
    xf = f32(x).reshape(rows, K // 64, 64)
    rec = (v.reshape(rows, K // 64, 64) * E[..., None]).astype(np.float64)
    gmax = np.abs(xf).max(axis=2, keepdims=True)
    assert np.all(np.abs(rec - xf) <= gmax * 2.0 ** -14 + 1e-45)


def _h_oracle(tens, bits, x, inds, k, I):
    ex = LazyExperts(tens["experts"], bits)
    xf = f32(x)
    href = np.zeros((inds.size, I), np.float32)
    for p, e in enumerate(inds.reshape(-1)):
        if e < 0:
            continue
        ew = ex[e]
        xr = xf[p // k: p // k + 1]
        href[p] = orc.swiglu(orc._mm_bf16(xr, ew.up), orc._mm_bf16(xr, ew.gate))[0]
    return href


def _exact_down(tens, e, bits):
    """scale * q + bias of expert e's down projection in float64 (no rounding)."""
    q = orc.unpack_affine(tens["experts"]["down_proj.weight"][int(e)].cpu().numpy().view(np.uint32), bits)
    sc = f32(tens["experts"]["down_proj.scales"][int(e)]).astype(np.float64)
    bi = f32(tens["experts"]["down_proj.biases"][int(e)]).astype(np.float64)
    return q.astype(np.float64) * np.repeat(sc, 64, axis=1) + np.repeat(bi, 64, axis=1)


@pytest.fixture
def i8_path():
    ops.set_glu_path("i8")
    yield
    ops.set_glu_path("auto")
    ops.set_glu_tile(0)
    assert ops.device_status(reset=True) == 0


@pytest.mark.parametrize("H,I,E,T,k", [(512, 128, 8, 5, 2), (2048, 512, 64, 33, 8), (1024, 256, 6, 1, 6),
                                       (4096, 1024, 16, 9, 4), (512, 512, 8, 7, 3),
                                       # ~40 pairs per group: three 16-pair tiles per group, the last partial
                                       (1024, 384, 4, 80, 2), (1024, 512, 4, 80, 2)])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("tile", [8, 16])
def test_gate_up_i8_matches_oracle(i8_path, tile, bits, H, I, E, T, k):
    ops.set_glu_tile(tile)
    cfg = LayerConfig("t", 9, H, E, k, I, None, bits, E)
    block, tens = make_layer(cfg, device=DEV)
    x = _bf16((T, H), 11)
    g = np.random.default_rng(T * 7 + E)
    inds = np.stack([g.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(inds).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    arena = block.switch_mlp
    assert _abi.load().sg_glu_gate_up_work_bytes(ctypes.byref(arena.desc()), T * k, k, d.grid_groups, 0) > 0
    h = ops.glu_gate_up(arena, x, d, pair_div=k)
    href = _h_oracle(tens, bits, x, inds, k, I)
    assert_close(f32(h), href, max_abs=2e-2 * max(1.0, float(np.abs(href).max())), what="h")
    # against the dequantising tensor-core kernel
    ops.set_glu_path("tc")
    h_tc = ops.glu_gate_up(arena, x, d, pair_div=k)
    ops.set_glu_path("i8")
    assert_close(f32(h), f32(h_tc), max_abs=2e-2 * max(1.0, float(np.abs(href).max())), what="h vs tc")
    # down projection of the device's h: the integer-operand kernel where the
    # shape allows it (I % 512, H % 256), against the oracle's down of that h
    down_i8 = _abi.load().sg_glu_down_work_bytes(ctypes.byref(arena.desc()), T * k, d.grid_groups) > 0
    assert down_i8 == (I % 512 == 0 and H % 256 == 0)
    y = ops.glu_down(arena, h, d)
    ex = LazyExperts(tens["experts"], bits)
    hdev = f32(h)
    ydown = np.stack([orc._mm_bf16(hdev[p: p + 1], ex[inds.reshape(-1)[p]].down)[0] for p in range(T * k)])
    if down_i8:
        # the layer tolerance against the oracle (whose weights are rounded to
        # bf16); against the exact affine weights scale * q + bias, which the
        # integer kernel uses: the output rounding (half a bf16 ulp, < 2^-8
        # relative) plus the piece rounding of h (each element to within 2^-14
        # of its group's largest magnitude), summed through |w| as a bound
        assert_close(f32(y), ydown, what="y|h")
        for p in range(T * k):
            w = _exact_down(tens, inds.reshape(-1)[p], bits)
            hp = hdev[p].astype(np.float64)
            gmax = np.repeat(np.abs(hp).reshape(-1, 64).max(axis=1), 64)
            bound = 2.0 ** -8 * np.abs(hp @ w.T) + 2.0 ** -14 * (np.abs(w) @ gmax) + 1e-6
            assert np.all(np.abs(f32(y[p]) - hp @ w.T) <= bound), (p, float(np.abs(f32(y[p]) - hp @ w.T).max()))
    else:
        assert_close(f32(y), ydown, max_abs=1e-2, rel=4e-3, what="y|h")
    # the fused layer call takes the same paths (work area from sg_glu_forward_scratch_bytes)
    y = ops.gather_forward(arena, x, d, k)
    y2 = ops.glu_down(arena, ops.glu_gate_up(arena, x, d, k, _abi.SG_OUT_DISPATCH_ORDER), d,
                      _abi.SG_IN_DISPATCH_ORDER)
    assert torch.equal(y, y2)
    # repeatable: the same bits on a second call
    assert torch.equal(ops.glu_gate_up(arena, x, d, pair_div=k), h)


@pytest.mark.parametrize("bits", [8, 4])
def test_gate_up_i8_rows_in_dispatch_order(i8_path, bits):
    H, I, E, T, k = 1024, 256, 8, 24, 2
    cfg = LayerConfig("t", 9, H, E, k, I, None, bits, E)
    block, tens = make_layer(cfg, device=DEV)
    x = _bf16((T, H), 13)
    g = np.random.default_rng(3)
    inds = np.stack([g.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(inds).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    arena = block.switch_mlp
    xs = ops.permute_rows(x, d, k)
    h_pos = ops.glu_gate_up(arena, xs, d, 1, _abi.SG_IN_DISPATCH_ORDER | _abi.SG_OUT_DISPATCH_ORDER)
    h_ref = ops.glu_gate_up(arena, x, d, k, _abi.SG_OUT_DISPATCH_ORDER)
    assert torch.equal(h_pos, h_ref)


@pytest.mark.parametrize("bits", [8, 4])
def test_gate_up_i8_missing_slots(i8_path, bits):
    H, I, E = 512, 512, 4
    cfg = LayerConfig("t", 9, H, E, 1, I, None, bits, E)
    block, tens = make_layer(cfg, device=DEV)
    x = _bf16((3, H), 12)
    inds = torch.tensor([[0], [1], [2]], dtype=torch.int32, device=DEV)
    d = ops.dispatch(inds, E, torch.tensor([0, -1, 2, 3], dtype=torch.int32, device=DEV))
    h = ops.glu_gate_up(block.switch_mlp, x, d, pair_div=1)
    assert torch.all(h[1] == 0) and torch.any(h[0] != 0)
    href = _h_oracle(tens, bits, x, np.array([0, -1, 2]), 1, I)
    assert_close(f32(h[[0, 2]]), href[[0, 2]], max_abs=2e-2 * max(1.0, float(np.abs(href).max())), what="h")
    # the down projection writes zeros for the pairs of the missing slot too
    y = ops.glu_down(block.switch_mlp, h, d)
    assert torch.all(y[1] == 0) and torch.any(y[0] != 0)


@pytest.mark.parametrize("bits", [8, 4])
def test_i8_padded_inbox_rows(i8_path, bits):
    """Rows per pair with unused entries (an expert-parallel inbox: id -1):
    only the filled entries are split into pieces and computed, and they match
    the dequantising kernels."""
    H, I, E, N = 1024, 512, 8, 96
    cfg = LayerConfig("t", 9, H, E, 1, I, None, bits, E)
    block, _ = make_layer(cfg, device=DEV)
    arena = block.switch_mlp
    rows = _bf16((N, H), 21)
    g = np.random.default_rng(5)
    eids = g.integers(0, E, N).astype(np.int32)
    eids[g.random(N) < 0.6] = -1  # about 60 % of the inbox unused
    d = ops.dispatch(torch.from_numpy(eids).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    valid = torch.from_numpy(eids >= 0).to(DEV)
    h = ops.glu_gate_up(arena, rows, d, 1, _abi.SG_OUT_DISPATCH_ORDER)
    y = ops.glu_down(arena, h, d, _abi.SG_IN_DISPATCH_ORDER)
    ops.set_glu_path("tc")
    h_tc = ops.glu_gate_up(arena, rows, d, 1, _abi.SG_OUT_DISPATCH_ORDER)
    y_tc = ops.glu_down(arena, h_tc, d, _abi.SG_IN_DISPATCH_ORDER)
    ops.set_glu_path("i8")
    nvalid = int(valid.sum().item())
    scale = max(1.0, float(f32(h_tc[:nvalid]).__abs__().max()))
    assert_close(f32(h[:nvalid]), f32(h_tc[:nvalid]), max_abs=2e-2 * scale, what="h")
    # y rows of filled entries (pair order), against the dequantising kernels
    assert_close(f32(y[valid]), f32(y_tc[valid]), what="y")
