"""GPU: sg_glu_forward_noalloc (intermediate rows in the library's fixed
device scratch area) gives exactly what sg_glu_forward with caller scratch
gives, on two calls in a row with different inputs and routings (the second
call reuses the scratch area the first one wrote).  Collected last."""

import ctypes

import numpy as np
import pytest
import torch

from preemptlm_b200 import _abi, ops
from preemptlm_b200.synthetic import LayerConfig, make_layer

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(block, E, T, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn((T, block.switch_mlp.hidden), generator=g, device=DEV).to(torch.bfloat16)
    rng = np.random.default_rng(seed)
    inds = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d = ops.dispatch(torch.from_numpy(inds).to(DEV), E, torch.arange(E, dtype=torch.int32, device=DEV))
    return x, d


@pytest.mark.parametrize("path", ["auto", "tc-perm"])
@pytest.mark.parametrize("bits", [8, 4])
def test_noalloc_matches_caller_scratch_twice(bits, path):
    """"tc-perm" forces the token rows into dispatch order first, so the
    permuted rows are placed in the scratch area after h."""
    ops.set_glu_path(path)
    try:
        E, k = 32, 4
        cfg = LayerConfig("noalloc", 10, 1024, E, k, 512, None, bits, E)
        block, _ = make_layer(cfg, device=DEV)
        for T, seed in ((96, 1), (40, 2)):  # second call: fewer pairs, other rows, same scratch area
            x, d = _case(block, E, T, k, seed)
            permute = _abi.load().sg_glu_use_permute(ctypes.byref(block.switch_mlp.desc()), T * k, d.grid_groups)
            assert permute == (1 if path == "tc-perm" else 0)
            want = ops.gather_forward(block.switch_mlp, x, d, k)
            got = ops.gather_forward_noalloc(block.switch_mlp, x, d, k)
            torch.cuda.synchronize()
            assert torch.equal(got, want)
        assert ops.device_status(reset=True) == 0
    finally:
        ops.set_glu_path("auto")


def test_noalloc_rejects_oversized_problems():
    E, k = 8, 2
    cfg = LayerConfig("noalloc", 10, 1024, E, k, 512, None, 8, E)
    block, _ = make_layer(cfg, device=DEV)
    P = (32 << 20) // (512 * 2) + 64  # h alone exceeds the 32 MiB area
    d = ops.dispatch(torch.zeros(P, dtype=torch.int32, device=DEV), E, torch.arange(E, dtype=torch.int32,
                                                                                     device=DEV))
    x = torch.zeros((P, 1024), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(_abi.SlottedGLUError) as e:
        ops.gather_forward_noalloc(block.switch_mlp, x, d, 1)
    assert e.value.status == _abi.SG_ERR_CAPACITY


def test_noalloc_rejects_h_plus_permuted_rows_over_capacity():
    """h alone fits the 32 MiB area but h plus the permuted token rows do not
    (prefill-sized groups permute): rejected before any launch."""
    E, k = 8, 1
    cfg = LayerConfig("noalloc", 10, 1024, E, k, 512, None, 8, E)
    block, _ = make_layer(cfg, device=DEV)
    P = 16000  # h: 16000 x 512 x 2 = 16.4 MB; + rows 16000 x 1024 x 2 = 49 MB in all
    ids = torch.arange(P, dtype=torch.int32, device=DEV) % E
    d = ops.dispatch(ids, E, torch.arange(E, dtype=torch.int32, device=DEV))
    assert _abi.load().sg_glu_use_permute(ctypes.byref(block.switch_mlp.desc()), P, d.grid_groups) == 1
    x = torch.zeros((P, 1024), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(_abi.SlottedGLUError) as e:
        ops.gather_forward_noalloc(block.switch_mlp, x, d, 1)
    assert e.value.status == _abi.SG_ERR_CAPACITY
    # half as many pairs fit (24.6 MB) and match the caller-scratch call
    d2 = ops.dispatch(ids[: P // 2].contiguous(), E, torch.arange(E, dtype=torch.int32, device=DEV))
    g = torch.Generator(device=DEV).manual_seed(3)
    x2 = torch.randn((P // 2, 1024), generator=g, device=DEV).to(torch.bfloat16)
    assert torch.equal(ops.gather_forward_noalloc(block.switch_mlp, x2, d2, 1),
                       ops.gather_forward(block.switch_mlp, x2, d2, 1))
    assert ops.device_status(reset=True) == 0
