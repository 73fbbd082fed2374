"""GPU: the layer call captured as a CUDA graph (Qwen3_xMoEWrapper.capture /
replay) gives the eager call's bits on new tokens, with and without a shared
expert, for decode- and prefill-sized groups."""

import pytest
import torch

from preemptlm_b200.layer import Qwen3_xMoEWrapper
from preemptlm_b200.synthetic import LayerConfig, make_layer, make_tokens

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,shared,T", [(8, 512, 64), (4, None, 200), (16, 256, 8)])
def test_graph_replay_matches_eager_call(bits, shared, T):
    cfg = LayerConfig("g", 7, 1024, 32, 4, 256, shared, bits, 32)
    block, _ = make_layer(cfg, device="cuda")
    moe = Qwen3_xMoEWrapper(block, "fp", "model.layers.0.mlp", 0)
    moe.capture(1, T)
    for step in range(3):
        x = make_tokens(cfg, T, device="cuda", step=step).view(1, T, cfg.hidden)
        got = moe.replay(x).clone()
        want = moe(x)
        assert torch.equal(got, want), f"step {step}"


def test_streaming_wrapper_refuses_capture():
    cfg = LayerConfig("g", 7, 1024, 32, 4, 256, None, 8, 32)
    block, _ = make_layer(cfg, device="cuda")
    moe = Qwen3_xMoEWrapper(block, "fp", "model.layers.0.mlp", 0)
    moe.expert_cache = object()  # a streaming wrapper reads slot misses on the host
    with pytest.raises(ValueError):
        moe.capture(1, 8)


def test_host_pipeline_gives_each_steps_output():
    """Replays fed from pinned host buffers through the overlapped pipeline:
    every step's host output equals the eager call on that step's tokens."""
    T = 48
    cfg = LayerConfig("g", 7, 1024, 32, 4, 256, 256, 8, 32)
    block, _ = make_layer(cfg, device="cuda")
    moe = Qwen3_xMoEWrapper(block, "fp", "model.layers.0.mlp", 0)
    moe.capture(1, T)
    pipe = moe.host_pipeline()
    steps = 5
    xs = [make_tokens(cfg, T, device="cuda", step=10 + i).view(1, T, cfg.hidden) for i in range(steps)]
    x_host = [x.cpu().pin_memory() for x in xs]
    outs = [torch.empty((1, T, cfg.hidden), dtype=torch.bfloat16).pin_memory() for _ in range(steps)]
    for i in range(steps):
        pipe.step(x_host[i], outs[i])
    pipe.drain()
    torch.cuda.synchronize()
    for i in range(steps):
        assert torch.equal(outs[i].cuda(), moe(xs[i])), f"step {i}"
