"""GPU, 2 ranks (skipped with fewer than 2 GPUs): the expert-parallel layer on
the CUDA kernels gives the single-GPU layer's output for every rank's tokens
(same seeded weights; each rank holds half of the experts), over the
library's NVLink peer-memory exchange (three steps in a row, so inbox and
output buffers are reused) and over NCCL all-to-alls."""

import os
import socket
import sys
import traceback
from datetime import timedelta

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errfile, transport):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import torch.distributed as dist

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from preemptlm_b200.ep import ExpertParallelMoE, shard_layer
        from preemptlm_b200.layer import Qwen3_xMoEWrapper
        from preemptlm_b200.synthetic import LayerConfig, make_layer, make_tokens

        from preemptlm_b200 import ops

        cfg = LayerConfig("ep", 8, 1024, 64, 6, 256, 256, 8, 64)
        backend, _ = shard_layer(cfg, rank, world, dev)
        ep = ExpertParallelMoE(backend, cfg.num_experts, cfg.hidden, cfg.top_k, transport=transport, max_tokens=64)
        block, _ = make_layer(cfg, device=dev)
        single = Qwen3_xMoEWrapper(block, "fp", "l", 0)
        for step in range(3 if transport == "p2p" else 1):
            T = 40 + 8 * (rank % 4) - 7 * step  # ragged token counts across ranks and steps (<= 64)
            x = make_tokens(cfg, T, device=dev, step=10 * step + rank)
            out = ep(x)
            ref = single.forward_resident(x)
            err = (out.float() - ref.float()).abs().max().item()
            assert err <= 1e-2, f"rank {rank} step {step}: max-abs {err} vs the single-GPU layer"
        if transport == "collective":
            send, recv = ep.last_counts
            assert sum(send) == T * cfg.top_k
        else:  # the step captured in a CUDA graph, replayed on new tokens
            ep.capture(T)
            for step in range(2):
                x = make_tokens(cfg, T, device=dev, step=100 + 10 * step + rank)
                out = ep.replay(x).clone()
                ref = single.forward_resident(x)
                err = (out.float() - ref.float()).abs().max().item()
                assert err <= 1e-2, f"rank {rank} replay {step}: max-abs {err} vs the single-GPU layer"
        torch.cuda.synchronize()
        assert ops.device_status(reset=True) == 0  # no exchange wait gave up
        ep.close()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        with open(errfile, "a") as f:
            f.write(f"rank {rank}:\n{traceback.format_exc()}\n")
        raise


def test_ep_one_rank_exchange_and_graph(tmp_path):
    """One rank exchanging with itself over the same peer-memory kernels
    (inboxes, flags, outputs written back), eager and as a replayed CUDA
    graph, against the single-GPU layer: the exchange path runs on one GPU."""
    import torch.multiprocessing as mp

    err = tmp_path / "err.txt"
    p = mp.get_context("spawn").Process(target=_worker, args=(0, 1, _free_port(), str(err), "p2p"))
    p.start()
    p.join(timeout=300)
    if p.is_alive():
        p.kill()
        pytest.fail("EP rank hung")
    assert p.exitcode == 0, err.read_text() if err.exists() else ""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "collective"])
def test_ep_two_gpus_matches_single_gpu(tmp_path, transport):
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    err = tmp_path / "err.txt"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(err), transport)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("EP rank hung")
    msg = err.read_text() if err.exists() else ""
    assert all(p.exitcode == 0 for p in procs), msg


@pytest.mark.skipif(torch.cuda.device_count() < 3, reason="needs more than 2 GPUs")
def test_ep_all_gpus_matches_single_gpu(tmp_path):
    """The peer transport over every GPU of the box (the largest power of two
    that divides the 64 experts): ragged tokens, eager steps and graph
    replays, against the single-GPU layer."""
    import torch.multiprocessing as mp

    world = 1
    while world * 2 <= min(8, torch.cuda.device_count()):
        world *= 2
    port = _free_port()
    err = tmp_path / "err.txt"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(err), "p2p")) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("EP rank hung")
    msg = err.read_text() if err.exists() else ""
    assert all(p.exitcode == 0 for p in procs), msg
