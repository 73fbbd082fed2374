"""GPU, 2 ranks over NCCL (skipped with fewer than 2 GPUs): the expert-parallel
layer on the CUDA kernels gives the single-GPU layer's output for every rank's
tokens (same seeded weights; each rank holds half of the experts)."""

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


def _worker(rank, world, port, errfile):
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

        cfg = LayerConfig("ep", 8, 1024, 64, 6, 256, 256, 8, 64)
        backend, _ = shard_layer(cfg, rank, world, dev)
        ep = ExpertParallelMoE(backend, cfg.num_experts, cfg.hidden, cfg.top_k)
        T = 40 + 24 * rank  # ragged token counts across ranks
        x = make_tokens(cfg, T, device=dev, step=rank)
        out = ep(x)
        block, _ = make_layer(cfg, device=dev)
        ref = Qwen3_xMoEWrapper(block, "fp", "l", 0).forward_resident(x)
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 1e-2, f"rank {rank}: max-abs {err} vs the single-GPU layer"
        send, recv = ep.last_counts
        assert sum(send) == T * cfg.top_k
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        with open(errfile, "a") as f:
            f.write(f"rank {rank}:\n{traceback.format_exc()}\n")
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_matches_single_gpu(tmp_path):
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    err = tmp_path / "err.txt"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(err))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("EP rank hung")
    msg = err.read_text() if err.exists() else ""
    assert all(p.exitcode == 0 for p in procs), msg
