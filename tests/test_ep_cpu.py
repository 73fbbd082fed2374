"""CPU, 2 ranks over gloo: the expert-parallel exchange (counts, dispatch,
combine all-to-alls) gives the single-process oracle's layer output, and a
rank that fails before the exchange makes the others fail fast instead of
hanging."""

import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(H=256, E=32, k=4, I=128, bits=8, seed=77):
    """A tiny seeded q8 layer with a shared expert, as host tensors."""
    sys.path.insert(0, ROOT)
    from oracle import slotted_glu_oracle as orc
    from preemptlm_b200.quant import quantize_affine

    g = torch.Generator().manual_seed(seed)

    def rnd(*shape, std=0.02):
        return (torch.randn(shape, generator=g) * std).to(torch.bfloat16)

    def bits16(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    def expert(inter):
        mats = []
        for shape in ((inter, H), (inter, H), (H, inter)):
            q, s, b = quantize_affine(rnd(*shape), bits, 64)
            mats.append(orc.dequant_affine(q.numpy().view(np.uint32), bits16(s), bits16(b), bits))
        return orc.ExpertWeights(*mats)

    router = bits16(rnd(E, H))
    experts = [expert(I) for _ in range(E)]
    shared = expert(I)
    sgate = bits16(rnd(1, H))
    return router, experts, shared, sgate


class OracleBackend:
    """Per-rank math done by the CPU oracle (test stand-in for CudaBackend)."""

    def __init__(self, router, top_k, local_experts, shared, sgate):
        self.router, self.k, self.local, self.shared, self.sgate = router, top_k, local_experts, shared, sgate

    @staticmethod
    def _bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    @staticmethod
    def _f32(t):
        from oracle import slotted_glu_oracle as orc

        return orc.bf16_bits_to_f32(OracleBackend._bits(t))

    def route(self, x):
        from oracle import slotted_glu_oracle as orc

        inds, sc, _ = orc.get_routings(orc.router_logits(self._bits(x), self.router), self.k, True)
        return torch.from_numpy(inds), torch.from_numpy(orc.bf16_bits_to_f32(sc)).to(torch.bfloat16)

    def experts(self, rows, local_eids):
        from oracle import slotted_glu_oracle as orc

        x = self._f32(rows)
        out = np.zeros((x.shape[0], x.shape[1]), np.float32)
        for i, e in enumerate(local_eids.tolist()):
            out[i] = orc.expert_forward(x[i: i + 1], self.local[e])[0]
        return torch.from_numpy(out).to(torch.bfloat16)

    def shared_terms(self, x):
        from oracle import slotted_glu_oracle as orc

        sy = orc.expert_forward(self._f32(x), self.shared)
        sg = orc.bf16_bits_to_f32(orc.router_logits(self._bits(x), self.sgate)).reshape(-1)
        return torch.from_numpy(sy).to(torch.bfloat16), torch.from_numpy(sg).to(torch.bfloat16)

    def combine(self, y, scores, sy, sg):
        from oracle import slotted_glu_oracle as orc

        T, k = scores.shape
        out = orc.combine_shared(self._f32(y).reshape(T, k, -1), self._f32(scores), self._f32(sy),
                                 self._f32(sg))
        return torch.from_numpy(out).to(torch.bfloat16)


def _worker(rank, world, port, mode, errfile):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        from oracle import slotted_glu_oracle as orc
        from preemptlm_b200.ep import ExpertParallelMoE

        H, E, k = 256, 32, 4
        router, experts, shared, sgate = _layer(H=H, E=E, k=k)
        per = E // world
        local = {e - rank * per: experts[e] for e in range(rank * per, (rank + 1) * per)}
        moe = ExpertParallelMoE(OracleBackend(router, k, local, shared, sgate), E, H, k)
        g = torch.Generator().manual_seed(1000 + rank)
        T = 5 + 3 * rank  # ragged: ranks hold different token counts
        x = torch.randn((T, H), generator=g).to(torch.bfloat16)
        if mode == "fail" and rank == 1:
            raise SystemExit(3)  # leaves before the first collective
        if mode == "fail":
            try:
                moe(x)
            except Exception:
                dist.destroy_process_group()
                return  # the survivor saw an error instead of hanging
            raise AssertionError("rank 0 completed a collective with a dead peer")
        out = moe(x)
        ref = orc.layer_forward(OracleBackend._bits(x), router, k, True, experts, shared, sgate)
        got = OracleBackend._f32(out)
        err = np.abs(got - ref["out"]).max()
        assert err <= 1e-2, f"rank {rank}: max-abs {err}"
        send, recv = moe.last_counts
        assert sum(send) == T * k
        dist.barrier()
        dist.destroy_process_group()
    except SystemExit:
        raise
    except BaseException:
        with open(errfile, "a") as f:
            f.write(f"rank {rank}:\n{traceback.format_exc()}\n")
        raise


def _stack_worker(rank, world, port, errfile):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
        from oracle import slotted_glu_oracle as orc
        from preemptlm_b200.ep import ExpertParallelMoE, ExpertParallelStack

        H, E, k, L = 256, 32, 4, 3
        per = E // world
        layers, full = [], []
        for li in range(L):
            router, experts, shared, sgate = _layer(H=H, E=E, k=k, seed=77 + li)
            full.append((router, experts, shared, sgate))
            local = {e - rank * per: experts[e] for e in range(rank * per, (rank + 1) * per)}
            layers.append(ExpertParallelMoE(OracleBackend(router, k, local, shared, sgate), E, H, k))
        stack = ExpertParallelStack(layers)
        g = torch.Generator().manual_seed(2000 + rank)
        T = 4 + 3 * rank
        x = torch.randn((T, H), generator=g).to(torch.bfloat16)
        out = stack(x)
        # the oracle's layers on the residual stream, in one process
        ref = x
        for router, experts, shared, sgate in full:
            y = orc.layer_forward(OracleBackend._bits(ref), router, k, True, experts, shared, sgate)["out"]
            ref = ref + torch.from_numpy(y).to(torch.bfloat16)
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 3e-2, f"rank {rank}: max-abs {err} after {L} layers"
        stack.close()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        with open(errfile, "a") as f:
            f.write(f"rank {rank}:\n{traceback.format_exc()}\n")
        raise


def test_ep_stack_two_ranks_gloo(tmp_path):
    """Three expert-parallel layers on the residual stream (x <- x + layer(x))
    over 2 gloo ranks, against the oracle's layers chained in one process."""
    world, port = 2, _free_port()
    err = tmp_path / "err.txt"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_stack_worker, args=(r, world, port, str(err))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        if p.is_alive():
            p.kill()
            pytest.fail("EP rank hung")
    msg = err.read_text() if err.exists() else ""
    assert all(p.exitcode == 0 for p in procs), msg


@pytest.mark.parametrize("mode", ["parity", "fail"])
def test_ep_two_ranks_gloo(mode, tmp_path):
    world, port = 2, _free_port()
    err = tmp_path / "err.txt"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, str(err))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("EP rank hung")
    msg = err.read_text() if err.exists() else ""
    if mode == "parity":
        assert all(p.exitcode == 0 for p in procs), msg
    else:
        assert procs[0].exitcode == 0, msg
        assert procs[1].exitcode == 3
