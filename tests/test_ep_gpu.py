"""GPU: the expert-parallel layer on the CUDA kernels (each rank holds its
share of the same seeded experts) gives, for every rank's tokens, the
single-GPU layer's output and -- on a sample of tokens -- the CPU oracle's,
over the library's NVLink peer-memory exchange (three steps in a row, so
inbox and output buffers are reused, then graph replays) and over NCCL
all-to-alls: one rank exchanging with itself on any GPU, 2 ranks, and every
GPU of the box (up to 8).  Plus the exchange's bounded waits running out on
one GPU (a rank that never takes part)."""

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


class _OracleLayer:
    """The CPU oracle of the whole layer on a sample of one rank's tokens:
    routing of every token bit-exact, outputs within the bf16 tolerance."""

    def __init__(self, cfg, tens):
        from tests._util import LazyExperts, bits16

        self.cfg, self.tens = cfg, tens
        self.ex = LazyExperts(tens["experts"], cfg.bits)
        self.shared = LazyExperts(tens["shared"], cfg.bits)[0]
        self.router = bits16(tens["router"])
        self.sgate = bits16(tens["shared_gate"])

    def check(self, x, out, n_sample, seed, what):
        import numpy as np

        from oracle import slotted_glu_oracle as orc
        from tests._util import assert_close, bits16, f32

        cfg = self.cfg
        T = x.shape[0]
        inds, sc, _ = orc.get_routings(orc.router_logits(bits16(x), self.router), cfg.top_k, cfg.norm_topk_prob)
        sample = np.sort(np.random.default_rng(seed).choice(T, n_sample, replace=False))
        xs = f32(x)[sample]
        y = np.stack([np.stack([orc.expert_forward(xs[i: i + 1], self.ex[inds[t, j]])[0]
                                for j in range(cfg.top_k)]) for i, t in enumerate(sample)])
        sg = orc.bf16_bits_to_f32(orc.router_logits(bits16(x[sample]), self.sgate))
        ref = orc.combine_shared(y, orc.bf16_bits_to_f32(sc[sample]), orc.expert_forward(xs, self.shared), sg)
        assert_close(f32(out)[sample], ref, what=f"{what} vs the oracle")


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
        block, tens = make_layer(cfg, device=dev)
        single = Qwen3_xMoEWrapper(block, "fp", "l", 0)
        oracle = _OracleLayer(cfg, tens)
        for step in range(3 if transport == "p2p" else 1):
            T = 40 + 8 * (rank % 4) - 7 * step  # ragged token counts across ranks and steps (<= 64)
            x = make_tokens(cfg, T, device=dev, step=10 * step + rank)
            out = ep(x)
            ref = single.forward_resident(x)
            err = (out.float() - ref.float()).abs().max().item()
            assert err <= 1e-2, f"rank {rank} step {step}: max-abs {err} vs the single-GPU layer"
            oracle.check(x, out, n_sample=4, seed=step * 8 + rank, what=f"rank {rank} step {step}")
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
                oracle.check(x, out, n_sample=4, seed=100 + step * 8 + rank, what=f"rank {rank} replay {step}")
        torch.cuda.synchronize()
        if transport == "p2p":
            ep.check()  # raises if an exchange wait gave up
        assert ops.device_status(reset=True) == 0
        ep.close()
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        with open(errfile, "a") as f:
            f.write(f"rank {rank}:\n{traceback.format_exc()}\n")
        raise


def _stack_worker(rank, world, port, errfile):
    """Three layers (their own seeds) sharing one peer exchange, on the
    residual stream: eager steps with ragged tokens, then graph replays of the
    whole stack, against the single-GPU layers chained the same way."""
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        import torch.distributed as dist

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        from preemptlm_b200.ep import ExpertParallelMoE, ExpertParallelStack, PeerExchange, shard_layer
        from preemptlm_b200.layer import Qwen3_xMoEWrapper
        from preemptlm_b200.synthetic import LayerConfig, make_layer, make_tokens

        from preemptlm_b200 import ops

        cfg = LayerConfig("ep", 8, 1024, 64, 6, 256, 256, 8, 64)
        L, Tmax = 3, 48
        ex = PeerExchange(None, world, rank, Tmax, cfg.top_k, cfg.hidden, dev)
        layers, singles = [], []
        for li in range(L):
            backend, _ = shard_layer(cfg, rank, world, dev, layer=li)
            layers.append(ExpertParallelMoE(backend, cfg.num_experts, cfg.hidden, cfg.top_k, transport="p2p",
                                            max_tokens=Tmax, exchange=ex))
            block, _ = make_layer(cfg.scaled(cfg_id=cfg.cfg_id + 1_000_000 * li), device=dev)
            singles.append(Qwen3_xMoEWrapper(block, "fp", f"l{li}", li))
        stack = ExpertParallelStack(layers)

        def reference(x):
            for single in singles:
                x = x + single.forward_resident(x)
            return x

        def check(out, ref, what):
            tol = 2.0 ** -6 * L * max(1.0, ref.float().abs().max().item())
            err = (out.float() - ref.float()).abs().max().item()
            assert err <= tol, f"rank {rank} {what}: max-abs {err} (tolerance {tol}) vs the single-GPU layers"

        for step in range(2):
            T = 40 + 4 * (rank % 2) - 5 * step
            x = make_tokens(cfg, T, device=dev, step=10 * step + rank)
            check(stack(x), reference(x), f"step {step}")
        stack.capture(T)
        for step in range(2):
            x = make_tokens(cfg, T, device=dev, step=200 + 10 * step + rank)
            check(stack.replay(x).clone(), reference(x), f"replay {step}")
        torch.cuda.synchronize()
        stack.check()
        assert ops.device_status(reset=True) == 0
        stack.close()
        assert ex.region is None  # the shared exchange was freed once, by the stack
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        with open(errfile, "a") as f:
            f.write(f"rank {rank}:\n{traceback.format_exc()}\n")
        raise


def _spawn(target, world, tmp_path, *extra):
    import torch.multiprocessing as mp

    port, err = _free_port(), tmp_path / "err.txt"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=target, args=(r, world, port, str(err), *extra)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
            pytest.fail("EP rank hung")
    assert all(p.exitcode == 0 for p in procs), err.read_text() if err.exists() else ""


def test_ep_stack_one_rank_shared_exchange(tmp_path):
    """A three-layer expert-parallel stack, one rank exchanging with itself."""
    _spawn(_stack_worker, 1, tmp_path)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_stack_two_gpus_shared_exchange(tmp_path):
    """The same stack over 2 GPUs."""
    _spawn(_stack_worker, 2, tmp_path)


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


def test_ep_wait_timeout_reports_and_zeroes_rows():
    """Failure detection without a fault: two ranks' regions on one GPU, and
    'rank 1' never takes part.  Rank 0's sends land (its own flag is raised),
    but the flags of rank 1 are never set, so sg_ep_wait_inbox and
    sg_ep_wait_back give up after the (shortened) wait limit: they return,
    sg_device_status reports SG_ERR_TIMEOUT, rank 1's inbox is marked empty and
    the output rows of the pairs rank 1 owns are zeroed, while rank 0's own
    pairs come back intact."""
    import ctypes
    import time

    import numpy as np

    from preemptlm_b200 import _abi, ops
    from preemptlm_b200.ep import _view, set_wait_limit

    lib = _abi.load()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    R, T, k, H, per = 2, 16, 4, 256, 8  # 16 experts, 8 per rank
    cap = T * k
    assert ops.device_status(reset=True) == 0
    nbytes = lib.sg_ep_region_bytes(R, cap, H)
    regions = []
    for _ in range(R):
        p = ctypes.c_void_p()
        _abi.check(lib.sg_ep_alloc(nbytes, ctypes.byref(p)), "sg_ep_alloc")
        regions.append(p.value)
    arr = (ctypes.c_void_p * R)(*regions)
    off = (ctypes.c_longlong * 5)()
    _abi.check(lib.sg_ep_layout(R, cap, H, off), "sg_ep_layout")
    try:
        g = torch.Generator(device=dev).manual_seed(7)
        x = torch.randn((T, H), generator=g, device=dev).to(torch.bfloat16)
        rng = np.random.default_rng(7)
        inds_np = np.stack([rng.permutation(R * per)[:k] for _ in range(T)]).astype(np.int32)
        inds = torch.from_numpy(inds_np).to(dev)
        dcnt = torch.zeros(R, dtype=torch.int32, device=dev)
        rows0 = _view(regions[0] + off[0], (R * cap, H), torch.bfloat16, dev)
        eids0 = _view(regions[0] + off[1], (R * cap,), torch.int32, dev)
        ybuf0 = _view(regions[0] + off[4], (cap, H), torch.bfloat16, dev)
        ybuf0.fill_(1.0)  # stale contents that the timed-out rows must not keep
        set_wait_limit(0.05)
        s = torch.cuda.current_stream().cuda_stream
        t0 = time.perf_counter()
        _abi.check(lib.sg_ep_send(arr, R, 0, cap, H, x.data_ptr(), inds.data_ptr(), T, k, per, dcnt.data_ptr(), s),
                   "sg_ep_send")
        _abi.check(lib.sg_ep_wait_inbox(ctypes.c_void_p(regions[0]), R, cap, H, s), "sg_ep_wait_inbox")
        # the 'experts' return each received row unchanged
        y = rows0.clone()
        _abi.check(lib.sg_ep_send_back(arr, R, 0, cap, H, y.data_ptr(), s), "sg_ep_send_back")
        _abi.check(lib.sg_ep_wait_back(ctypes.c_void_p(regions[0]), R, cap, H, inds.data_ptr(), T, k, per, s),
                   "sg_ep_wait_back")
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        assert ops.device_status(reset=True) == _abi.SG_ERR_TIMEOUT
        assert elapsed < 1.5, f"the waits took {elapsed:.2f} s with a 50 ms limit"
        mine = (inds_np.reshape(-1) // per) == 0
        assert torch.all(eids0[cap:] == -1)  # rank 1's inbox: marked empty
        n_mine = int(mine.sum())
        assert int((eids0[:cap] >= 0).sum()) == n_mine
        yb = ybuf0.float().cpu().numpy()
        xr = x.float().cpu().numpy()[np.arange(T * k) // k]
        assert np.array_equal(yb[mine], xr[mine])  # own pairs came back through the exchange
        assert np.all(yb[~mine] == 0)  # the late rank's pairs were zeroed
    finally:
        set_wait_limit(2.0)
        torch.cuda.synchronize()
        ops.device_status(reset=True)
        for r in regions:
            lib.sg_ep_free(ctypes.c_void_p(r))
