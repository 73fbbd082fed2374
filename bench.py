#!/usr/bin/env python
"""SlottedGLU MoE layer throughput on B200 (tokens/s) with its roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (default ``cfg3``): the Qwen3-Next-style slotted MoE layer -- hidden
2048, 512 experts, top-10 renormalised routing, expert intermediate 512, an
always-on shared SwiGLU expert (intermediate 512) with a sigmoid gate,
affine 8-bit group-64 weights -- at a decode batch of ``--tokens`` (256)
tokens per GPU.  Every expert of the GPU's shard is resident in the arena
(the reference's non-streaming branch), so a step is router -> routing ->
dispatch -> gathered gate/up+SwiGLU -> down -> combine.  One step reads about
1.7 GB of expert weights, well above the 126 MB L2, so no flush is needed.

One JSON line on rank 0:
  value     whole-job tokens/s, inputs resident in HBM, CUDA-event timed
  e2e       tokens/s through the public layer call with the tokens copied
            host->device and the output device->host every step
  roofline  the routed gate/up kernel: algorithmic bytes / its event time;
            ``traffic`` scales the DRAM bytes per unique expert of the
            committed ncu summary named in ``traffic_source``
  cpu_baseline  the CPU oracle port on the same 256-token step (rank 0, N=1)
  sweep     (N=1) every configuration at its benchmark sizes on one GPU:
            decode tokens/s with the HBM fraction, prefill with the tensor
            fraction, and the streaming miss path
  strong    (N>1) a fixed global batch of 256 tokens split over the N GPUs
``--impl reference`` times that CPU port alone (the reference itself runs on
MLX, which is not installed here; the line records the import probe) on the
same 256-token step, all host cores.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import re
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
# A committed ncu summary states the DRAM bytes (read + write) of the routed
# gate/up launch per unique expert on a smaller case of a workload, on a line
#   roofline-traffic: <workload> <bytes> bytes per unique expert
# The launch streams each unique expert's weights once, so the traffic of a
# bench launch is that figure times its unique experts.
TRAFFIC_RE = re.compile(r"^roofline-traffic:\s+(\S+)\s+(\d+)\s+bytes per unique expert", re.M)
QUEUE_AHEAD_CYCLES = 1_000_000_000  # ~0.5 s of device spin before the device-resident timed region
METRIC = "SlottedGLU tokens/s at 1/2/4/8 B200; expert-GEMM HBM GB/s vs 8 TB/s peak"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default="cfg3")
    ap.add_argument("--tokens", type=int, default=256, help="decode tokens per GPU per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--experts", type=int, default=None, help="override the expert count (profiling cases)")
    ap.add_argument("--no-shared", action="store_true", help="drop the shared expert (profiling cases)")
    ap.add_argument("--glu-path", choices=("auto", "gemv", "tc", "tc-perm"), default="auto")
    ap.add_argument("--microbatches", type=int, default=None,
                    help="expert-parallel micro-batches per step (default: 1 with the p2p exchange, 2 with NCCL)")
    ap.add_argument("--no-graph", action="store_true",
                    help="e2e steps issued eagerly instead of as a captured CUDA graph of the layer call")
    ap.add_argument("--ep", action="store_true",
                    help="run the expert-parallel layer even on one GPU (one rank exchanging with itself)")
    ap.add_argument("--ep-transport", choices=("p2p", "collective"), default="p2p",
                    help="expert-parallel exchange: the library's NVLink peer-memory kernels or NCCL all-to-alls")
    ap.add_argument("--profile", action="store_true",
                    help="only warm-up + timed device-resident steps (for ncu captures); prints ms/step")
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-configuration sweep (N=1)")
    ap.add_argument("--sweep-steps", type=int, default=20, help="timed steps per sweep point")
    ap.add_argument("--sweep-only", default=None,
                    help="comma-separated sweep configurations to run (default: all)")
    ap.add_argument("--layers", type=int, default=1,
                    help="L > 1: an L-layer stack of the workload's MoE block, expert-parallel over the GPUs "
                         "(cfg4 with 60: the 397B-style stack), one pass of the tokens through every layer per step")
    return ap.parse_args()


def hbm_peak():
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    """Dense bf16 TFLOP/s of this pool's B200s (burst: a kernel timed alone)."""
    try:
        p = json.loads(PEAKS_FILE.read_text())
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic(workload: str):
    """(bytes per unique expert, summary file) from the committed ncu summaries."""
    for f in sorted((ROOT / "profiles").glob("*.md")):
        for m in TRAFFIC_RE.finditer(f.read_text()):
            if m.group(1) == workload:
                return int(m.group(2)), f"profiles/{f.name}"
    return None, None


def mlx_probe() -> str:
    """Whether the reference's own numerics (mlx, mlx_lm) import on this host."""
    try:
        import mlx.core  # noqa: F401
        import mlx_lm  # noqa: F401

        return "mlx and mlx_lm import"
    except Exception as e:  # ModuleNotFoundError on the images this runs on
        return f"{type(e).__name__}: {e}"


# --------------------------------------------------------------------------- clocks


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"sg_clocks_{os.getpid()}.csv"
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------- CPU port (oracle)


def cpu_port_step(cfg, x_bits, host, threads):
    """The CPU oracle's layer on one batch of tokens, experts spread over
    threads (one BLAS thread each)."""
    import numpy as np
    from threadpoolctl import threadpool_limits

    from oracle import slotted_glu_oracle as orc

    T = x_bits.shape[0]
    x = orc.bf16_bits_to_f32(x_bits)
    logits = orc.router_logits(x_bits, host["router"])
    inds, sc, _ = orc.get_routings(logits, cfg.top_k, cfg.norm_topk_prob)
    flat = inds.reshape(-1)
    y = np.zeros((T * cfg.top_k, cfg.hidden), np.float32)
    experts = host["experts"]

    def run(eid):
        pairs = np.nonzero(flat == eid)[0]
        y[pairs] = orc.expert_forward(x[pairs // cfg.top_k], experts[int(eid)])

    with threadpool_limits(1), ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(run, np.unique(flat)))
    sy = sg = None
    if host["shared"] is not None:
        sy = orc.expert_forward(x, host["shared"])
        sg = orc.bf16_bits_to_f32(orc.router_logits(x_bits, host["shared_gate"]))
    return orc.combine_shared(y.reshape(T, cfg.top_k, cfg.hidden), orc.bf16_bits_to_f32(sc), sy, sg)


def _sample_tokens(cfg, n, i):
    from preemptlm_b200.synthetic import _gen, _randn

    return _randn((n, cfg.hidden), _gen(1000 * cfg.cfg_id + 500 + i, "cpu"), "cpu", 1.0)


def _b16(t):
    import numpy as np
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _deq(cfg, ts, i):
    """Dequantised weights of expert ``i`` of a host tensor dict."""
    import numpy as np

    from oracle import slotted_glu_oracle as orc

    mats = []
    for p in ("gate_proj", "up_proj", "down_proj"):
        if cfg.bits == 16:
            mats.append(orc.bf16_bits_to_f32(_b16(ts[f"{p}.weight"][i])))
        else:
            mats.append(orc.dequant_affine(ts[f"{p}.weight"][i].numpy().view(np.uint32),
                                           _b16(ts[f"{p}.scales"][i]), _b16(ts[f"{p}.biases"][i]), cfg.bits))
    return orc.ExpertWeights(*mats)


def host_layer(cfg, T, n_steps, tens=None):
    """Host copy of the layer for the CPU port, made once before any timing:
    router and shared-gate bits, and the weights of every routed expert the
    timed token batches reach, dequantised once (the reference's arena holds
    bf16 expert weights, expert_cache.py:198-224, so its step does no
    dequantisation either).  Copied from the GPU layer's tensors, or generated
    on the host (reference arm: no GPU use; routed experts then come from
    per-expert seeds, with the layer's shapes and distributions)."""
    import numpy as np
    import torch

    from oracle import slotted_glu_oracle as orc
    from preemptlm_b200.synthetic import _gen, _randn, make_expert_tensors

    c = cfg.cfg_id
    threads = os.cpu_count() or 1
    if tens is not None:
        router = tens["router"].cpu()
        sgate = None if tens["shared_gate"] is None else tens["shared_gate"].cpu()
        shared_t = None if tens["shared"] is None else {k: v.cpu() for k, v in tens["shared"].items()}
    else:
        router = _randn((cfg.num_experts, cfg.hidden), _gen(1000 * c + 1, "cpu"), "cpu", 0.02)
        shared_t = sgate = None
        if cfg.shared_inter is not None:
            shared_t = make_expert_tensors(cfg, 1, cfg.shared_inter, 1000 * c + 3, "cpu")
            sgate = _randn((1, cfg.hidden), _gen(1000 * c + 4, "cpu"), "cpu", 0.02)
    rb = _b16(router)
    needed = set()
    for i in range(n_steps):
        lg = orc.router_logits(_b16(_sample_tokens(cfg, T, i)), rb)
        needed.update(orc.get_routings(lg, cfg.top_k, cfg.norm_topk_prob)[0].reshape(-1).tolist())
    needed = sorted(needed)
    if tens is not None:
        idx = torch.tensor(needed, device=tens["router"].device)
        host_t = {k: v.index_select(0, idx).cpu() for k, v in tens["experts"].items()}
        load = lambda j: _deq(cfg, host_t, j)  # noqa: E731
    else:
        def load(j):
            e = needed[j]
            return _deq(cfg, make_expert_tensors(cfg, 1, cfg.inter, 1000 * c + 2 + 7919 * (e + 1), "cpu"), 0)
    from threadpoolctl import threadpool_limits

    with threadpool_limits(1), ThreadPoolExecutor(max_workers=threads) as ex:
        mats = list(ex.map(load, range(len(needed))))
    return {"router": rb, "experts": dict(zip(needed, mats)),
            "shared": None if shared_t is None else _deq(cfg, shared_t, 0),
            "shared_gate": None if sgate is None else _b16(sgate)}


def time_cpu_port(cfg, T, steps, host, warmup=0):
    """Seconds per step of the CPU port on batches of T tokens, all host threads."""
    threads = os.cpu_count() or 1
    times = []
    for i in range(warmup + steps):
        xb = _b16(_sample_tokens(cfg, T, i))
        t0 = time.perf_counter()
        cpu_port_step(cfg, xb, host, threads)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return times, threads


# --------------------------------------------------------------------------- our arm


def _kernel_roofline(cfg, timing, rows_per_step, T_local):
    """Algorithmic bytes / CUDA-event time of the routed gate/up (and down)
    launches recorded in ``timing``."""
    import statistics as st

    H, I, k = cfg.hidden, cfg.inter, cfg.top_k
    if cfg.bits == 16:
        per_gu, per_dn = 2 * I * H * 2, H * I * 2
    else:
        per_gu = 2 * (I * H * cfg.bits // 8 + (I * H // 64) * 4)
        per_dn = H * I * cfg.bits // 8 + (H * I // 64) * 4
    gu_ms, dn_ms, gu_b, dn_b, us, gu_f, dn_f = [], [], 0, 0, [], 0, 0
    for i, (ev, cnt) in enumerate(zip(timing["events"], timing["dispatch"])):
        U = int(cnt[0].item())
        P = rows_per_step[i] if rows_per_step else T_local * k
        if not isinstance(P, int):  # (counts, group_off) of a dispatch over padded inboxes: filled entries
            P = int(P[1][int(P[0][0].item())].item())
        n_in = T_local if not rows_per_step else P  # distinct input rows read
        us.append(U)
        gu_ms.append(ev[0].elapsed_time(ev[1]))
        dn_ms.append(ev[1].elapsed_time(ev[2]))
        gu_b += U * per_gu + n_in * H * 2 + P * I * 2
        dn_b += U * per_dn + P * I * 2 + P * H * 2
        gu_f += 4 * P * H * I  # gate and up, 2 flops per multiply-add
        dn_f += 2 * P * H * I
    return {"gu_ms": gu_ms, "dn_ms": dn_ms, "gu_bytes": gu_b, "dn_bytes": dn_b, "unique": us,
            "gu_gbs": gu_b / (sum(gu_ms) * 1e-3) / 1e9, "dn_gbs": dn_b / (sum(dn_ms) * 1e-3) / 1e9,
            "gu_tflops": gu_f / (sum(gu_ms) * 1e-3) / 1e12, "dn_tflops": dn_f / (sum(dn_ms) * 1e-3) / 1e12,
            "pairs_per_expert": (gu_f / (4 * H * I)) / max(1, sum(us)),
            "mean_unique": st.mean(us)}


def _abi_check_status(where: str) -> None:
    """Raise if a kernel of the library recorded an error (a bounded wait that
    gave up) since the last check; synchronises, so never inside a timed region."""
    from preemptlm_b200 import ops

    st = ops.device_status(reset=True)
    if st != 0:
        raise RuntimeError(f"{where}: a kernel recorded status {st} (bounded wait expired)")


# (configuration, token counts) of the one-GPU sweep: the sizes BASELINE's configurations name
SWEEP = (("cfg3", (1, 8, 32, 128)), ("cfg1", (1, 4, 16, 32)), ("cfg2", (512, 2048, 8192)), ("cfg4", (64, 4096)))


def _step_roofline(cfg, T, U, ms):
    """Fraction of the binding roofline of a whole layer step: algorithmic
    bytes (every byte once: the unique experts' weights, router, shared
    expert, tokens in and out) over the measured copy bandwidth, or
    algorithmic FLOPs over the measured bf16 tensor peak, whichever takes
    longer."""
    hbm, _ = hbm_peak()
    tpk, _ = tensor_peak()
    H, E, k, I = cfg.hidden, cfg.num_experts, cfg.top_k, cfg.inter
    nbytes = U * cfg.expert_bytes() + cfg.shared_bytes() + E * H * 2 + 2 * T * H * 2
    flops = 2 * T * k * 3 * H * I + 2 * T * H * E
    if cfg.shared_inter is not None:
        nbytes += H * 2
        flops += 2 * T * 3 * H * cfg.shared_inter + 2 * T * H
    t_hbm, t_tc = nbytes / (hbm * 1e9), flops / (tpk * 1e12)
    bound = "hbm" if t_hbm >= t_tc else "tensor"
    return {"bound": bound, "step_frac": round(max(t_hbm, t_tc) / (ms * 1e-3), 4),
            "step_GBs": round(nbytes / (ms * 1e-3) / 1e9, 1), "step_TFLOPs": round(flops / (ms * 1e-3) / 1e12, 1)}


def _sweep_point(moe, cfg, T, steps, warmup, dev, flush):
    """One (configuration, T) point: the layer step captured as a CUDA graph
    and replayed on new tokens, an L2 flush (a 256 MB read) before every
    timed replay, CUDA events around each replay; then the same steps eagerly
    with events around the routed gate/up and down launches."""
    import torch

    from preemptlm_b200.synthetic import make_tokens

    H = cfg.hidden
    xs = [make_tokens(cfg, T, device=dev, step=5000 + i) for i in range(warmup + steps)]
    for i in range(warmup):
        moe.forward_resident(xs[i], timing={})
    moe.capture(1, T)
    g_in = moe.graph_input.view(T, H)
    for i in range(warmup):
        g_in.copy_(xs[i], non_blocking=True)
        moe.replay()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    torch.cuda._sleep(QUEUE_AHEAD_CYCLES // 4)
    for i in range(steps):
        g_in.copy_(xs[warmup + i], non_blocking=True)
        flush()
        ev[i][0].record()
        moe.replay()
        ev[i][1].record()
    timing: dict = {}
    torch.cuda._sleep(QUEUE_AHEAD_CYCLES // 4)  # the host queues the eager steps ahead of the GPU
    for i in range(steps):
        flush()
        moe.forward_resident(xs[warmup + i], timing=timing)
    torch.cuda.synchronize()
    _abi_check_status(f"sweep {cfg.name} T={T}")
    ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    rl = _kernel_roofline(cfg, timing, None, T)
    hbm, _ = hbm_peak()
    tpk, _ = tensor_peak()
    gu_ms, dn_ms = statistics.mean(rl["gu_ms"]), statistics.mean(rl["dn_ms"])
    pt = {"T": T, "tokens_per_s": round(T / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
          "unique_experts": round(rl["mean_unique"], 1), "pairs_per_expert": round(rl["pairs_per_expert"], 1),
          **_step_roofline(cfg, T, rl["mean_unique"], ms),
          "gate_up": {"ms": round(gu_ms, 4), "GBs": round(rl["gu_gbs"], 1), "hbm_frac": round(rl["gu_gbs"] / hbm, 4),
                      "TFLOPs": round(rl["gu_tflops"], 1), "tensor_frac": round(rl["gu_tflops"] / tpk, 4)},
          "down": {"ms": round(dn_ms, 4), "GBs": round(rl["dn_gbs"], 1), "hbm_frac": round(rl["dn_gbs"] / hbm, 4),
                   "TFLOPs": round(rl["dn_tflops"], 1), "tensor_frac": round(rl["dn_tflops"] / tpk, 4)}}
    return pt


def run_sweep(args, dev):
    """Every configuration at its benchmark sizes on one GPU (all experts of
    the layer resident), plus the streaming miss path."""
    import torch

    from preemptlm_b200 import ops
    from preemptlm_b200.layer import Qwen3_xMoEWrapper
    from preemptlm_b200.synthetic import CONFIGS, make_layer

    only = set(args.sweep_only.split(",")) if args.sweep_only else None
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev)  # 256 MB, twice the L2
    sink = torch.empty(1, dtype=torch.float32, device=dev)

    def flush():
        torch.amax(flush_buf, dim=0, keepdim=True, out=sink)

    ops.set_glu_path("auto")
    out = {"l2": "a 256 MB read before every timed step", "timed_steps": "CUDA graph replays",
           "steps": args.sweep_steps}
    for name, Ts in SWEEP:
        if only and name not in only:
            continue
        cfg = CONFIGS[name]
        block, tens = make_layer(cfg, device=dev)
        del tens  # the arena holds its own copy
        torch.cuda.empty_cache()
        moe = Qwen3_xMoEWrapper(block, "synthetic", "model.layers.0.mlp", 0)
        pts = [_sweep_point(moe, cfg, T, args.sweep_steps, 3, dev, flush) for T in Ts]
        out[name] = {"workload": f"{cfg.name}: H{cfg.hidden} E{cfg.num_experts} k{cfg.top_k} I{cfg.inter} "
                                 f"shared{cfg.shared_inter} {'bf16' if cfg.bits == 16 else f'affine-q{cfg.bits} g64'}, "
                                 f"all {cfg.num_experts} experts resident", "points": pts}
        del moe, block
        torch.cuda.empty_cache()
    if not only or "cfg5" in only:
        out["cfg5"] = stream_points(dev, steps=max(10, args.sweep_steps), warmup=3)
    return out


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from preemptlm_b200 import ops
    from preemptlm_b200.layer import Qwen3_xMoEWrapper
    from preemptlm_b200.synthetic import CONFIGS, make_layer, make_tokens

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = CONFIGS[args.workload]
    if args.experts:
        cfg = cfg.scaled(num_experts=args.experts, num_slots=args.experts)
    if args.no_shared:
        cfg = cfg.scaled(shared_inter=None)
    ops.set_glu_path(args.glu_path)
    T = args.tokens
    H = cfg.hidden
    use_ep = world > 1 or args.ep
    if use_ep:
        if world == 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            os.environ.setdefault("MASTER_PORT", "29533")
            dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=180), device_id=dev)
        else:
            dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        from preemptlm_b200.ep import ExpertParallelMoE, shard_layer

        backend, _ = shard_layer(cfg, rank, world, dev)
        mb = args.microbatches or (1 if args.ep_transport == "p2p" else 2)
        ep = ExpertParallelMoE(backend, cfg.num_experts, H, cfg.top_k, transport=args.ep_transport,
                               max_tokens=-(-T // mb))

        def step(x):
            # the step's tokens in mb micro-batches, every count exchange queued
            # before the host waits on the first
            return torch.cat(ep.forward_many(x.chunk(mb))) if mb > 1 else ep.forward(x)
        tens = None
    else:
        block, tens = make_layer(cfg, device=dev)
        moe = Qwen3_xMoEWrapper(block, "synthetic", "model.layers.0.mlp", 0)
        backend = None
    n_in = args.warmup + args.steps
    xs = [make_tokens(cfg, T, device=dev, step=i + 1000 * rank) for i in range(n_in)]
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def run_step(x, timing=None):
        if use_ep:
            backend.timing = timing
            return step(x)
        return moe.forward_resident(x, timing=timing)

    for i in range(args.warmup):
        # the per-kernel timing pass's own code path, so nothing runs for the
        # first time inside a timed region
        run_step(xs[i], timing={})
    torch.cuda.synchronize()

    # The timed steps replay the step captured as a CUDA graph (the public
    # capture/replay calls): a step then costs the host one input copy and one
    # graph launch, so host-side stalls on a shared machine cannot idle the GPU
    # inside the timed region.  Per-kernel times come from a separate eager pass.
    graph_ok = not args.no_graph and not args.profile and (
        not use_ep or (args.ep_transport == "p2p" and mb == 1))
    if graph_ok:
        if use_ep:
            ep.capture(T)
            g_in, g_replay = ep.graph_input, ep.replay
        else:
            moe.capture(1, T)
            g_in, g_replay = moe.graph_input.view(T, H), moe.replay

    def timed_step(x, timing):
        if graph_ok:
            g_in.copy_(x, non_blocking=True)
            return g_replay()
        return run_step(x, timing=timing)

    # ---------------------------------------------------------------- device-resident timing
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    timing: dict = {}
    launches0 = ops.LAUNCHES[0]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    host_t = []
    gc.collect()
    gc.disable()  # host-side collector pauses would leave the GPU idle between launches
    # a bounded device spin ahead of the timed region lets the host queue the
    # steps before the GPU reaches them, so a host-side hiccup (driver lock,
    # allocator) cannot idle the GPU inside the timed region
    torch.cuda._sleep(QUEUE_AHEAD_CYCLES)
    if world > 1:
        # one untimed exchange step after the spin: the ranks' spins end a
        # little apart, and this step (which waits on every peer) lines up
        # their timed regions
        timed_step(xs[0], {})
    start.record()
    for i in range(args.steps):
        step_ev[i].record()
        h0 = time.perf_counter()
        timed_step(xs[args.warmup + i], timing)
        host_t.append(time.perf_counter() - h0)
    step_ev[args.steps].record()
    end.record()
    torch.cuda.synchronize()
    gc.enable()
    barrier()
    clk = clocks.stop()
    launches = ops.LAUNCHES[0] - launches0
    ms_step = start.elapsed_time(end) / args.steps
    if graph_ok:  # per-kernel events: the same steps again, issued eagerly behind the same spin
        gc.disable()
        torch.cuda._sleep(QUEUE_AHEAD_CYCLES)
        if world > 1:
            run_step(xs[0], timing={})
        for i in range(args.steps):
            run_step(xs[args.warmup + i], timing=timing)
        torch.cuda.synchronize()
        gc.enable()
        barrier()
    per_step = [step_ev[i].elapsed_time(step_ev[i + 1]) for i in range(args.steps)]
    step_stats = {"min_ms": round(min(per_step), 4), "median_ms": round(statistics.median(per_step), 4),
                  "max_ms": round(max(per_step), 4), "host_median_ms": round(1e3 * statistics.median(host_t), 4),
                  "host_max_ms": round(1e3 * max(host_t), 4)}
    if use_ep:
        backend.timing = None
        if timing.get("phases"):  # per-phase device time of the exchange step, mean over the timed steps
            names = ("route_shared", "send", "wait_inbox", "experts", "send_back", "wait_back", "combine")
            ph = timing["phases"]
            step_stats["phases_ms"] = {n: round(statistics.mean(m[j].elapsed_time(m[j + 1]) for m in ph), 4)
                                       for j, n in enumerate(names)}
    if world > 1:
        t = torch.tensor([ms_step], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step = float(t.item())

    if args.profile:
        if rank == 0:
            print(json.dumps({"profile": cfg.name, "experts": cfg.num_experts, "tokens": T, "ms_per_step": ms_step,
                          "steps_detail": step_stats}))
        if use_ep:
            ep.close()
            dist.destroy_process_group()
        return
    rl = _kernel_roofline(cfg, timing, timing.get("rows"), T)
    peak, peak_kind = hbm_peak()
    tpeak, tpeak_kind = tensor_peak()
    us_mean = rl["mean_unique"]
    step_bytes = (us_mean * cfg.expert_bytes() + cfg.shared_bytes() + cfg.num_experts * H * 2 + 2 * T * H * 2)
    step_gbs = step_bytes / (ms_step * 1e-3) / 1e9

    # ---------------------------------------------------------------- end to end (host buffers)
    x_host = [torch.empty((T, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    for i, xh in enumerate(x_host):
        xh.copy_(xs[i].cpu())
    out_host = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()

    graphed = use_ep and args.ep_transport == "p2p" and mb == 1 and not args.no_graph
    if graphed and not graph_ok:
        # the expert-parallel step as one CUDA graph (captured once, collective):
        # the host's per-step cost is the input copy, one graph launch and the
        # output copy
        ep.capture(T)

    if not use_ep and not args.no_graph and not graph_ok:
        moe.capture(1, T)  # the public layer call as one CUDA graph

    # the captured step fed from pinned host memory through the public
    # pipeline: host->device and device->host copies overlap the neighbouring
    # steps' compute
    pipe = ep.host_pipeline() if graphed else (
        moe.host_pipeline() if not use_ep and not args.no_graph else None)

    def e2e_step(i):
        if pipe is not None:
            pipe.step(x_host[i % 2], out_host)
            return
        else:
            xd = x_host[i % 2].to(dev, non_blocking=True)
            out = step(xd) if use_ep else moe(xd.view(1, T, H)).view(T, H)
        out_host.copy_(out, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    gc.collect()
    gc.disable()
    e_start.record()
    for i in range(args.steps):
        e2e_step(i)
    if pipe is not None:
        pipe.drain()  # the last step's output is on the host inside the timed region
    e_end.record()
    torch.cuda.synchronize()
    gc.enable()
    barrier()
    e2e_ms = e_start.elapsed_time(e_end) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    # a bounded wait that gave up inside any of the steps above fails the run
    if use_ep:
        ep.check()
    else:
        _abi_check_status("timed steps")

    # ---------------------------------------------------------------- strong scaling (N > 1)
    strong = None
    if use_ep and world > 1 and graph_ok:
        Ts = max(1, 256 // world)
        ep.capture(Ts)
        xs_s = [make_tokens(cfg, Ts, device=dev, step=3000 + i + 1000 * rank) for i in range(args.steps)]
        for i in range(min(3, args.steps)):
            ep.replay(xs_s[i])
        torch.cuda.synchronize()
        barrier()
        gc.disable()
        torch.cuda._sleep(QUEUE_AHEAD_CYCLES)
        ep.replay(xs_s[0])  # lines up the ranks after the spin (untimed)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for i in range(args.steps):
            ep.replay(xs_s[i])
        s1.record()
        torch.cuda.synchronize()
        gc.enable()
        barrier()
        ep.check()
        t = torch.tensor([s0.elapsed_time(s1) / args.steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_s = float(t.item())
        strong = {"tokens_global": Ts * world, "tokens_per_gpu": Ts, "value": round(Ts * world / (ms_s * 1e-3), 1),
                  "unit": "tokens/s", "ms_per_step": round(ms_s, 4), "scaling": "strong",
                  "timed_steps": "CUDA graph replays"}

    # ---------------------------------------------------------------- CPU baseline (oracle port)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n = 2
        times, threads = time_cpu_port(cfg, T, n, host_layer(cfg, T, n + 1, tens), warmup=1)
        cpu = {"value": round(T * len(times) / sum(times), 3), "unit": "tokens/s", "cores": threads,
               "kind": "port",
               "sample": f"{len(times)} steps of the same {T}-token step through the CPU oracle of the layer "
                         f"(router, routing, fp32 matmuls of weights dequantised once at set-up, combine), "
                         f"experts over {threads} threads"}

    # ---------------------------------------------------------------- per-configuration sweep (one GPU)
    sweep = None
    if world == 1 and not use_ep and not args.no_sweep and not args.experts:
        del moe, block, tens
        torch.cuda.empty_cache()
        sweep = run_sweep(args, dev)

    shard = cfg.num_experts // world
    value = T * world / (ms_step * 1e-3)
    # DRAM bytes per unique expert of the same kernel from the committed ncu
    # summary (a 1-GPU capture of this workload's layer shape)
    traffic_pe, traffic_src = profile_traffic(cfg.name) if not args.experts else (None, None)
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": f"u{cfg.bits}" if cfg.bits != 16 else "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) tokens)",
        "config": {
            "workload": f"{cfg.name}: H{cfg.hidden} E{cfg.num_experts} k{cfg.top_k} I{cfg.inter} "
                        f"shared{cfg.shared_inter} affine-q{cfg.bits} g64, decode {T} tokens/GPU, "
                        f"expert-parallel over {world} GPU(s), all {shard} experts of each shard resident",
            "tokens_per_gpu": T, "hidden": H, "experts": cfg.num_experts, "top_k": cfg.top_k, "inter": cfg.inter,
            "shared_inter": cfg.shared_inter, "bits": cfg.bits, "slots_per_gpu": shard,
            "unique_experts_per_step_per_gpu": round(us_mean, 1),
            "l2": "no flush: each step streams >126 MB (L2) of expert weights per GPU",
            "queue": "device-resident steps are queued behind a bounded device spin (not timed); e2e is not",
            "parallelism": f"ep{world}",
            "microbatches": mb if use_ep else 1,
            "exchange": args.ep_transport if use_ep else None,
            "e2e_graph": not args.no_graph and (graphed or not use_ep),
            "timed_steps": "CUDA graph replays" if graph_ok else "eager",
        },
        "roofline": {
            "bound": "hbm", "kernel": f"{ops.LAST_GATE_UP[0]} (routed, q{cfg.bits})", "achieved": round(rl["gu_gbs"], 1),
            "peak": peak, "unit": "GB/s", "frac": round(rl["gu_gbs"] / peak, 4), "peak_kind": peak_kind,
            "traffic": round(traffic_pe * us_mean) if traffic_pe else None,
            "traffic_source": traffic_src,
            "bytes_per_launch": round(rl["gu_bytes"] / len(rl["gu_ms"])),
            "ms_per_launch": round(statistics.mean(rl["gu_ms"]), 5),
            "down": {"achieved": round(rl["dn_gbs"], 1), "frac": round(rl["dn_gbs"] / peak, 4),
                     "ms_per_launch": round(statistics.mean(rl["dn_ms"]), 5)},
            "step_achieved": round(step_gbs, 1), "step_frac": round(step_gbs / peak, 4),
            "tensor": {"achieved": round(rl["gu_tflops"], 1), "peak": tpeak, "unit": "TFLOP/s",
                       "frac": round(rl["gu_tflops"] / tpeak, 4), "peak_kind": tpeak_kind,
                       "down_achieved": round(rl["dn_tflops"], 1)},
            "pairs_per_expert": round(rl["pairs_per_expert"], 1),
        },
        "e2e": {"value": round(T * world / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2, "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": launches,
        "step_detail": step_stats,
        "clocks": clk,
        "cpu_baseline": cpu,
    }
    if strong is not None:
        line["strong"] = strong
    if sweep is not None:
        line["sweep"] = sweep
    if rl["pairs_per_expert"] >= 64:
        # prefill-sized expert groups: the gate/up launch is tensor-core bound
        r = line["roofline"]
        hbm = {k: r[k] for k in ("achieved", "peak", "unit", "frac", "peak_kind")}
        r.update(bound="tensor", achieved=r["tensor"]["achieved"], peak=tpeak, unit="TFLOP/s",
                 frac=r["tensor"]["frac"], peak_kind=tpeak_kind, hbm=hbm)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if use_ep:
        barrier()
        ep.close()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- reference arm


def run_stack(args, rank, world, local_rank):
    """``--layers L``: the MoE blocks of an L-layer decoder stack, each split
    expert-parallel over the N GPUs and all sharing one peer exchange.  A step
    is one pass of ``--tokens`` tokens per GPU through every layer on the
    residual stream (x <- x + layer(x)); the whole step is one CUDA graph.
    Per-kernel figures are layer 0's, from an eager pass."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from preemptlm_b200 import ops
    from preemptlm_b200.ep import ExpertParallelMoE, ExpertParallelStack, PeerExchange, shard_layer
    from preemptlm_b200.synthetic import CONFIGS, make_tokens

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cfg = CONFIGS[args.workload]
    L, T, H = args.layers, args.tokens, cfg.hidden
    if world == 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=300), device_id=dev)
    else:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        dist.barrier(device_ids=[local_rank])

    t_build = time.perf_counter()
    ex = PeerExchange(None, world, rank, T, cfg.top_k, H, dev)
    layers = []
    for li in range(L):
        backend, _ = shard_layer(cfg, rank, world, dev, layer=li)
        layers.append(ExpertParallelMoE(backend, cfg.num_experts, H, cfg.top_k, transport="p2p", max_tokens=T,
                                        exchange=ex))
        torch.cuda.empty_cache()
    stack = ExpertParallelStack(layers)
    build_s = time.perf_counter() - t_build
    mem_gb = torch.cuda.memory_allocated(dev) / 1e9
    xs = [make_tokens(cfg, T, device=dev, step=i + 1000 * rank) for i in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        stack(xs[i])
    torch.cuda.synchronize()
    mem_before = torch.cuda.memory_allocated(dev)
    stack.capture(T)
    graph_pool_gb = (torch.cuda.memory_allocated(dev) - mem_before) / 1e9  # buffers the graph keeps
    for i in range(args.warmup):
        stack.replay(xs[i])
    torch.cuda.synchronize()
    barrier()

    # device-resident: graph replays queued behind a bounded device spin
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    launches0 = ops.LAUNCHES[0]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gc.collect()
    gc.disable()
    torch.cuda._sleep(QUEUE_AHEAD_CYCLES)
    stack.replay(xs[0])  # lines up the ranks after the spin (untimed)
    start.record()
    for i in range(args.steps):
        stack.replay(xs[args.warmup + i])
    end.record()
    torch.cuda.synchronize()
    gc.enable()
    barrier()
    clk = clocks.stop()
    launches = ops.LAUNCHES[0] - launches0
    t = torch.tensor([start.elapsed_time(end) / args.steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_step = float(t.item())

    # layer 0's kernels and exchange phases: an eager pass behind the same spin
    timing: dict = {}
    n_eager = min(args.steps, 5)
    gc.disable()
    torch.cuda._sleep(QUEUE_AHEAD_CYCLES)
    layers[0].backend.timing = timing
    for i in range(n_eager):
        stack(xs[args.warmup + i])
    torch.cuda.synchronize()
    layers[0].backend.timing = None
    gc.enable()
    barrier()
    rl = _kernel_roofline(cfg, timing, timing.get("rows"), T)
    phases = None
    if timing.get("phases"):
        names = ("route_shared", "send", "wait_inbox", "experts", "send_back", "wait_back", "combine")
        phases = {n: round(statistics.mean(m[j].elapsed_time(m[j + 1]) for m in timing["phases"]), 4)
                  for j, n in enumerate(names)}
    peak, peak_kind = hbm_peak()
    us_mean = rl["mean_unique"]
    step_bytes = L * (us_mean * cfg.expert_bytes() + cfg.shared_bytes() + cfg.num_experts * H * 2 + 2 * T * H * 2)
    step_gbs = step_bytes / (ms_step * 1e-3) / 1e9

    # end to end: the captured stack fed from pinned host memory through the pipeline
    x_host = [torch.empty((T, H), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    for i, xh in enumerate(x_host):
        xh.copy_(xs[i].cpu())
    out_host = torch.empty((T, H), dtype=torch.bfloat16).pin_memory()
    pipe = stack.host_pipeline()
    for i in range(args.warmup):
        pipe.step(x_host[i % 2], out_host)
    pipe.drain()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gc.disable()
    e0.record()
    for i in range(args.steps):
        pipe.step(x_host[i % 2], out_host)
    pipe.drain()
    e1.record()
    torch.cuda.synchronize()
    gc.enable()
    barrier()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    stack.check()

    shard = cfg.num_experts // world
    value = T * world / (ms_step * 1e-3)
    line = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": f"u{cfg.bits}" if cfg.bits != 16 else "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, every layer its own seeds; N(0,1) tokens)",
        "config": {
            "workload": f"{cfg.name} x {L} layers: H{cfg.hidden} E{cfg.num_experts} k{cfg.top_k} I{cfg.inter} "
                        f"shared{cfg.shared_inter} affine-q{cfg.bits} g64, {'prefill' if T >= 1024 else 'decode'} {T} "
                        f"tokens/GPU through every layer "
                        f"(x <- x + moe(x)), expert-parallel over {world} GPU(s), {shard} experts of each "
                        f"layer resident per GPU",
            "layers": L, "tokens_per_gpu": T, "hidden": H, "experts": cfg.num_experts, "top_k": cfg.top_k,
            "inter": cfg.inter, "shared_inter": cfg.shared_inter, "bits": cfg.bits, "slots_per_gpu_per_layer": shard,
            "weights_gb_per_gpu": round(mem_gb, 1), "graph_pool_gb_per_gpu": round(graph_pool_gb, 2),
            "peak_gb_per_gpu": round(torch.cuda.max_memory_allocated(dev) / 1e9, 1), "build_s": round(build_s, 1),
            "unique_experts_per_layer_per_gpu": round(us_mean, 1),
            "l2": "no flush: each step streams every layer's experts (GBs per GPU)",
            "queue": "device-resident steps are queued behind a bounded device spin (not timed); e2e is not",
            "parallelism": f"ep{world}", "exchange": "p2p, one region shared by the layers",
            "timed_steps": "CUDA graph replays of the whole stack",
        },
        "roofline": {
            "bound": "hbm", "kernel": f"{ops.LAST_GATE_UP[0]} (routed, q{cfg.bits}, layer 0)",
            "achieved": round(rl["gu_gbs"], 1), "peak": peak, "unit": "GB/s", "frac": round(rl["gu_gbs"] / peak, 4),
            "peak_kind": peak_kind, "traffic": None, "traffic_source": None,
            "ms_per_launch": round(statistics.mean(rl["gu_ms"]), 5),
            "down": {"achieved": round(rl["dn_gbs"], 1), "frac": round(rl["dn_gbs"] / peak, 4),
                     "ms_per_launch": round(statistics.mean(rl["dn_ms"]), 5)},
            "step_achieved": round(step_gbs, 1), "step_frac": round(step_gbs / peak, 4),
            "pairs_per_expert": round(rl["pairs_per_expert"], 1),
        },
        "e2e": {"value": round(T * world / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 2, "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": launches,
        "step_detail": {"ms_per_layer": round(ms_step / L, 4), "layer0_phases_ms": phases},
        "clocks": clk,
        "cpu_baseline": None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    barrier()
    stack.close()
    dist.destroy_process_group()


def run_reference(args, rank, world):
    """The CPU port of the layer (the oracle; the reference's own MLX numerics
    do not import here) on the same step as our arm: a batch of --tokens
    tokens (256) of the cfg3 layer, all host cores."""
    if rank != 0:
        return
    from preemptlm_b200.synthetic import CONFIGS

    cfg = CONFIGS[args.workload]
    T = args.tokens
    probe = mlx_probe()
    warm = min(args.warmup, 1)  # CPU steps need no long warm-up; the run stays within minutes
    t0 = time.perf_counter()
    host = host_layer(cfg, T, warm + args.steps)
    setup_s = time.perf_counter() - t0
    times, threads = time_cpu_port(cfg, T, args.steps, host, warmup=warm)
    value = T * len(times) / sum(times)
    sample = (f"{len(times)} steps of {T} tokens of the {cfg.name} layer through the CPU oracle port (router, "
              f"routing, fp32 matmuls of expert weights dequantised once at set-up, combine), experts over "
              f"{threads} threads; mlx probe: {probe}")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
        "steps": len(times), "warmup": warm, "ms_per_step": round(1e3 * sum(times) / len(times), 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"u{cfg.bits}" if cfg.bits != 16 else "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) tokens)",
        "config": {"workload": f"{cfg.name}: H{cfg.hidden} E{cfg.num_experts} k{cfg.top_k} I{cfg.inter} "
                               f"shared{cfg.shared_inter} affine-q{cfg.bits} g64, decode {T} tokens per step "
                               f"(CPU port, one host)",
                   "tokens_per_gpu": T, "parallelism": "cpu", "setup_s": round(setup_s, 1)},
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "mlx_probe": probe,
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _fs_of(path) -> str:
    """File-system type of the mount holding ``path`` (from /proc/mounts)."""
    try:
        best, fs = "", "unknown"
        p = str(Path(path).resolve())
        for line in Path("/proc/mounts").read_text().splitlines():
            parts = line.split()
            if len(parts) >= 3 and p.startswith(parts[1]) and len(parts[1]) > len(best):
                best, fs = parts[1], f"{parts[2]} ({parts[0]} on {parts[1]})"
        return fs
    except Exception:
        return "unknown"


def stream_points(dev, steps, warmup, batches=(1, 16)):
    """Streaming miss path (config-2 layer shape: H2048 E128 k8 I768, affine
    q4 g64, 64 slots): a seeded expert bank written to local disk, Zipf(1.1)
    expert popularity, demand refills through DiskBackedExpertLoader (pread
    into pinned host buffers, cudaMemcpyAsync into slots on a side stream),
    end-to-end decode tokens/s (tokens host->device, output device->host every
    step)."""
    import shutil
    import tempfile

    import torch

    from preemptlm_b200.bank import PreadExpertBank
    from preemptlm_b200.cache_manager import ExpertCacheManager
    from preemptlm_b200.layer import Qwen3_xMoEWrapper
    from preemptlm_b200.loader import DiskBackedExpertLoader, HostExpertCache
    from preemptlm_b200.synthetic import CONFIGS, make_layer, make_zipf_tokens, write_bank

    cfg = CONFIGS["cfg2"].scaled(name="cfg5-stream-q4", num_slots=64)
    block, tens = make_layer(cfg, device=dev)
    tmp = Path(tempfile.mkdtemp(prefix="sg_bank_", dir=os.environ.get("SG_BANK_DIR")))
    t0 = time.perf_counter()
    write_bank(tmp, cfg, tens["experts"], block.switch_mlp.tensor_names())
    os.sync()
    write_s = time.perf_counter() - t0
    results = {"workload": f"{cfg.name}: H{cfg.hidden} E{cfg.num_experts} k{cfg.top_k} I{cfg.inter} affine-q4 g64, "
                           f"{cfg.num_slots} slots, host blob cache of 32 experts, lfru slots, Zipf(1.1) routing",
               "bank_fs": _fs_of(tmp), "bank_write_s": round(write_s, 2)}
    try:
        for batch in batches:
            bank = PreadExpertBank(tmp, bypass_page_cache=True)
            nbytes = bank.manifest.expert_num_bytes()
            cache = HostExpertCache(ExpertCacheManager(budget_bytes=32 * nbytes))
            loader = DiskBackedExpertLoader(expert_bank=bank, cache=cache)

            class Cand:
                layer_path, block_idx = "model.layers.0.mlp", 0

            moe = Qwen3_xMoEWrapper.make_wrapper_factory(model_fingerprint=bank.model_fingerprint,
                                                         expert_loader=loader, expert_cache=cache,
                                                         num_slots=cfg.num_slots, slot_size=nbytes,
                                                         slot_policy="lfru")(block, Cand())
            n = warmup + steps
            xs = make_zipf_tokens(tens["router"], n * batch, cfg.top_k, seed=500 + batch, device=dev)
            x_host = xs.cpu().pin_memory().view(n, batch, cfg.hidden)
            out_host = torch.empty((batch, cfg.hidden), dtype=torch.bfloat16).pin_memory()

            def step(i):
                xd = x_host[i].to(dev, non_blocking=True)
                out_host.copy_(moe(xd.view(1, batch, cfg.hidden)).view(batch, cfg.hidden), non_blocking=True)

            for i in range(warmup):
                step(i)
            torch.cuda.synchronize()
            moe.admit_stats.update(steps=0, unique=0, missed=0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(warmup, n):
                step(i)
            e1.record()
            torch.cuda.synchronize()
            _abi_check_status(f"streaming batch {batch}")
            ms = e0.elapsed_time(e1) / steps
            st = moe.admit_stats
            results[f"batch{batch}"] = {"tokens_per_s": round(batch * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
                                        "hit_rate": round(1 - st["missed"] / max(1, st["unique"]), 4),
                                        "refills_per_step": round(st["missed"] / max(1, st["steps"]), 2)}
            loader.close()
            bank.close()
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return results


def run_stream(args, rank, world, local_rank):
    """``--workload cfg5``: the streaming miss path alone (one GPU)."""
    import torch

    if world > 1:
        raise SystemExit("the streaming workload runs on one GPU")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    results = stream_points(dev, args.steps, args.warmup)
    if rank == 0:
        b16 = results["batch16"]
        print(json.dumps({
            "metric": "streaming decode tokens/s (end to end, demand refills from disk)", "value": b16["tokens_per_s"],
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": b16["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u4", "data": "synthetic (seeded bank on local disk, Zipf(1.1) routing)",
            "config": results,
        }))


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    if args.gpus > 1 and world == 1:
        raise SystemExit("--gpus N > 1 runs under torch.distributed.run (one process per GPU)")
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "cfg5":
        run_stream(args, rank, world, local_rank)
        return
    if args.layers > 1:
        run_stack(args, rank, world, local_rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
