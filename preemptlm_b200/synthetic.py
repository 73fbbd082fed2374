"""Seeded synthetic MoE layers with the shapes of the benchmark configurations.

Weights are N(0, 0.02) bf16, router N(0, 0.02), activations N(0, 1) bf16;
quantised layers use per-group-64 min/max affine 4/8-bit.  Tensor t of
configuration c is drawn from a generator seeded ``1000 * c + t``.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from .arena import SlottedGLU
from .layer import SparseMoeBlock
from .quant import QuantSettings, quantize_affine


@dataclass(frozen=True)
class LayerConfig:
    name: str
    cfg_id: int
    hidden: int
    num_experts: int
    top_k: int
    inter: int
    shared_inter: int | None
    bits: int  # 16 = bf16
    num_slots: int
    norm_topk_prob: bool = True

    @property
    def quant(self) -> QuantSettings | None:
        return None if self.bits == 16 else QuantSettings("affine", self.bits, 64)

    def expert_bytes(self) -> int:
        n = 3 * self.hidden * self.inter
        return n * 2 if self.bits == 16 else n * self.bits // 8 + n // 64 * 4

    def shared_bytes(self) -> int:
        if self.shared_inter is None:
            return 0
        n = 3 * self.hidden * self.shared_inter
        return n * 2 if self.bits == 16 else n * self.bits // 8 + n // 64 * 4

    def scaled(self, **kw) -> "LayerConfig":
        return replace(self, **kw)


CONFIGS = {
    # single layer, bf16 decode; T in {1, 4, 16, 32}
    "cfg1": LayerConfig("cfg1-bf16-decode", 1, 2048, 128, 8, 768, None, 16, 64),
    # same shape, affine q4 g64 prefill; T in {512, 2048, 8192}
    "cfg2": LayerConfig("cfg2-q4-prefill", 2, 2048, 128, 8, 768, None, 4, 64),
    # Qwen3-Next-style: q8, shared expert 512, 128 slots; decode T = 1..256
    "cfg3": LayerConfig("cfg3-q8-decode-shared", 3, 2048, 512, 10, 512, 512, 8, 128),
    # Qwen3.5-397B-style layer of the 60-layer stack: q4, shared 1024, 256 slots
    "cfg4": LayerConfig("cfg4-q4-397b-layer", 4, 4096, 512, 10, 1024, 1024, 4, 256),
}


def _randn(shape, gen, device, std):
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_expert_tensors(cfg: LayerConfig, n: int, inter: int, seed: int, device) -> dict[str, torch.Tensor]:
    """Weights of ``n`` experts in blob-name form: ``gate_proj.weight`` ...
    bf16 [n, out, in], or packed/scales/biases when quantised."""
    g = _gen(seed, device)
    H = cfg.hidden
    out = {}
    for p, shape in (("gate_proj", (n, inter, H)), ("up_proj", (n, inter, H)), ("down_proj", (n, H, inter))):
        w = _randn(shape, g, device, 0.02)
        if cfg.bits == 16:
            out[f"{p}.weight"] = w
        else:
            parts = [quantize_affine(w[i: i + 32], cfg.bits, 64) for i in range(0, n, 32)]
            for j, part in enumerate(("weight", "scales", "biases")):
                out[f"{p}.{part}"] = torch.cat([q[j] for q in parts]) if len(parts) > 1 else parts[0][j]
            del w, parts
    return out


def fill_arena(arena: SlottedGLU, tensors: dict[str, torch.Tensor]) -> None:
    for name, t in tensors.items():
        arena._tensor(name).copy_(t)


def make_layer(cfg: LayerConfig, device="cuda", gen_device=None, experts: dict | None = None):
    """A non-streaming SparseMoeBlock with every routed expert resident
    (``switch_mlp`` arena of num_experts slots).  Returns (block, tensors)."""
    gen_device = gen_device or device
    c = cfg.cfg_id
    router = _randn((cfg.num_experts, cfg.hidden), _gen(1000 * c + 1, gen_device), gen_device, 0.02)
    if experts is None:
        experts = make_expert_tensors(cfg, cfg.num_experts, cfg.inter, 1000 * c + 2, gen_device)
    arena = SlottedGLU(cfg.num_experts, (cfg.inter, cfg.hidden), (cfg.hidden, cfg.inter), quant=cfg.quant,
                       device=device)
    fill_arena(arena, experts)
    shared = shared_t = sgate = None
    if cfg.shared_inter is not None:
        shared_t = make_expert_tensors(cfg, 1, cfg.shared_inter, 1000 * c + 3, gen_device)
        shared = SlottedGLU(1, (cfg.shared_inter, cfg.hidden), (cfg.hidden, cfg.shared_inter), quant=cfg.quant,
                            device=device)
        fill_arena(shared, shared_t)
        sgate = _randn((1, cfg.hidden), _gen(1000 * c + 4, gen_device), gen_device, 0.02)
    block = SparseMoeBlock(gate=router.to(device), top_k=cfg.top_k, norm_topk_prob=cfg.norm_topk_prob,
                           moe_intermediate_size=cfg.inter, quant=cfg.quant, switch_mlp=arena, shared_expert=shared,
                           shared_expert_gate=None if sgate is None else sgate.to(device))
    return block, {"router": router, "experts": experts, "shared": shared_t, "shared_gate": sgate}


def make_tokens(cfg: LayerConfig, T: int, device="cuda", step: int = 0) -> torch.Tensor:
    return _randn((T, cfg.hidden), _gen(1000 * cfg.cfg_id + 100 + step, device), device, 1.0)


def write_bank(path, cfg: LayerConfig, experts: dict[str, torch.Tensor], tensor_names, block_idx: int = 0):
    """Write ``experts`` (blob-name tensors, [E, ...]) as an expert bank of one
    MoE block with ExpertBankWriter: the seeded synthetic bank of the streaming
    workload."""
    from .bank import ExpertBankWriter, ModelMoESpec, assemble_expert_blob, derive_tensor_specs, make_encoding_tag

    names = tuple(tensor_names)
    specs = derive_tensor_specs({n: experts[n][0] for n in names}, names)
    spec = ModelMoESpec(moe_block_idxs=(block_idx,), num_routed_experts=cfg.num_experts, top_k=cfg.top_k)
    enc = make_encoding_tag(None if cfg.bits == 16 else cfg.bits, 64)
    with ExpertBankWriter(path, model_id=cfg.name, model_fingerprint=f"synthetic-{cfg.cfg_id}", encoding=enc,
                          tensor_specs=specs, model_moe_spec=spec, overwrite=True) as w:
        for e in range(cfg.num_experts):
            w.add_expert(block_idx, e, assemble_expert_blob({n: experts[n][e] for n in names}, specs))
    return None


def make_zipf_tokens(router: torch.Tensor, T: int, top_k: int, seed: int, s: float = 1.1, device="cuda",
                     noise: float = 0.1) -> torch.Tensor:
    """Tokens whose routing follows a Zipf(s) expert popularity: each token is
    a sum of the (normalised) router rows of top_k experts drawn by Zipf rank
    over a seeded random ranking of the experts, plus N(0, noise) -- so the
    real router sends it (almost always) to those experts."""
    import numpy as np

    E, H = router.shape
    rng = np.random.default_rng(seed)
    rank = rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1) ** s
    p /= p.sum()
    w = router.float().to(device)
    wn = w / (w * w).sum(1, keepdim=True)
    picks = np.stack([rank[rng.choice(E, size=top_k, replace=False, p=p)] for _ in range(T)])
    idx = torch.from_numpy(picks).to(device)
    x = 3.0 * wn[idx].sum(1)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = x + noise * torch.randn((T, H), generator=g, device=device)
    return x.to(torch.bfloat16)
