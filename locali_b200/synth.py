"""Seeded synthetic routed-MoE layers with the shapes and value distributions
of the benchmark configurations (no checkpoint or dataset is involved).

C0  hidden 1024, 16 experts, top-6, inter 512, 4-bit g64, scaling 1.0, 8 tokens
C1  hidden 4096, 256 experts, top-6, inter 2048, 2-bit g64, scaling 2.5, 1 token
C2  C1 with gate/up 2-bit and down 4-bit, 1/4/16/64 tokens, Zipf expert popularity
C3  C1 prefill: 4096 tokens, uniform or Zipf routing
C4  43 layers of C2 shapes, expert parallel over 1/2/4/8 GPUs, 256 tokens

Values: activations N(0,1) bf16; router weight N(0,0.02) bf16; router bias
N(0,0.01) fp32; codes uniformly random over all bits; scales |N(0,0.01)| and
biases N(0,0.01) in bf16.  Arena slot 0 is the reserved all-zero slot and
expert e lives in slot e + 1.

Zipf popularity (C2-C4) is a per-expert selection-bias tilt
``beta * ln(p_e / p_max)`` with ``p_e`` proportional to ``rank_e^-1.1`` over a
seeded random ranking; ``beta = 0.032`` puts about 60% of the top-6 selections
on the 64 most popular experts.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from .ops import ExpertArrays, QProjArrays, RouterArrays

ZIPF_S = 1.1
ZIPF_BETA = 0.032


@dataclass(frozen=True)
class MoEConfig:
    name: str
    hidden: int
    n_experts: int
    top_k: int
    inter: int
    bits_gate: int
    bits_up: int
    bits_down: int
    group_size: int
    swiglu_limit: float = 10.0
    routed_scaling: float = 1.0
    tokens: int = 1
    zipf: bool = False
    scoring: str = "sigmoid"

    def expert_bytes(self) -> int:
        """Code + scale + bias bytes of one expert (all three projections)."""
        H, I, gs = self.hidden, self.inter, self.group_size
        sb = 2 * 2  # scale + bias, 2 bytes each
        gate = I * H * self.bits_gate // 8 + I * (H // gs) * sb
        up = I * H * self.bits_up // 8 + I * (H // gs) * sb
        down = H * I * self.bits_down // 8 + H * (I // gs) * sb
        return gate + up + down

    def gateup_bytes(self) -> int:
        H, I, gs = self.hidden, self.inter, self.group_size
        return I * H * (self.bits_gate + self.bits_up) // 8 + 2 * I * (H // gs) * 4

    def down_bytes(self) -> int:
        H, I, gs = self.hidden, self.inter, self.group_size
        return H * I * self.bits_down // 8 + H * (I // gs) * 4

    def router_bytes(self) -> int:
        return self.n_experts * self.hidden * 2 + self.n_experts * 4


CONFIGS = {
    "c0": MoEConfig("c0", 1024, 16, 6, 512, 4, 4, 4, 64, 10.0, 1.0, 8),
    "c1": MoEConfig("c1", 4096, 256, 6, 2048, 2, 2, 2, 64, 10.0, 2.5, 1),
    "c2": MoEConfig("c2", 4096, 256, 6, 2048, 2, 2, 4, 64, 10.0, 2.5, 1, zipf=True),
    "c3": MoEConfig("c3", 4096, 256, 6, 2048, 2, 2, 2, 64, 10.0, 2.5, 4096),
    "c4": MoEConfig("c4", 4096, 256, 6, 2048, 2, 2, 4, 64, 10.0, 2.5, 256, zipf=True),
}


def config(name: str, **over) -> MoEConfig:
    return replace(CONFIGS[name], **over)


def zipf_bias(n_experts: int, generator: torch.Generator) -> torch.Tensor:
    rank = torch.randperm(n_experts, generator=generator, device=generator.device)
    p = (rank.double() + 1.0).pow(-ZIPF_S)
    return (ZIPF_BETA * torch.log(p / p.max())).float()


def _qproj(rows: int, cols: int, bits: int, gs: int, n_slots: int, g: torch.Generator,
           dtype: torch.dtype) -> QProjArrays:
    dev = g.device
    w = torch.randint(-(2**31), 2**31, (n_slots, rows, cols * bits // 32), generator=g, dtype=torch.int32,
                      device=dev)
    s = (torch.randn((n_slots, rows, cols // gs), generator=g, device=dev) * 0.01).abs().to(dtype)
    b = (torch.randn((n_slots, rows, cols // gs), generator=g, device=dev) * 0.01).to(dtype)
    w[0].zero_()
    s[0].zero_()
    b[0].zero_()
    return QProjArrays(w, s, b, bits, gs)


@dataclass
class SynthLayer:
    cfg: MoEConfig
    router: RouterArrays
    experts: ExpertArrays
    expert_slot: torch.Tensor


def make_layer(cfg: MoEConfig, seed: int = 0, device: str | torch.device = "cpu",
               dtype: torch.dtype = torch.bfloat16, extra_slots: int = 0) -> SynthLayer:
    """All tensors are generated on ``device`` with a generator seeded by
    ``seed``.  ``extra_slots`` more arena slots after the experts' (slot
    ``E + 1``: e.g. the block's shared expert) hold random weights too."""
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    E, H, I = cfg.n_experts, cfg.hidden, cfg.inter
    rw = (torch.randn((E, H), generator=g, device=device) * 0.02).to(torch.bfloat16)
    rb = torch.randn((E,), generator=g, device=device) * 0.01
    if cfg.zipf:
        rb = rb + zipf_bias(E, g)
    router = RouterArrays(rw, rb.float().contiguous(), cfg.top_k, cfg.scoring, cfg.routed_scaling, True)
    n_slots = E + 1 + extra_slots
    gate = _qproj(I, H, cfg.bits_gate, cfg.group_size, n_slots, g, dtype)
    up = _qproj(I, H, cfg.bits_up, cfg.group_size, n_slots, g, dtype)
    down = _qproj(H, I, cfg.bits_down, cfg.group_size, n_slots, g, dtype)
    slot = torch.arange(1, E + 1, dtype=torch.int32, device=device)
    return SynthLayer(cfg, router, ExpertArrays(gate, up, down), slot)


def make_tokens(cfg: MoEConfig, tokens: int | None = None, seed: int = 1,
                device: str | torch.device = "cpu", dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    device = torch.device(device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    T = cfg.tokens if tokens is None else tokens
    return torch.randn((T, cfg.hidden), generator=g, device=device).to(dtype)


def layer_to(layer: SynthLayer, device: str | torch.device) -> SynthLayer:
    def mv(q: QProjArrays) -> QProjArrays:
        return QProjArrays(q.weight.to(device), q.scales.to(device), q.biases.to(device), q.bits, q.group_size)

    r = layer.router
    return SynthLayer(layer.cfg,
                      RouterArrays(r.weight.to(device), None if r.bias is None else r.bias.to(device), r.top_k,
                                   r.scoring, r.routed_scaling, r.norm_topk),
                      ExpertArrays(mv(layer.experts.gate), mv(layer.experts.up), mv(layer.experts.down)),
                      layer.expert_slot.to(device))

