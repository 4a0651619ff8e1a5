"""Convert torch layers/tensors of locali_b200 into oracle numpy inputs.

TEST INFRASTRUCTURE ONLY (see the package docstring).
"""

from __future__ import annotations

import numpy as np

from .moe_oracle import ExpertsNP, LayerNP, QProjNP


def t2np(t) -> np.ndarray:
    """torch tensor -> numpy (bf16/f16 values as exact float32; ints as-is)."""
    import torch

    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().numpy()
    if t.dtype == torch.int32:
        return t.numpy()
    return t.numpy()


def qproj_np(q) -> QProjNP:
    return QProjNP(t2np(q.weight).view(np.uint32), t2np(q.scales), t2np(q.biases), int(q.bits), int(q.group_size))


def layer_np(layer, swiglu_mode: str = "fused", dtype: str = "bf16") -> LayerNP:
    """From a ``locali_b200.synth.SynthLayer`` (or anything with the same fields)."""
    r = layer.router
    ex = layer.experts
    return LayerNP(
        router_weight=t2np(r.weight),
        router_bias=None if r.bias is None else t2np(r.bias),
        experts=ExpertsNP(qproj_np(ex.gate), qproj_np(ex.up), qproj_np(ex.down)),
        expert_slot=t2np(layer.expert_slot).astype(np.int64),
        top_k=int(r.top_k),
        scoring=r.scoring,
        routed_scaling=float(r.routed_scaling),
        norm_topk=bool(r.norm_topk),
        swiglu_limit=float(layer.cfg.swiglu_limit),
        swiglu_mode=swiglu_mode,
        dtype=dtype,
    )
