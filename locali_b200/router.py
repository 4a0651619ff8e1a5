"""Resident V4 MoE gate running on the router kernel.

Plays the role of the checkpoint's MoEGate that ``V4ArenaMoE.route`` calls
(dsv4_arena.py:165-166): ``gate(x, input_ids) -> (indices, weights)``.  The
arithmetic is arena.py:501-506 plus the V4 routed scaling: fp32 logits of
bf16 activations and weights, sigmoid (or sqrt-softplus / softmax) scores,
top-k on ``score + bias`` (bias is selection-only), weights from the raw
scores normalised by ``sum + 1e-20`` and multiplied by ``routed_scaling``.
"""

from __future__ import annotations

import torch

from . import ops
from .ops import RouterArrays


class V4Gate:
    def __init__(self, router: RouterArrays):
        self.router = router
        self._ws = None

    @property
    def top_k(self) -> int:
        return self.router.top_k

    @property
    def weight(self) -> torch.Tensor:
        return self.router.weight

    def __call__(self, x: torch.Tensor, input_ids=None):
        if self._ws is None:
            self._ws = ops.Workspace(x.device)
        lead = x.shape[:-1]
        if x.dtype not in (torch.bfloat16, torch.float16):
            x = x.to(torch.bfloat16)
        idx, w = ops.route(x.reshape(-1, x.shape[-1]), self.router, self._ws)
        k = self.router.top_k
        return idx.reshape(*lead, k), w.reshape(*lead, k)
