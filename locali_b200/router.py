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
    """The V4 gate on the device.  ``tid2eid`` (int [vocab, top_k], optional)
    is the token-id -> expert table of a hash-routed layer (the first layers
    of DeepSeek-V4, dsv4_arena.py:149-152): with it, a call with ``input_ids``
    takes the experts from the table and weights them by their scores; without
    it (or without ``input_ids``) the layer is scored (top-k on score + bias)."""

    def __init__(self, router: RouterArrays, tid2eid: torch.Tensor | None = None):
        self.router = router
        self.tid2eid = None if tid2eid is None else tid2eid.to(device=router.weight.device, dtype=torch.int32)
        self._ws = None

    @property
    def top_k(self) -> int:
        return self.router.top_k

    @property
    def weight(self) -> torch.Tensor:
        return self.router.weight

    def hash_idx(self, input_ids) -> torch.Tensor | None:
        """[T, top_k] experts of the tokens of a hash-routed layer, else None."""
        if self.tid2eid is None or input_ids is None:
            return None
        ids = torch.as_tensor(input_ids, device=self.tid2eid.device).reshape(-1).long()
        return self.tid2eid.index_select(0, ids)

    def __call__(self, x: torch.Tensor, input_ids=None):
        if self._ws is None:
            self._ws = ops.Workspace(x.device)
        lead = x.shape[:-1]
        if x.dtype not in (torch.bfloat16, torch.float16):
            x = x.to(torch.bfloat16)
        idx, w = ops.route(x.reshape(-1, x.shape[-1]), self.router, self._ws, hash_idx=self.hash_idx(input_ids))
        k = self.router.top_k
        return idx.reshape(*lead, k), w.reshape(*lead, k)
