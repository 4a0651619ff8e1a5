"""Drop-in for the reference's kernel module (dsv4_kernels.py).

Same two entry points and signatures:

* ``eligible(inputs, indices, weight_up, scales_up, biases_up, *, group_size,
  bits)`` -- whether the decode geometry fits the fused kernel
  (dsv4_kernels.py:217-243).  Like the reference it accepts decode only
  (``inputs.shape[0] == 1``), but for 2-, 4- and 8-bit codes and groups of
  64/128 (32 for 4/8-bit) instead of 2-bit / group 128 only.
* ``fused_affine2_swiglu(inputs, indices, wu, su, bu, wg, sg, bg, *,
  group_size, limit)`` -> ``[tokens, top_k, 1, n]`` post-SwiGLU activations
  (dsv4_kernels.py:246-300): gate and up products over arena slots with one
  rounding of ``silu_f32(min(gate, L)) * clip(up, -L, L)``.  The reference
  passes ``int(limit)`` to its kernel (:293); here the limit is used as given
  (identical for the V4 value 10.0).

Both run on the sm_100a kernels of liblmoe.so through the C ABI; there is no
Metal/CUDA-JIT/CPU alternative.
"""

from __future__ import annotations

import torch

from . import ops

_SUPPORTED = {(2, 64), (2, 128), (4, 32), (4, 64), (4, 128), (8, 32), (8, 64), (8, 128)}


def eligible(inputs: torch.Tensor, indices: torch.Tensor, weight_up: torch.Tensor, scales_up: torch.Tensor,
             biases_up: torch.Tensor, *, group_size: int, bits: int) -> bool:
    if inputs.ndim != 4 or indices.ndim != 2 or int(inputs.shape[0]) != 1:
        return False
    k = int(inputs.shape[-1])
    n = int(scales_up.shape[-2])
    return (
        (bits, group_size) in _SUPPORTED
        and inputs.dtype in (torch.float16, torch.bfloat16)
        and weight_up.dtype in (torch.int32, getattr(torch, "uint32", torch.int32))
        and scales_up.dtype == inputs.dtype
        and biases_up.dtype == inputs.dtype
        and k % group_size == 0
        and n % 16 == 0
        and int(weight_up.shape[-1]) == k * bits // 32
        and int(scales_up.shape[-1]) == k // group_size
    )


def fused_affine2_swiglu(inputs: torch.Tensor, indices: torch.Tensor, weight_up: torch.Tensor,
                         scales_up: torch.Tensor, biases_up: torch.Tensor, weight_gate: torch.Tensor,
                         scales_gate: torch.Tensor, biases_gate: torch.Tensor, *, group_size: int,
                         limit: float) -> torch.Tensor:
    tokens = int(inputs.shape[0])
    top_k = int(indices.shape[-1])
    k = int(inputs.shape[-1])
    n = int(scales_up.shape[-2])
    bits = int(weight_up.shape[-1]) * 32 // k
    up = ops.QProjArrays(weight_up, scales_up, biases_up, bits, group_size)
    gate = ops.QProjArrays(weight_gate, scales_gate, biases_gate, bits, group_size)
    ex = ops.ExpertArrays(gate, up, gate)  # the down projection is not read by this call
    h = ops.gateup_swiglu(inputs.reshape(tokens, k), indices.reshape(tokens, top_k), ex, limit, "fused")
    return h.reshape(tokens, top_k, 1, n)


__all__ = ["eligible", "fused_affine2_swiglu"]
