"""numpy restatement of Locali's routed-MoE layer (TEST INFRASTRUCTURE ONLY).

What is restated, and from where (paths within gabrielekarra/locali):

* Code layout: affine codes packed LSB-first into little-endian uint32 words.
  Element ``j`` of a row occupies bits ``[j*b, (j+1)*b)`` of the row's bit
  stream (``dsv4_kernels.py:59-73`` for the Metal body, ``:135-150`` for the
  CUDA body: word ``w`` holds columns ``[w*32/b, (w+1)*32/b)``, low bits first).
  3-bit rows are the same continuous bit stream (MLX packs 8 codes per 3 bytes
  LSB-first); no in-repo source pins that, so 3-bit is marked unpinned.
* Dequantised product (``mx.gather_qmm``, MLX 0.32.0, third party, called at
  ``dsv4_arena.py:198-221`` and ``arena.py:676-681``): per output row ``n`` and
  group ``g`` of ``group_size`` columns, ``scale[n,g] * sum_j x_j q_nj +
  bias[n,g] * sum_j x_j``, accumulated in fp32 and rounded once to the
  activation dtype (``dsv4_kernels.py:152-154`` and ``:165-166`` state the same
  arithmetic for the fused decode kernel).  The oracle accumulates in float64,
  which is closer to exact than any fp32 order.
* Clamped SwiGLU (``dsv4_arena.py:223-235``): ``up`` and ``gate`` are rounded to
  the activation dtype first, then ``up = clip(up, -L, L)``,
  ``gate = min(gate, L)``.  Two rounding modes:
  ``"fused"`` = ``T(silu_f32(gate) * up)`` with one rounding
  (``dsv4_kernels.py:165-170``; also ``fp32_swiglu`` at ``dsv4_arena.py:228-232``);
  ``"stock"`` = MLX ``nn.silu(gate) * up`` evaluated op by op in bf16
  (``dsv4_arena.py:234``; the per-op rounding of MLX's compiled silu is not
  pinned here).
* Router (``arena.py:501-506``): ``s = sigmoid(x_f32 @ Wg^T)``; the top-k is
  chosen on ``s + bias`` (bias is selection-only); weights are the raw scores of
  the chosen experts normalised by ``sum + 1e-20``; the V4 gate then applies
  ``routed_scaling_factor`` (``tests/test_dsv4_engine_small.py:50,113-116``).
  Ties in the selection are broken towards the lower expert id (MLX's
  argpartition leaves them unspecified).
* Combine (``arena.py:543`` and ``:619-624``): weights cast to the activation
  dtype, ``y * w`` rounded per element, summed over k (fp32 accumulation in
  route order, one final rounding; MLX's bf16 reduction order is not pinned).
* Prefill weights (``weights="rounded"``): the build's prefill path
  dequantises each weight to the activation dtype before the matrix product
  (one rounding of the exact ``scale * q + bias``), the dequantise-then-GEMM
  form MLX's quantized matmul takes for large batches (not pinned here).  The
  decode path and ``weights="exact"`` never round a weight.
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace

import numpy as np

__all__ = [
    "bf16_bits_to_f32",
    "f32_to_bf16_bits",
    "bf16_round",
    "f16_round",
    "round_act",
    "pack_codes",
    "unpack_codes",
    "dequantize",
    "gather_qmm",
    "round_act_exact",
    "swiglu",
    "router",
    "near_ties",
    "combine",
    "moe_layer",
    "rel_l2",
    "ExpertsNP",
    "LayerNP",
    "QProjNP",
    "silu_f32",
]


# ---------------------------------------------------------------- bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 values (exact)."""
    bits = np.asarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bf16 bit patterns (uint16)."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = u.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float values to bf16 (nearest even); returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(a, dtype=np.float32)))


def f16_round(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_act(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round to the activation dtype ('bf16' or 'f16'), as float32."""
    if dtype == "bf16":
        return bf16_round(a)
    if dtype == "f16":
        return f16_round(a)
    raise ValueError(dtype)


# ---------------------------------------------------------------- code layout
def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """[..., K] integer codes -> [..., K*bits/32] uint32, LSB-first bit stream.

    Follows the layout read by ``dsv4_kernels.py:135-150`` (2-bit) and its
    generalisation to b bits; element j sits at bits [j*b, (j+1)*b).
    """
    codes = np.asarray(codes)
    K = codes.shape[-1]
    if (K * bits) % 32:
        raise ValueError("row bit length must be a multiple of 32")
    lead = codes.shape[:-1]
    c = codes.reshape(-1, K).astype(np.uint64) & ((1 << bits) - 1)
    nwords = K * bits // 32
    out = np.zeros((c.shape[0], nwords), dtype=np.uint64)
    for j in range(K):
        bit = j * bits
        w, sh = divmod(bit, 32)
        out[:, w] |= (c[:, j] << sh) & 0xFFFFFFFF
        if sh + bits > 32:  # straddles into the next word (3-bit)
            out[:, w + 1] |= c[:, j] >> (32 - sh)
    return out.astype(np.uint32).reshape(*lead, nwords)


def unpack_codes(words: np.ndarray, bits: int, K: int | None = None) -> np.ndarray:
    """Inverse of :func:`pack_codes`: [..., W] uint32 -> [..., K] uint8 codes."""
    words = np.asarray(words, dtype=np.uint32)
    W = words.shape[-1]
    if K is None:
        K = W * 32 // bits
    lead = words.shape[:-1]
    flat = words.reshape(-1, W)
    mask = (1 << bits) - 1
    if 32 % bits == 0:
        per = 32 // bits
        shifts = (np.arange(per, dtype=np.uint32) * bits)[None, None, :]
        out = (flat[:, :, None] >> shifts) & mask
        return out.reshape(*lead, W * per)[..., :K].astype(np.uint8)
    # general bit stream (3-bit): view as little-endian bytes, then bits
    by = flat.view(np.uint8).reshape(flat.shape[0], W * 4)
    bitarr = np.unpackbits(by, axis=1, bitorder="little")
    idx = np.arange(K)[:, None] * bits + np.arange(bits)[None, :]
    sel = bitarr[:, idx]  # [rows, K, bits]
    weights = (1 << np.arange(bits)).astype(np.uint16)
    out = (sel.astype(np.uint16) * weights).sum(-1)
    return out.reshape(*lead, K).astype(np.uint8)


def round_act_exact(a, dtype: str = "bf16") -> np.ndarray:
    """Round float64 values once to the activation dtype (nearest, ties to
    even), without an intermediate float32 rounding."""
    a = np.asarray(a, np.float64)
    prec, qmin = (8, -133) if dtype == "bf16" else (11, -24)
    _, e = np.frexp(a)
    q = np.ldexp(1.0, np.maximum(e - prec, qmin))
    return (np.rint(a / q) * q).astype(np.float32)


def dequantize(words, scales, biases, bits, group_size, K=None):
    """Affine dequantisation ``scale*q + bias`` per group (float64)."""
    q = unpack_codes(words, bits, K).astype(np.float64)
    N, Kq = q.shape[-2], q.shape[-1]
    s = np.repeat(np.asarray(scales, np.float64), group_size, axis=-1)[..., :Kq]
    b = np.repeat(np.asarray(biases, np.float64), group_size, axis=-1)[..., :Kq]
    return s * q + b


# ---------------------------------------------------------------- projections
@dataclass
class QProjNP:
    """One projection's arena arrays for all slots (MLX SwitchGLU layout).

    weight uint32 [n_slots, rows, cols*bits/32]; scales/biases float32 values
    (already exact bf16/f16 numbers) [n_slots, rows, cols/group_size].
    """

    weight: np.ndarray
    scales: np.ndarray
    biases: np.ndarray
    bits: int
    group_size: int

    @property
    def rows(self) -> int:
        return int(self.weight.shape[-2])

    @property
    def cols(self) -> int:
        return int(self.scales.shape[-1]) * self.group_size


def gather_qmm(x: np.ndarray, proj: QProjNP, slots: np.ndarray, dtype: str = "bf16",
               acc=np.float64, weights: str = "exact") -> np.ndarray:
    """``mx.gather_qmm(x, w, s, b, rhs_indices=slots, transpose=True)``.

    x: [R, K] float (values already in the activation dtype), one row per
    route; slots: [R] arena slot per route.  Returns [R, N] rounded to dtype.
    Arithmetic per ``dsv4_kernels.py:152-154``: per group
    ``scale * sum(x*q) + bias * sum(x)``.  ``weights="rounded"``: each
    dequantised weight rounded once to dtype first (the prefill path).
    """
    x = np.asarray(x, dtype=np.float32)
    slots = np.asarray(slots).reshape(-1)
    R, K = x.shape
    gs = proj.group_size
    G = K // gs
    out = np.zeros((R, proj.rows), dtype=np.float64)
    if weights == "rounded":
        for slot in np.unique(slots):
            rows = np.nonzero(slots == slot)[0]
            wq = dequantize(proj.weight[slot], proj.scales[slot], proj.biases[slot], proj.bits, gs, K)
            wr = round_act_exact(wq, dtype).astype(np.float64)
            out[rows] = x[rows].astype(np.float64) @ wr.T
        return round_act(out, dtype)
    if weights != "exact":
        raise ValueError(weights)
    xg = x.astype(acc).reshape(R, G, gs)
    xsum = xg.sum(-1)  # [R, G]
    for slot in np.unique(slots):
        rows = np.nonzero(slots == slot)[0]
        q = unpack_codes(proj.weight[slot], proj.bits, K).astype(acc)  # [N, K]
        qg = q.reshape(proj.rows, G, gs)
        # dots[g, r, n] = sum_j x[r, g, j] * q[n, g, j]
        dots = np.matmul(xg[rows].transpose(1, 0, 2), qg.transpose(1, 2, 0))
        s = proj.scales[slot].astype(acc)  # [N, G]
        b = proj.biases[slot].astype(acc)
        out[rows] = np.einsum("grn,ng->rn", dots, s) + xsum[rows] @ b.T
    return round_act(out.astype(np.float32) if acc == np.float32 else out, dtype)


def swiglu(up: np.ndarray, gate: np.ndarray, limit: float, mode: str = "fused",
           dtype: str = "bf16") -> np.ndarray:
    """Clamped SwiGLU on dtype-rounded ``up``/``gate`` (``dsv4_arena.py:223-235``)."""
    up = np.asarray(up, np.float32)
    gate = np.asarray(gate, np.float32)
    if limit > 0:
        up = np.clip(up, np.float32(-limit), np.float32(limit))
        gate = np.minimum(gate, np.float32(limit))
    with np.errstate(over="ignore"):
        if mode == "fused":
            # dsv4_kernels.py:169-170: silu in fp32, one rounding of silu*up
            silu = gate / (np.float32(1.0) + np.exp(-gate, dtype=np.float32))
            return round_act(silu.astype(np.float32) * up, dtype)
        if mode == "stock":
            # nn.silu(gate) * up op by op in the activation dtype
            sig = round_act(np.float32(1.0) / (np.float32(1.0) + np.exp(-gate, dtype=np.float32)), dtype)
            s = round_act(gate * sig, dtype)
            return round_act(s * up, dtype)
    raise ValueError(mode)


# ---------------------------------------------------------------- router
def _score(logits: np.ndarray, scoring: str) -> np.ndarray:
    lg = logits.astype(np.float64)
    if scoring == "sigmoid":
        s = 1.0 / (1.0 + np.exp(-lg))
    elif scoring == "sqrtsoftplus":
        s = np.sqrt(np.logaddexp(0.0, lg))
    elif scoring == "softmax":
        m = lg.max(-1, keepdims=True)
        e = np.exp(lg - m)
        s = e / e.sum(-1, keepdims=True)
    else:
        raise ValueError(scoring)
    return s.astype(np.float32)


def router(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None, top_k: int,
           scoring: str = "sigmoid", routed_scaling: float = 1.0, norm_topk: bool = True,
           hash_idx: np.ndarray | None = None):
    """``ArenaMoE.route`` (``arena.py:501-506``) plus V4 routed scaling.

    x [T, H] values, weight [E, H] values (bf16 numbers).  Returns
    (idx [T,k] int32 ordered by biased score desc, w [T,k] float32,
    scores [T,E] float32, biased [T,E] float32).

    ``hash_idx`` [T, k]: token-id hash routing (the V4 gate's first layers,
    ``dsv4_arena.py:149-152``; the gate itself is not in the reference
    repository): the experts are given and weighted by their scores,
    normalised and scaled as for scored layers (ids outside [0, E) score 0).
    """
    x64 = np.asarray(x, np.float64)
    w64 = np.asarray(weight, np.float64)
    logits = (x64 @ w64.T).astype(np.float32)
    scores = _score(logits, scoring)
    biased = scores if bias is None else (scores + np.asarray(bias, np.float32)).astype(np.float32)
    T, E = scores.shape
    if hash_idx is not None:
        idx = np.asarray(hash_idx).reshape(T, top_k).astype(np.int32)
        ok = (idx >= 0) & (idx < E)
        g = np.where(ok, np.take_along_axis(scores, np.clip(idx, 0, E - 1), axis=-1), 0).astype(np.float32)
    else:
        # stable descending order: ties -> lower expert id first
        order = np.argsort(-biased, axis=-1, kind="stable")
        idx = order[:, :top_k].astype(np.int32)
        g = np.take_along_axis(scores, idx, axis=-1).astype(np.float32)
    if norm_topk:
        w = g / (g.sum(-1, keepdims=True, dtype=np.float32) + np.float32(1e-20))
    else:
        w = g
    w = (w * np.float32(routed_scaling)).astype(np.float32)
    return idx, w, scores, biased


def near_ties(biased: np.ndarray, top_k: int, eps: float = 1e-5) -> np.ndarray:
    """Tokens whose k-th and (k+1)-th biased scores differ by less than eps."""
    srt = -np.sort(-np.asarray(biased, np.float32), axis=-1)
    if srt.shape[-1] <= top_k:
        return np.zeros(srt.shape[0], dtype=bool)
    gap = srt[:, top_k - 1] - srt[:, top_k]
    return gap < eps


def combine(y: np.ndarray, w: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    """``(y * w.astype(dtype)[..., None]).sum(-2)`` (``arena.py:543,619-624``).

    y [T, k, H] dtype values; w [T, k] float32.  Products rounded per element,
    summed in route order in fp32, rounded once.
    """
    wb = round_act(np.asarray(w, np.float32), dtype)
    prod = round_act(np.asarray(y, np.float32) * wb[..., None], dtype)
    acc = np.zeros(prod.shape[0:1] + prod.shape[2:], dtype=np.float32)
    for j in range(prod.shape[1]):
        acc = (acc + prod[:, j]).astype(np.float32)
    return round_act(acc, dtype)


# ---------------------------------------------------------------- full layer
@dataclass
class ExpertsNP:
    gate: QProjNP
    up: QProjNP
    down: QProjNP


@dataclass
class LayerNP:
    """Host copy of one layer: router + experts + expert->slot map."""

    router_weight: np.ndarray          # [E, H] float32 (bf16 values)
    router_bias: np.ndarray | None     # [E] float32
    experts: ExpertsNP
    expert_slot: np.ndarray            # [E] int
    top_k: int = 6
    scoring: str = "sigmoid"
    routed_scaling: float = 1.0
    norm_topk: bool = True
    swiglu_limit: float = 10.0
    swiglu_mode: str = "fused"
    dtype: str = "bf16"
    extra: dict = field(default_factory=dict)


def expert_ffn(x: np.ndarray, idx: np.ndarray, layer: LayerNP, acc=np.float64, weights: str = "exact"):
    """``V4ArenaMoE._gather`` for [T,k] routes: returns (up, gate, h, y)."""
    T, k = idx.shape
    slots = np.asarray(layer.expert_slot)[idx.reshape(-1)]
    xr = np.repeat(np.asarray(x, np.float32), k, axis=0)  # route r = t*k + j
    ex = layer.experts
    up = gather_qmm(xr, ex.up, slots, layer.dtype, acc, weights)
    gate = gather_qmm(xr, ex.gate, slots, layer.dtype, acc, weights)
    h = swiglu(up, gate, layer.swiglu_limit, layer.swiglu_mode, layer.dtype)
    y = gather_qmm(h, ex.down, slots, layer.dtype, acc, weights)
    return (up.reshape(T, k, -1), gate.reshape(T, k, -1), h.reshape(T, k, -1),
            y.reshape(T, k, -1))


def moe_layer(x: np.ndarray, layer: LayerNP, idx: np.ndarray | None = None,
              w: np.ndarray | None = None, acc=np.float64, weights: str = "exact") -> dict:
    """One routed-MoE layer, ``ArenaMoE.__call__`` single-tier path
    (``arena.py:508-547`` with ``_apply`` ``:569-624``)."""
    x = np.asarray(x, np.float32)
    out = {}
    if idx is None:
        idx, w, scores, biased = router(x, layer.router_weight, layer.router_bias, layer.top_k,
                                        layer.scoring, layer.routed_scaling, layer.norm_topk)
        out["scores"], out["biased"] = scores, biased
        out["ties"] = near_ties(biased, layer.top_k)
    up, gate, h, y = expert_ffn(x, idx, layer, acc, weights)
    out.update(idx=idx, w=w, up=up, gate=gate, h=h, y=y, out=combine(y, w, layer.dtype))
    return out


def moe_block(x: np.ndarray, layer: LayerNP, shared_slot: int | None = None, residual: np.ndarray | None = None,
              acc=np.float64, weights: str = "exact") -> dict:
    """The patched V4 MoE block (``dsv4_engine.py:255-261``: ``routed +
    block.shared_experts(x)``) followed by the decoder layer's residual add.
    The shared expert is a SwitchGLU expert of the same arena (slot
    ``shared_slot``) taken by every token; each sum is rounded to the
    activation dtype: ``T(residual + T(T(routed) + T(shared)))``."""
    out = moe_layer(x, layer, acc=acc, weights=weights)
    o = out["out"]
    T = np.asarray(x).shape[0]
    if shared_slot is not None:
        shared_layer = replace(layer, expert_slot=np.array([shared_slot]))
        _, _, _, ys = expert_ffn(x, np.zeros((T, 1), np.int64), shared_layer, acc, weights)
        out["shared"] = ys[:, 0]
        o = round_act(o + ys[:, 0], layer.dtype)
    if residual is not None:
        o = round_act(np.asarray(residual, np.float32) + o, layer.dtype)
    out["block"] = o
    return out


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b.ravel())
    num = np.linalg.norm((a - b).ravel())
    return float(num / den) if den > 0 else float(num)


def silu_f32(g):
    g = np.asarray(g, np.float32)
    return g / (np.float32(1.0) + np.exp(-g, dtype=np.float32))

