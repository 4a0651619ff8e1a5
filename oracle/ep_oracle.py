"""CPU restatement of the expert-parallel exchange (TEST INFRASTRUCTURE ONLY).

Only ``tests/`` import this module.  It restates, byte for byte where the
device writes bytes, the protocol of ``locali_b200/csrc/lmoe_ep.cu`` as
declared in ``include/lmoe.h`` (lmoe_ep_*):

* dispatch: for every destination rank ``d`` the rows of the tokens with at
  least one expert owned by ``d``, in token order, then padding rows; each
  row is the token's activations followed by a trailer of int32 local expert
  ids (``-1``: owned elsewhere), fp32 weights (0 where not local), the int32
  token id, zero padding to 16 bytes.  A padding row's trailer has ids
  ``-1``, weights 0 and token ``-1``; its activation bytes are unspecified
  (zero here).  ``slot_of[t, d]`` is the row of token ``t`` in ``d``'s block.
* partials (expert side): per real received row, the rounded ``y * w`` rows
  of its local routes (the single-device combine's per-route terms,
  ``arena.py:543,619-624``) summed in route order in fp32.
* combine (source side): per token, the partials of its owning ranks added
  in rank order in fp32 and rounded once; with a residual, rounded again
  after adding it.

The reference has no expert-parallel mode (``dsv4_engine.py:256-257`` runs
every expert of a layer on one device); the arithmetic restated here is the
single-device layer's (``arena.py:508-672``) split by expert owner, and is
checked against that layer in the tests.
"""

from __future__ import annotations

import numpy as np

from . import moe_oracle as O


def trailer_bytes(k: int) -> int:
    return (8 * k + 4 + 15) // 16 * 16


def row_bytes(H: int, k: int) -> int:
    return 2 * H + trailer_bytes(k)


def dispatch(x_bits: np.ndarray, idx: np.ndarray, w: np.ndarray, n_experts: int, world: int):
    """x_bits uint16 [T, H] (activation bits), idx [T, k], w [T, k] fp32 ->
    (send uint8 [world, T, row_bytes], slot_of int32 [T, world])."""
    x_bits = np.asarray(x_bits, np.uint16)
    idx = np.asarray(idx, np.int64)
    w = np.asarray(w, np.float32)
    T, H = x_bits.shape
    k = idx.shape[1]
    per = n_experts // world
    RB, TW = row_bytes(H, k), trailer_bytes(k) // 4
    send = np.zeros((world, T, RB), np.uint8)
    slot_of = np.full((T, world), -1, np.int32)
    valid = (idx >= 0) & (idx < n_experts)
    owner = np.where(valid, idx // per, -1)
    cnt = [0] * world
    for t in range(T):
        for d in range(world):
            own = owner[t] == d
            if not own.any():
                continue
            s = cnt[d]
            cnt[d] += 1
            slot_of[t, d] = s
            tr = np.zeros(TW, np.int32)
            tr[:k] = np.where(own, idx[t] - d * per, -1)
            tr[k:2 * k] = np.where(own, w[t], np.float32(0)).astype(np.float32).view(np.int32)
            tr[2 * k] = t
            send[d, s, :2 * H] = x_bits[t].view(np.uint8)
            send[d, s, 2 * H:] = tr.view(np.uint8)
    for d in range(world):
        for s in range(cnt[d], T):
            tr = np.zeros(TW, np.int32)
            tr[:k] = -1
            tr[2 * k] = -1
            send[d, s, 2 * H:] = tr.view(np.uint8)
    return send, slot_of


def parse(recv: np.ndarray, H: int, k: int):
    """recv uint8 [n, row_bytes] -> (x_bits uint16 [n, H], ids [n, k], w fp32 [n, k], token [n])."""
    recv = np.ascontiguousarray(recv, np.uint8).reshape(-1, row_bytes(H, k))
    xb = recv[:, :2 * H].copy().view(np.uint16)
    tr = recv[:, 2 * H:].copy().view(np.int32)
    return xb, tr[:, :k].copy(), tr[:, k:2 * k].copy().view(np.float32), tr[:, 2 * k].copy()


def bits_to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    bits = np.asarray(bits, np.uint16)
    if dtype == "f16":
        return bits.view(np.float16).astype(np.float32)
    return O.bf16_bits_to_f32(bits)


def partials(recv: np.ndarray, H: int, k: int, local: O.LayerNP, acc=np.float32) -> np.ndarray:
    """Expert side: fp32 [n, H]; padding rows are NaN (never read)."""
    xb, ids, w, tok = parse(recv, H, k)
    n = xb.shape[0]
    n_local = len(local.expert_slot)
    out = np.full((n, H), np.nan, np.float32)
    x = bits_to_f32(xb, local.dtype)
    rows, js = np.nonzero((ids >= 0) & (ids < n_local) & (tok[:, None] >= 0))
    for r in range(n):
        if tok[r] >= 0:
            out[r] = 0.0
    if rows.size == 0:
        return out
    _, _, _, y = O.expert_ffn(x[rows], ids[rows, js][:, None], local, acc)
    y = y.reshape(rows.size, H)
    wr = O.round_act(w[rows, js].astype(np.float32), local.dtype)
    yw = O.round_act(y * wr[:, None], local.dtype)
    order = np.lexsort((js, rows))  # per row, route order
    for i in order:
        out[rows[i]] += yw[i]
    return out


def combine(back: np.ndarray, slot_of: np.ndarray, dtype: str = "bf16", residual: np.ndarray | None = None):
    """Source side: back fp32 [world, T, H] -> out [T, H] (activation values)."""
    world, T, H = back.shape
    acc = np.zeros((T, H), np.float32)
    for d in range(world):  # rank order
        for t in range(T):
            s = slot_of[t, d]
            if s >= 0:
                acc[t] += back[d, s]
    out = O.round_act(acc, dtype)
    if residual is not None:
        out = O.round_act(out + np.asarray(residual, np.float32), dtype)
    return out


def normed(out: np.ndarray, dtype: str = "bf16", eps: float = 1e-6) -> np.ndarray:
    """Weightless LayerNorm of the combined rows (mean and variance over the
    row), rounded: the next layer's MoE input the expert-parallel combine
    writes."""
    o = np.asarray(out, np.float64)
    mean = np.mean(o, axis=-1, keepdims=True)
    var = np.mean((o - mean) ** 2, axis=-1, keepdims=True)
    return O.round_act(((o - mean) / np.sqrt(var + eps)).astype(np.float32), dtype)
