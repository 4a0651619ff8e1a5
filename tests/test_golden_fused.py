"""Parity pins against outputs of the reference's own CUDA fused 2-bit gate/up
+ clamped SwiGLU kernel (dsv4_kernels.py:100-173, built from the reference
sources by oracle/build_ref.py and run by tests/golden/make_golden.py on a
B200; the fixture stores seeds, shapes and the output bits only).

* CPU: the numpy oracle (fused rounding mode) reproduces the reference
  kernel's bits except for last-place differences from fp32 summation order.
* GPU: the sm_100a gate/up + SwiGLU kernel (lmoe_gateup_swiglu) reproduces
  them to the same bar, from the row-major arrays and from the pre-tiled copy.
"""

import json

import numpy as np
import pytest

from oracle import moe_oracle as O
from tests.golden.make_golden import HERE, fused_inputs

GOLDEN = HERE / "ref_fused_swiglu.npz"
LIMIT = 10.0


def _cases():
    z = np.load(GOLDEN)
    return [(tuple(c), z[c[0]]) for c in json.loads(str(z["meta"]))]


def _to_f32(bits, dtype):
    bits = np.asarray(bits, np.uint16)
    if dtype == "f16":
        return bits.view(np.float16).astype(np.float32)
    return O.bf16_bits_to_f32(bits)


def _oracle(inp, K, N, GS, top_k, dtype):
    x = np.repeat(inp["x"].astype(np.float32), top_k, axis=0)
    up = O.gather_qmm(x, O.QProjNP(inp["wu"], inp["su"], inp["bu"], 2, GS), inp["slots"], dtype)
    gate = O.gather_qmm(x, O.QProjNP(inp["wg"], inp["sg"], inp["bg"], 2, GS), inp["slots"], dtype)
    return O.swiglu(up, gate, LIMIT, "fused", dtype)


def _check(got, ref):
    # rel L2 (the parity bar is 1e-2) and last-place agreement
    assert O.rel_l2(got, ref) < 3e-3
    assert float(np.mean(got != ref)) < 0.05


@pytest.mark.parametrize("case", range(4))
def test_oracle_matches_reference_kernel(case):
    (name, K, N, GS, top_k, dtype, n_slots, seed), bits = _cases()[case]
    inp = fused_inputs(K, N, GS, top_k, dtype, n_slots, seed)
    ref = _to_f32(bits, dtype)
    _check(_oracle(inp, K, N, GS, top_k, dtype), ref)


@pytest.mark.gpu
@pytest.mark.parametrize("tiled", [False, True])
@pytest.mark.parametrize("case", range(4))
def test_kernel_matches_reference_kernel(built, case, tiled):
    import torch

    from locali_b200 import ops

    (name, K, N, GS, top_k, dtype, n_slots, seed), bits = _cases()[case]
    inp = fused_inputs(K, N, GS, top_k, dtype, n_slots, seed)
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16

    def act(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(tdt).cuda()

    def words(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()

    up = ops.QProjArrays(words(inp["wu"]), act(inp["su"]), act(inp["bu"]), 2, GS)
    gate = ops.QProjArrays(words(inp["wg"]), act(inp["sg"]), act(inp["bg"]), 2, GS)
    if tiled:
        if up.tile_bytes() == 0:
            pytest.skip(f"K={K} is below one 8-group chunk of g{GS}: no stream tile layout")
        up.pack_tiles()
        gate.pack_tiles()
    ex = ops.ExpertArrays(gate, up, gate)  # down is not read by this call
    slots = torch.from_numpy(inp["slots"].astype(np.int32)).reshape(1, top_k).cuda()
    h = ops.gateup_swiglu(act(inp["x"]), slots, ex, LIMIT, "fused")
    torch.cuda.synchronize()
    got = h.float().cpu().numpy()
    ref = _to_f32(bits, dtype)
    _check(got, ref)


def test_oracle_hash_router_weights():
    """The hash-routed oracle takes the given experts and normalises their scores."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, 64)).astype(np.float32)
    wg = (rng.standard_normal((8, 64)) * 0.1).astype(np.float32)
    hidx = np.array([[0, 1], [7, 3], [5, 5]], dtype=np.int32)
    idx, w, scores, _ = O.router(x, wg, None, 2, "sigmoid", 2.0, True, hash_idx=hidx)
    assert np.array_equal(idx, hidx)
    g = np.take_along_axis(scores, hidx, axis=-1)
    np.testing.assert_allclose(w, 2.0 * g / (g.sum(-1, keepdims=True) + 1e-20), rtol=1e-6)


def test_oracle_three_bit_stream_layout():
    """3-bit rows are one LSB-first bit stream (MLX packs 8 codes per 3 bytes):
    element j at bits [3j, 3j+3) of the row's little-endian bytes."""
    rng = np.random.default_rng(1)
    c = rng.integers(0, 8, (4, 96)).astype(np.uint8)
    w = O.pack_codes(c, 3)
    assert w.shape == (4, 9)
    assert np.array_equal(O.unpack_codes(w, 3, 96), c)
    bits = np.unpackbits(w.view(np.uint8).reshape(4, -1), axis=1, bitorder="little")
    for j in (0, 10, 11, 21, 31, 95):
        assert int(bits[2, 3 * j] + 2 * bits[2, 3 * j + 1] + 4 * bits[2, 3 * j + 2]) == c[2, j]
