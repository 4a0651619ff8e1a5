"""The C-ABI libraries load and export every symbol their headers declare;
host-side validation works without a GPU (no kernel is launched here)."""

import ctypes
import re
from pathlib import Path

import pytest

from locali_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def _declared(header: Path) -> list[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b(lmoe_\w+|locali_cache_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_headers_declare_entry_points():
    lm = _declared(ROOT / "include" / "lmoe.h")
    assert "lmoe_moe_layer" in lm and "lmoe_gateup_swiglu" in lm and "lmoe_route" in lm
    core = _declared(ROOT / "include" / "locali_core.h")
    assert set(core) == set(_lib.CORE_SYMBOLS)


@pytest.mark.parametrize("header,lib", [("lmoe.h", "liblmoe.so"), ("locali_core.h", "liblocali_core.so")])
def test_library_exports_every_declared_symbol(built, header, lib):
    dll = ctypes.CDLL(str(ROOT / "locali_b200" / lib))
    for name in _declared(ROOT / "include" / header):
        assert hasattr(dll, name), f"{lib} does not export {name}"


def _layer(bits=2, gs=64, hidden=1024, inter=512, E=16, k=6):
    fake = 256  # non-null dummy pointers: nothing is dereferenced on the host
    q = lambda b: _lib.QProj(fake, fake, fake, b, gs)  # noqa: E731
    ex = _lib.Experts(E + 1, hidden, inter, _lib.LMOE_BF16, q(bits), q(bits), q(bits))
    r = _lib.Router(fake, None, E, k, 0, 1, 1.0)
    return _lib.Layer(r, ex, fake, 10.0, 0)


def test_workspace_size_and_validation(built):
    lib = _lib.lmoe()
    L = _layer()
    n1 = lib.lmoe_workspace_size(ctypes.byref(L), 1)
    n64 = lib.lmoe_workspace_size(ctypes.byref(L), 64)
    assert 0 < n1 < n64
    # unsupported bit width / group size
    assert lib.lmoe_workspace_size(ctypes.byref(_layer(bits=5)), 1) == 0
    assert lib.lmoe_workspace_size(ctypes.byref(_layer(bits=2, gs=32)), 1) == 0
    # top_k > n_experts
    assert lib.lmoe_workspace_size(ctypes.byref(_layer(E=4, k=6)), 1) == 0
    # zero tokens is a successful no-op; null pointers with tokens are rejected
    assert lib.lmoe_moe_layer(ctypes.byref(L), None, 0, None, None, None, None, 0, None) == _lib.LMOE_OK
    assert lib.lmoe_moe_layer(ctypes.byref(L), None, 4, None, None, None, None, 0, None) == _lib.LMOE_EINVAL
    assert lib.lmoe_moe_layer(None, None, 4, None, None, None, None, 0, None) == _lib.LMOE_EINVAL
    # host-buffer entry: zero tokens is a no-op; null buffers are rejected
    # before any CUDA call
    assert lib.lmoe_moe_layer_host(ctypes.byref(L), None, 0, None, None, None, 0, None, 0) == _lib.LMOE_OK
    assert lib.lmoe_moe_layer_host(ctypes.byref(L), None, 4, None, None, None, 0, None, 0) == _lib.LMOE_EINVAL
    assert lib.lmoe_moe_layer_host(ctypes.byref(L), 256, 4, 256, None, 256, 1 << 30, None, 0) == _lib.LMOE_EINVAL
    # too small a workspace is reported before any launch
    rc = lib.lmoe_moe_layer(ctypes.byref(L), 256, 4, 256, None, None, 256, 16, None)
    assert rc == _lib.LMOE_EWORKSPACE
    bad = _layer()
    bad.swiglu_mode = 7
    assert lib.lmoe_moe_layer(ctypes.byref(bad), 256, 4, 256, None, None, 256, 1 << 30, None) == \
        _lib.LMOE_EUNSUPPORTED


def test_strerror_and_version(built):
    lib = _lib.lmoe()
    assert lib.lmoe_version() == 2
    assert lib.lmoe_strerror(_lib.LMOE_EINDEX).decode().startswith("expert id")
    assert lib.lmoe_workspace_size_routes(8, 512, 256, 5) > 0


def test_tile_geometry(built):
    """Pre-tiled stream format: 16-row tiles of 8-group K chunks (codes +
    scales + biases, 128-byte padded), tiles paired, per slot in (pair, chunk)
    order."""
    lib = _lib.lmoe()
    # 2-bit g64, K=4096: chunks of 512 columns; a chunk tile holds codes
    # 16*128, scales and biases 16*16 each (2560 B), 8 chunks x 128 tiles
    assert lib.lmoe_tile_bytes(2048, 4096, 2, 64) == 128 * 8 * (16 * 128 + 2 * 16 * 16)
    # 4-bit g32, K=2048: chunks of 256 columns, same tile bytes
    assert lib.lmoe_tile_bytes(4096, 2048, 4, 32) == 256 * 8 * (16 * 128 + 2 * 16 * 16)
    # hidden 7168 at 2 bits: 14 chunks
    assert lib.lmoe_tile_bytes(2048, 7168, 2, 64) == 128 * 14 * (16 * 128 + 2 * 16 * 16)
    assert lib.lmoe_tile_bytes(16, 128, 2, 128) == 0       # K below one 8-group chunk; 16 rows are not a pair
    assert lib.lmoe_tile_bytes(2048, 4096, 3, 64) == 0     # bits not compiled
    assert lib.lmoe_tile_bytes(2040, 4096, 2, 64) == 0     # rows not a multiple of 32 (tile pairs)
    assert lib.lmoe_tile_bytes(2048, 3520, 2, 64) == 0     # K not a multiple of the 512-column chunk
    q = _lib.QProj(None, None, None, 2, 64, None)
    assert lib.lmoe_tile_pack(ctypes.byref(q), 1, 16, 256, 0, 1, None, None) == _lib.LMOE_EINVAL


def test_product_path_fails_loudly_without_cuda(built):
    import torch

    from locali_b200 import ops

    x = torch.zeros((1, 512), dtype=torch.bfloat16)
    slots = torch.zeros((1, 1), dtype=torch.int32)
    q = ops.QProjArrays(torch.zeros((2, 64, 32), dtype=torch.int32), torch.zeros((2, 64, 8), dtype=torch.bfloat16),
                        torch.zeros((2, 64, 8), dtype=torch.bfloat16), 2, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.gather_qmm(x, slots, q)


def test_prefill_path_selection(built):
    """Path choice and workspace sizing of lmoe_moe_layer_path (host logic)."""
    lib = _lib.lmoe()
    P = _lib.PATH
    L = _layer()  # hidden 1024, inter 512, 2-bit g64, 16 experts: both paths available
    ws = lambda layer, T, p: lib.lmoe_workspace_size_path(ctypes.byref(layer), T, P[p])  # noqa: E731
    dec, pre, auto = ws(L, 4096, "decode"), ws(L, 4096, "prefill"), ws(L, 4096, "auto")
    assert dec > 0 and pre > 0 and auto == max(dec, pre)
    assert lib.lmoe_workspace_size(ctypes.byref(L), 4096) == auto
    # below the AUTO threshold AUTO sizes the decode path
    assert not _lib.auto_takes_prefill(8, 6, 16)
    assert ws(L, 8, "auto") == ws(L, 8, "decode")
    # inter not a multiple of 128: no prefill path, AUTO falls back to decode
    odd = _layer(inter=320)
    assert ws(odd, 64, "prefill") == 0
    assert ws(odd, 4096, "auto") == ws(odd, 4096, "decode")
    big = 1 << 40
    rc = lib.lmoe_moe_layer_path(ctypes.byref(odd), 256, 4, 256, None, None, 256, big, None, P["prefill"], None, None)
    assert rc == _lib.LMOE_EUNSUPPORTED
    # code rows the decode GEMVs cannot stage (7168 x 2 bits: 112 16-byte
    # chunks; 8192: two stages do not fit): decode unavailable, AUTO = prefill
    for hidden in (7168, 8192):
        wide = _layer(hidden=hidden)
        assert ws(wide, 1, "decode") == 0
        assert ws(wide, 1, "auto") == ws(wide, 1, "prefill") > 0
    # unknown path value
    assert lib.lmoe_moe_layer_path(ctypes.byref(L), 256, 4, 256, None, None, 256, big, None, 9, None, None) == \
        _lib.LMOE_EUNSUPPORTED
    # the prefill workspace is checked before any launch
    small = ws(L, 512, "decode")
    assert ws(L, 512, "prefill") > small
    rc = lib.lmoe_moe_layer_path(ctypes.byref(L), 256, 512, 256, None, None, 256, small, None, P["prefill"], None,
                                 None)
    assert rc == _lib.LMOE_EWORKSPACE


def test_three_bit_layers_take_the_prefill_path(built):
    """3-bit projections have no decode GEMV: AUTO sizes (and takes) the
    prefill path at any token count; DECODE reports them unsupported."""
    lib = _lib.lmoe()
    P = _lib.PATH
    L3 = _layer(bits=3)
    ws = lambda layer, T, p: lib.lmoe_workspace_size_path(ctypes.byref(layer), T, P[p])  # noqa: E731
    assert ws(L3, 1, "decode") == 0
    assert ws(L3, 1, "auto") >= ws(L3, 1, "prefill") > 0
    big = 1 << 40
    rc = lib.lmoe_moe_layer_path(ctypes.byref(L3), 256, 1, 256, None, None, 256, big, None, P["decode"], None, None)
    assert rc == _lib.LMOE_EUNSUPPORTED
    assert lib.lmoe_tile_bytes(2048, 4096, 3, 64) == 0  # no tile layout for 3-bit rows


def test_auto_rule_mirror_matches_library(built):
    """_lib.auto_takes_prefill (used by tests and the bench) is the library's
    AUTO choice: AUTO sizes the decode layout below the threshold and the
    larger of both layouts from it on."""
    lib = _lib.lmoe()
    P = _lib.PATH
    for E in (16, 64, 256):
        L = _layer(E=E, k=6)
        for T in (1, 8, 42, 43, 64, 74, 75, 96, 300):
            dec = lib.lmoe_workspace_size_path(ctypes.byref(L), T, P["decode"])
            pre = lib.lmoe_workspace_size_path(ctypes.byref(L), T, P["prefill"])
            auto = lib.lmoe_workspace_size_path(ctypes.byref(L), T, P["auto"])
            want = max(dec, pre) if _lib.auto_takes_prefill(T, 6, E) else dec
            assert auto == want, (E, T)
