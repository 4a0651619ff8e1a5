"""Expert index (the reference's JSON format, dsv4_index.py:127-143) and an
expert-major pack writer.

Index records are ``[root, shard, offset, nbytes, shape, dtype]`` per
``L{layer}.E{expert}`` -> projection -> {weight, scales, biases}, with a
``tier`` per expert and per-tier quantisation.  :func:`build_index` reads the
safetensors headers of an MLX checkpoint (stacked ``[E, ...]`` switch_mlp
tensors, dsv4_index.py:63-143); :func:`write_pack` lays in-memory experts out
expert-major (every expert's nine arrays contiguous and 16 KiB aligned, the
property pack_experts.py gives the reference) so one read fills a slot.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import torch

from .arena import ARRS, DT_NAME, PROJS

DTSIZE = {"U8": 1, "I8": 1, "F16": 2, "BF16": 2, "U16": 2, "I16": 2, "U32": 4, "I32": 4, "F32": 4, "U64": 8,
          "I64": 8, "F64": 8}
ALIGN = 16384


def shard_header(path: Path) -> tuple[dict, int]:
    with Path(path).open("rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"invalid safetensors header: {path}")
        size = struct.unpack("<Q", raw)[0]
        header = json.loads(f.read(size))
    header.pop("__metadata__", None)
    return header, 8 + size


def build_index(snapshot) -> dict:
    snapshot = Path(snapshot).expanduser().resolve()
    config = json.loads((snapshot / "config.json").read_text())
    weights = json.loads((snapshot / "model.safetensors.index.json").read_text())["weight_map"]
    layers, experts, top_k = int(config["num_hidden_layers"]), int(config["n_routed_experts"]), \
        int(config["num_experts_per_tok"])
    quant = config.get("quantization_config", {})
    bits, group, mode = int(quant.get("bits", 2)), int(quant.get("group_size", 128)), quant.get("mode", "affine")
    if mode != "affine":
        raise ValueError(f"the arena requires affine MLX experts, checkpoint mode is {mode!r}")
    headers, entries, total = {}, {}, 0
    root = str(snapshot)
    for layer in range(layers):
        for proj in PROJS:
            for arr in ARRS:
                name = f"model.layers.{layer}.ffn.switch_mlp.{proj}.{arr}"
                if name not in weights:
                    raise ValueError(f"checkpoint is missing {name}")
                shard = weights[name]
                if shard not in headers:
                    headers[shard] = shard_header(snapshot / shard)
                header, start = headers[shard]
                meta = header[name]
                shape, dt = meta["shape"], meta["dtype"]
                if not shape or shape[0] != experts:
                    raise ValueError(f"{name}: expected first dimension {experts}, got {shape}")
                stride = DTSIZE[dt]
                for d in shape[1:]:
                    stride *= d
                base = start + meta["data_offsets"][0]
                for e in range(experts):
                    entries.setdefault(f"L{layer}.E{e}", {"tier": "cold"}).setdefault(proj, {})[arr] = \
                        [root, shard, base + e * stride, stride, shape[1:], dt]
                    total += stride
    return {"format": 1, "snapshot": root, "layers": layers, "num_experts": experts, "top_k": top_k,
            "quantization": {"cold": {"bits": bits, "group_size": group, "mode": mode}}, "expert_bytes": total,
            "experts": entries}


def write_pack(directory, experts_per_layer, top_k: int, tier: str = "cold") -> Path:
    """Write ``experts.bin`` + ``index.json`` for ``ops.ExpertArrays`` per layer
    (arrays ``[E + 1, ...]``, slot 0 is the zero slot and is not written)."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    data = d / "experts.bin"
    entries = {}
    off = 0
    E = int(experts_per_layer[0].gate.weight.shape[0]) - 1
    with data.open("wb") as f:
        for l, ex in enumerate(experts_per_layer):
            for e in range(E):
                pad = (-off) % ALIGN
                if pad:
                    f.write(b"\0" * pad)
                    off += pad
                rec = {"tier": tier}
                for p, q in zip(PROJS, (ex.gate, ex.up, ex.down)):
                    rec[p] = {}
                    for k, a in zip(ARRS, (q.weight, q.scales, q.biases)):
                        t = a[e + 1].contiguous().cpu()
                        raw = t.view(-1).view(torch.uint8).numpy().tobytes()
                        rec[p][k] = [str(d), data.name, off, len(raw), list(t.shape), DT_NAME[a.dtype]]
                        f.write(raw)
                        off += len(raw)
                entries[f"L{l}.E{e}"] = rec
    ex = experts_per_layer[0]
    idx = {"format": 1, "pack": True, "layers": len(experts_per_layer), "num_experts": E, "top_k": top_k,
           "quantization": {tier: {"bits": ex.gate.bits, "group_size": ex.gate.group_size, "mode": "affine"}},
           "experts": entries}
    out = d / "index.json"
    out.write_text(json.dumps(idx))
    return out
