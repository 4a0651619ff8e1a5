"""Generate the golden fixtures under tests/golden/ from the reference itself.

* ``ref_planner.json`` (CPU): plans recorded from the reference slot planner
  (native/locali_core.c, built into oracle/_ref/ by ``python -m
  oracle.build_ref``) over fixed and seeded-random operation sequences.
* ``ref_fused_swiglu.npz`` (GPU): outputs of the reference's own CUDA fused
  2-bit gate/up + clamped SwiGLU kernel (dsv4_kernels.py:100-173, built into
  oracle/_ref/libref_dsv4.so) on inputs regenerated from a seed by
  :func:`fused_inputs`; only the seeds, shapes and output bits are stored.

Usage: ``python -m tests.golden.make_golden planner`` (here) and
``python -m tests.golden.make_golden fused`` (on a GPU box).
"""

from __future__ import annotations

import ctypes
import json
import random
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF_DIR = ROOT / "oracle" / "_ref"


# ---------------------------------------------------------------- planner
def random_ops(seed: int, policy: str) -> dict:
    rng = random.Random(seed)
    slots = rng.choice([3, 5, 8, 12])
    prot = 0 if policy == "lfu-decay" else rng.randrange(0, slots - 1)
    keys = rng.choice([10, 24, 64])
    ops = []
    for _ in range(150):
        if policy == "lfu-decay" and rng.random() < 0.15:
            ops.append(["note"])
            continue
        n = rng.randrange(1, 4)
        plan_keys = [rng.randrange(keys) for _ in range(n)]
        pinned = rng.sample(range(0, slots + 1), rng.randrange(0, 3))
        ops.append(["plan", plan_keys, pinned, int(rng.random() < 0.85)])
    return {"name": f"{policy}-{seed}", "keys": keys, "slots": slots, "protected": prot, "policy": policy,
            "ops": ops}


def fixed_cases() -> list[dict]:
    seq = [0, 1, 2, 3, 0, 4, 5, 1, 6, 7, 2, 8, 0, 9, 3, 10]
    cases = []
    for prot in (0, 3):
        ops = [["plan", [k], [1] if i % 4 == 3 else [], 1] for i, k in enumerate(seq)]
        cases.append({"name": f"fixed-slru-{prot}", "keys": 64, "slots": 8, "protected": prot, "policy": "slru",
                      "ops": ops})
    cases.append({"name": "lfu-decay-basic", "keys": 16, "slots": 3, "protected": 0, "policy": "lfu-decay",
                  "ops": [["plan", [1], [], 1], ["plan", [1], [], 1], ["plan", [2], [], 1], ["plan", [3], [], 1]]
                  + [["note"]] * 16 + [["plan", [4], [], 1]]})
    return cases


def make_planner_golden() -> Path:
    sys.path.insert(0, str(ROOT))
    from locali_b200.native import NativeCache

    lib = REF_DIR / "liblocali_core_ref.so"
    if not lib.exists():
        raise SystemExit("build the reference core first: python -m oracle.build_ref")
    cases = fixed_cases() + [random_ops(s, p) for p in ("slru", "lfu-decay") for s in range(4)]
    for case in cases:
        c = NativeCache(case["keys"], case["slots"], case["protected"], policy=case["policy"], library=lib)
        expect = []
        for op in case["ops"]:
            if op[0] == "plan":
                _, keys, pinned, touch = op
                expect.append([[r.slot, int(r.hit), r.evicted_key, int(r.placed)]
                               for r in c.plan(keys, pinned_slots=pinned, touch_hits=bool(touch))])
                expect.append([c.probation_size, c.protected_size])
            else:
                c.note_token()
        case["expect"] = expect
        c.close()
    out = HERE / "ref_planner.json"
    out.write_text(json.dumps({"source": "reference native/locali_core.c", "cases": cases}))
    return out


# ---------------------------------------------------------------- fused kernel
FUSED_CASES = [
    # name, K, N, GS, top_k, dtype, n_slots, seed
    ("ref-test-geometry-f16", 256, 128, 128, 2, "f16", 4, 19),
    ("c0-width-g64-bf16", 1024, 512, 64, 6, "bf16", 9, 7),
    ("c0-width-g128-bf16", 1024, 512, 128, 6, "bf16", 9, 8),
    ("c0-width-g64-f16", 1024, 512, 64, 6, "f16", 9, 9),
]


def _round(a: np.ndarray, dtype: str) -> np.ndarray:
    sys.path.insert(0, str(ROOT))
    from oracle.moe_oracle import round_act

    return round_act(a, dtype)


def fused_inputs(K: int, N: int, GS: int, top_k: int, dtype: str, n_slots: int, seed: int) -> dict:
    """Deterministic inputs (numpy PCG64) for one fused-kernel case.

    Values follow the benchmark distributions: x N(0,1); codes uniform;
    scales |N(0,0.01)|; biases N(0,0.01); all rounded to ``dtype``.
    """
    rng = np.random.default_rng(seed)
    words = rng.integers(0, 2**32, size=(n_slots, N, K // 16), dtype=np.uint64).astype(np.uint32)
    scales = _round(np.abs(rng.standard_normal((n_slots, N, K // GS))) * 0.01, dtype)
    biases = _round(rng.standard_normal((n_slots, N, K // GS)) * 0.01, dtype)
    x = _round(rng.standard_normal((1, K)), dtype)
    slots = rng.choice(np.arange(1, n_slots), size=top_k, replace=False).astype(np.uint32)
    return {"wu": words, "su": scales, "bu": biases,
            "wg": rng.integers(0, 2**32, size=(n_slots, N, K // 16), dtype=np.uint64).astype(np.uint32),
            "sg": _round(np.abs(rng.standard_normal((n_slots, N, K // GS))) * 0.01, dtype),
            "bg": _round(rng.standard_normal((n_slots, N, K // GS)) * 0.01, dtype),
            "x": x, "slots": slots}


def run_reference_fused(inp: dict, K, N, GS, top_k, dtype) -> np.ndarray:
    """Run the reference CUDA kernel (oracle/_ref/libref_dsv4.so) on cuda:0."""
    import torch

    lib = ctypes.CDLL(str(REF_DIR / "libref_dsv4.so"))
    f = lib.ref_affine2_swiglu_launch
    f.restype = ctypes.c_int
    tdt = torch.float16 if dtype == "f16" else torch.bfloat16
    dev = torch.device("cuda", 0)

    def act(a):
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(tdt).to(dev)

    def u32(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(dev)

    t = {k: (u32(v) if k in ("wu", "wg", "slots") else act(v)) for k, v in inp.items()}
    out = torch.empty((top_k, N), dtype=tdt, device=dev)
    ptr = lambda v: ctypes.c_void_p(v.data_ptr())  # noqa: E731
    rc = f(K, N, GS, top_k, top_k, 10, int(dtype == "f16"), ptr(t["x"]), ptr(t["slots"]), ptr(t["wu"]),
           ptr(t["su"]), ptr(t["bu"]), ptr(t["wg"]), ptr(t["sg"]), ptr(t["bg"]), ptr(out),
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    if rc != 0:
        raise RuntimeError(f"reference kernel launch failed ({rc})")
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


def make_fused_golden() -> Path:
    rec = {}
    for name, K, N, GS, top_k, dtype, n_slots, seed in FUSED_CASES:
        inp = fused_inputs(K, N, GS, top_k, dtype, n_slots, seed)
        out = run_reference_fused(inp, K, N, GS, top_k, dtype)
        bits = out.astype(np.float16).view(np.uint16) if dtype == "f16" else \
            (out.view(np.uint32) >> 16).astype(np.uint16)
        rec[name] = bits
    meta = np.array(json.dumps([list(c) for c in FUSED_CASES]))
    out_path = HERE / "ref_fused_swiglu.npz"
    np.savez_compressed(out_path, meta=meta, **rec)
    return out_path


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "planner"
    if what == "planner":
        print(make_planner_golden())
    elif what == "fused":
        print(make_fused_golden())
    else:
        raise SystemExit("usage: make_golden.py planner|fused")
