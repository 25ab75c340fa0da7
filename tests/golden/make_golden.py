"""Generate the golden fixtures in this directory from the reference itself.

Run in a container where the VQLab reference checkout is available (pass its
root as the first argument, or set VQLAB_REF).  It is NOT run by the tests:
the tests read the committed .npz files, so they also work where the
reference is absent (the GPU boxes).

  vq_pack_golden.npz  -- pack/unpack vectors produced by the reference's own
                         numpy writer/reader src/vqlab/runtime/vq_pack.py
                         (pack :48-76, unpack :79-97, words_per_row :41-45),
                         bit widths 1..16, aligned and ragged NSUB, and the
                         benchmark geometries (14-bit NSUB 512/128, 12-bit
                         NSUB 512, 8-bit NSUB 2560, ragged 14-bit NSUB 80).
  moe_block_golden.npz -- the reference's float64 numpy MoE block
                         `ref_moe` (tests/test_qwen3_5_parity.py:180-204) on a
                         tiny dense model, shared expert zeroed so only the
                         router/top-k/renormalise/SwiGLU/combine remain.
  writer_artifacts.json -- the VQ-layer part of the reference's writer
                         fixtures tests/golden/writers/{pack,pack_straddle,
                         sz_pack}.json (artifacts its own writers produced):
                         config.json `vq_modules` / `vq_skipzero`, and the
                         dtype, shape and shard of every tensor of those
                         layers (the loader's input contract,
                         src/vqlab/bundle/add_model_file.py:70-131).

vq_pack.py imports only numpy, so it is loaded straight from its file; the
parity test module imports mlx at the top, so its four numpy functions are
taken out with `ast` and executed alone.
"""
from __future__ import annotations

import ast
import importlib.util
import os
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def _load_vq_pack(ref: pathlib.Path):
    path = ref / "src" / "vqlab" / "runtime" / "vq_pack.py"
    spec = importlib.util.spec_from_file_location("ref_vq_pack", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _load_ref_moe(ref: pathlib.Path):
    path = ref / "tests" / "test_qwen3_5_parity.py"
    tree = ast.parse(path.read_text())
    keep = {"_silu", "_sigmoid", "ref_mlp", "ref_moe"}
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in keep]
    assert {n.name for n in body} == keep, "reference MoE helpers moved"
    ns = {"np": np}
    exec(compile(ast.Module(body=body, type_ignores=[]), str(path), "exec"), ns)
    return ns["ref_moe"]


def make_pack(vq_pack) -> dict:
    rng = np.random.default_rng(20261201)
    out = {}
    cases = []
    for bits in range(1, 17):
        for nsub in (32, 64, 40, 80, 7):
            cases.append((f"b{bits}_n{nsub}", 2, 3, nsub, bits))
    cases += [("c2_gateup", 1, 4, 512, 14), ("c2_down", 1, 4, 128, 14),
              ("c1", 1, 4, 512, 12), ("c4_attn", 1, 2, 2560, 8),
              ("ragged80_b14", 2, 3, 80, 14), ("c4_mlp_down", 1, 2, 2176, 14)]
    names = []
    for name, e, o, nsub, bits in cases:
        codes = rng.integers(0, 1 << bits, (e, o, nsub)).astype(np.uint16)
        packed = vq_pack.pack(codes, bits)
        assert packed.shape[-1] == vq_pack.words_per_row(nsub, bits)
        back = vq_pack.unpack(packed, nsub, bits)
        assert np.array_equal(back.astype(np.uint16), codes)
        out[f"{name}__codes"] = codes
        out[f"{name}__packed"] = packed
        out[f"{name}__meta"] = np.array([e, o, nsub, bits, vq_pack.words_per_row(nsub, bits)],
                                        dtype=np.int64)
        names.append(name)
    out["cases"] = np.array(names)
    out["bits_for_k"] = np.array([[k, vq_pack.bits_for_k(k)] for k in
                                  (2, 4, 16, 256, 512, 1024, 2048, 4096, 8192, 16384, 65536)],
                                 dtype=np.int64)
    return out


def make_moe(ref_moe) -> dict:
    rng = np.random.default_rng(7)
    T, D, E, I, k = 6, 64, 8, 32, 3
    x = rng.standard_normal((T, D))
    p = {
        "gate.weight": rng.standard_normal((E, D)) * 0.3,
        "experts.gate_up_proj": rng.standard_normal((E, 2 * I, D)) * 0.1,
        "experts.down_proj": rng.standard_normal((E, D, I)) * 0.1,
        "shared_expert.gate_proj.weight": np.zeros((I, D)),
        "shared_expert.up_proj.weight": np.zeros((I, D)),
        "shared_expert.down_proj.weight": np.zeros((D, I)),
        "shared_expert_gate.weight": np.zeros((1, D)),
    }
    y = ref_moe(x, p, {"num_experts_per_tok": k})
    return {"x": x, "router": p["gate.weight"], "gate_up": p["experts.gate_up_proj"],
            "down": p["experts.down_proj"], "k": np.array(k), "y": y}


def make_writer_artifacts(ref: pathlib.Path) -> dict:
    import json
    out = {}
    for name in ("pack", "pack_straddle", "sz_pack"):
        fx = json.loads((ref / "tests" / "golden" / "writers" / f"{name}.json").read_text())
        cfg = fx["config"]
        prefixes = set(cfg.get("vq_modules") or {})
        sz = cfg.get("vq_skipzero")
        if sz:
            prefixes |= set(sz.get("modules") or {})
        tensors = {k: {"dtype": v["dtype"], "shape": v["shape"], "shard": v["shard"]}
                   for k, v in fx["tensors"].items() if any(k.startswith(p + ".") for p in prefixes)}
        keep = {k: cfg[k] for k in ("vq_modules", "vq_skipzero") if k in cfg}
        if "vq_skipzero" in keep:
            keep["vq_skipzero"] = {"format": sz.get("format"), "version": sz.get("version"),
                                   "modules": sz.get("modules")}
        out[name] = {"config": keep, "tensors": tensors}
    return out


def main(argv) -> int:
    ref = pathlib.Path(argv[1] if len(argv) > 1 else os.environ.get("VQLAB_REF", ""))
    if not (ref / "src" / "vqlab" / "runtime" / "vq_pack.py").exists():
        print("usage: make_golden.py <VQLab checkout>", file=sys.stderr)
        return 2
    np.savez_compressed(HERE / "vq_pack_golden.npz", **make_pack(_load_vq_pack(ref)))
    np.savez_compressed(HERE / "moe_block_golden.npz", **make_moe(_load_ref_moe(ref)))
    import json
    (HERE / "writer_artifacts.json").write_text(json.dumps(make_writer_artifacts(ref), indent=1, sort_keys=True) + "\n")
    print("wrote", HERE / "vq_pack_golden.npz", HERE / "moe_block_golden.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
