"""A small synthetic VQLab artifact (written with the repo's own safetensors
writer): one plain packed d8 switch layer, one SKIPZERO packed d4 switch
layer, one dense d2 layer (unpacked uint8 codes)."""
import json
import pathlib

import numpy as np
import torch

from oracle import oracle as orc
from vqlab_b200.artifact import write_safetensors

SW = "model.layers.0.mlp.switch_mlp.gate_proj"
SZ = "model.layers.0.mlp.switch_mlp.down_proj"
DN = "model.layers.0.self_attn.q_proj"


def make_artifact(root, seed=0):
    root = pathlib.Path(root)
    root.mkdir(parents=True, exist_ok=True)
    r = np.random.default_rng(seed)
    t, meta = {}, {}
    # packed d8 K4096 switch layer
    E, OUT, IN = 4, 96, 512
    c = r.integers(0, 4096, (E, OUT, IN // 8)).astype(np.uint16)
    t[SW + ".codes"] = torch.from_numpy(orc.pack(c, 12).view(np.int32))
    t[SW + ".codebook"] = torch.from_numpy((r.standard_normal((4096, 8)) * 0.02).astype(np.float16))
    t[SW + ".vq_scales"] = torch.from_numpy(r.uniform(0.5, 1.5, (E, OUT, IN // 64)).astype(np.float16))
    meta[SW] = {"experts": E, "out": OUT, "in": IN, "group": 64, "dim": 8, "k": 4096, "pack_bits": 12}
    # SKIPZERO packed d4 K2048 switch layer (live rows only + bit-packed mask)
    E2, OUT2, IN2 = 4, 40, 256
    c2 = r.integers(0, 2048, (E2, OUT2, IN2 // 4)).astype(np.uint16)
    s2 = r.uniform(0.5, 1.5, (E2, OUT2, IN2 // 64)).astype(np.float16)
    live = r.random((E2, OUT2)) < 0.6
    live[1] = False
    packed = orc.pack(c2, 11)
    t[SZ + ".sz_codes"] = torch.from_numpy(np.ascontiguousarray(packed[live]).view(np.int32))
    t[SZ + ".sz_scales"] = torch.from_numpy(np.ascontiguousarray(s2[live]))
    mask = np.packbits(np.pad(live, ((0, 0), (0, (-OUT2) % 8))), axis=1, bitorder="little")
    t[SZ + ".sz_rowmask"] = torch.from_numpy(mask)
    t[SZ + ".codebook"] = torch.from_numpy((r.standard_normal((2048, 4)) * 0.02).astype(np.float16))
    meta[SZ] = {"experts": E2, "out": OUT2, "in": IN2, "group": 64, "dim": 4, "k": 2048, "pack_bits": 11}
    # dense d2 K256, unpacked uint8
    OUT3, IN3 = 64, 256
    t[DN + ".codes"] = torch.from_numpy(r.integers(0, 256, (OUT3, IN3 // 2)).astype(np.uint8))
    t[DN + ".codebook"] = torch.from_numpy((r.standard_normal((256, 2)) * 0.02).astype(np.float16))
    t[DN + ".vq_scales"] = torch.from_numpy(r.uniform(0.5, 1.5, (OUT3, IN3 // 64)).astype(np.float16))
    dense = {DN: {"out": OUT3, "in": IN3, "group": 64, "dim": 2, "k": 256}}
    # two shards and an index
    keys = sorted(t)
    half = {k: t[k] for k in keys[: len(keys) // 2]}
    rest = {k: t[k] for k in keys[len(keys) // 2:]}
    write_safetensors(root / "model-00001-of-00002.safetensors", half)
    write_safetensors(root / "model-00002-of-00002.safetensors", rest)
    wm = {k: "model-00001-of-00002.safetensors" for k in half}
    wm.update({k: "model-00002-of-00002.safetensors" for k in rest})
    (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    (root / "config.json").write_text(json.dumps({"model_type": "qwen3_5_moe", "vq_modules": meta,
                                                  "vq_linear": dense}))
    return {"tensors": t, "live": live, "c2": c2, "s2": s2, "packed2": packed}
