"""The artifact loader against the reference's own writer fixtures.

tests/golden/writer_artifacts.json holds the VQ-layer part of three artifacts
the reference's writers produced (its tests/golden/writers/{pack,
pack_straddle,sz_pack}.json; extracted by tests/golden/make_golden.py): the
config.json `vq_modules` / `vq_skipzero` blocks and the dtype, shape and
shard of every tensor of those layers.  The weights themselves are not in the
fixture (only their hashes), so each test lays out an artifact directory with
exactly those keys, dtypes, shapes and shard files, filled with seeded values,
and loads it through `vqlab_b200.artifact` -- the config reader of
src/vqlab/bundle/add_model_file.py:70-131 restated.  On the GPU the loaded
layers are run and compared with the oracle.
"""
import json
import pathlib

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import max_rel
from vqlab_b200 import VQSwitchLinear
from vqlab_b200.artifact import Artifact, load_vq_layers, write_safetensors

FIX = json.loads((pathlib.Path(__file__).parent / "golden" / "writer_artifacts.json").read_text())
_NP = {"U8": np.uint8, "U32": np.uint32, "F16": np.float16, "I32": np.int32}


def _fill(key, meta, cfg, rng):
    """Seeded values for one fixture tensor, consistent with its layer's config."""
    shape, dt = tuple(meta["shape"]), meta["dtype"]
    prefix = key.rsplit(".", 1)[0]
    mod = (cfg.get("vq_modules") or {}).get(prefix, {})
    k = int(mod.get("k", 16))
    if key.endswith(".sz_rowmask"):
        szm = cfg["vq_skipzero"]["modules"][prefix]
        E, OUT = int(szm["experts"]), int(szm["out"])
        live = np.ones(E * OUT, bool)
        live[rng.choice(E * OUT, size=int(szm["dead_rows"]), replace=False)] = False
        bits = np.zeros((E, shape[1] * 8), np.uint8)
        bits[:, :OUT] = live.reshape(E, OUT)
        return np.packbits(bits.reshape(E, -1, 8), axis=-1, bitorder="little").reshape(shape)
    if key.endswith(".sz_shape"):
        return np.zeros(shape, np.int32)
    if dt == "F16":
        if key.endswith("scales"):
            return rng.uniform(0.5, 1.5, shape).astype(np.float16)
        return (rng.standard_normal(shape) * 0.05).astype(np.float16)
    if dt == "U32":  # packed words: uniform codes when K = 2^bits and NSUB % 32 == 0
        return rng.integers(0, 2 ** 32, shape, dtype=np.uint32)
    return rng.integers(0, k, shape).astype(_NP[dt])


def _build(root: pathlib.Path, name: str, seed=0):
    fx = FIX[name]
    rng = np.random.default_rng(seed)
    root.mkdir(parents=True)
    (root / "config.json").write_text(json.dumps(fx["config"]))
    shards, arrays = {}, {}
    for key, meta in sorted(fx["tensors"].items()):
        arrays[key] = _fill(key, meta, fx["config"], rng)
        shards.setdefault(meta["shard"], {})[key] = torch.from_numpy(arrays[key])
    for shard, tensors in shards.items():
        write_safetensors(root / shard, tensors)
    (root / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {k: m["shard"] for k, m in fx["tensors"].items()}}))
    return fx, arrays


@pytest.mark.parametrize("name", sorted(FIX))
def test_loader_reads_reference_writer_layout(tmp_path, name):
    fx, arrays = _build(tmp_path / name, name)
    cfg = fx["config"]
    art = Artifact(tmp_path / name)
    assert set(art.modules()) == set(cfg["vq_modules"])
    layers = load_vq_layers(tmp_path / name, device="cpu")
    sz_mods = (cfg.get("vq_skipzero") or {}).get("modules") or {}
    for p, m in cfg["vq_modules"].items():
        L = layers[p]
        assert isinstance(L, VQSwitchLinear)
        assert (L.num_experts, L.output_dims, L.input_dims) == (m["experts"], m["out"], m["in"])
        assert tuple(L.codebook.shape) == (m["k"], m["dim"]) and L.group_size == m["group"]
        assert L.pack_bits == int(m.get("pack_bits", 0))
        if p in sz_mods:
            s = sz_mods[p]
            assert L.skipzero and tuple(L.row_table.shape) == (s["experts"], s["out"])
            nlive = int((L.row_table >= 0).sum())
            assert nlive == s["live_rows"] == L.codes.shape[0] and int((L.row_table < 0).sum()) == s["dead_rows"]
            assert np.array_equal(L.codes.numpy().view(np.uint8), arrays[p + ".sz_codes"])
        else:
            assert not L.skipzero
            assert np.array_equal(L.codes.numpy().view(arrays[p + ".codes"].dtype), arrays[p + ".codes"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(FIX))
def test_loaded_reference_layout_matches_oracle(tmp_path, name):
    """Each loaded layer on the GPU against the oracle (walk order, fp32 output
    with the fp16 output rounding): max relative error <= 2e-3."""
    fx, arrays = _build(tmp_path / name, name, seed=1)
    layers = load_vq_layers(tmp_path / name, device="cuda")
    rng = np.random.default_rng(2)
    for p, m in fx["config"]["vq_modules"].items():
        L = layers[p]
        T, k, IN = 3, 2, int(m["in"])
        x = rng.standard_normal((T, 1, 1, IN)).astype(np.float16)
        idx = rng.integers(0, int(m["experts"]), (T, k)).astype(np.int32)
        y = L(torch.from_numpy(x).cuda(), torch.from_numpy(idx).cuda(), out_dtype=torch.float32)
        y = y.cpu().numpy().reshape(T * k, -1)
        nsub = IN // int(m["dim"])
        cb = arrays[p + ".codebook"].view(np.uint16)
        xh = x.reshape(T, IN).view(np.uint16)
        if L.skipzero:
            codes = arrays[p + ".sz_codes"].astype(np.uint16)
            ref = orc.switch_fused_rowtable(codes, cb, arrays[p + ".sz_scales"].view(np.uint16), xh,
                                            idx.reshape(-1).astype(np.uint32), k, L.row_table.cpu().numpy())
        else:
            c = arrays[p + ".codes"]
            codes = orc.unpack(c, nsub, L.pack_bits) if L.pack_bits else c.astype(np.uint16)
            ref = orc.switch_fused(codes, cb, arrays[p + ".vq_scales"].view(np.uint16), xh,
                                   idx.reshape(-1).astype(np.uint32), k)
        assert max_rel(orc.round_f16(ref), y) <= 2e-3, p
