"""Artifact loading on the host: the safetensors reader against a hand-built
file, a writer/reader round trip, and VQ layers built from a synthetic
artifact (plain, SKIPZERO and dense)."""
import json
import struct

import numpy as np
import torch

from artifact_cases import DN, SW, SZ, make_artifact
from vqlab_b200 import VQLinear, VQSwitchLinear
from vqlab_b200.artifact import Artifact, load_vq_layers, read_safetensors, write_safetensors


def test_reader_known_file(tmp_path):
    """A file laid out by hand from the format description."""
    hdr = {"b": {"dtype": "I32", "shape": [2], "data_offsets": [4, 12]},
           "a": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]}, "__metadata__": {"format": "pt"}}
    h = json.dumps(hdr).encode()
    data = np.array([1.5, -2.0], np.float16).tobytes() + np.array([7, -9], np.int32).tobytes()
    p = tmp_path / "x.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + data)
    t = read_safetensors(p)
    assert t["a"].dtype == torch.float16 and t["a"].tolist() == [1.5, -2.0]
    assert t["b"].dtype == torch.int32 and t["b"].tolist() == [7, -9]
    assert set(read_safetensors(p, ["b"])) == {"b"}


def test_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    t = {"f16": torch.randn((3, 5), generator=g).half(), "bf16": torch.randn((4,), generator=g).bfloat16(),
         "i32": torch.randint(-2 ** 31, 2 ** 31 - 1, (2, 3, 4), dtype=torch.int32, generator=g),
         "u8": torch.randint(0, 255, (7,), dtype=torch.uint8, generator=g), "empty": torch.zeros((0, 3))}
    write_safetensors(tmp_path / "r.safetensors", t, metadata={"k": "v"})
    back = read_safetensors(tmp_path / "r.safetensors")
    assert set(back) == set(t)
    for k in t:
        assert back[k].dtype == t[k].dtype and torch.equal(back[k], t[k])


def test_load_layers_host(tmp_path):
    case = make_artifact(tmp_path / "art")
    art = Artifact(tmp_path / "art")
    assert set(art.modules()) == {SW, SZ, DN}
    L = load_vq_layers(tmp_path / "art", device="cpu")
    sw, sz, dn = L[SW], L[SZ], L[DN]
    assert isinstance(sw, VQSwitchLinear) and isinstance(sz, VQSwitchLinear) and isinstance(dn, VQLinear)
    assert (sw.num_experts, sw.output_dims, sw.input_dims, sw.pack_bits, sw.skipzero) == (4, 96, 512, 12, False)
    assert (sz.num_experts, sz.output_dims, sz.input_dims, sz.pack_bits, sz.skipzero) == (4, 40, 256, 11, True)
    assert dn.pack_bits == 0 and dn.output_dims == 64 and dn.input_dims == 256
    live = case["live"]
    want = np.full(live.shape, -1, np.int32)
    want[live] = np.arange(int(live.sum()), dtype=np.int32)
    assert np.array_equal(sz.row_table.numpy(), want)
    assert torch.equal(sw.codes, case["tensors"][SW + ".codes"])
    assert sz.codes.shape[0] == int(live.sum())
