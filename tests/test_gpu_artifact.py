"""Layers loaded from an artifact compute exactly what modules built from the
same tensors compute (plain and SKIPZERO switch layers, a dense layer)."""
import numpy as np
import pytest
import torch

from artifact_cases import DN, SW, SZ, make_artifact
from vqlab_b200 import VQLinear, VQSwitchLinear
from vqlab_b200.artifact import load_vq_layers

pytestmark = pytest.mark.gpu


def test_loaded_layers_match_direct_modules(tmp_path):
    case = make_artifact(tmp_path / "art")
    t = {k: v.cuda() for k, v in case["tensors"].items()}
    L = load_vq_layers(tmp_path / "art")
    rng = np.random.default_rng(3)
    idx = torch.from_numpy(rng.integers(0, 4, (6, 2)).astype(np.int32)).cuda()
    x = torch.from_numpy(rng.standard_normal((6, 1, 1, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    direct = VQSwitchLinear(t[SW + ".codes"], t[SW + ".codebook"], t[SW + ".vq_scales"], group_size=64, pack_bits=12,
                            in_features=512)
    assert torch.equal(L[SW](x, idx), direct(x, idx))
    # SKIPZERO layer vs the expanded layout (dead rows code 0, scale +0)
    live, c2, s2 = case["live"], case["c2"].copy(), case["s2"].copy()
    c2[~live] = 0
    s2[~live] = 0
    from oracle import oracle as orc
    exp = VQSwitchLinear(torch.from_numpy(orc.pack(c2, 11).view(np.int32)).cuda(), t[SZ + ".codebook"],
                         torch.from_numpy(s2).cuda(), group_size=64, pack_bits=11, in_features=256)
    x2 = torch.from_numpy(rng.standard_normal((6, 1, 1, 256)).astype(np.float32)).cuda().to(torch.bfloat16)
    assert torch.equal(L[SZ](x2, idx).view(torch.int16), exp(x2, idx).view(torch.int16))
    xd = torch.from_numpy(rng.standard_normal((3, 256)).astype(np.float32)).cuda().to(torch.bfloat16)
    dd = VQLinear(t[DN + ".codes"], t[DN + ".codebook"], t[DN + ".vq_scales"], group_size=64)
    assert torch.equal(L[DN](xd), dd(xd))
