"""A dense model's VQ MLP in one launch (vqb_dense_mlp_forward, VQDenseMLP)
against the oracle's composition of the per-step calls: each projection is
vq_dense._decode_matmul (vq_dense.py:267-312: weights bf16(fp16(cb * s)) for
bf16 x, fp16 for fp16 x, fp32 accumulation, one rounding to x's dtype --
oracle.dense_decode_matmul), h = dtype(silu(g) * u) (oracle.swiglu_bf16).
The bound is 2e-3 of the output's scale plus one ULP of each value for the
final rounding: y is the down projection's rounded output, and the earlier
stages' one-ULP flips move its fp32 sums by far less than that."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import bf16_ulp
from vqlab_b200 import VQLinear, _lib
from vqlab_b200.mlp import FUSED_MAX_TOKENS, VQDenseMLP

pytestmark = pytest.mark.gpu

G = 64


def _lin(rng, out, inn, K):
    bits = int(K - 1).bit_length()
    codes = rng.integers(0, K, (out, inn // 8)).astype(np.uint16)
    cb = (rng.standard_normal((K, 8)) * 0.02).astype(np.float16)
    sc = rng.uniform(0.5, 1.5, (out, inn // G)).astype(np.float16)
    mod = VQLinear(torch.from_numpy(orc.pack(codes[None], bits)[0].view(np.int32)).cuda(),
                   torch.from_numpy(cb).cuda(), torch.from_numpy(sc).cuda(), group_size=G, pack_bits=bits,
                   in_features=inn)
    return (codes, cb, sc), mod


def _mlp(seed, H, I, K, fused="on"):
    rng = np.random.default_rng(seed)
    P = [_lin(rng, I, H, K), _lin(rng, I, H, K), _lin(rng, H, I, K)]
    return [p[0] for p in P], VQDenseMLP(P[0][1], P[1][1], P[2][1], fused=fused), rng


def _oracle(P, x_vals, bf16=True):
    rnd = orc.round_bf16 if bf16 else orc.round_f16
    proj = lambda p, v: rnd(orc.dense_decode_matmul(p[0], p[1].view(np.uint16), p[2].view(np.uint16), v,  # noqa: E731
                                                    wbf16=bf16))
    g, u = proj(P[0], x_vals), proj(P[1], x_vals)
    h = orc.swiglu_bf16(g, u) if bf16 else orc.round_f16(orc.silu(g) * u)
    return proj(P[2], h)


def _ulp16(v):
    v = np.abs(np.asarray(v, dtype=np.float64))
    return np.exp2(np.floor(np.log2(np.maximum(v, 2.0 ** -14))) - 10)


@pytest.mark.parametrize("H,I,K,T", [(512, 1024, 4096, 1), (512, 1024, 4096, 3), (512, 1024, 4096, 8),
                                     (1024, 512, 16384, 1), (1024, 512, 16384, 5), (512, 512, 4096, 40)])
def test_dense_mlp_matches_oracle(H, I, K, T):
    P, mlp, rng = _mlp(H + I + T, H, I, K)
    assert mlp.fused_status(T) == 0
    x = orc.round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    y = mlp.forward_fused(torch.from_numpy(x).cuda().to(torch.bfloat16)).float().cpu().numpy()
    ref = _oracle(P, x)
    lim = 2e-3 * np.abs(ref).max() + bf16_ulp(ref)
    assert np.all(np.abs(y - ref) <= lim), float(np.max(np.abs(y - ref) / lim))


def test_dense_mlp_c4_shape():
    """BASELINE C4's MLP: hidden 5120, intermediate 17408, d8 / K16384 / 14-bit, one token."""
    P, mlp, rng = _mlp(44, 5120, 17408, 16384)
    x = orc.round_bf16(rng.standard_normal((1, 5120)).astype(np.float32))
    y = mlp(torch.from_numpy(x).cuda().to(torch.bfloat16)).float().cpu().numpy()
    ref = _oracle(P, x)
    lim = 2e-3 * np.abs(ref).max() + bf16_ulp(ref)
    assert np.all(np.abs(y - ref) <= lim), float(np.max(np.abs(y - ref) / lim))


def test_dense_mlp_fp16_x():
    P, mlp, rng = _mlp(7, 512, 1024, 4096)
    x = rng.standard_normal((4, 512)).astype(np.float16).astype(np.float32)
    y = mlp.forward_fused(torch.from_numpy(x).cuda().to(torch.float16))
    assert y.dtype == torch.float16
    ref = _oracle(P, x, bf16=False)
    yv = y.float().cpu().numpy()
    assert np.all(np.abs(yv - ref) <= 2e-3 * np.abs(ref).max() + _ulp16(ref))


def test_dense_mlp_auto_path_one_launch_and_fallback():
    """auto: one launch up to FUSED_MAX_TOKENS rows (repeatable bytes, close to
    the per-step calls), the per-step calls above it (byte-equal to 'off')."""
    _, mlp, rng = _mlp(9, 512, 1024, 4096, fused="auto")
    x = torch.from_numpy(rng.standard_normal((FUSED_MAX_TOKENS, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    y0 = mlp(x)
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    y1 = mlp(x)
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 1
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))
    mlp.fused = "off"
    ys = mlp(x).float().cpu().numpy()
    lim = 4e-3 * np.abs(ys).max() + 2 * bf16_ulp(ys)
    assert np.all(np.abs(y1.float().cpu().numpy() - ys) <= lim)
    xb = torch.from_numpy(rng.standard_normal((FUSED_MAX_TOKENS + 1, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    mlp.fused = "auto"
    ya = mlp(xb)
    mlp.fused = "off"
    assert torch.equal(ya.view(torch.int16), mlp(xb).view(torch.int16))


def test_dense_mlp_refuses_switch_layers_and_bad_shapes():
    rng = np.random.default_rng(3)
    _, lin = _lin(rng, 1024, 512, 4096)
    mlp = VQDenseMLP(lin, lin, _lin(rng, 512, 1024, 4096)[1])
    assert mlp.fused_status(2) == 0
    assert mlp.fused_status(2, torch.float32) == _lib.VQB_UNSUPPORTED_GEOMETRY
    bad = VQDenseMLP(lin, lin, lin)  # down must be [H, I]
    assert bad.fused_status(2) == _lib.VQB_BAD_SHAPE
    d = mlp.mlp_desc()
    assert _lib.lib().vqb_dense_mlp_workspace_size(ctypes.byref(d), 2) > 0
