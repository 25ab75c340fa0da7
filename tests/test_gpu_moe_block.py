"""The whole MoE block on the GPU (router, gate/up/down VQ projections,
fused SwiGLU, fused slot combine) against the oracle's composition of the
same steps (router_topk, switch_fused, swiglu_bf16, combine_bf16 -- the
reference block of tests/test_qwen3_5_parity.py:180-204), each projection
restated in the reference arm the B200 kernel family reproduces."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import bf16_ulp
from vqlab_b200 import VQSwitchLinear
from vqlab_b200.moe import VQMoEBlock

pytestmark = pytest.mark.gpu

E, H, I, K, BITS, G, TOPK = 16, 512, 256, 4096, 12, 64, 4


def _proj(rng, out, inn):
    codes = rng.integers(0, K, (E, out, inn // 8)).astype(np.uint16)
    cb = (rng.standard_normal((K, 8)) * 0.02).astype(np.float16)
    sc = rng.uniform(0.5, 1.5, (E, out, inn // G)).astype(np.float16)
    return codes, orc.pack(codes, BITS), cb, sc


def _vq(p, inn):
    _, packed, cb, sc = p
    return VQSwitchLinear(torch.from_numpy(packed.view(np.int32)).cuda(), torch.from_numpy(cb).cuda(),
                          torch.from_numpy(sc).cuda(), group_size=G, pack_bits=BITS, in_features=inn)


@pytest.mark.parametrize("T", [3, 64, 300])  # decode kernel, decode kernel, grouped GEMM (> 512 pairs, 75/expert)
def test_moe_block_matches_oracle_composition(T):
    rng = np.random.default_rng(T)
    P = [_proj(rng, I, H), _proj(rng, I, H), _proj(rng, H, I)]
    blk = VQMoEBlock(_vq(P[0], H), _vq(P[1], H), _vq(P[2], I), TOPK)
    x = orc.round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    lg = rng.standard_normal((T, E)).astype(np.float32)
    y = blk(torch.from_numpy(x).cuda().to(torch.bfloat16), torch.from_numpy(lg).cuda()).float().cpu().numpy()

    idx, w = orc.router_topk(lg, TOPK)
    li = idx.reshape(-1)
    xh = orc.f16_bits(x)
    out = lambda a: orc.round_bf16(orc.round_f16(a))
    # each projection against the reference arm whose numerics the kernel family
    # it runs on implements: the walk (decode kernel), or gemmseg2 without ACCS
    # (the grouped GEMM: W = fp16(cb * s), fp32 accumulation)
    mode = lambda m, n, k: orc.MODE_PRESCALED if m.kernel_path(n, k) == "gemm" else orc.MODE_WALK
    mg, mu, md = mode(blk.gate_proj, T, TOPK), mode(blk.up_proj, T, TOPK), mode(blk.down_proj, T * TOPK, 1)
    g = out(orc.switch_fused(P[0][0], P[0][2].view(np.uint16), P[0][3].view(np.uint16), xh, li, TOPK, mode=mg))
    u = out(orc.switch_fused(P[1][0], P[1][2].view(np.uint16), P[1][3].view(np.uint16), xh, li, TOPK, mode=mu))
    h = orc.swiglu_bf16(g, u)
    d = out(orc.switch_fused(P[2][0], P[2][2].view(np.uint16), P[2][3].view(np.uint16), orc.f16_bits(h), li, 1,
                             mode=md))
    ref = orc.combine_bf16(d.reshape(T, TOPK, H), w)
    # The north-star bound on the block output, 2e-3 of its scale, plus one bf16
    # ULP of each value for the final rounding (the combine's fp32 sums of GPU
    # and oracle may straddle a bf16 boundary).  The earlier stages' roundings
    # (g, u, h, d in bf16) need no allowance of their own: a one-ULP difference
    # in a few of the 256 h values moves the down projection's sums by far less
    # than 2e-3 of their scale.
    lim = 2e-3 * np.abs(ref).max() + bf16_ulp(ref)
    assert np.all(np.abs(y - ref) <= lim), float(np.max(np.abs(y - ref) / lim))


@pytest.mark.parametrize("T,K_", [(5, 16384), (64, 16384), (300, 4096)])
def test_shared_workspace_is_identical_to_separate_calls(T, K_):
    """gate / up / down on one workspace (routing from gate, x gathered once,
    VQB_REUSE_*) give the same bytes as three independent calls."""
    from vqlab_b200.moe import expert_mlp, swiglu
    rng = np.random.default_rng(T + K_)
    bits = int(K_ - 1).bit_length()

    def proj(out, inn):
        codes = rng.integers(0, K_, (E, out, inn // 8)).astype(np.uint16)
        cb = (rng.standard_normal((K_, 8)) * 0.02).astype(np.float16)
        sc = rng.uniform(0.5, 1.5, (E, out, inn // G)).astype(np.float16)
        return VQSwitchLinear(torch.from_numpy(orc.pack(codes, bits).view(np.int32)).cuda(), torch.from_numpy(cb).cuda(),
                              torch.from_numpy(sc).cuda(), group_size=G, pack_bits=bits, in_features=inn)

    gp, up, dp = proj(I, H), proj(I, H), proj(H, I)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, H)).astype(np.float32)).cuda().to(torch.bfloat16)
    idx = torch.from_numpy(np.stack([rng.permutation(E)[:TOPK] for _ in range(T)]).astype(np.int32)).cuda()
    shared = expert_mlp(gp, up, dp, x, idx)
    separate = dp(swiglu(gp(x, idx), up(x, idx)), idx)
    assert torch.equal(shared.view(torch.int16), separate.view(torch.int16))
