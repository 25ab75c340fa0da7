"""The MoE block in one launch (vqb_moe_block_forward) against the oracle's
composition of the reference block (tests/test_qwen3_5_parity.py:180-204:
router_topk, the three projections, swiglu_bf16, combine_bf16), each
projection in the reference's non-ACCS arm (W = fp16(cb * s), fp32 sums --
oracle.MODE_PRESCALED, the weights the fused kernel builds), with the block
output bound of the north star, 2e-3 of the output's scale, plus one rounding
allowance for each of the two roundings that reach y with weight ~1: the final
one (one ULP of y) and the down projection's output (sum_j w_j * one ULP of
d_j -- the fused kernel sums the partials in another order than the oracle,
so a d value can round to the neighbouring bf16 value; the earlier stages' flips
move d by far less than its own ULP).  Also: the routing is bit-identical to vqb_moe_route, the
launch is one kernel, repeated calls are bit-identical, and shapes the fused
kernel does not serve take the per-step path."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import bf16_ulp
from vqlab_b200 import VQSwitchLinear, _lib
from vqlab_b200.moe import VQMoEBlock, route

pytestmark = pytest.mark.gpu

G = 64


def _proj(rng, E, out, inn, K):
    bits = int(K - 1).bit_length()
    codes = rng.integers(0, K, (E, out, inn // 8)).astype(np.uint16)
    cb = (rng.standard_normal((K, 8)) * 0.02).astype(np.float16)
    sc = rng.uniform(0.5, 1.5, (E, out, inn // G)).astype(np.float16)
    mod = VQSwitchLinear(torch.from_numpy(orc.pack(codes, bits).view(np.int32)).cuda(), torch.from_numpy(cb).cuda(),
                         torch.from_numpy(sc).cuda(), group_size=G, pack_bits=bits, in_features=inn)
    return (codes, cb, sc), mod


def _block(seed, E, H, I, K, topk, fused="on"):
    rng = np.random.default_rng(seed)
    P = [_proj(rng, E, I, H, K), _proj(rng, E, I, H, K), _proj(rng, E, H, I, K)]
    blk = VQMoEBlock(P[0][1], P[1][1], P[2][1], topk, fused=fused)
    return [p[0] for p in P], blk, rng


def _oracle_block(P, x_vals, lg, topk, x_f16=False):
    T = x_vals.shape[0]
    idx, w = orc.router_topk(lg, topk)
    li = idx.reshape(-1)
    xh = orc.f16_bits(x_vals)
    out = (lambda a: orc.round_f16(a)) if x_f16 else (lambda a: orc.round_bf16(orc.round_f16(a)))
    pres = orc.MODE_PRESCALED
    g = out(orc.switch_fused(P[0][0], P[0][1].view(np.uint16), P[0][2].view(np.uint16), xh, li, topk, mode=pres))
    u = out(orc.switch_fused(P[1][0], P[1][1].view(np.uint16), P[1][2].view(np.uint16), xh, li, topk, mode=pres))
    if x_f16:
        h = orc.round_f16(orc.silu(g) * u)
    else:
        h = orc.swiglu_bf16(g, u)
    d = out(orc.switch_fused(P[2][0], P[2][1].view(np.uint16), P[2][2].view(np.uint16), orc.f16_bits(h), li, 1,
                             mode=pres))
    dd = d.reshape(T, topk, -1)
    ulp = _f16_ulp if x_f16 else bf16_ulp
    d_allow = np.einsum("tj,tjh->th", w.astype(np.float64), ulp(dd))
    if x_f16:
        acc = np.zeros((T, d.shape[1]), np.float32)
        for j in range(topk):
            acc = (acc + (dd[:, j, :] * w[:, j:j + 1]).astype(np.float32)).astype(np.float32)
        return orc.round_f16(acc), idx, w, d_allow
    return orc.combine_bf16(dd, w), idx, w, d_allow


def _f16_ulp(v):
    v = np.abs(np.asarray(v, dtype=np.float64))
    return np.exp2(np.floor(np.log2(np.maximum(v, 2.0 ** -14))) - 10)


def _check(y, ref, d_allow, ulp=bf16_ulp):
    lim = 2e-3 * np.abs(ref).max() + ulp(ref) + d_allow
    assert np.all(np.abs(y - ref) <= lim), float(np.max(np.abs(y - ref) / lim))


@pytest.mark.parametrize("E,H,I,K,topk,T", [
    (16, 512, 512, 4096, 4, 1), (16, 512, 512, 4096, 4, 3), (16, 512, 512, 4096, 4, 8),
    (16, 512, 512, 4096, 4, 17), (16, 512, 512, 4096, 4, 64), (16, 512, 512, 4096, 4, 160),
    (8, 1024, 512, 16384, 2, 2), (8, 1024, 512, 16384, 2, 33),
])
def test_fused_block_matches_oracle(E, H, I, K, topk, T):
    P, blk, rng = _block(T * 7 + K, E, H, I, K, topk)
    assert blk.fused_status(T) == 0
    x = orc.round_bf16(rng.standard_normal((T, H)).astype(np.float32))
    lg = rng.standard_normal((T, E)).astype(np.float32)
    y, idx, w = blk.forward_fused(torch.from_numpy(x).cuda().to(torch.bfloat16), torch.from_numpy(lg).cuda())
    ref, ridx, rw, allow = _oracle_block(P, x, lg, topk)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    _check(y.float().cpu().numpy(), ref, allow)


@pytest.mark.parametrize("T", [1, 8, 64])
def test_fused_block_c2_shape(T):
    """BASELINE C2's layer: 512 experts, hidden 4096, intermediate 1024,
    d8 / K16384 / 14-bit codes, top-10, at decode batches 1, 8 and 64 (the
    headline: 640 pairs, the most the fused launch serves)."""
    P, blk, rng = _block(100 + T, 512, 4096, 1024, 16384, 10)
    x = orc.round_bf16(rng.standard_normal((T, 4096)).astype(np.float32))
    lg = rng.standard_normal((T, 512)).astype(np.float32)
    y, idx, _ = blk.forward_fused(torch.from_numpy(x).cuda().to(torch.bfloat16), torch.from_numpy(lg).cuda())
    ref, ridx, _, allow = _oracle_block(P, x, lg, 10)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    _check(y.float().cpu().numpy(), ref, allow)


def test_fused_block_fp16_x():
    P, blk, rng = _block(5, 16, 512, 512, 4096, 4)
    T = 6
    x = rng.standard_normal((T, 512)).astype(np.float16).astype(np.float32)
    lg = rng.standard_normal((T, 16)).astype(np.float32)
    y, _, _ = blk.forward_fused(torch.from_numpy(x).cuda().to(torch.float16), torch.from_numpy(lg).cuda())
    assert y.dtype == torch.float16
    ref, _, _, allow = _oracle_block(P, x, lg, 4, x_f16=True)
    _check(y.float().cpu().numpy(), ref, allow, ulp=_f16_ulp)


def test_fused_routing_is_the_router_kernels():
    """indices and weights bit-identical to vqb_moe_route on the same logits."""
    _, blk, rng = _block(9, 16, 512, 512, 4096, 4)
    T = 40
    x = torch.from_numpy(rng.standard_normal((T, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    lg = torch.from_numpy(rng.standard_normal((T, 16)).astype(np.float32)).cuda()
    lg[3, 5] = lg[3, 6]  # a tie: the lower expert id first
    _, idx, w = blk.forward_fused(x, lg)
    ridx, rw = route(lg, 4)
    assert torch.equal(idx, ridx) and torch.equal(w.view(torch.int32), rw.view(torch.int32))


def test_fused_block_one_launch_deterministic_status():
    _, blk, rng = _block(11, 16, 512, 512, 4096, 4)
    T = 12
    x = torch.from_numpy(rng.standard_normal((T, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    lg = torch.from_numpy(rng.standard_normal((T, 16)).astype(np.float32)).cuda()
    nb = int(_lib.lib().vqb_moe_block_workspace_size(ctypes.byref(blk.block_desc()), T))
    ws = torch.full((nb,), 0x5A, dtype=torch.uint8, device="cuda")  # stale status and partials
    y0 = blk(x, lg)  # builds the codebook halves once
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    y1, _, _ = blk.forward_fused(x, lg, workspace=ws)
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 1
    assert int(ws[:16].view(torch.int32)[1]) == 0
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))


def test_fused_block_close_to_per_step_path():
    P, blk, rng = _block(13, 16, 512, 512, 4096, 4, fused="auto")
    T = 20
    x = torch.from_numpy(rng.standard_normal((T, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    lg = torch.from_numpy(rng.standard_normal((T, 16)).astype(np.float32)).cuda()
    yf = blk(x, lg).float().cpu().numpy()
    blk.fused = "off"
    ys = blk(x, lg).float().cpu().numpy()
    lim = 4e-3 * np.abs(ys).max() + 2 * bf16_ulp(ys)
    assert np.all(np.abs(yf - ys) <= lim)


def test_unserved_shapes_take_the_per_step_path():
    """n_tokens * top_k > 640 (and 12-bit codes with K < 4096) are not fused:
    auto runs the per-step kernels, 'on' refuses."""
    _, blk, rng = _block(17, 16, 512, 512, 4096, 4, fused="auto")
    T = 161
    assert blk.fused_status(T) == _lib.VQB_UNSUPPORTED_GEOMETRY
    x = torch.from_numpy(rng.standard_normal((T, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    lg = torch.from_numpy(rng.standard_normal((T, 16)).astype(np.float32)).cuda()
    ya = blk(x, lg)
    blk.fused = "off"
    assert torch.equal(ya.view(torch.int16), blk(x, lg).view(torch.int16))
    blk.fused = "on"
    with pytest.raises(ValueError):
        blk(x, lg)
    _, blk2, _ = _block(18, 16, 512, 512, 3000, 4)
    assert blk2.fused_status(4) == _lib.VQB_UNSUPPORTED_GEOMETRY


def test_fused_block_bounded_wait_reports_timeout():
    """The failure path without a fault: one CTA waits for a signal nothing
    sends (vqb_moe_block_options.stall_cta) and gives up after 20 ms; the call
    ends, the status block reads VQB_TIMEOUT, and the next call on the same
    device is correct again (every CTA still arrived at every grid barrier)."""
    _, blk, rng = _block(23, 16, 512, 512, 4096, 4)
    T = 9
    x = torch.from_numpy(rng.standard_normal((T, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    lg = torch.from_numpy(rng.standard_normal((T, 16)).astype(np.float32)).cuda()
    good, _, _ = blk.forward_fused(x, lg)
    nb = int(_lib.lib().vqb_moe_block_workspace_size(ctypes.byref(blk.block_desc()), T))
    ws = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    opts = _lib.MoeBlockOptions(wait_limit_us=20000, stall_cta=5)
    blk.forward_fused(x, lg, workspace=ws, options=opts)
    torch.cuda.synchronize()
    assert int(ws[:16].view(torch.int32)[1]) == _lib.VQB_TIMEOUT
    again, _, _ = blk.forward_fused(x, lg, workspace=ws)
    torch.cuda.synchronize()
    assert int(ws[:16].view(torch.int32)[1]) == 0
    assert torch.equal(again.view(torch.int16), good.view(torch.int16))
