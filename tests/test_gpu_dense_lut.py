"""The small-codebook dense kernels: dense_lut_kernel (d2, K <= 256, 8-bit
codes, up to 8 rows -- the attention projections of benchmark configuration C4)
against the oracle's fused dense arm (vq_switch.py:2319-2327 restated by
oracle.switch_fused: x narrowed to fp16, fp32 group partials times the
group's scale, y rounded once to the output dtype).

Tolerance (written here, applied below): the kernel sums each group's
products in the MMA's order and a row block's split-K partials in split
order, so a bf16 / fp16 output is within 2e-3 * max|ref| + 1 ULP of the
oracle's (the north-star bound plus one output rounding step), an fp32
output within max relative error 2e-3 (the reference's metric,
tests/test_vq_prefill_paths.py:209-210); a repeated call is bit-identical.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import bf16_ulp, make_layer, max_rel, to_torch, within_tol_bf16
from vqlab_b200 import VQLinear, _lib

pytestmark = pytest.mark.gpu


def _lin(L):
    codes, cb, sc = to_torch(L)
    return VQLinear(codes[0], cb, sc[0], group_size=L.G, pack_bits=L.bits, in_features=L.IN)


def _ref(L, xv):
    return orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, orc.f16_bits(xv), np.zeros(xv.shape[0], np.uint32), 1)


def _ulp16(v):
    v = np.abs(np.asarray(v, dtype=np.float64))
    return np.exp2(np.floor(np.log2(np.maximum(v, 2.0 ** -14))) - 10)


def _x(rng, n, IN, dt):
    return torch.from_numpy(rng.standard_normal((n, IN)).astype(np.float32)).to(dt)


@pytest.mark.parametrize("OUT,IN,n", [(5120, 5120, 1), (5120, 5120, 8), (1024, 5120, 1), (1024, 5120, 5),
                                      (1000, 2048, 3), (256, 512, 8), (300, 1536, 2), (8192, 512, 4),
                                      (40000, 1024, 2)])
def test_lut_matches_oracle_bf16(OUT, IN, n):
    """C4's q / o (5120 x 5120) and k / v (1024 x 5120) projections at one and
    eight rows, a ragged last row block, one window per row (no split), and
    more row blocks than fit on the GPU at once."""
    L = make_layer(E=1, OUT=OUT, IN=IN, D=2, K=256, G=64, seed=OUT + IN + n)
    lin = _lin(L)
    rng = np.random.default_rng(n)
    xb = _x(rng, n, IN, torch.bfloat16)
    n0 = _lib.launch_count()
    y = lin(xb.cuda())
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 1, "one launch: no routing step"
    ref = orc.round_bf16(_ref(L, xb.float().numpy()))
    assert within_tol_bf16(ref, y.float().cpu().numpy())


@pytest.mark.parametrize("ydt", [torch.float16, torch.float32])
def test_lut_fp16_x_and_output_dtypes(ydt):
    L = make_layer(E=1, OUT=768, IN=3072, D=2, K=256, G=64, seed=5)
    lin = _lin(L)
    x = _x(np.random.default_rng(6), 7, 3072, torch.float16)
    y = lin(x.cuda(), out_dtype=ydt).float().cpu().numpy()
    ref = _ref(L, x.float().numpy())
    if ydt == torch.float32:
        assert max_rel(ref, y) <= 2e-3
    else:
        r16 = orc.round_f16(ref)
        assert np.all(np.abs(y - r16) <= 2e-3 * np.abs(r16).max() + _ulp16(r16))


@pytest.mark.parametrize("K", [2, 200, 256])
def test_lut_smaller_codebooks(K):
    """K < 256 stored as 8-bit codes (every code < K)."""
    L = make_layer(E=1, OUT=512, IN=1024, D=2, K=K, G=64, seed=K)
    if L.bits != 8:  # pack_bits follows K; an 8-bit store is what this kernel serves
        L = type(L)(L.E, L.OUT, L.IN, L.D, L.K, L.G, 8, L.codes, orc.pack(L.codes, 8), L.cb_bits, L.sc_bits)
    lin = _lin(L)
    xb = _x(np.random.default_rng(K + 1), 4, 1024, torch.bfloat16)
    y = lin(xb.cuda()).float().cpu().numpy()
    assert within_tol_bf16(orc.round_bf16(_ref(L, xb.float().numpy())), y)


def test_lut_repeatable_and_graph_replay():
    """Repeated eager calls and replays of one captured graph give the same bytes."""
    L = make_layer(E=1, OUT=5120, IN=5120, D=2, K=256, G=64, seed=9)
    lin = _lin(L)
    x = _x(np.random.default_rng(10), 2, 5120, torch.bfloat16).cuda()
    y0 = lin(x)
    y1 = lin(x)
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))
    out = torch.empty_like(y0)
    lin(x, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lin(x, out=out)
    for _ in range(5):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), y0.view(torch.int16))
    del g


@pytest.mark.parametrize("fill", [0x00, 0xFF])
def test_lut_status_block_through_the_c_abi(fill):
    """Through the C ABI with a workspace full of garbage: y is right and the
    status block's int32 [1] is 0 after the call."""
    L = make_layer(E=1, OUT=2048, IN=5120, D=2, K=256, G=64, seed=11)
    lin = _lin(L)
    n = 3
    xb = _x(np.random.default_rng(12), n, 5120, torch.bfloat16).cuda()
    y = torch.empty((n, 2048), dtype=torch.bfloat16, device="cuda")
    d = lin.desc()
    lib = _lib.lib()
    wsb = lib.vqb_dense_workspace_size(ctypes.byref(d), n, None)
    ws = torch.full((wsb,), fill, dtype=torch.uint8, device="cuda")
    st = lib.vqb_dense_forward(ctypes.byref(d), ctypes.c_void_p(xb.data_ptr()), _lib.VQB_BF16, n,
                               ctypes.c_void_p(y.data_ptr()), _lib.VQB_BF16, ctypes.c_void_p(ws.data_ptr()), wsb,
                               None, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    assert int(ws[4:8].view(torch.int32).item()) == 0
    ref = orc.round_bf16(_ref(L, xb.float().cpu().numpy()))
    assert within_tol_bf16(ref, y.float().cpu().numpy())


def test_lut_agrees_with_the_grouped_decode_kernel():
    """The explicit decode path (the grouped MMA kernel after the routing
    step) and AUTO (this kernel) compute the same fused-arm numerics: within
    two output roundings."""
    from vqlab_b200.vq_switch import make_options
    L = make_layer(E=1, OUT=1536, IN=4096, D=2, K=256, G=64, seed=13)
    a = _lin(L)
    b = _lin(L)
    b.options = make_options(path=_lib.PATH_DECODE)
    xb = _x(np.random.default_rng(14), 6, 4096, torch.bfloat16).cuda()
    ya = a(xb).float().cpu().numpy()
    yb = b(xb).float().cpu().numpy()
    assert np.all(np.abs(ya - yb) <= 4e-3 * np.abs(yb).max() + 2 * bf16_ulp(yb))


# ------------------------------------------------------------------ d8 variant
# dense_lut8_kernel: a d8 codebook of <= 4096 entries (C1: 4096 x 4096, K4096,
# 12-bit) at <= 8 rows, in the _decode_matmul arithmetic (vq_dense.py:267-312
# restated by oracle.dense_decode_matmul: W = fp16(cb * s), bf16 for bf16 x,
# fp32 accumulation, one rounding).  Same tolerance as above.

def _ref8(L, xv, bf16):
    return orc.dense_decode_matmul(L.codes[0], L.cb_bits, L.sc_bits[0], xv, wbf16=bf16)


@pytest.mark.parametrize("OUT,IN,K,n", [(4096, 4096, 4096, 1), (4096, 4096, 4096, 3), (4096, 4096, 4096, 8),
                                        (1000, 2048, 4096, 2), (512, 512, 4096, 5), (768, 1536, 1000, 4),
                                        (2048, 1024, 256, 7), (37888, 512, 4096, 2)])
def test_lut8_matches_oracle_bf16(OUT, IN, K, n):
    """C1's matvec at one, three and eight rows; a ragged last row block; one
    window per row (no split); 10-bit and 8-bit codebooks; 37888 rows of one
    window, where 256-row CTAs (148 of them) tie 128-row ones and are taken,
    while the other shapes take 128-row CTAs."""
    L = make_layer(E=1, OUT=OUT, IN=IN, D=8, K=K, G=64, seed=OUT + IN + K + n)
    lin = _lin(L)
    xb = _x(np.random.default_rng(n + 3), n, IN, torch.bfloat16)
    lin(xb.cuda())  # a d8 module's first call also builds its codebook halves (one more launch)
    torch.cuda.synchronize()
    n0 = _lib.launch_count()
    y = lin(xb.cuda())
    torch.cuda.synchronize()
    assert _lib.launch_count() - n0 == 1, "one launch: no routing step"
    ref = orc.round_bf16(_ref8(L, xb.float().numpy(), True))
    assert within_tol_bf16(ref, y.float().cpu().numpy())


@pytest.mark.parametrize("ydt", [torch.float16, torch.float32])
def test_lut8_fp16_x_and_output_dtypes(ydt):
    L = make_layer(E=1, OUT=1024, IN=2048, D=8, K=4096, G=64, seed=21)
    lin = _lin(L)
    x = _x(np.random.default_rng(22), 6, 2048, torch.float16)
    y = lin(x.cuda(), out_dtype=ydt).float().cpu().numpy()
    ref = _ref8(L, x.float().numpy(), False)
    if ydt == torch.float32:
        assert max_rel(ref, y) <= 2e-3
    else:
        r16 = orc.round_f16(ref)
        assert np.all(np.abs(y - r16) <= 2e-3 * np.abs(r16).max() + _ulp16(r16))


def test_lut8_repeatable_graph_replay_and_decode_path():
    """Repeated calls and graph replays give the same bytes; the explicit
    decode path (routing step + grouped MMA kernel) agrees within two output
    roundings."""
    from vqlab_b200.vq_switch import make_options
    L = make_layer(E=1, OUT=4096, IN=4096, D=8, K=4096, G=64, seed=23)
    lin = _lin(L)
    x = _x(np.random.default_rng(24), 2, 4096, torch.bfloat16).cuda()
    y0 = lin(x)
    assert torch.equal(y0.view(torch.int16), lin(x).view(torch.int16))
    out = torch.empty_like(y0)
    lin(x, out=out)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        lin(x, out=out)
    for _ in range(3):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), y0.view(torch.int16))
    del g
    b = _lin(L)
    b.options = make_options(path=_lib.PATH_DECODE)
    ya, yb = y0.float().cpu().numpy(), b(x).float().cpu().numpy()
    assert np.all(np.abs(ya - yb) <= 4e-3 * np.abs(yb).max() + 2 * bf16_ulp(yb))
