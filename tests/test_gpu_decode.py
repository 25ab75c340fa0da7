"""Parity of the sm_100a decode kernel (through the C ABI) with the CPU oracle.

Tolerances (written here, applied below):
  * the per-pair kernel (decode_variant 1) at k_split 1 performs the
    reference walk's float operations in the reference's order (per-code dot,
    group partial, fma per group), so its result must be BIT-IDENTICAL to the
    oracle's restatement (vq_switch.py:1316-1392), NaN patterns included.
  * the tensor-core kernel (default) sums each group's products in the MMA's
    order: fp32-level max relative error (the reference's metric,
    max|a-b|/max|a|, tests/test_vq_prefill_paths.py:209-210) <= 2e-3, and a
    bf16 output within 2e-3*max|ref| + 1 bf16 ULP of the oracle's
    (the ULP admits one output rounding step).
"""
import pathlib

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import make_layer, max_rel, skewed_routing, to_torch, within_tol_bf16
from vqlab_b200 import VQLinear, VQSwitchLinear, vq_pack
from vqlab_b200.vq_switch import make_options

pytestmark = pytest.mark.gpu

GOLD = np.load(pathlib.Path(__file__).parent / "golden" / "vq_pack_golden.npz")


def _switch(L, ks=0, variant=0, stage=0):
    codes, cb, sc = to_torch(L)
    m = VQSwitchLinear(codes, cb, sc, group_size=L.G, pack_bits=L.bits, in_features=L.IN)
    if ks or variant or stage:
        m.options = make_options(k_split=ks, decode_variant=variant, stage_codebook=stage)
    return m


def _oracle_switch(L, x_vals, idx, krep, mode=orc.MODE_WALK):
    xh = orc.f16_bits(x_vals)
    return orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, xh, idx, krep, mode=mode)


@pytest.mark.parametrize("case", [str(c) for c in GOLD["cases"]])
def test_device_unpack_bit_exact(case):
    e, o, nsub, bits, wpr = (int(v) for v in GOLD[f"{case}__meta"])
    packed = torch.from_numpy(GOLD[f"{case}__packed"].view(np.int32)).cuda()
    got = vq_pack.unpack_device(packed, nsub, bits).cpu().numpy().astype(np.uint16)
    assert np.array_equal(got, GOLD[f"{case}__codes"])


GEOMS = [  # (D, K, IN, OUT, G)
    (8, 16384, 512, 96, 64),
    (8, 4096, 256, 64, 256),      # per-row scale (G = IN)
    (8, 1024, 640, 40, 64),       # NSUB 80: ragged tail block
    (8, 16384, 320, 33, 64),      # NSUB 40, OUT not a multiple of 32
    (4, 2048, 256, 64, 64),
    (4, 256, 512, 48, 64),
    (2, 256, 256, 64, 64),
    (2, 512, 128, 32, 64),
    # shapes the tensor-core kernel serves (IN % 512 == 0, G % 64 == 0 or G = IN)
    (8, 16384, 1024, 96, 64),
    (8, 4096, 1024, 64, 1024),    # per-row scale
    (8, 256, 512, 40, 64),        # OUT not a multiple of 16
    (8, 16384, 2048, 48, 128),
    (4, 2048, 512, 64, 64),
    (2, 256, 512, 64, 64),
    (2, 2048, 1024, 32, 64),      # 11-bit d2 codes
]


@pytest.mark.parametrize("D,K,IN,OUT,G", GEOMS)
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("variant,stage", [(1, 0)])
def test_switch_walk_bit_exact(D, K, IN, OUT, G, xdt, variant, stage):
    """The per-pair kernel repeats the reference walk exactly at k_split 1."""
    L = make_layer(E=6, OUT=OUT, IN=IN, D=D, K=K, G=G, seed=K + IN)
    T, k = 5, 3
    idx = skewed_routing(T, k, 6, seed=3)
    rng = np.random.default_rng(4)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, IN)).astype(np.float32)).to(xdt)
    m = _switch(L, ks=1, variant=variant, stage=stage)
    y = m(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda())
    assert y.shape == (T, k, 1, OUT) and y.dtype == xdt
    xv = x.float().numpy().reshape(T, IN)
    ref = orc.round_f16(_oracle_switch(L, xv, idx.reshape(-1), krep=k))
    got = y.float().cpu().numpy().reshape(T * k, OUT)
    if xdt == torch.float32 or xdt == torch.float16:
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    else:
        assert np.array_equal(got.view(np.uint32), orc.round_bf16(ref).view(np.uint32))


@pytest.mark.parametrize("D,K,IN,OUT,G", GEOMS)
@pytest.mark.parametrize("ks,stage", [(0, 0), (1, 1), (2, 2), (4, 0), (8, 1), (16, 0)])
def test_switch_split_within_tolerance(D, K, IN, OUT, G, ks, stage):
    L = make_layer(E=5, OUT=OUT, IN=IN, D=D, K=K, G=G, seed=7 + K)
    T, k = 4, 4
    idx = skewed_routing(T, k, 5, seed=5)
    rng = np.random.default_rng(8)
    xb = torch.from_numpy(rng.standard_normal((T, 1, 1, IN)).astype(np.float32)).to(torch.bfloat16)
    m = _switch(L, ks=ks, stage=stage)
    y = m(xb.cuda(), torch.from_numpy(idx).to(torch.int32).cuda()).float().cpu().numpy().reshape(T * k, OUT)
    ref32 = _oracle_switch(L, xb.float().numpy().reshape(T, IN), idx.reshape(-1), krep=k)
    ref = orc.round_bf16(orc.round_f16(ref32))
    assert within_tol_bf16(ref, y)
    # fp32-level: the f32 output carries only the fp16 rounding
    y32 = m(xb.float().cuda(), torch.from_numpy(idx).to(torch.int32).cuda()).cpu().numpy().reshape(T * k, OUT)
    assert max_rel(orc.round_f16(ref32), y32) <= 2e-3
    # and accuracy vs the float64 exact reconstruction is at least the oracle's
    ex = orc.exact_f64(L.codes, L.cb_bits, L.sc_bits, orc.f16_vals(orc.f16_bits(xb.float().numpy().reshape(T, IN))),
                       idx=idx.reshape(-1), krep=k)
    rms = lambda a: float(np.sqrt(np.mean((np.asarray(a, np.float64) - ex) ** 2)))
    assert rms(y32) <= 1.01 * rms(orc.round_f16(ref32)) + 1e-12


@pytest.mark.parametrize("T,k,E", [(16, 3, 4), (40, 8, 8), (7, 6, 2), (64, 10, 16)])
@pytest.mark.parametrize("ppc", [0, 1, 2, 4, 8, 16])
def test_switch_many_pairs_per_expert(T, k, E, ppc):
    """More pairs than experts: chunks of up to 16 pairs share each lookup
    (one or two MMA n-tiles); a hot expert spans several chunks."""
    L = make_layer(E=E, OUT=64, IN=512, D=8, K=16384, G=64, seed=T * k)
    idx = skewed_routing(T, k, E, seed=T)
    rng = np.random.default_rng(T)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, 512)).astype(np.float32)).to(torch.bfloat16)
    m = _switch(L, ks=1)
    m.options.pairs_per_chunk = ppc
    y = m(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy()
    ref = _oracle_switch(L, x.float().numpy().reshape(T, 512), idx.reshape(-1), krep=k)
    assert within_tol_bf16(orc.round_bf16(orc.round_f16(ref)), y.reshape(T * k, 64))
    y32 = m(x.float().cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).cpu().numpy().reshape(T * k, 64)
    assert max_rel(orc.round_f16(ref), y32) <= 2e-3


def test_bad_expert_index_is_reported_not_read():
    """An expert id >= E is reported in the workspace status block and computed
    as expert 0 (no out-of-range read); the module raises under
    VQB_CHECK_ROUTING=1."""
    import os
    L = make_layer(E=3, OUT=32, IN=128, D=8, K=256, G=64, seed=31)
    m = _switch(L)
    x = torch.randn((2, 1, 1, 128), device="cuda").to(torch.bfloat16)
    bad = torch.tensor([[0, 7], [1, 2]], dtype=torch.int32, device="cuda")
    os.environ["VQB_CHECK_ROUTING"] = "1"
    try:
        with pytest.raises(ValueError, match="out of range"):
            m(x, bad)
        m(x, torch.tensor([[0, 2], [1, 2]], dtype=torch.int32, device="cuda"))
    finally:
        del os.environ["VQB_CHECK_ROUTING"]


def test_switch_per_pair_x_and_unsorted_pairs():
    """x given per pair ([T, k, 1, IN], the SwitchGLU down_proj call shape)
    and a pair order that interleaves experts."""
    L = make_layer(E=4, OUT=64, IN=256, D=8, K=4096, G=64, seed=11)
    T, k = 3, 4
    idx = np.array([[3, 0, 3, 1], [2, 2, 0, 1], [1, 3, 0, 2]], dtype=np.int32)
    rng = np.random.default_rng(12)
    x = torch.from_numpy(rng.standard_normal((T, k, 1, 256)).astype(np.float32)).to(torch.float16)
    y = _switch(L, ks=1, variant=1)(x.cuda(), torch.from_numpy(idx).cuda()).float().cpu().numpy().reshape(T * k, 64)
    ref = orc.round_f16(_oracle_switch(L, x.float().numpy().reshape(T * k, 256), idx.reshape(-1).astype(np.uint32), 1))
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("K,dtype", [(256, np.uint8), (4096, np.uint16)])
def test_switch_unpacked_codes(K, dtype):
    """pack_bits == 0: plain uint8/uint16 codes (the BITS=0 arm the reference
    guards against reading row 0 everywhere, tests/test_vq_prefill_paths.py:215)."""
    L = make_layer(E=3, OUT=48, IN=256, D=4, K=K, G=64, packed=False, seed=13)
    assert L.packed.dtype == dtype
    T, k = 4, 2
    idx = skewed_routing(T, k, 3, seed=6)
    rng = np.random.default_rng(14)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, 256)).astype(np.float32))
    y = _switch(L, ks=1, variant=1)(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).cpu().numpy().reshape(T * k, 48)
    ref = orc.round_f16(_oracle_switch(L, x.numpy().reshape(T, 256), idx.reshape(-1), krep=k))
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))
    assert float(np.max(np.abs(y[0] - y[-1]))) > 0


def test_special_values_propagate_like_the_oracle():
    """Subnormal codebook entries, inf and NaN scales (tests/test_vq_wdec.py:148):
    compared as bit patterns, so NaN positions must agree too."""
    L = make_layer(E=2, OUT=32, IN=256, D=8, K=256, G=64, seed=15)
    cb = L.cb_bits.view(np.float16).copy()
    cb[:16] = np.float16(3e-6)            # fp16 subnormals
    L.cb_bits = cb.view(np.uint16)
    sc = L.sc_bits.view(np.float16).copy()
    sc[0, 3, 1] = np.float16(np.inf)
    sc[1, 5, 2] = np.float16(np.nan)
    sc[0, 7, 0] = np.float16(6e-8)        # subnormal scale
    L.sc_bits = sc.view(np.uint16)
    idx = np.array([[0, 1], [1, 0]], dtype=np.uint32)
    rng = np.random.default_rng(16)
    x = torch.from_numpy(rng.standard_normal((2, 1, 1, 256)).astype(np.float32))
    y = _switch(L, ks=1, variant=1)(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).cpu().numpy().reshape(4, 32)
    ref = orc.round_f16(_oracle_switch(L, x.numpy().reshape(2, 256), idx.reshape(-1), krep=2))
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(y[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_empty_and_single_pair():
    L = make_layer(E=2, OUT=32, IN=128, D=8, K=256, G=64, seed=17)
    m = _switch(L)
    x = torch.zeros((0, 1, 1, 128), dtype=torch.bfloat16, device="cuda")
    y = m(x, torch.zeros((0, 2), dtype=torch.int32, device="cuda"))
    assert y.shape == (0, 2, 1, 32)
    x1 = torch.randn((1, 1, 1, 128), device="cuda").to(torch.bfloat16)
    y1 = m(x1, torch.ones((1, 1), dtype=torch.int32, device="cuda"))
    assert y1.shape == (1, 1, 1, 32)


def test_c2_shapes_at_batch_1_and_8():
    """benchmark configuration C2 projection shapes (d8, K16384/14-bit, hidden 4096,
    intermediate 1024, top-10) on 16 experts, with the default auto split."""
    rng = np.random.default_rng(18)
    for OUT, IN in ((1024, 4096), (4096, 1024)):
        L = make_layer(E=16, OUT=OUT, IN=IN, D=8, K=16384, G=64, seed=OUT)
        m = _switch(L)
        for T in (1, 8):
            idx = np.stack([rng.choice(16, 10, replace=False) for _ in range(T)]).astype(np.uint32)
            xb = torch.from_numpy(rng.standard_normal((T, 1, 1, IN)).astype(np.float32)).to(torch.bfloat16)
            y = m(xb.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy().reshape(-1, OUT)
            ref = _oracle_switch(L, xb.float().numpy().reshape(T, IN), idx.reshape(-1), krep=10)
            assert within_tol_bf16(orc.round_bf16(orc.round_f16(ref)), y)


# ------------------------------------------------------------------ dense

def _dense_path_is_fused(D, packed, n):
    """vq_dense.py:94-102 / :401-441: fused only for d2/d4 at N <= cutoff."""
    maxn = 12 if not packed else {2: 72, 4: 32}.get(D, 0)
    return D != 8 and n <= maxn


def _dense(L, ks=0, variant=0):
    codes, cb, sc = to_torch(L)
    lin = VQLinear(codes[0], cb, sc[0], group_size=L.G, pack_bits=L.bits, in_features=L.IN)
    if ks or variant:
        lin.options = make_options(k_split=ks, decode_variant=variant)
    return lin


def _dense_oracle(L, xv, xdt, fused):
    if fused:
        return orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, orc.f16_bits(xv), np.zeros(xv.shape[0], np.uint32), 1)
    return orc.dense_decode_matmul(L.codes[0], L.cb_bits, L.sc_bits[0], xv, wbf16=(xdt == torch.bfloat16))


DENSE_GEOMS = [(8, 4096, 512, 128, 512), (8, 16384, 640, 64, 64), (2, 256, 512, 96, 64), (4, 4096, 256, 64, 64),
               (8, 4096, 1024, 96, 1024), (8, 16384, 1024, 64, 64), (2, 256, 1024, 80, 64)]


@pytest.mark.parametrize("D,K,IN,OUT,G", DENSE_GEOMS)
@pytest.mark.parametrize("n", [1, 3, 32, 80])
def test_dense_matches_reference_path(D, K, IN, OUT, G, n):
    L = make_layer(E=1, OUT=OUT, IN=IN, D=D, K=K, G=G, seed=19 + D)
    lin = _dense(L)
    rng = np.random.default_rng(20)
    xb = torch.from_numpy(rng.standard_normal((n, IN)).astype(np.float32)).to(torch.bfloat16)
    y = lin(xb.cuda()).float().cpu().numpy()
    xv = xb.float().numpy()
    fused = _dense_path_is_fused(D, True, n)
    ref = _dense_oracle(L, xv, torch.bfloat16, fused)
    assert within_tol_bf16(orc.round_bf16(ref), y)
    ex = orc.exact_f64(L.codes[0], L.cb_bits, L.sc_bits[0], xv)
    rms = lambda a: float(np.sqrt(np.mean((np.asarray(a, np.float64) - ex) ** 2)))
    assert rms(y) <= 1.01 * rms(orc.round_bf16(ref)) + 1e-12


@pytest.mark.parametrize("D,K,IN,OUT,G", DENSE_GEOMS)
@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n", [2, 100])
def test_dense_ks1_bit_exact(D, K, IN, OUT, G, xdt, n):
    """k_split 1: the fused arm repeats the walk order, the _decode_matmul arm
    the ascending-k GEMM order with exactly representable products, so both
    are bit-identical to the oracle before and after the output rounding."""
    L = make_layer(E=1, OUT=OUT, IN=IN, D=D, K=K, G=G, seed=21 + K)
    lin = _dense(L, ks=1, variant=1)
    rng = np.random.default_rng(22)
    x = torch.from_numpy(rng.standard_normal((n, IN)).astype(np.float32)).to(xdt)
    y = lin(x.cuda()).float().cpu().numpy()
    xv = x.float().numpy()
    ref = _dense_oracle(L, xv, xdt, _dense_path_is_fused(D, True, n))
    ref = orc.round_bf16(ref) if xdt == torch.bfloat16 else orc.round_f16(ref)
    assert np.array_equal(y.view(np.uint32), ref.view(np.uint32))


def test_dense_unpacked_cutoff_12():
    """Unpacked d2 codes: fused up to 12 rows, _decode_matmul above."""
    L = make_layer(E=1, OUT=64, IN=256, D=2, K=256, G=64, packed=False, seed=23)
    lin = _dense(L, ks=1, variant=1)
    rng = np.random.default_rng(24)
    for n in (12, 13):
        x = torch.from_numpy(rng.standard_normal((n, 256)).astype(np.float32)).to(torch.bfloat16)
        y = lin(x.cuda()).float().cpu().numpy()
        ref = orc.round_bf16(_dense_oracle(L, x.float().numpy(), torch.bfloat16, _dense_path_is_fused(2, False, n)))
        assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), n


@pytest.mark.parametrize("IN,OUT,n", [(5120, 17408, 1), (5120, 17408, 32), (17408, 5120, 1), (17408, 5120, 7)])
def test_dense_c4_mlp_shapes(IN, OUT, n):
    """benchmark configuration C4 MLP projections at full size (d8/K16384, 14-bit) on
    the grouped GEMM's dimension-split passes: 136 row tiles of 5120 k, and
    40 row tiles of 17408 k cut over three CTAs each (split-K)."""
    L = make_layer(E=1, OUT=OUT, IN=IN, D=8, K=16384, G=64, seed=IN + n)
    lin = _dense(L)
    rng = np.random.default_rng(n + 5)
    xb = torch.from_numpy(rng.standard_normal((n, IN)).astype(np.float32)).to(torch.bfloat16)
    y = lin(xb.cuda()).float().cpu().numpy()
    ref = _dense_oracle(L, xb.float().numpy(), torch.bfloat16, fused=False)
    assert within_tol_bf16(orc.round_bf16(ref), y)
