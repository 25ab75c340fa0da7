"""Self-consistency of the CPU oracle's matmul restatements and the MoE block.

The restated kernels are checked against the float64 exact reconstruction
(score/kernel_truth_moe.py:37-50) and against each other; the MoE block
restatement is checked against the reference's own float64 numpy MoE block
(`ref_moe`, tests/test_qwen3_5_parity.py:180-204) through the golden file."""
import pathlib

import numpy as np
import pytest

from oracle import oracle as orc
from vq_cases import make_layer, max_rel

GM = np.load(pathlib.Path(__file__).parent / "golden" / "moe_block_golden.npz")


def test_moe_block_restatement_matches_reference_ref_moe():
    x, router, gu, dn, k, y_ref = (GM[n] for n in ("x", "router", "gate_up", "down", "k", "y"))
    k = int(k)
    logits = x @ router.T
    idx, w = orc.router_topk(logits.astype(np.float32), k)
    # the same composition in float64 with the oracle's routing decisions
    I = gu.shape[1] // 2
    y = np.zeros_like(x)
    for t in range(x.shape[0]):
        for j in range(k):
            e = idx[t, j]
            h = gu[e] @ x[t]
            a = h[:I] / (1.0 + np.exp(-h[:I])) * h[I:]
            y[t] += float(w[t, j]) * (dn[e] @ a)
    assert np.max(np.abs(y - y_ref)) <= 1e-5 * np.max(np.abs(y_ref))


@pytest.mark.parametrize("D,K,IN,G", [(8, 4096, 512, 64), (8, 16384, 256, 256), (4, 256, 256, 64),
                                      (2, 256, 256, 64), (8, 1024, 640, 64)])
@pytest.mark.parametrize("mode", [orc.MODE_WALK, orc.MODE_SS])
def test_fused_restatement_close_to_exact(D, K, IN, G, mode):
    L = make_layer(E=3, OUT=40, IN=IN, D=D, K=K, G=G, seed=D + K)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((4, IN)).astype(np.float32)
    xh = orc.f16_bits(x)
    idx = np.array([0, 2, 1, 1, 0, 2, 2, 0], dtype=np.uint32)
    y32 = orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, xh, idx, krep=2, mode=mode)
    ex = orc.exact_f64(L.codes, L.cb_bits, L.sc_bits, orc.f16_vals(xh), idx=idx, krep=2)
    assert max_rel(ex, y32) < 1e-5
    # packed reader gives the identical accumulators
    yp = orc.switch_fused(L.packed, L.cb_bits, L.sc_bits, xh, idx, krep=2, mode=mode, packed_bits=L.bits)
    assert np.array_equal(y32.view(np.uint32), yp.view(np.uint32))


def test_decode_matmul_restatement():
    L = make_layer(E=1, OUT=64, IN=512, D=8, K=4096, G=512, seed=3)
    rng = np.random.default_rng(2)
    xb = orc.round_bf16(rng.standard_normal((2, 512)).astype(np.float32))
    y = orc.dense_decode_matmul(L.codes[0], L.cb_bits, L.sc_bits[0], xb, wbf16=True)
    ex = orc.exact_f64(L.codes[0], L.cb_bits, L.sc_bits[0], xb)
    # the bf16 weight rounding of vq_dense.py:294 costs ~2^-9 relative per weight
    assert max_rel(ex, y) < 4e-3
    y16 = orc.dense_decode_matmul(L.codes[0], L.cb_bits, L.sc_bits[0], xb, wbf16=False)
    assert max_rel(ex, y16) < 1e-3


def test_rounding_helpers():
    v = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9, -2.5, 65504.0, 1e-40], dtype=np.float32)
    b = orc.bf16_vals(orc.bf16_bits(v))
    assert b[0] == 1.0 and b[1] == 1.0  # tie to even
    assert b[2] == np.float32(1.0 + 2 ** -7)
    assert b[3] == -2.5
    nan = orc.bf16_vals(orc.bf16_bits(np.array([np.nan], dtype=np.float32)))
    assert np.isnan(nan[0])


def test_router_topk_renormalised_and_tie_order():
    lg = np.array([[0.0, 1.0, 1.0, -1.0]], dtype=np.float32)
    idx, w = orc.router_topk(lg, 2)
    assert idx.tolist() == [[1, 2]]
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_rowtable_restatement_equals_expanded_layout():
    """oracle.switch_fused_rowtable on compact live rows is bit-identical to
    switch_fused on the expanded layout (dead rows: code 0, scale +0, whose walk
    gives fma(+0, gacc, +0) = +0), the reference's own SKIPZERO claim
    (tests/test_vq_skipzero.py:83-113); an out-of-table compact index is dead."""
    r = np.random.default_rng(5)
    E, OUT, IN, D, K, G = 4, 24, 128, 8, 512, 64
    codes = r.integers(0, K, (E, OUT, IN // D)).astype(np.uint16)
    cb = (r.standard_normal((K, D)) * 0.05).astype(np.float16).view(np.uint16)
    sc = r.uniform(0.5, 1.5, (E, OUT, IN // G)).astype(np.float16)
    live = r.random((E, OUT)) >= 0.5
    live[0] = False
    tbl = np.full((E, OUT), -1, np.int32)
    tbl[live] = np.arange(int(live.sum()), dtype=np.int32)
    full_c, full_s = codes.copy(), sc.copy()
    full_c[~live] = 0
    full_s[~live] = 0
    x = orc.f16_bits(r.standard_normal((3, IN)))
    idx = np.array([0, 1, 2, 3, 1, 2], dtype=np.uint32)
    a = orc.switch_fused(full_c, cb, full_s.view(np.uint16), x, idx, 2)
    b = orc.switch_fused_rowtable(codes[live], cb, sc[live].view(np.uint16), x, idx, 2, tbl)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    bad = tbl.copy()
    bad[2, 0] = int(live.sum()) + 7
    c = orc.switch_fused_rowtable(codes[live], cb, sc[live].view(np.uint16), x, idx, 2, bad)
    assert np.all(c[2][0:1] == 0) and np.all(c[idx == 2][:, 0] == 0)


def test_prescaled_arm_equals_dense_decode_matmul_fp16():
    """MODE_PRESCALED (gemmseg2 without ACCS: W = fp16(cb*s), ascending-k fp32
    sum) on one expert is the dense _decode_matmul with fp16 weights and fp16 x,
    bit for bit: the same weight rounding and the same summation order."""
    L = make_layer(E=1, OUT=40, IN=256, D=8, K=1024, G=64, seed=9)
    r = np.random.default_rng(10)
    xv = orc.f16_vals(orc.f16_bits(r.standard_normal((3, 256))))
    a = orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, orc.f16_bits(xv), np.zeros(3, np.uint32), 1,
                         mode=orc.MODE_PRESCALED)
    b = orc.dense_decode_matmul(L.codes[0], L.cb_bits, L.sc_bits[0], xv, wbf16=False)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    ex = orc.exact_f64(L.codes, L.cb_bits, L.sc_bits, xv, idx=np.zeros(3, np.uint32))
    assert max_rel(ex, a) < 2e-3
