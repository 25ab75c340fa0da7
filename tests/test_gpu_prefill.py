"""Parity of the grouped tcgen05 GEMM (the large-N path) with the CPU oracle.

The GEMM materialises each weight as fp16(cb * s) (one RNE rounding, the
reference's non-ACCS and dense arms) and accumulates in fp32 in the tensor
core's order, so it is compared within the north-star tolerance, written
here: fp32-level max relative error (max|a-b|/max|a|, the reference's
metric, tests/test_vq_prefill_paths.py:209-210) <= 2e-3 against the
restated gemmseg2-ACCS accumulators, bf16 outputs within 2e-3*max|ref| + 1
bf16 ULP, and accuracy against the float64 reconstruction no worse than the
reference's own non-ACCS arm (the same one weight rounding) by more than 1%.
The reference's gates use skewed routing on purpose (hot expert, one
never-used and one single-row expert, a duplicated expert in a token,
tests/test_vq_prefill_paths.py:32-43) and Zipf(1.1) popularity (benchmark
configuration C3).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import make_layer, max_rel, skewed_routing, to_torch, within_tol_bf16, zipf_routing
from vqlab_b200 import VQLinear, VQSwitchLinear
from vqlab_b200.vq_switch import make_options

pytestmark = pytest.mark.gpu


def _switch(L, path=0):
    codes, cb, sc = to_torch(L)
    m = VQSwitchLinear(codes, cb, sc, group_size=L.G, pack_bits=L.bits, in_features=L.IN)
    if path:
        m.options = make_options(path=path)
    return m


def _prescaled_oracle(L, x_vals, idx, krep):
    """fp64 reference of W = fp16(cb*s) (the weight the GEMM multiplies)."""
    E, OUT, NSUB = L.codes.shape
    cb = orc.f16_vals(L.cb_bits)
    sc = orc.f16_vals(L.sc_bits)
    y = np.empty((idx.size, OUT), dtype=np.float64)
    xh = orc.f16_vals(orc.f16_bits(x_vals))
    for e in np.unique(idx):
        W = cb[L.codes[e].astype(np.int64)].reshape(OUT, L.IN)
        W = orc.round_f16(W * np.repeat(sc[e], L.G, axis=1)).astype(np.float64)
        sel = np.nonzero(idx == e)[0]
        y[sel] = xh[sel // krep].astype(np.float64) @ W.T
    return y


def _check(L, x, idx, krep, y):
    """y: module output as float32 [N, OUT] (x dtype bf16 -> fp16 -> bf16 rounding)."""
    xv = x.float().cpu().numpy().reshape(-1, L.IN)
    ref32 = orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, orc.f16_bits(xv), idx, krep, mode=orc.MODE_ACCS)
    ref = orc.round_bf16(orc.round_f16(ref32))
    assert within_tol_bf16(ref, y)
    return ref32


GEOMS = [  # (D, K, IN, OUT, G)
    (8, 16384, 1024, 256, 64),
    (8, 4096, 512, 128, 512),     # per-row scale
    (8, 1024, 640, 200, 64),      # OUT not a multiple of 128, ragged NSUB
    (4, 2048, 512, 128, 64),
    (2, 256, 512, 128, 64),
]


@pytest.mark.parametrize("D,K,IN,OUT,G", GEOMS)
def test_grouped_gemm_skewed_routing(D, K, IN, OUT, G):
    E = 8
    L = make_layer(E=E, OUT=OUT, IN=IN, D=D, K=K, G=G, seed=100 + K + IN)
    T, k = 80, 8  # 640 pairs > 512: the grouped GEMM serves it
    idx = skewed_routing(T, k, E, seed=9)
    rng = np.random.default_rng(10)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, IN)).astype(np.float32)).to(torch.bfloat16)
    m = _switch(L)
    y = m(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy().reshape(T * k, OUT)
    ref32 = _check(L, x, idx.reshape(-1), k, y)
    # fp32-level (fp32 output: only the fp16 output rounding remains)
    y32 = m(x.float().cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).cpu().numpy().reshape(T * k, OUT)
    assert max_rel(orc.round_f16(ref32), y32) <= 2e-3
    # accuracy: within 1% of the rms error of the same fp16 weight rounding
    xv = x.float().numpy().reshape(T, IN)
    ex = orc.exact_f64(L.codes, L.cb_bits, L.sc_bits, orc.f16_vals(orc.f16_bits(xv)), idx=idx.reshape(-1), krep=k)
    pre = orc.round_f16(_prescaled_oracle(L, xv, idx.reshape(-1), k))
    rms = lambda a: float(np.sqrt(np.mean((np.asarray(a, np.float64) - ex) ** 2)))
    assert rms(y32) <= 1.01 * rms(pre) + 1e-12


DSPLIT_GEOMS = [  # (K, IN, OUT, G): d8 codebooks over the shared-memory budget
    (16384, 1536, 200, 64),    # dimension split: ragged OUT, 3 windows per pass, two groups per position
    (16384, 512, 128, 128),    # dimension split: one group per position, scales from global (NGRP < 8)
    (12000, 1024, 128, 64),    # dimension split with K between the one-pass limit and 2^14
    (16384, 1536, 128, 192),   # dimension split, G not a power of two
    (16384, 576, 136, 64),     # IN not a multiple of 512: entry-slice passes instead
]


@pytest.mark.parametrize("K,IN,OUT,G", DSPLIT_GEOMS)
def test_large_codebook_passes(K, IN, OUT, G):
    """d8 codebooks larger than shared memory: each pass keeps half of every
    entry's dims (or, where the split does not apply, a slice of the entries)
    resident; the sum over passes must equal the one-pass product."""
    E = 6
    L = make_layer(E=E, OUT=OUT, IN=IN, D=8, K=K, G=G, seed=K + IN + G)
    T, k = 90, 6  # 540 pairs
    idx = skewed_routing(T, k, E, seed=11)
    rng = np.random.default_rng(12)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, IN)).astype(np.float32)).to(torch.bfloat16)
    m = _switch(L, path=2)
    ii = torch.from_numpy(idx.astype(np.int32)).cuda()
    y = m(x.cuda(), ii).float().cpu().numpy().reshape(T * k, OUT)
    ref32 = _check(L, x, idx.reshape(-1), k, y)
    y32 = m(x.float().cuda(), ii).cpu().numpy().reshape(T * k, OUT)
    assert max_rel(orc.round_f16(ref32), y32) <= 2e-3
    xv = x.float().numpy().reshape(T, IN)
    ex = orc.exact_f64(L.codes, L.cb_bits, L.sc_bits, orc.f16_vals(orc.f16_bits(xv)), idx=idx.reshape(-1), krep=k)
    pre = orc.round_f16(_prescaled_oracle(L, xv, idx.reshape(-1), k))
    rms = lambda a: float(np.sqrt(np.mean((np.asarray(a, np.float64) - ex) ** 2)))
    assert rms(y32) <= 1.01 * rms(pre) + 1e-12
    # deterministic: the same call gives the same bytes
    assert np.array_equal(y32, m(x.float().cuda(), ii).cpu().numpy().reshape(T * k, OUT))


def test_hot_expert_spans_several_tiles():
    """One expert with > 256 tokens: several 256-token tiles of the same rows."""
    E = 4
    L = make_layer(E=E, OUT=128, IN=512, D=8, K=16384, G=64, seed=41)
    T, k = 300, 2
    idx = np.zeros((T, k), dtype=np.uint32)
    idx[:, 1] = np.arange(T) % E
    rng = np.random.default_rng(42)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, 512)).astype(np.float32)).to(torch.bfloat16)
    y = _switch(L)(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy().reshape(T * k, 128)
    _check(L, x, idx.reshape(-1), k, y)


@pytest.mark.parametrize("T,k", [(1, 1), (3, 5), (17, 2)])
def test_forced_gemm_on_tiny_batches(T, k):
    """path=PREFILL at a few pairs: tiles of 1..17 tokens (N rounded to 16)."""
    E = 6
    L = make_layer(E=E, OUT=256, IN=512, D=8, K=4096, G=64, seed=T * 7 + k)
    idx = np.random.default_rng(T).integers(0, E, (T, k)).astype(np.uint32)
    rng = np.random.default_rng(43)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, 512)).astype(np.float32)).to(torch.bfloat16)
    y = _switch(L, path=2)(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy()
    _check(L, x, idx.reshape(-1), k, y.reshape(T * k, 256))


def test_zipf_prefill_small():
    """benchmark configuration C3 in miniature: Zipf(1.1) popularity, 10 distinct experts per token."""
    E, T, k = 64, 256, 10
    L = make_layer(E=E, OUT=256, IN=1024, D=8, K=16384, G=64, seed=77)
    idx = zipf_routing(T, k, E, seed=5)
    rng = np.random.default_rng(78)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, 1024)).astype(np.float32)).to(torch.bfloat16)
    y = _switch(L)(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy().reshape(T * k, 256)
    _check(L, x, idx.reshape(-1), k, y)


def test_down_projection_per_pair_input():
    """SwitchGLU down_proj shape: x given per pair, N > 512."""
    E = 8
    L = make_layer(E=E, OUT=512, IN=256 * 2, D=8, K=16384, G=64, seed=91)
    T, k = 70, 8
    idx = skewed_routing(T, k, E, seed=92)
    rng = np.random.default_rng(93)
    x = torch.from_numpy(rng.standard_normal((T, k, 1, 512)).astype(np.float32)).to(torch.bfloat16)
    y = _switch(L)(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy().reshape(T * k, 512)
    xv = x.float().numpy().reshape(T * k, 512)
    ref = orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, orc.f16_bits(xv), idx.reshape(-1), 1, mode=orc.MODE_ACCS)
    assert within_tol_bf16(orc.round_bf16(orc.round_f16(ref)), y)


@pytest.mark.parametrize("D,K,IN,OUT,G", [(8, 16384, 1024, 256, 64), (8, 4096, 512, 384, 512), (2, 256, 512, 128, 64)])
@pytest.mark.parametrize("n,xdt", [(17, torch.bfloat16), (100, torch.bfloat16), (300, torch.float16)])
def test_dense_large_n_decode_matmul_numerics(D, K, IN, OUT, G, n, xdt):
    """Dense N > 16 off the fused kernel: W = fp16(cb*s) in x's dtype (bf16 for
    bf16 x), fp32 accumulation -- the reference's _decode_matmul numerics up
    to the GEMM's summation order (vq_dense.py:267-312)."""
    L = make_layer(E=1, OUT=OUT, IN=IN, D=D, K=K, G=G, seed=n + D)
    codes, cb, sc = to_torch(L)
    lin = VQLinear(codes[0], cb, sc[0], group_size=G, pack_bits=L.bits, in_features=IN)
    rng = np.random.default_rng(n)
    x = torch.from_numpy(rng.standard_normal((n, IN)).astype(np.float32)).to(xdt)
    y = lin(x.cuda()).float().cpu().numpy()
    fused = D != 8 and n <= {2: 72, 4: 32}.get(D, 0)
    xv = x.float().numpy()
    if fused:
        ref = orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, orc.f16_bits(xv), np.zeros(n, np.uint32), 1)
    else:
        ref = orc.dense_decode_matmul(L.codes[0], L.cb_bits, L.sc_bits[0], xv, wbf16=(xdt == torch.bfloat16))
    rounded = orc.round_bf16(ref) if xdt == torch.bfloat16 else orc.round_f16(ref)
    assert within_tol_bf16(rounded, y)


@pytest.mark.parametrize("OUT,IN", [(384, 4096), (200, 2048)])
@pytest.mark.parametrize("n,xdt", [(1, torch.bfloat16), (5, torch.float16), (130, torch.bfloat16)])
def test_dense_split_k(OUT, IN, n, xdt):
    """Dense d8/K16384 layers with few row tiles: the GEMM cuts each tile's K
    windows over several CTAs and sums the fp32 partials in split order.
    The result stays within the _decode_matmul tolerance and is deterministic."""
    L = make_layer(E=1, OUT=OUT, IN=IN, D=8, K=16384, G=64, seed=n + OUT)
    codes, cb, sc = to_torch(L)
    lin = VQLinear(codes[0], cb, sc[0], group_size=64, pack_bits=L.bits, in_features=IN)
    rng = np.random.default_rng(n + 1)
    x = torch.from_numpy(rng.standard_normal((n, IN)).astype(np.float32)).to(xdt)
    y = lin(x.cuda())
    ref = orc.dense_decode_matmul(L.codes[0], L.cb_bits, L.sc_bits[0], x.float().numpy(), wbf16=(xdt == torch.bfloat16))
    rounded = orc.round_bf16(ref) if xdt == torch.bfloat16 else orc.round_f16(ref)
    assert within_tol_bf16(rounded, y.float().cpu().numpy())
    assert torch.equal(y, lin(x.cuda()))


@pytest.mark.parametrize("T", [1, 2])
def test_switch_decode_batch_split_k(T):
    """A decode batch over a few experts on the dimension-split GEMM: 10-20
    pairs give 80-160 tiles, each cut over 2-3 CTAs, and most CTAs run two
    work items, the second in the reversed codebook-slice order -- each
    item must still cover its own K range."""
    E, OUT, IN, k = 16, 1024, 4096, 10
    L = make_layer(E=E, OUT=OUT, IN=IN, D=8, K=16384, G=64, seed=300 + T)
    idx = np.stack([np.random.default_rng(T * 10 + t).permutation(E)[:k] for t in range(T)]).astype(np.uint32)
    rng = np.random.default_rng(301)
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, IN)).astype(np.float32)).to(torch.bfloat16)
    m = _switch(L)
    assert m.kernel_path(T, k) == "gemm"
    y = m(x.cuda(), torch.from_numpy(idx.astype(np.int32)).cuda()).float().cpu().numpy().reshape(T * k, OUT)
    _check(L, x, idx.reshape(-1), k, y)


class _NoHalves:
    """Stands in for a module's CodebookHalves: always NULL, so every call
    derives the dimension halves itself."""

    def pointer(self, codebook):
        return None


def test_codebook_halves_built_once_give_the_same_bytes():
    """A module passes its d8 codebook's dimension halves, built once
    (vqb_codebook_halves), to every call; the result must be byte-equal to a
    call that derives them inside, for the switch and the dense entry point,
    and the halves must follow an in-place change of the codebook."""
    L = make_layer(E=5, OUT=256, IN=1024, D=8, K=16384, G=64, seed=77)
    T, k = 40, 3
    idx = torch.from_numpy(skewed_routing(T, k, 5, seed=3).astype(np.int32)).cuda()
    x = torch.randn((T, 1, 1, 1024), generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).cuda()
    a, b = _switch(L, path=2), _switch(L, path=2)
    b._halves = _NoHalves()
    ya = a(x, idx)
    assert a._halves.pointer(a.codebook) is not None
    assert torch.equal(ya.view(torch.int16), b(x, idx).view(torch.int16))
    # in place: the cached halves are rebuilt (the tensor's version counter moved)
    a.codebook.mul_(0.5)
    b.codebook.mul_(0.5)
    assert torch.equal(a(x, idx).view(torch.int16), b(x, idx).view(torch.int16))
    assert not torch.equal(a(x, idx).view(torch.int16), ya.view(torch.int16))
    codes, cb, sc = to_torch(L)
    da = VQLinear(codes[0], cb, sc[0], group_size=64, pack_bits=L.bits, in_features=1024)
    db = VQLinear(codes[0], cb.clone(), sc[0], group_size=64, pack_bits=L.bits, in_features=1024)
    db._halves = _NoHalves()
    xd = x.reshape(T, 1024)
    assert torch.equal(da(xd).view(torch.int16), db(xd).view(torch.int16))
