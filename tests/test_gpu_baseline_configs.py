"""Parity at the benchmark configurations' full sizes, through the shipped AUTO path.

Every call here goes through the public modules with the library's default
kernel choice, at the shapes the benchmark times, and is compared with the CPU
oracle's restatement of the reference arm that serves the same call:

  C1  dense 4096 x 4096, d8/K4096/12-bit, N = 1 ........ _decode_matmul (vq_dense.py:267-312)
  C2  512 experts, gate 1024 x 4096 and down 4096 x 1024, d8/K16384/14-bit, top-10,
      batch 1: gate simd_sum arm, down walk arm (vq_switch.py:1575-1660, :1316-1392);
      batch 8: walk arm; batch 64: gemmseg2 ACCS arm (:4171-4203)
  C3  4096 tokens, Zipf(1.1) top-10 over 512 experts ........ gemmseg2 ACCS, on a seeded sample
      of >= 2048 pairs that covers every pair of the single-row experts and every tile of the
      hottest expert
  C4  attention q/o 5120 x 5120 and k/v 1024 x 5120, d2/K256/8-bit, N = 1 and 32
      ..................................................... dense d2 simd_sum arm (:2432-2439)
      MLP 17408 x 5120 (d8/K16384), N = 1 and 32 .......... _decode_matmul

Tolerance (written here): the output stored as float32
(`out_dtype=torch.float32`: the switch keeps its fp16 output rounding, the
dense projections their fp32 accumulators) is within max relative error
max|y - ref| / max|ref| <= 2e-3 of the oracle's (the reference's metric,
tests/test_vq_prefill_paths.py:209-210).  The bf16 output the modules return
by default is checked too, within 2e-3 * max|ref| + one bf16 ULP of each
reference value: the ULP is the one output rounding step by which two fp32
results that straddle a bf16 rounding boundary differ.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import max_rel, within_tol_bf16, zipf_routing
from vqlab_b200 import VQLinear, VQSwitchLinear

pytestmark = pytest.mark.gpu

HIDDEN, INTER, E, TOPK, D, K, BITS, G = 4096, 1024, 512, 10, 8, 16384, 14, 64
TOL = 2e-3


def _wpr(nsub, bits):
    return (nsub + 31) // 32 * bits


class SwitchWeights:
    """One C2/C3 projection: packed codes uint32 [E, OUT, WPR] (uniform random
    words are uniform 14-bit codes: K = 2^14 and NSUB % 32 == 0), codebook fp16
    ~N(0, 0.02), scales fp16 ~U(0.5, 1.5), on the host and on the GPU."""

    def __init__(self, out, inn, seed):
        rng = np.random.default_rng(seed)
        self.OUT, self.IN = out, inn
        self.packed = rng.integers(0, 2 ** 32, (E, out, _wpr(inn // D, BITS)), dtype=np.uint32)
        self.cb = (rng.standard_normal((K, D)) * 0.02).astype(np.float16)
        self.sc = rng.uniform(0.5, 1.5, (E, out, inn // G)).astype(np.float16)
        self.module = VQSwitchLinear(torch.from_numpy(self.packed.view(np.int32)).cuda(),
                                     torch.from_numpy(self.cb).cuda(), torch.from_numpy(self.sc).cuda(),
                                     group_size=G, pack_bits=BITS, in_features=inn)

    def oracle(self, x_vals, idx, krep, mode):
        """Pre-rounding accumulators [N, OUT] of the oracle for pairs idx (pair p reads x row p // krep),
        computed on the experts the pairs use only."""
        idx = np.asarray(idx, dtype=np.uint32).reshape(-1)
        used, local = np.unique(idx, return_inverse=True)
        return orc.switch_fused(np.ascontiguousarray(self.packed[used]), self.cb.view(np.uint16),
                                np.ascontiguousarray(self.sc[used]).view(np.uint16), orc.f16_bits(x_vals),
                                local.astype(np.uint32), krep, mode=mode, packed_bits=BITS)


@pytest.fixture(scope="module")
def c2_layer():
    return {"gate": SwitchWeights(INTER, HIDDEN, seed=0), "down": SwitchWeights(HIDDEN, INTER, seed=1)}


def _router_idx(T, seed):
    rng = np.random.default_rng(seed)
    lg = rng.standard_normal((T, E)).astype(np.float32)
    idx, _ = orc.router_topk(lg, TOPK)
    return idx


def _check_switch(W, x_bf16, idx, krep, mode, sel=None):
    """Run the module on the whole call (bf16 x), compare the pairs `sel` (all
    when None) with the oracle at the fp32 level and as bf16."""
    xt = torch.from_numpy(x_bf16).cuda().to(torch.bfloat16)
    it = torch.from_numpy(idx.astype(np.int32)).cuda()
    N = idx.size
    y32 = W.module(xt, it, out_dtype=torch.float32).reshape(N, W.OUT)
    yb = W.module(xt, it).reshape(N, W.OUT)
    torch.cuda.synchronize()
    sel = np.arange(N) if sel is None else np.asarray(sel)
    xrows = x_bf16.reshape(-1, W.IN)[sel // krep]
    ref32 = W.oracle(xrows, idx.reshape(-1)[sel], 1, mode)
    st = torch.from_numpy(sel).cuda()
    got32 = y32.index_select(0, st).cpu().numpy()
    gotb = yb.index_select(0, st).float().cpu().numpy()
    err = max_rel(orc.round_f16(ref32), got32)
    assert err <= TOL, f"fp32-level max rel {err:.3e}"
    assert within_tol_bf16(orc.round_bf16(orc.round_f16(ref32)), gotb)
    return err


# ------------------------------------------------------------------ C2 decode

# the reference arm of each (batch, projection) at the C2 shapes (benchmark
# configuration notes: simd_sum only when N <= 20 and IN / G >= 32, walk up to
# 512 pairs, gemmseg2 ACCS above)
C2_MODES = {(1, "gate"): orc.MODE_SS, (1, "down"): orc.MODE_WALK, (8, "gate"): orc.MODE_WALK,
            (8, "down"): orc.MODE_WALK, (64, "gate"): orc.MODE_ACCS, (64, "down"): orc.MODE_ACCS}


@pytest.mark.parametrize("batch", [1, 8, 64])
@pytest.mark.parametrize("proj", ["gate", "down"])
def test_c2_full_size(c2_layer, batch, proj):
    """C2 at 512 experts: gate (x per token, top-10 pairs) and down (x per pair)."""
    W = c2_layer[proj]
    idx = _router_idx(batch, seed=100 + batch)
    rng = np.random.default_rng(200 + batch)
    if proj == "gate":
        x = orc.round_bf16(rng.standard_normal((batch, 1, 1, HIDDEN)).astype(np.float32))
        krep = TOPK
    else:
        x = orc.round_bf16(rng.standard_normal((batch, TOPK, 1, INTER)).astype(np.float32))
        krep = 1
    assert W.module.kernel_path(x.reshape(-1, W.IN).shape[0], krep) in ("gemm", "decode")
    _check_switch(W, x, idx, krep, C2_MODES[(batch, proj)])


# ------------------------------------------------------------------ C3 prefill

def _c3_sample(idx, seed=3, n_other=1000):
    """Pairs to check: every pair of the 24 experts with the fewest rows
    (Zipf(1.1) over 4096 tokens leaves no expert with a single row -- the
    smallest hold 5; single-row experts are the C2 batch-1/8 case above and the
    skewed-routing fixtures), every third pair of the hottest expert (its
    128-token tiles all get covered, the first and last pair included), and a
    seeded random draw of the others."""
    flat = idx.reshape(-1)
    counts = np.bincount(flat, minlength=E)
    hot = int(np.argmax(counts))
    small = np.argsort(counts, kind="stable")[:24]
    small = small[counts[small] > 0]
    pairs_small = np.nonzero(np.isin(flat, small))[0]
    pairs_hot = np.nonzero(flat == hot)[0]
    pick_hot = np.unique(np.concatenate([pairs_hot[::3], pairs_hot[-1:]]))
    rest = np.setdiff1d(np.arange(flat.size), np.concatenate([pairs_small, pick_hot]))
    rng = np.random.default_rng(seed)
    pick_rest = rng.choice(rest, size=min(n_other, rest.size), replace=False)
    sel = np.unique(np.concatenate([pairs_small, pick_hot, pick_rest]))
    return sel, hot, counts


@pytest.fixture(scope="module")
def c3_routing():
    return zipf_routing(4096, TOPK, E, s=1.1, seed=2)


def test_c3_full_size_gate(c2_layer, c3_routing):
    idx = c3_routing
    sel, hot, counts = _c3_sample(idx)
    assert sel.size >= 2048 and counts[hot] > 1000
    rng = np.random.default_rng(300)
    x = orc.round_bf16(rng.standard_normal((4096, 1, 1, HIDDEN)).astype(np.float32))
    W = c2_layer["gate"]
    assert W.module.kernel_path(4096, TOPK) == "gemm"
    _check_switch(W, x, idx, TOPK, orc.MODE_ACCS, sel=sel)


def test_c3_full_size_down(c2_layer, c3_routing):
    idx = c3_routing
    sel, _, _ = _c3_sample(idx, seed=4)
    rng = np.random.default_rng(301)
    x = orc.round_bf16(rng.standard_normal((4096, TOPK, 1, INTER)).astype(np.float32))
    W = c2_layer["down"]
    assert W.module.kernel_path(4096 * TOPK, 1) == "gemm"
    _check_switch(W, x, idx, 1, orc.MODE_ACCS, sel=sel)


# ------------------------------------------------------------------ dense C1 / C4

def _dense_layer(out, inn, d, k, bits, g, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, k, (out, inn // d)).astype(np.uint16)
    cb = (rng.standard_normal((k, d)) * 0.02).astype(np.float16)
    sc = rng.uniform(0.5, 1.5, (out, inn // g)).astype(np.float16)
    packed = orc.pack(codes, bits)
    lin = VQLinear(torch.from_numpy(packed.view(np.int32)).cuda(), torch.from_numpy(cb).cuda(),
                   torch.from_numpy(sc).cuda(), group_size=g, pack_bits=bits, in_features=inn)
    return lin, codes, cb.view(np.uint16), sc.view(np.uint16)


def _check_dense(lin, codes, cb, sc, x_bf16, fused, rms_check=True):
    """fused: the reference's fused dense arm (x narrowed to fp16, group
    partials, simd_sum over 32-group blocks, y stored directly); else
    _decode_matmul (W = bf16(fp16(cb * s)), y = x @ W^T in fp32)."""
    xt = torch.from_numpy(x_bf16).cuda().to(torch.bfloat16)
    y32 = lin(xt, out_dtype=torch.float32).cpu().numpy()
    yb = lin(xt).float().cpu().numpy()
    if fused:
        ref32 = orc.switch_fused(codes[None], cb, sc[None], orc.f16_bits(x_bf16),
                                 np.zeros(x_bf16.shape[0], np.uint32), 1, mode=orc.MODE_SS)
    else:
        ref32 = orc.dense_decode_matmul(codes, cb, sc, x_bf16, wbf16=True)
    err = max_rel(ref32, y32)
    assert err <= TOL, f"fp32-level max rel {err:.3e}"
    assert within_tol_bf16(orc.round_bf16(ref32), yb)
    if rms_check:
        # the delivered bf16 output no less accurate against the float64
        # reconstruction than the reference arm's (1 % slack); the fp32
        # accumulators themselves differ from it by summation order only, at the
        # level of fp32 round-off, where a relative rule means nothing
        xv = orc.f16_vals(orc.f16_bits(x_bf16)) if fused else x_bf16
        ex = orc.exact_f64(codes, cb, sc, xv)
        rms = lambda a: float(np.sqrt(np.mean((np.asarray(a, np.float64) - ex) ** 2)))
        assert rms(yb) <= 1.01 * rms(orc.round_bf16(ref32)) + 1e-12
    return err


@pytest.mark.parametrize("g", [64, 4096])
def test_c1_dense_matvec(g):
    """C1: 4096 x 4096, d8/K4096 (12-bit codes), N = 1, per-group (G = 64) and
    per-output-row (G = IN) scales."""
    lin, codes, cb, sc = _dense_layer(4096, 4096, 8, 4096, 12, g, seed=g)
    rng = np.random.default_rng(41)
    x = orc.round_bf16(rng.standard_normal((1, 4096)).astype(np.float32))
    _check_dense(lin, codes, cb, sc, x, fused=False)


@pytest.mark.parametrize("out", [5120, 1024])
@pytest.mark.parametrize("n", [1, 32])
def test_c4_attention_projections(out, n):
    """C4 attention q/o (5120 x 5120) and k/v (1024 x 5120), d2/K256 8-bit packed:
    the fused dense arm (N <= 72) -- the decode kernel at N = 1, the grouped
    GEMM with fp16 operands at N = 32."""
    lin, codes, cb, sc = _dense_layer(out, 5120, 2, 256, 8, 64, seed=out + n)
    rng = np.random.default_rng(out * 3 + n)
    x = orc.round_bf16(rng.standard_normal((n, 5120)).astype(np.float32))
    _check_dense(lin, codes, cb, sc, x, fused=True, rms_check=(n == 1))


@pytest.mark.parametrize("n", [1, 32])
def test_c4_mlp_fp32_level(n):
    """C4 MLP gate 17408 x 5120, d8/K16384 (the grouped GEMM's dimension split)."""
    lin, codes, cb, sc = _dense_layer(17408, 5120, 8, 16384, 14, 64, seed=500 + n)
    rng = np.random.default_rng(n + 51)
    x = orc.round_bf16(rng.standard_normal((n, 5120)).astype(np.float32))
    _check_dense(lin, codes, cb, sc, x, fused=False, rms_check=False)


def test_c4_mlp_decode_kernel_instantiation():
    """The decode kernel's bf16-weight arm with the codebook prefix in shared
    memory (the rest read through L1) at the C4 MLP gate shape: 16-bit codes
    of a K16384 codebook are not a dimension-split geometry, so a one-row call
    takes the decode kernel with its largest shared-memory request."""
    lin, codes, cb, sc = _dense_layer(17408, 5120, 8, 16384, 16, 64, seed=777)
    rng = np.random.default_rng(52)
    x = orc.round_bf16(rng.standard_normal((1, 5120)).astype(np.float32))
    _check_dense(lin, codes, cb, sc, x, fused=False, rms_check=False)
