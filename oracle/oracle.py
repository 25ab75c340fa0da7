"""CPU oracle for the VQ expert runtime hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module, and only as the checker (or the timed CPU baseline).  The
product package `vqlab_b200` never imports it and has no CPU fallback.

Two layers:
  * `liboracle.so` (vq_oracle.c, built by oracle/Makefile): the C restatement
    of the reference arithmetic, OpenMP over rows.  Citations are in the C.
  * numpy restatements here: the vq_pack reader/writer (vq_pack.py:34-101),
    IEEE fp16/bf16 rounding helpers, and the MoE block around the projections
    (router softmax, top-k, renormalise, SwiGLU, weighted combine), after the
    reference's numpy MoE block tests/test_qwen3_5_parity.py:180-204 and the
    router convention family/qwen3_5.py:110-118.

Parity status: the vq_pack reader is pinned by golden vectors generated with
the reference's own vq_pack.py (tests/golden/make_golden.py).  The matmul
arithmetic is a restatement of kernels that only run on Apple GPUs; their
float orders that Metal leaves unspecified are chosen and named in the C, so
bit-level parity with the Metal kernels is UNPINNED.  The float64 exact
reconstruction (score/kernel_truth_moe.py:37-50) is the accuracy arbiter.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build(force: bool = False) -> pathlib.Path:
    """Compile liboracle.so with oracle/Makefile (gcc, no CUDA)."""
    if force or not LIB_PATH.exists() or (
            LIB_PATH.stat().st_mtime < (HERE / "vq_oracle.c").stat().st_mtime):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        i32, i64 = ctypes.c_int, ctypes.c_int64
        L.orc_unpack.argtypes = [P, i64, i64, i64, i32, P]
        L.orc_pack.argtypes = [P, i64, i64, i32, P]
        L.orc_pack.restype = i32
        L.orc_words_per_row.argtypes = [i64, i32]
        L.orc_words_per_row.restype = i64
        L.orc_switch_fused.argtypes = [P, P, P, i32, i32, i32, i32, i32, i32,
                                       P, i32, P, i32, i32, i32, P]
        L.orc_switch_fused_packed.argtypes = [P, i32, P, P, i32, i32, i32, i32, i32, i32,
                                              P, i32, P, i32, i32, i32, P]
        L.orc_dense_decode_matmul.argtypes = [P, P, P, i32, i32, i32, i32, P, i32, i32, P]
        L.orc_exact_f64.argtypes = [P, P, P, i32, i32, i32, i32, i32, P, i32, P, i32, i32, P]
        for f in ("orc_f32_to_f16", "orc_f32_to_bf16", "orc_f16_to_f32", "orc_bf16_to_f32"):
            getattr(L, f).argtypes = [P, P, i64]
        L.orc_num_threads.restype = i32
        L.orc_set_num_threads.argtypes = [i32]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------ numbers

def f16_bits(a) -> np.ndarray:
    """float values -> IEEE fp16 bit patterns (RNE)."""
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32).astype(np.float16)).view(np.uint16)


def f16_vals(bits) -> np.ndarray:
    return np.ascontiguousarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16_bits(a) -> np.ndarray:
    """float32 values -> bfloat16 bit patterns, round-to-nearest-even."""
    u = np.ascontiguousarray(np.asarray(a, dtype=np.float32)).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_vals(bits) -> np.ndarray:
    return (np.ascontiguousarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    return bf16_vals(bf16_bits(a))


def round_f16(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


# ------------------------------------------------------------------ vq_pack

BLOCK = 32


def words_per_row(nsub: int, bits: int) -> int:
    """vq_pack.py:41-45: ceil(NSUB/32) blocks of `bits` words each."""
    return (nsub + BLOCK - 1) // BLOCK * bits


def unpack(packed: np.ndarray, nsub: int, bits: int) -> np.ndarray:
    """[..., WPR] uint32 -> [..., NSUB] codes via the C reader (vq_pack.py:79-97)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    lead = packed.shape[:-1]
    wpr = packed.shape[-1]
    assert wpr == words_per_row(nsub, bits), (wpr, nsub, bits)
    rows = int(np.prod(lead)) if lead else 1
    out = np.empty(rows * nsub, dtype=np.uint16)
    lib().orc_unpack(_p(packed), rows, wpr, nsub, bits, _p(out))
    return out.reshape(*lead, nsub)


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """[..., NSUB] codes -> [..., WPR] uint32 via the C writer (vq_pack.py:48-76)."""
    codes = np.ascontiguousarray(codes, dtype=np.uint16)
    lead = codes.shape[:-1]
    nsub = codes.shape[-1]
    rows = int(np.prod(lead)) if lead else 1
    wpr = words_per_row(nsub, bits)
    out = np.empty(rows * wpr, dtype=np.uint32)
    bad = lib().orc_pack(_p(codes), rows, nsub, bits, _p(out))
    assert not bad, "code exceeds bit width"
    return out.reshape(*lead, wpr)


def unpack_numpy(packed: np.ndarray, nsub: int, bits: int) -> np.ndarray:
    """Pure-numpy reader of the same bit stream (an independent second
    restatement, used to cross-check the C reader): code j of a row occupies
    bits [j*bits, (j+1)*bits) of the row's little-endian word stream."""
    packed = np.asarray(packed, dtype=np.uint32)
    j = np.arange(nsub, dtype=np.int64)
    bit = j * bits
    w, sh = bit >> 5, (bit & 31).astype(np.uint64)
    lo = packed[..., w].astype(np.uint64) >> sh
    w1 = np.minimum(w + 1, packed.shape[-1] - 1)
    hi = packed[..., w1].astype(np.uint64) << (np.uint64(32) - sh)
    straddle = (sh + bits) > 32
    v = np.where(straddle, lo | hi, lo) & np.uint64((1 << bits) - 1)
    return v.astype(np.uint16)


# ------------------------------------------------------------ matmul paths

MODE_WALK, MODE_SS, MODE_ACCS, MODE_PRESCALED = 0, 1, 2, 3


def switch_fused(codes, codebook_bits, scales_bits, x_f16_bits, idx, krep, mode=MODE_WALK,
                 packed_bits: int = 0):
    """Fused expert decode accumulators y32 [N, OUT] (pre output rounding).

    codes: [E, OUT, NSUB] unpacked uint16, or [E, OUT, WPR] uint32 when
    packed_bits > 0.  codebook_bits [K, D], scales_bits [E, OUT, NGRP] and
    x_f16_bits [T, IN] are fp16 bit patterns.  Pair p reads token p // krep.
    mode: MODE_WALK / MODE_SS / MODE_ACCS (the group reductions of the walk,
    simd_sum and gemmseg2-ACCS kernels) or MODE_PRESCALED (gemmseg2 without
    ACCS: W = fp16(cb * s), one fp32 sum over k); orders are named in the C.
    """
    cb = np.ascontiguousarray(codebook_bits, dtype=np.uint16)
    sc = np.ascontiguousarray(scales_bits, dtype=np.uint16)
    xh = np.ascontiguousarray(x_f16_bits, dtype=np.uint16)
    idx = np.ascontiguousarray(idx, dtype=np.uint32).reshape(-1)
    K, D = cb.shape
    E, OUT, NGRP = sc.shape
    T, IN = xh.shape
    G = IN // NGRP
    N = idx.shape[0]
    y = np.empty((N, OUT), dtype=np.float32)
    if packed_bits:
        c = np.ascontiguousarray(codes, dtype=np.uint32)
        lib().orc_switch_fused_packed(_p(c), packed_bits, _p(cb), _p(sc), E, OUT, IN, D, G, K,
                                      _p(xh), T, _p(idx), N, krep, mode, _p(y))
    else:
        c = np.ascontiguousarray(codes, dtype=np.uint16)
        lib().orc_switch_fused(_p(c), _p(cb), _p(sc), E, OUT, IN, D, G, K,
                               _p(xh), T, _p(idx), N, krep, mode, _p(y))
    return y


def switch_fused_rowtable(codes, codebook_bits, scales_bits, x_f16_bits, idx, krep, row_table,
                          mode=MODE_WALK, packed_bits: int = 0):
    """The SKIPZERO switch (vq_switch.py:4958-5013 builds the row table; the
    kernels' row hook, e.g. the packed d8 walk :1395-1415): codes
    [R, NSUB] (or [R, WPR] packed) and scales_bits [R, NGRP] hold the R live
    rows only, row_table int32 [E, OUT] maps (expert, out row) to its compact
    row, -1 = dead (an entry >= R counts as dead too).  A live row is computed
    exactly as switch_fused computes the same row of the expanded layout; a
    dead row reads no code or scale and its output is +0.  Returns y32 [N, OUT]."""
    rt = np.ascontiguousarray(row_table, dtype=np.int32)
    E, OUT = rt.shape
    R = np.asarray(codes).shape[0]
    live = (rt >= 0) & (rt < R)
    take = np.where(live, rt, 0).reshape(-1)
    full_codes = np.ascontiguousarray(np.asarray(codes)[take]).reshape(E, OUT, -1)
    full_sc = np.ascontiguousarray(np.asarray(scales_bits, dtype=np.uint16)[take]).reshape(E, OUT, -1)
    y = switch_fused(full_codes, codebook_bits, full_sc, x_f16_bits, idx, krep, mode=mode, packed_bits=packed_bits)
    idx = np.ascontiguousarray(idx, dtype=np.uint32).reshape(-1)
    y[~live[idx]] = 0.0
    return y


def dense_decode_matmul(codes, codebook_bits, scales_bits, x_vals, wbf16: bool):
    """vq_dense._decode_matmul accumulators y32 [N, OUT]; x_vals are float32
    values already in the input dtype; codes [OUT, NSUB] unpacked."""
    c = np.ascontiguousarray(codes, dtype=np.uint16)
    cb = np.ascontiguousarray(codebook_bits, dtype=np.uint16)
    sc = np.ascontiguousarray(scales_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x_vals, dtype=np.float32)
    OUT, NSUB = c.shape
    K, D = cb.shape
    N, IN = x.shape
    G = IN // sc.shape[-1]
    y = np.empty((N, OUT), dtype=np.float32)
    lib().orc_dense_decode_matmul(_p(c), _p(cb), _p(sc), OUT, IN, D, G, _p(x), N, int(wbf16), _p(y))
    return y


def exact_f64(codes, codebook_bits, scales_bits, x_vals, idx=None, krep=1):
    """float64 exact reconstruction y [N, OUT]; codes [E, OUT, NSUB] unpacked
    (or [OUT, NSUB] for a dense layer with idx None)."""
    c = np.ascontiguousarray(codes, dtype=np.uint16)
    sc = np.ascontiguousarray(scales_bits, dtype=np.uint16)
    if c.ndim == 2:
        c, sc = c[None], sc[None]
    cb = np.ascontiguousarray(codebook_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x_vals, dtype=np.float32)
    E, OUT, NSUB = c.shape
    K, D = cb.shape
    T, IN = x.shape
    G = IN // sc.shape[-1]
    if idx is None:
        N = T
        idxa = None
    else:
        idxa = np.ascontiguousarray(idx, dtype=np.uint32).reshape(-1)
        N = idxa.shape[0]
    y = np.empty((N, OUT), dtype=np.float64)
    lib().orc_exact_f64(_p(c), _p(cb), _p(sc), E, OUT, IN, D, G, _p(x), T,
                        None if idxa is None else _p(idxa), N, krep, _p(y))
    return y


# ------------------------------------------------------------- MoE block

def router_topk(logits, k: int):
    """fp32 softmax over experts, top-k by probability (ties -> lower expert
    id), weights renormalised to sum 1 (tests/test_qwen3_5_parity.py:187-193,
    family/qwen3_5.py:110-118).  Returns (idx [T,k] uint32, w [T,k] fp32)."""
    lg = np.asarray(logits, dtype=np.float32)
    m = lg.max(-1, keepdims=True)
    pr = np.exp(lg - m)
    pr = pr / pr.sum(-1, keepdims=True)
    order = np.argsort(-pr, axis=-1, kind="stable")[:, :k]
    w = np.take_along_axis(pr, order, -1)
    w = w / w.sum(-1, keepdims=True)
    return order.astype(np.uint32), w.astype(np.float32)


def silu(v):
    v = np.asarray(v, dtype=np.float32)
    return v / (np.float32(1.0) + np.exp(-v))


def swiglu_bf16(gate_bf16_vals, up_bf16_vals):
    """h = bf16(silu(gate) * up), computed in fp32 from bf16 inputs."""
    return round_bf16(silu(gate_bf16_vals) * np.asarray(up_bf16_vals, dtype=np.float32))


def combine_bf16(down_bf16_vals, w):
    """y[t] = bf16(sum_j w[t,j] * down[t,j]) with an fp32 ascending-j sum."""
    d = np.asarray(down_bf16_vals, dtype=np.float32)
    T, k, OUT = d.shape
    acc = np.zeros((T, OUT), dtype=np.float32)
    for j in range(k):
        acc = acc + w[:, j:j + 1].astype(np.float32) * d[:, j]
    return round_bf16(acc)


def num_threads() -> int:
    return int(lib().orc_num_threads())


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))
