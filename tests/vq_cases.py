"""Seeded synthetic VQ layers for the tests (numpy side) and their torch twins.

Value distributions follow the reference tests and benchmark configurations: codes
uniform over [0, K), codebook fp16 ~N(0, sigma), scales fp16 ~U(0.5, 1.5)
(or ~N(1, 0.1) like tests/test_vq_prefill_paths.py:26-27), x ~N(0, 1).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import oracle as orc


@dataclass
class VQLayer:
    E: int
    OUT: int
    IN: int
    D: int
    K: int
    G: int
    bits: int            # pack_bits (0 = unpacked)
    codes: np.ndarray    # [E, OUT, NSUB] uint16 unpacked
    packed: np.ndarray   # [E, OUT, WPR] uint32 (bits > 0) or codes in storage dtype
    cb_bits: np.ndarray  # [K, D] fp16 bits
    sc_bits: np.ndarray  # [E, OUT, NGRP] fp16 bits

    @property
    def NSUB(self):
        return self.IN // self.D

    @property
    def NGRP(self):
        return self.IN // self.G


def make_layer(E, OUT, IN, D, K, G=64, packed=True, seed=0, cb_sigma=0.02, scale="uniform") -> VQLayer:
    rng = np.random.default_rng(seed)
    nsub = IN // D
    codes = rng.integers(0, K, (E, OUT, nsub)).astype(np.uint16)
    cb = (rng.standard_normal((K, D)) * cb_sigma).astype(np.float16)
    if scale == "uniform":
        sc = rng.uniform(0.5, 1.5, (E, OUT, IN // G)).astype(np.float16)
    else:
        sc = (rng.standard_normal((E, OUT, IN // G)) * 0.1 + 1).astype(np.float16)
    if packed:
        bits = int(K - 1).bit_length()
        store = orc.pack(codes, bits)
    else:
        bits = 0
        store = codes.astype(np.uint8 if K <= 256 else np.uint16)
    return VQLayer(E, OUT, IN, D, K, G, bits, codes, store, cb.view(np.uint16), sc.view(np.uint16))


def skewed_routing(T, k, E, seed=1):
    """The reference's skewed fixture (tests/test_vq_prefill_paths.py:32-43):
    expert 0 hot (~10x mean), expert E-2 never, expert E-1 exactly once, one
    token routed to the same expert twice."""
    r = np.random.default_rng(seed)
    p = np.ones(E)
    p[0] = 10
    p[E - 2] = 0
    p /= p.sum()
    idx = r.choice(E, size=(T, k), p=p).astype(np.uint32)
    idx[0, :2] = 3 % E
    idx[idx == (E - 1)] = 1 % E
    if T > 5:
        idx[5, 0] = E - 1
    return idx


def zipf_routing(T, k, E, s=1.1, seed=2):
    """Zipf(s) expert popularity over a seeded permutation of the experts,
    k distinct experts per token (benchmark configuration C3)."""
    r = np.random.default_rng(seed)
    perm = r.permutation(E)
    w = 1.0 / np.arange(1, E + 1) ** s
    w = w / w.sum()
    pop = np.empty(E)
    pop[perm] = w
    idx = np.empty((T, k), dtype=np.uint32)
    for t in range(T):
        idx[t] = r.choice(E, size=k, replace=False, p=pop)
    return idx


def to_torch(layer: VQLayer, device="cuda"):
    import torch
    if layer.bits:
        codes = torch.from_numpy(layer.packed.view(np.int32)).to(device)
    elif layer.packed.dtype == np.uint8:
        codes = torch.from_numpy(layer.packed).to(device)
    else:
        codes = torch.from_numpy(layer.packed.view(np.int16)).to(device)
    cb = torch.from_numpy(layer.cb_bits.view(np.float16)).to(device)
    sc = torch.from_numpy(layer.sc_bits.view(np.float16)).to(device)
    return codes, cb, sc


def max_rel(a, b):
    """The reference's metric (tests/test_vq_prefill_paths.py:209-210):
    max|a-b| / max|a|, with a the reference side."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(1e-30, float(np.max(np.abs(a)))))


def bf16_ulp(v):
    """One bfloat16 unit in the last place at |v| (for values that took a bf16
    rounding: 2^(floor(log2|v|) - 7))."""
    v = np.abs(np.asarray(v, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(v, 1e-38)))
    return np.exp2(e - 7)


def within_tol_bf16(ref, got, rel=2e-3):
    """Elementwise: |got - ref| <= rel * max|ref| + 1 bf16 ULP of ref.  The
    extra ULP admits the one rounding step a bf16 output can differ by when
    the two fp32 accumulators straddle a rounding boundary."""
    ref = np.asarray(ref, dtype=np.float64)
    got = np.asarray(got, dtype=np.float64)
    lim = rel * np.max(np.abs(ref)) + bf16_ulp(ref)
    return bool(np.all(np.abs(got - ref) <= lim))
