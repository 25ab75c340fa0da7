"""The CPU oracle and the product's host format code against golden vectors
produced by the reference's own vq_pack.py (tests/golden/make_golden.py).

Mirrors the reference's T1 extraction-equivalence test
(tests/test_vq_wdec.py:91-102: every lane, bits 2..16) and its ragged-tail
cases (tests/test_kswarm_d8_walk.py:45, tests/test_vq_prefill_paths.py:410)."""
import pathlib

import numpy as np
import pytest

from oracle import oracle as orc
from vqlab_b200 import vq_pack

G = np.load(pathlib.Path(__file__).parent / "golden" / "vq_pack_golden.npz")
CASES = [str(c) for c in G["cases"]]


@pytest.mark.parametrize("case", CASES)
def test_oracle_unpack_matches_reference(case):
    e, o, nsub, bits, wpr = (int(v) for v in G[f"{case}__meta"])
    packed = G[f"{case}__packed"]
    assert packed.shape == (e, o, wpr)
    assert orc.words_per_row(nsub, bits) == wpr
    assert np.array_equal(orc.unpack(packed, nsub, bits), G[f"{case}__codes"])
    assert np.array_equal(orc.unpack_numpy(packed, nsub, bits), G[f"{case}__codes"])


@pytest.mark.parametrize("case", CASES)
def test_oracle_pack_matches_reference(case):
    e, o, nsub, bits, wpr = (int(v) for v in G[f"{case}__meta"])
    assert np.array_equal(orc.pack(G[f"{case}__codes"], bits), G[f"{case}__packed"])


@pytest.mark.parametrize("case", CASES)
def test_product_vq_pack_matches_reference(case):
    e, o, nsub, bits, wpr = (int(v) for v in G[f"{case}__meta"])
    codes, packed = G[f"{case}__codes"], G[f"{case}__packed"]
    assert vq_pack.words_per_row(nsub, bits) == wpr
    assert vq_pack.packed_bytes(e, o, nsub, bits) == packed.nbytes
    assert np.array_equal(vq_pack.pack(codes, bits), packed)
    back = vq_pack.unpack(packed, nsub, bits)
    assert back.dtype == (np.uint8 if bits <= 8 else np.uint16)
    assert np.array_equal(back.astype(np.uint16), codes)


def test_bits_for_k_matches_reference():
    for k, b in G["bits_for_k"]:
        assert vq_pack.bits_for_k(int(k)) == int(b)
    with pytest.raises(ValueError):
        vq_pack.bits_for_k(3000)


def test_pack_rejects_overwide_codes():
    with pytest.raises(ValueError):
        vq_pack.pack(np.array([[[16]]], dtype=np.uint16), 4)
    with pytest.raises(ValueError):
        vq_pack.unpack(np.zeros((1, 1, 5), dtype=np.uint32), 32, 4)


def test_t1_extraction_equivalence_all_lanes_all_bits():
    """T1: the per-lane two-word formula (the Metal VQ_CODE / the CUDA bit
    walker) agrees with the block reader for every lane and bits 1..16."""
    rng = np.random.default_rng(7)
    for bits in range(1, 17):
        words = rng.integers(0, 2 ** 32, size=(1, 1, 2 * bits), dtype=np.uint64).astype(np.uint32)
        a = orc.unpack(words, 64, bits)
        b = orc.unpack_numpy(words, 64, bits)
        c = vq_pack.unpack(words, 64, bits).astype(np.uint16)
        assert np.array_equal(a, b) and np.array_equal(a, c), bits
