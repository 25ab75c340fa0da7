"""vq_pack v1 packed-code format: host writer/reader and the device reader.

Same API and byte layout as the reference's src/vqlab/runtime/vq_pack.py
(bits_for_k :34, words_per_row :41, pack :48, unpack :79, packed_bytes :100),
implemented differently: a packed row is read here as what it is, an
LSB-first bit stream in which code j occupies bits [j*BITS, (j+1)*BITS)
(32 codes fill exactly BITS words, so the reference's blocks of 32 are this
stream cut at word boundaries; the tail block is zero-padded).  The host
writer expands codes to bits and lets numpy pack them little-endian; the
device reader is the vqb_unpack kernel.
"""
from __future__ import annotations

import ctypes

import numpy as np

BLOCK = 32  # codes per block: 32 codes * BITS bits == BITS whole words


def bits_for_k(k: int) -> int:
    """Field width of a K-entry codebook (K must be a power of two)."""
    b = int(k - 1).bit_length()
    if (1 << b) != k:
        raise ValueError(f"K={k} is not a power of two")
    return b


def words_per_row(nsub: int, bits: int) -> int:
    """uint32 words per packed row: ceil(NSUB/32) blocks of BITS words."""
    return (nsub + BLOCK - 1) // BLOCK * bits


def packed_bytes(e: int, out: int, nsub: int, bits: int) -> int:
    return e * out * words_per_row(nsub, bits) * 4


def _rows_chunks(n_rows: int, row_elems: int, budget: int = 1 << 26):
    step = max(1, budget // max(1, row_elems))
    for r0 in range(0, n_rows, step):
        yield r0, min(n_rows, r0 + step)


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """[..., NSUB] integer codes -> [..., WPR] uint32 (the reference's [E, OUT, NSUB] included)."""
    codes = np.asarray(codes)
    if not 1 <= bits <= 16:
        raise ValueError(f"bits={bits} outside 1..16")
    if codes.size and int(codes.max()) >= (1 << bits):
        raise ValueError("code exceeds bit width")
    lead, nsub = codes.shape[:-1], codes.shape[-1]
    nsub_p = -(-nsub // BLOCK) * BLOCK
    flat = codes.reshape(-1, nsub).astype(np.uint32)
    rows = flat.shape[0]
    wpr = words_per_row(nsub, bits)
    out = np.zeros((rows, wpr), dtype=np.uint32)
    shifts = np.arange(bits, dtype=np.uint32)
    for r0, r1 in _rows_chunks(rows, nsub_p * bits):
        c = np.zeros((r1 - r0, nsub_p), dtype=np.uint32)
        c[:, :nsub] = flat[r0:r1]
        bitplane = ((c[:, :, None] >> shifts) & 1).astype(np.uint8).reshape(r1 - r0, nsub_p * bits)
        out[r0:r1] = np.packbits(bitplane, axis=-1, bitorder="little").view("<u4")
    return out.reshape(*lead, wpr)


def unpack(packed: np.ndarray, nsub: int, bits: int) -> np.ndarray:
    """Inverse of pack(): [..., WPR] uint32 -> [..., NSUB] (uint8 if bits <= 8 else uint16)."""
    packed = np.ascontiguousarray(packed, dtype="<u4")
    lead, wpr = packed.shape[:-1], packed.shape[-1]
    if wpr != words_per_row(nsub, bits):
        raise ValueError(f"packed rows are {wpr} words, expected {words_per_row(nsub, bits)} "
                         f"for NSUB={nsub}, bits={bits}")
    flat = packed.reshape(-1, wpr)
    rows = flat.shape[0]
    nsub_p = wpr // bits * BLOCK
    weights = (np.uint32(1) << np.arange(bits, dtype=np.uint32))
    out = np.empty((rows, nsub), dtype=np.uint8 if bits <= 8 else np.uint16)
    for r0, r1 in _rows_chunks(rows, nsub_p * bits):
        bitplane = np.unpackbits(flat[r0:r1].view(np.uint8), axis=-1, bitorder="little")
        vals = bitplane.reshape(r1 - r0, nsub_p, bits).astype(np.uint32) @ weights
        out[r0:r1] = vals[:, :nsub]
    return out.reshape(*lead, nsub)


def unpack_device(packed, nsub: int, bits: int):
    """Device reader: torch uint32-compatible CUDA tensor [..., WPR] -> int16-view
    uint16 codes [..., NSUB] (returned as torch.int32 for convenience of indexing)."""
    import torch

    from . import _lib

    if not packed.is_cuda:
        raise ValueError("unpack_device needs a CUDA tensor")
    packed = packed.contiguous()
    wpr = packed.shape[-1]
    if wpr != words_per_row(nsub, bits):
        raise ValueError(f"packed rows are {wpr} words, expected {words_per_row(nsub, bits)}")
    rows = packed.numel() // wpr
    out = torch.empty((*packed.shape[:-1], nsub), dtype=torch.int16, device=packed.device)
    st = _lib.lib().vqb_unpack(ctypes.c_void_p(packed.data_ptr()), rows, wpr, nsub, bits,
                               ctypes.c_void_p(out.data_ptr()),
                               ctypes.c_void_p(torch.cuda.current_stream(packed.device).cuda_stream))
    _lib.check(st, "vqb_unpack")
    return out.to(torch.int32) & 0xFFFF
