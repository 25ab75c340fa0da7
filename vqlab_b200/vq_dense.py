"""VQLinear for PyTorch on B200: a bias-free dense linear whose weight is VQ-coded.

Drop-in for the reference module src/vqlab/runtime/vq_dense.py:315-441:
constructor (codes, codebook, vq_scales, group_size, pack_bits, in_features),
properties input_dims / output_dims, and `__call__(x) -> [*x.shape[:-1], OUT]`
in x's dtype.  codes are [OUT, WPR] uint32 (packed) or [OUT, NSUB] uint8 /
uint16.  The work is one call into libvqb200.so (vqb_dense_forward).
VQEmbedding is not part of the hot path and is not provided.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .vq_switch import _DTYPES, _code_meta, _stream_ptr


class VQLinear(torch.nn.Module):
    def __init__(self, codes, codebook, vq_scales, group_size: int = 64, pack_bits: int = 0,
                 in_features: int | None = None):
        super().__init__()
        if pack_bits and in_features is None:
            raise ValueError("packed codes need explicit in_features")
        self.register_buffer("codes", codes, persistent=True)
        self.register_buffer("codebook", codebook, persistent=True)
        self.register_buffer("vq_scales", vq_scales, persistent=True)
        self.group_size = int(group_size)
        self.pack_bits = int(pack_bits)
        self._in_features = in_features
        self._k_expect = int(codebook.shape[0])
        self._code_bytes = _code_meta(codes, self.pack_bits)
        self.options = None
        self._halves = _lib.CodebookHalves()  # d8: the GEMM's codebook layout, built once per codebook

    @property
    def input_dims(self) -> int:
        if self.pack_bits:
            return int(self._in_features)
        return int(self.codes.shape[-1]) * int(self.codebook.shape[1])

    @property
    def output_dims(self) -> int:
        return int(self.codes.shape[0])

    def desc(self) -> _lib.LinearDesc:
        d = _lib.LinearDesc()
        d.num_experts = 1
        d.out_features = self.output_dims
        d.in_features = self.input_dims
        d.dim = int(self.codebook.shape[1])
        d.num_codes = int(self.codebook.shape[0])
        d.group_size = int(self.input_dims // self.vq_scales.shape[-1])
        d.pack_bits = self.pack_bits
        d.code_bytes = self._code_bytes
        d.expected_num_codes = self._k_expect
        d.codes_last_dim = int(self.codes.shape[-1])
        d.codes = self.codes.data_ptr()
        d.codebook = self.codebook.data_ptr()
        d.scales = self.vq_scales.data_ptr()
        d.row_table = None
        d.codebook_halves = self._halves.pointer(self.codebook)
        return d

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """The reference call (vq_dense.py:346).  Extension: `out_dtype` stores y
        in another dtype than x's (float32 keeps the fp32 accumulators)."""
        if int(self.codebook.shape[0]) != self._k_expect:
            raise RuntimeError(
                f"VQ codebook was sharded: K={self.codebook.shape[0]}, expected {self._k_expect}. The "
                f"codebook is a SHARED lookup table and must be REPLICATED across tensor-parallel ranks.")
        for name in ("codes", "codebook", "vq_scales"):
            t = getattr(self, name)
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous CUDA tensor")
        if self.codebook.dtype != torch.float16 or self.vq_scales.dtype != torch.float16:
            raise ValueError("codebook and vq_scales must be float16")
        IN, OUT = self.input_dims, self.output_dims
        if x.shape[-1] != IN:
            raise ValueError(f"x last dim {x.shape[-1]} != in_features {IN}")
        if x.dtype not in _DTYPES:
            raise ValueError(f"x dtype {x.dtype} not supported")
        if not x.is_cuda or x.device != self.codes.device:
            raise ValueError("x must be a CUDA tensor on the module's device")
        xf = x.reshape(-1, IN).contiguous()
        n = xf.shape[0]
        ydt = x.dtype if out_dtype is None else out_dtype
        if ydt not in _DTYPES:
            raise ValueError(f"out_dtype {ydt} not supported")
        if out is None:
            y = torch.empty((n, OUT), dtype=ydt, device=x.device)
        else:
            y = out
            if y.shape != (n, OUT) or y.dtype != ydt or not y.is_contiguous():
                raise ValueError("out must be a contiguous [N, OUT] tensor of the output dtype")
        d = self.desc()
        optp = ctypes.byref(self.options) if self.options is not None else None
        L = _lib.lib()
        ws_bytes = L.vqb_dense_workspace_size(ctypes.byref(d), n, optp)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        st = L.vqb_dense_forward(ctypes.byref(d), ctypes.c_void_p(xf.data_ptr()), _DTYPES[x.dtype], n,
                                 ctypes.c_void_p(y.data_ptr()), _DTYPES[ydt], ctypes.c_void_p(ws.data_ptr()),
                                 ws_bytes, optp, _stream_ptr(x.device))
        _lib.check(st, "vqb_dense_forward")
        return y.reshape(*x.shape[:-1], OUT)
