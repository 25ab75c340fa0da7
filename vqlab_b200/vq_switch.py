"""VQSwitchLinear for PyTorch on B200: routed MoE experts over VQ codes.

Drop-in for the reference module src/vqlab/runtime/vq_switch.py:5194-5423:
same constructor (codes, codebook, vq_scales, group_size, pack_bits,
in_features, row_table), same `from_weights`, same properties (input_dims,
output_dims, num_experts) and the same call
`__call__(x, indices, sorted_indices=False) -> [*indices.shape, 1, OUT]` in
x's dtype.  Tensors are torch CUDA tensors; the work is one call into
libvqb200.so (include/vqb.h: vqb_switch_forward) on the current stream.
There is no CPU path: a CPU tensor is an error.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_DTYPES = {torch.float16: _lib.VQB_F16, torch.bfloat16: _lib.VQB_BF16, torch.float32: _lib.VQB_F32}


def _code_meta(codes: torch.Tensor, pack_bits: int):
    """(code_bytes for unpacked codes, 0 when packed)."""
    if pack_bits:
        if codes.element_size() != 4:
            raise ValueError("packed codes must be 32-bit words (uint32/int32)")
        return 0
    if codes.dtype in (torch.uint8, torch.int8):
        return 1
    if codes.dtype in (torch.int16, torch.uint16):
        return 2
    raise ValueError(f"unpacked codes must be uint8 or uint16, got {codes.dtype}")


def _stream_ptr(dev) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def make_options(path: int = 0, k_split: int = 0, max_fused_pairs: int = 0, decode_variant: int = 0,
                 stage_codebook: int = 0, pairs_per_chunk: int = 0):
    o = _lib.Options()
    o.path, o.k_split, o.max_fused_pairs = path, k_split, max_fused_pairs
    o.decode_variant, o.stage_codebook, o.pairs_per_chunk = decode_variant, stage_codebook, pairs_per_chunk
    return o


def skipzero_row_table(rowmask: torch.Tensor, num_experts: int, out_features: int) -> torch.Tensor:
    """SKIPZERO on-disk live mask -> row table (vq_switch.py:4958-4976).

    rowmask: uint8 [E, ceil(OUT/8)], bit i of byte b = row 8*b + i (little bit
    order).  Returns int32 [E, OUT]: the compact row of each live (expert, row)
    in (expert, row) order, -1 for dead rows.  Integer work only; runs on the
    mask's device."""
    E, OUT = int(num_experts), int(out_features)
    rm = rowmask.to(torch.int32).reshape(E, -1)
    bits = (rm[..., None] >> torch.arange(8, device=rm.device, dtype=torch.int32)) & 1
    live = bits.reshape(E, -1)[:, :OUT].reshape(-1)
    pos = torch.cumsum(live, 0, dtype=torch.int32) - 1
    return torch.where(live > 0, pos, torch.full_like(pos, -1)).to(torch.int32).reshape(E, OUT)


class VQSwitchLinear(torch.nn.Module):
    """Routed VQ experts (bias-free), reading vq_pack codes in place."""

    def __init__(self, codes, codebook, vq_scales, group_size: int = 64, pack_bits: int = 0,
                 in_features: int | None = None, row_table=None):
        super().__init__()
        if row_table is not None:
            # SKIPZERO (vq_switch.py:5205-5216): codes / vq_scales hold live rows
            # only ([NLIVE, W] / [NLIVE, NGRP]) and row_table [E, OUT] int32 maps
            # (expert, out row) -> compact row, -1 = dead; dead rows read no
            # bytes and produce +0.
            if codes.dim() != 2 or vq_scales.dim() != 2:
                raise ValueError("skipzero codes/vq_scales must be compact 2-D")
            if row_table.dim() != 2 or row_table.dtype != torch.int32:
                raise ValueError("row_table must be int32 [num_experts, out_features]")
            self.register_buffer("row_table", row_table, persistent=True)
        if pack_bits and in_features is None:
            raise ValueError("packed codes need explicit in_features: a packed row is WPR words wide, so "
                             "its shape no longer implies the input dimension")
        self.register_buffer("codes", codes, persistent=True)
        self.register_buffer("codebook", codebook, persistent=True)
        self.register_buffer("vq_scales", vq_scales, persistent=True)
        self.group_size = int(group_size)
        self.pack_bits = int(pack_bits)
        self._in_features = in_features
        # sharding guard (vq_switch.py:5225-5233): K at construction
        self._k_expect = int(codebook.shape[0])
        self._code_bytes = _code_meta(codes, self.pack_bits)
        self.options = None  # optional _lib.Options for tests / A-B runs
        self._halves = _lib.CodebookHalves()  # d8: the GEMM's codebook layout, built once per codebook

    @classmethod
    def from_weights(cls, codes, codebook, vq_scales):
        """Geometry from the tensors (vq_switch.py:5236-5248): packed codes are
        32-bit words, BITS = bit_length(K-1), IN = scales.shape[-1] * 64."""
        if codes.element_size() == 4:
            k = int(codebook.shape[0])
            bits = int(k - 1).bit_length()
            return cls(codes, codebook, vq_scales, pack_bits=bits, in_features=int(vq_scales.shape[-1]) * 64)
        return cls(codes, codebook, vq_scales)

    @property
    def skipzero(self) -> bool:
        return getattr(self, "row_table", None) is not None

    @property
    def input_dims(self) -> int:
        # derived from the current tensors, never cached (vq_switch.py:5254-5270)
        if self.pack_bits:
            return int(self.vq_scales.shape[-1]) * self.group_size
        return int(self.codes.shape[-1]) * int(self.codebook.shape[1])

    @property
    def output_dims(self) -> int:
        if self.skipzero:
            return int(self.row_table.shape[1])
        return int(self.codes.shape[1])

    @property
    def num_experts(self) -> int:
        if self.skipzero:
            return int(self.row_table.shape[0])
        return int(self.codes.shape[0])

    def desc(self) -> _lib.LinearDesc:
        d = _lib.LinearDesc()
        d.num_experts = self.num_experts
        d.out_features = self.output_dims
        d.in_features = self.input_dims
        d.dim = int(self.codebook.shape[1])
        d.num_codes = int(self.codebook.shape[0])
        d.group_size = self.group_size
        d.pack_bits = self.pack_bits
        d.code_bytes = self._code_bytes
        d.expected_num_codes = self._k_expect
        d.codes_last_dim = int(self.codes.shape[-1])
        d.codes = self.codes.data_ptr()
        d.codebook = self.codebook.data_ptr()
        d.scales = self.vq_scales.data_ptr()
        if self.skipzero:
            d.row_table = self.row_table.data_ptr()
            d.num_rows = int(self.codes.shape[0])
        else:
            d.row_table = None
            d.num_rows = 0
        d.codebook_halves = self._halves.pointer(self.codebook)
        return d

    def _check_tensors(self):
        k_now = int(self.codebook.shape[0])
        if k_now != self._k_expect:
            raise RuntimeError(
                f"VQ codebook was sharded: K={k_now}, expected {self._k_expect}. The codebook is a SHARED "
                f"lookup table and must be replicated across tensor-parallel ranks, not sliced.")
        for name in ("codes", "codebook", "vq_scales") + (("row_table",) if self.skipzero else ()):
            t = getattr(self, name)
            if not t.is_cuda:
                raise ValueError(f"{name} must be a CUDA tensor (the B200 runtime has no CPU path)")
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
        if self.codebook.dtype != torch.float16 or self.vq_scales.dtype != torch.float16:
            raise ValueError("codebook and vq_scales must be float16")
        if int(self.vq_scales.shape[-1]) * self.group_size != self.input_dims:
            raise ValueError("vq_scales last axis must be in_features / group_size")

    def kernel_path(self, n_tokens: int, top_k: int) -> str:
        """Which kernel family a call of n_tokens x top_k pairs runs on: "decode"
        (the fused small-N kernel) or "gemm" (the grouped tcgen05 GEMM), for
        fp16 / bf16 x (the library's AUTO rule, or the forced path in options)."""
        d = self.desc()
        opts = self.options
        r = _lib.lib().vqb_switch_path(ctypes.byref(d), int(n_tokens), int(top_k),
                                       ctypes.byref(opts) if opts is not None else None)
        if r < 0:
            _lib.check(-r, "vqb_switch_path")
        return "gemm" if r == 2 else "decode"

    def workspace_bytes(self, n_tokens: int, top_k: int) -> int:
        """Scratch bytes a call of n_tokens rows x top_k pairs each needs (vqb_switch_workspace_size)."""
        d = self.desc()
        opts = self.options
        return int(_lib.lib().vqb_switch_workspace_size(ctypes.byref(d), int(n_tokens), int(top_k),
                                                         ctypes.byref(opts) if opts is not None else None))

    def forward(self, x: torch.Tensor, indices: torch.Tensor, sorted_indices: bool = False,
                out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                reuse: int = 0, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """The reference call (vq_switch.py:5284).  Extensions for a block that
        runs several projections on one routing: `workspace` (a uint8 CUDA
        tensor of at least workspace_bytes) is used instead of a fresh one, and
        `reuse` (VQB_REUSE_* flags) tells the library that it already holds
        this call's routing tables / gathered x from the previous call.
        `out_dtype` stores y in another dtype than x's (float32 keeps the
        fp16-rounded result without the second rounding to x's dtype)."""
        self._check_tensors()
        IN = self.input_dims
        OUT = self.output_dims
        if x.shape[-1] != IN:
            raise ValueError(f"x last dim {x.shape[-1]} != in_features {IN}")
        if x.dtype not in _DTYPES:
            raise ValueError(f"x dtype {x.dtype} not supported")
        if not x.is_cuda or x.device != self.codes.device:
            raise ValueError("x must be a CUDA tensor on the module's device")
        idx = indices
        if idx.dtype not in (torch.int32, torch.uint32):
            idx = idx.to(torch.int32)
        idx = idx.contiguous()
        N = idx.numel()
        T = x.numel() // IN
        # xkrep (vq_switch.py:4438-4451, :5341): pair p reads token p // krep
        # when x holds one row per token and the pairs of a token are adjacent.
        if T == N:
            x2, krep = x.reshape(N, IN), 1
        elif T > 0 and N % T == 0 and tuple(x.shape[:-1]) in (
                tuple(idx.shape[:-1]) + (1, 1), tuple(idx.shape[:-1]) + (1,), tuple(idx.shape[:-1])):
            x2, krep = x.reshape(T, IN), N // T
        else:
            x2 = torch.broadcast_to(x, (*idx.shape, 1, IN)).reshape(N, IN)
            krep = 1
        x2 = x2.contiguous()
        ntok = x2.shape[0]
        ydt = x.dtype if out_dtype is None else out_dtype
        if ydt not in _DTYPES:
            raise ValueError(f"out_dtype {ydt} not supported")
        if out is None:
            y = torch.empty((N, OUT), dtype=ydt, device=x.device)
        else:
            y = out
            if y.shape != (N, OUT) or y.dtype != ydt or not y.is_contiguous():
                raise ValueError("out must be a contiguous [N, OUT] tensor of the output dtype")
        d = self.desc()
        opts = self.options
        if reuse:
            base = opts if opts is not None else _lib.Options()
            opts = _lib.Options.from_buffer_copy(base)
            opts.reuse = int(reuse)
        optp = ctypes.byref(opts) if opts is not None else None
        L = _lib.lib()
        ws_bytes = L.vqb_switch_workspace_size(ctypes.byref(d), ntok, krep, optp)
        if workspace is not None:
            if workspace.dtype != torch.uint8 or workspace.device != x.device or workspace.numel() < ws_bytes:
                raise ValueError(f"workspace must be a uint8 tensor of >= {ws_bytes} bytes on {x.device}")
            ws = workspace
        else:
            if reuse:
                raise ValueError("reuse needs the workspace of the call that routed")
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        st = L.vqb_switch_forward(ctypes.byref(d), ctypes.c_void_p(x2.data_ptr()), _DTYPES[x.dtype], ntok,
                                  ctypes.c_void_p(idx.data_ptr()), krep, ctypes.c_void_p(y.data_ptr()),
                                  _DTYPES[ydt], ctypes.c_void_p(ws.data_ptr()), ws_bytes, optp,
                                  _stream_ptr(x.device))
        _lib.check(st, "vqb_switch_forward")
        if os.environ.get("VQB_CHECK_ROUTING") == "1":
            if int(ws[:16].view(torch.int32)[1].item()) != 0:
                raise ValueError("an expert index was out of range for this VQSwitchLinear")
        return y.reshape(*indices.shape, 1, OUT)

    __call__ = torch.nn.Module.__call__
