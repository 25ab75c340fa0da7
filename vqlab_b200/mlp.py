"""The dense model's MLP around three VQLinear projections, the caller of
VQLinear in the reference's serving stack (mlx_lm's MLP: down(silu(gate(x)) *
up(x)), each projection a VQLinear, src/vqlab/runtime/vq_dense.py:315-441).

Decode batches of d8 projections run the whole MLP as one library launch
(vqb_dense_mlp_forward: the fused block kernel with one expert and the dense
numerics -- bf16(fp16(cb * s)) weights for bf16 x, each projection's output
rounded once to x's dtype); everything else runs the three projections and
vqb_swiglu as separate calls.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .moe import swiglu
from .vq_dense import VQLinear
from .vq_switch import _DTYPES, _stream_ptr

# the fused launch decodes every weight once per 8 tokens, the per-step GEMM
# once per 128: the fused path is taken up to this many tokens
FUSED_MAX_TOKENS = 8


class VQDenseMLP(torch.nn.Module):
    """gate_proj / up_proj: VQLinear [I, H]; down_proj: VQLinear [H, I].

    fused: "auto" (one launch when the library serves the shape and x has at
    most FUSED_MAX_TOKENS rows), "on" (always the fused launch; ValueError when
    the shape is not served), "off" (the per-step calls)."""

    def __init__(self, gate_proj: VQLinear, up_proj: VQLinear, down_proj: VQLinear, fused: str = "auto"):
        super().__init__()
        if fused not in ("auto", "on", "off"):
            raise ValueError("fused must be 'auto', 'on' or 'off'")
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self.fused = fused

    def mlp_desc(self) -> _lib.DenseMlpDesc:
        d = _lib.DenseMlpDesc()
        d.gate, d.up, d.down = self.gate_proj.desc(), self.up_proj.desc(), self.down_proj.desc()
        return d

    def fused_status(self, n_tokens: int, dtype: torch.dtype = torch.bfloat16) -> int:
        """vqb_dense_mlp_supported at n_tokens rows (0 = served)."""
        if dtype not in (torch.bfloat16, torch.float16):
            return _lib.VQB_UNSUPPORTED_GEOMETRY
        d = self.mlp_desc()
        return int(_lib.lib().vqb_dense_mlp_supported(ctypes.byref(d), int(n_tokens), _DTYPES[dtype]))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [..., H] -> [..., H] in x's dtype."""
        lead, H = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, H)
        T = x2.shape[0]
        if self.fused != "off" and x.is_cuda and (self.fused == "on" or T <= FUSED_MAX_TOKENS):
            st = self.fused_status(T, x.dtype)
            if st == _lib.VQB_OK:
                return self.forward_fused(x2).reshape(*lead, -1)
            if self.fused == "on":
                raise ValueError(f"fused dense MLP: {_lib.status_string(st)}")
        return self.down_proj(swiglu(self.gate_proj(x2), self.up_proj(x2))).reshape(*lead, -1)

    def forward_fused(self, x: torch.Tensor, workspace: torch.Tensor | None = None,
                      options: _lib.MoeBlockOptions | None = None) -> torch.Tensor:
        """The MLP in one launch for x [T, H]; workspace / options as for
        VQMoEBlock.forward_fused."""
        T, H = x.shape
        x = x.contiguous()
        d = self.mlp_desc()
        L = _lib.lib()
        nbytes = int(L.vqb_dense_mlp_workspace_size(ctypes.byref(d), T))
        if workspace is None:
            ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
        else:
            if workspace.dtype != torch.uint8 or not workspace.is_cuda or workspace.numel() < nbytes:
                raise ValueError(f"workspace must be a uint8 CUDA tensor of >= {nbytes} bytes")
            ws = workspace
        y = torch.empty((T, self.down_proj.output_dims), dtype=x.dtype, device=x.device)
        _lib.check(L.vqb_dense_mlp_forward(ctypes.byref(d), ctypes.c_void_p(x.data_ptr()), _DTYPES[x.dtype], T,
                                           ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nbytes,
                                           ctypes.byref(options) if options is not None else None,
                                           _stream_ptr(x.device)), "vqb_dense_mlp_forward")
        return y
