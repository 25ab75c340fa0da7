"""The MoE block that calls the VQ experts: router top-k, SwiGLU, combine.

This is the caller of VQSwitchLinear in the reference's serving stack (mlx_lm
SwitchGLU / the Qwen3.5-MoE block, restated by the reference as the numpy
`ref_moe`, tests/test_qwen3_5_parity.py:180-204, with the router convention
of family/qwen3_5.py:110-118): fp32 softmax over the router logits, top-k,
weights always renormalised, gate and up projections of each (token, slot)
pair, h = silu(gate) * up, the down projection, and the weighted sum over
the k slots.  The three projections are the VQ kernels; SwiGLU and the slot
combine are one fused library kernel each (vqb_swiglu, vqb_moe_combine).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .vq_switch import VQSwitchLinear, _DTYPES, _stream_ptr


def swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """dtype(silu(f32 g) * f32 u) in one pass (vqb_swiglu)."""
    if g.shape != u.shape or g.dtype != u.dtype or not g.is_cuda or g.dtype not in _DTYPES:
        raise ValueError("swiglu: gate and up must be CUDA tensors of one shape and a 16/32-bit float dtype")
    g, u = g.contiguous(), u.contiguous()
    h = torch.empty_like(g)
    _lib.check(_lib.lib().vqb_swiglu(ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(u.data_ptr()),
                                     ctypes.c_void_p(h.data_ptr()), g.numel(), _DTYPES[g.dtype], _stream_ptr(g.device)),
               "vqb_swiglu")
    return h


def combine(d: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y[t] = dtype(sum_j w[t, j] * f32 d[t, j]) for expert outputs d [T, k, H] (vqb_moe_combine)."""
    if d.dim() != 3 or w.shape != d.shape[:2] or not d.is_cuda or d.dtype not in _DTYPES:
        raise ValueError("combine: expects d [T, k, H] on CUDA and weights [T, k]")
    T, k, H = d.shape
    d = d.contiguous()
    w = w.to(torch.float32).contiguous()
    y = torch.empty((T, H), dtype=d.dtype, device=d.device)
    _lib.check(_lib.lib().vqb_moe_combine(ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                          ctypes.c_void_p(y.data_ptr()), T, k, H, _DTYPES[d.dtype],
                                          _stream_ptr(d.device)), "vqb_moe_combine")
    return y


# vqb_options.reuse flags (include/vqb.h)
REUSE_ROUTING = 1
REUSE_X = 2


def expert_mlp(gate_proj: VQSwitchLinear, up_proj: VQSwitchLinear, down_proj: VQSwitchLinear, xe: torch.Tensor,
               idx: torch.Tensor) -> torch.Tensor:
    """down(swiglu(gate(x), up(x))) for the pairs of idx [R, k] (x per token,
    xe [R, 1, 1, H]) -> [R, k, 1, H].  When the three projections run the
    grouped GEMM they share one workspace: gate routes and gathers x, up reuses
    both, down reuses the routing (VQB_REUSE_*)."""
    R, k = idx.shape
    if (gate_proj.kernel_path(R, k) == "gemm" and up_proj.kernel_path(R, k) == "gemm"
            and down_proj.kernel_path(R * k, 1) == "gemm"):
        nbytes = max(gate_proj.workspace_bytes(R, k), up_proj.workspace_bytes(R, k),
                     down_proj.workspace_bytes(R * k, 1))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=xe.device)
        g = gate_proj(xe, idx, workspace=ws)
        u = up_proj(xe, idx, workspace=ws, reuse=REUSE_ROUTING | REUSE_X)
        return down_proj(swiglu(g, u), idx, workspace=ws, reuse=REUSE_ROUTING)
    return down_proj(swiglu(gate_proj(xe, idx), up_proj(xe, idx)), idx)


def combine_partial(d: torch.Tensor, w: torch.Tensor, ids: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 partial combine for expert parallelism: out[t] = sum over the slots
    j with ids[t, j] != -1 (VQB_SKIP_EXPERT) of w[t, j] * f32 d[t, j], in slot
    order, no rounding (vqb_moe_combine_partial); a skipped slot's row of d is
    never read."""
    if d.dim() != 3 or w.shape != d.shape[:2] or not d.is_cuda or d.dtype not in _DTYPES:
        raise ValueError("combine_partial: expects d [T, k, H] on CUDA and weights [T, k]")
    T, k, H = d.shape
    d = d.contiguous()
    w = w.to(torch.float32).contiguous()
    if ids is not None:
        if ids.shape != (T, k):
            raise ValueError("combine_partial: ids must be [T, k]")
        ids = ids.to(torch.int32).contiguous()
    y = torch.empty((T, H), dtype=torch.float32, device=d.device)
    _lib.check(_lib.lib().vqb_moe_combine_partial(
        ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(w.data_ptr()),
        ctypes.c_void_p(ids.data_ptr()) if ids is not None else None, ctypes.c_void_p(y.data_ptr()), T, k, H,
        _DTYPES[d.dtype], _stream_ptr(d.device)), "vqb_moe_combine_partial")
    return y


def route(router_logits: torch.Tensor, top_k: int):
    """fp32 softmax, top-k, renormalise.  Returns (indices int32 [T,k], weights fp32 [T,k]).
    On CUDA one library kernel (vqb_moe_route); CPU tensors (the host-side
    expert-parallel tests) take the same steps as torch ops."""
    if router_logits.is_cuda and router_logits.dim() == 2 and 1 <= top_k <= min(32, router_logits.shape[1]) \
            and router_logits.shape[1] <= 8192:
        lg = router_logits.float().contiguous()
        T, E = lg.shape
        idx = torch.empty((T, top_k), dtype=torch.int32, device=lg.device)
        w = torch.empty((T, top_k), dtype=torch.float32, device=lg.device)
        _lib.check(_lib.lib().vqb_moe_route(ctypes.c_void_p(lg.data_ptr()), T, E, top_k,
                                            ctypes.c_void_p(idx.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                            _stream_ptr(lg.device)), "vqb_moe_route")
        return idx, w
    pr = torch.softmax(router_logits.float(), dim=-1)
    w, idx = torch.topk(pr, top_k, dim=-1, sorted=True)
    w = w / w.sum(dim=-1, keepdim=True)
    return idx.to(torch.int32), w


class VQMoEBlock(torch.nn.Module):
    """gate_proj / up_proj: [E, I, H] experts; down_proj: [E, H, I].

    fused: "auto" runs the whole block as one library launch
    (vqb_moe_block_forward) whenever the library serves the shape -- decode
    batches of d8 layers, n_tokens * top_k <= 640 -- and the per-step kernels
    otherwise; "on" requires the fused launch (ValueError when the shape is not
    served); "off" always runs the per-step kernels."""

    def __init__(self, gate_proj: VQSwitchLinear, up_proj: VQSwitchLinear, down_proj: VQSwitchLinear,
                 top_k: int, fused: str = "auto"):
        super().__init__()
        if fused not in ("auto", "on", "off"):
            raise ValueError("fused must be 'auto', 'on' or 'off'")
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self.top_k = int(top_k)
        self.fused = fused

    def block_desc(self) -> _lib.MoeBlockDesc:
        d = _lib.MoeBlockDesc()
        d.gate, d.up, d.down = self.gate_proj.desc(), self.up_proj.desc(), self.down_proj.desc()
        d.top_k = self.top_k
        return d

    def fused_status(self, n_tokens: int, dtype: torch.dtype = torch.bfloat16) -> int:
        """vqb_moe_block_supported for this block at n_tokens (0 = served)."""
        if dtype not in (torch.bfloat16, torch.float16):
            return _lib.VQB_UNSUPPORTED_GEOMETRY
        d = self.block_desc()
        return int(_lib.lib().vqb_moe_block_supported(ctypes.byref(d), int(n_tokens), _DTYPES[dtype]))

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """x [T, H] (bf16), router_logits [T, E] -> y [T, H] in x's dtype."""
        T, H = x.shape
        if self.fused != "off" and x.is_cuda and router_logits.is_cuda:
            st = self.fused_status(T, x.dtype)
            if st == _lib.VQB_OK:
                return self.forward_fused(x, router_logits)[0]
            if self.fused == "on":
                raise ValueError(f"fused MoE block: {_lib.status_string(st)}")
        idx, w = route(router_logits, self.top_k)
        return self.project(x, idx, w)

    def forward_fused(self, x: torch.Tensor, router_logits: torch.Tensor, workspace: torch.Tensor | None = None,
                      options: _lib.MoeBlockOptions | None = None):
        """The block in one launch: returns (y [T, H], indices int32 [T, k],
        weights fp32 [T, k]) -- the routing is vqb_moe_route's, bit for bit.
        workspace: optional uint8 CUDA tensor of at least
        vqb_moe_block_workspace_size bytes (its first 16 bytes are the call's
        status block); allocated per call when None.  options: vqb_moe_block_options
        (bounded-wait limit; the failure-path test knob)."""
        T, H = x.shape
        x = x.contiguous()
        lg = router_logits.to(torch.float32).contiguous()
        if lg.dim() != 2 or lg.shape[0] != T:
            raise ValueError("router_logits must be [T, E]")
        d = self.block_desc()
        L = _lib.lib()
        nbytes = int(L.vqb_moe_block_workspace_size(ctypes.byref(d), T))
        if workspace is None:
            ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
        else:
            if workspace.dtype != torch.uint8 or not workspace.is_cuda or workspace.numel() < nbytes:
                raise ValueError(f"workspace must be a uint8 CUDA tensor of >= {nbytes} bytes")
            ws = workspace
        y = torch.empty((T, H), dtype=x.dtype, device=x.device)
        idx = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        _lib.check(L.vqb_moe_block_forward(ctypes.byref(d), ctypes.c_void_p(lg.data_ptr()),
                                           ctypes.c_void_p(x.data_ptr()), _DTYPES[x.dtype], T,
                                           ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(idx.data_ptr()),
                                           ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nbytes,
                                           ctypes.byref(options) if options is not None else None,
                                           _stream_ptr(x.device)), "vqb_moe_block_forward")
        return y, idx, w

    def project(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """The three projections, SwiGLU and combine for given routing."""
        T, H = x.shape
        d = expert_mlp(self.gate_proj, self.up_proj, self.down_proj, x.reshape(T, 1, 1, H), idx)
        return combine(d.reshape(T, self.top_k, -1), w)
