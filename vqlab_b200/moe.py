"""The MoE block that calls the VQ experts: router top-k, SwiGLU, combine.

This is the caller of VQSwitchLinear in the reference's serving stack (mlx_lm
SwitchGLU / the Qwen3.5-MoE block, restated by the reference as the numpy
`ref_moe`, tests/test_qwen3_5_parity.py:180-204, with the router convention
of family/qwen3_5.py:110-118): fp32 softmax over the router logits, top-k,
weights always renormalised, gate and up projections of each (token, slot)
pair, h = silu(gate) * up, the down projection, and the weighted sum over
the k slots.  Only the three projections are VQ kernels; the rest is small
elementwise work on [T, k, ...] tensors.
"""
from __future__ import annotations

import torch

from .vq_switch import VQSwitchLinear


def route(router_logits: torch.Tensor, top_k: int):
    """fp32 softmax, top-k, renormalise.  Returns (indices int32 [T,k], weights fp32 [T,k])."""
    pr = torch.softmax(router_logits.float(), dim=-1)
    w, idx = torch.topk(pr, top_k, dim=-1, sorted=True)
    w = w / w.sum(dim=-1, keepdim=True)
    return idx.to(torch.int32), w


class VQMoEBlock(torch.nn.Module):
    """gate_proj / up_proj: [E, I, H] experts; down_proj: [E, H, I]."""

    def __init__(self, gate_proj: VQSwitchLinear, up_proj: VQSwitchLinear, down_proj: VQSwitchLinear,
                 top_k: int):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self.top_k = int(top_k)

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """x [T, H] (bf16), router_logits [T, E] -> y [T, H] in x's dtype."""
        T, H = x.shape
        idx, w = route(router_logits, self.top_k)
        xe = x.reshape(T, 1, 1, H)
        g = self.gate_proj(xe, idx)                       # [T, k, 1, I]
        u = self.up_proj(xe, idx)
        h = (torch.nn.functional.silu(g.float()) * u.float()).to(x.dtype)
        d = self.down_proj(h, idx)                        # [T, k, 1, H]
        y = (d.float().squeeze(2) * w.unsqueeze(-1)).sum(dim=1)
        return y.to(x.dtype)
