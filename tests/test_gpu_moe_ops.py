"""Fused MoE elementwise kernels (vqb_swiglu, vqb_moe_combine) against the
plain PyTorch fp32 formulas they replace."""
import pytest
import torch

from vqlab_b200.moe import combine, swiglu

pytestmark = pytest.mark.gpu


def _ulp_close(a, b, dtype):
    """|a - b| within one unit in the last place of the output dtype (0 for fp32 within 2 ulp)."""
    a, b = a.float(), b.float()
    if dtype == torch.float32:
        return bool(torch.allclose(a, b, rtol=3e-7, atol=1e-30))
    eps = {torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}[dtype]
    return bool(((a - b).abs() <= eps * b.abs().clamp_min(2.0 ** -14) + 1e-30).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [8 * 1024, 1000 + 3])  # vector path, ragged scalar path
def test_swiglu_matches_torch(dtype, n):
    g = torch.Generator(device="cuda").manual_seed(n)
    a = (torch.randn(n, device="cuda", generator=g) * 4).to(dtype)
    b = torch.randn(n, device="cuda", generator=g).to(dtype)
    ref = (torch.nn.functional.silu(a.float()) * b.float()).to(dtype)
    got = swiglu(a, b)
    assert got.dtype == dtype and got.shape == a.shape
    assert _ulp_close(got, ref, dtype)


def test_swiglu_special_values():
    a = torch.tensor([0.0, -0.0, 80.0, -80.0, float("inf"), -float("inf"), 1e-30, 3.0], device="cuda")
    b = torch.ones_like(a)
    ref = torch.nn.functional.silu(a) * b
    got = swiglu(a, b)
    assert torch.equal(torch.isnan(got), torch.isnan(ref))
    m = ~torch.isnan(ref)
    assert torch.allclose(got[m], ref[m], rtol=3e-7, atol=0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("T,k,H", [(64, 10, 4096), (3, 1, 16), (5, 4, 24)])
def test_combine_matches_fp32_slot_sum(dtype, T, k, H):
    g = torch.Generator(device="cuda").manual_seed(T * k + H)
    d = torch.randn((T, k, H), device="cuda", generator=g).to(dtype)
    w = torch.softmax(torch.randn((T, k), device="cuda", generator=g), dim=-1)
    # slot order, each product rounded to fp32 (as the kernel)
    acc = torch.zeros((T, H), device="cuda")
    for j in range(k):
        acc = acc + d[:, j, :].float() * w[:, j:j + 1]
    ref = acc.to(dtype)
    got = combine(d, w)
    assert got.dtype == dtype and got.shape == (T, H)
    assert torch.equal(got, ref)


def test_empty_and_errors():
    e = torch.empty((0, 3, 8), device="cuda", dtype=torch.bfloat16)
    assert combine(e, torch.empty((0, 3), device="cuda")).shape == (0, 8)
    with pytest.raises(ValueError):
        swiglu(torch.ones(4, device="cuda"), torch.ones(5, device="cuda"))
    with pytest.raises(ValueError):
        combine(torch.ones((2, 3), device="cuda"), torch.ones((2, 3), device="cuda"))
