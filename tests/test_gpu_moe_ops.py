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


def _torch_route(lg, k):
    pr = torch.softmax(lg.float(), dim=-1)
    w, idx = torch.topk(pr, k, dim=-1, sorted=True)
    return idx.to(torch.int32), w / w.sum(dim=-1, keepdim=True)


@pytest.mark.parametrize("T,E,k", [(1, 512, 10), (64, 512, 10), (4096, 512, 10), (7, 600, 4), (33, 8, 1),
                                   (5, 64, 32), (3, 5000, 8)])
def test_router_kernel_matches_torch(T, E, k):
    """vqb_moe_route (one kernel) against torch softmax / topk / renormalise:
    the same experts in the same order, weights within a few fp32 ulp (the
    softmax and selected sums are added in another order)."""
    from vqlab_b200.moe import route
    g = torch.Generator(device="cuda").manual_seed(T * E + k)
    lg = torch.randn((T, E), device="cuda", generator=g) * 2
    lg[:, 0] += 3.0  # a popular expert
    idx, w = route(lg, k)
    ridx, rw = _torch_route(lg, k)
    assert idx.dtype == torch.int32 and w.dtype == torch.float32
    assert torch.equal(idx, ridx)
    assert torch.allclose(w, rw, rtol=2e-6, atol=1e-9)
    assert torch.allclose(w.sum(-1), torch.ones(T, device="cuda"), rtol=1e-5)


def test_router_kernel_ties_take_the_lower_expert():
    from vqlab_b200.moe import route
    lg = torch.zeros((2, 64), device="cuda")
    lg[1, 40] = 1.0
    idx, w = route(lg, 4)
    assert idx[0].tolist() == [0, 1, 2, 3]
    assert idx[1].tolist() == [40, 0, 1, 2]
    assert torch.allclose(w[0], torch.full((4,), 0.25, device="cuda"))


@pytest.mark.parametrize("E,k", [(512, 10), (96, 8), (1000, 16)])
def test_router_kernel_ties_within_and_across_lanes(E, k):
    """Integer logits with many exact ties (equal logits give equal
    probabilities in any correct arithmetic): the experts come out in the
    order (larger probability, then the lower id) -- also when the tied
    entries sit in the same lane of the register router (ids 32 apart)."""
    from vqlab_b200.moe import route
    g = torch.Generator(device="cpu").manual_seed(E + k)
    T = 48
    lg = torch.randint(0, 4, (T, E), generator=g).float()
    lg[0, :] = 0.0
    lg[0, 64] = lg[0, 32] = lg[0, 0] = 2.0  # one lane (0) holds all three of the top entries
    idx, w = route(lg.cuda(), k)
    keys = lg.numpy()
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-keys[t, e], e))[:k]
        assert idx[t].tolist() == order, t
    assert torch.allclose(w.sum(-1), torch.ones(T, device="cuda"), rtol=1e-5)
