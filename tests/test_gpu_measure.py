"""The library's measurement aids on a B200: the launch counter counts our
kernels, and the one-shot timer brackets exactly the dominant kernel."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vqlab_b200 import VQSwitchLinear, _lib
from vq_cases import make_layer, to_torch

pytestmark = pytest.mark.gpu


def _layer():
    L = make_layer(E=8, OUT=256, IN=512, D=8, K=4096, G=64, seed=5)
    codes, cb, sc = to_torch(L)
    return L, VQSwitchLinear(codes, cb, sc, group_size=64, pack_bits=L.bits, in_features=512)


# decode: route + decode kernel (x converted while it is staged); GEMM: route + gather + GEMM
@pytest.mark.parametrize("T,launches", [(4, 2), (600, 3)])
def test_launch_count_and_kernel_timer(T, launches):
    L, m = _layer()
    rng = np.random.default_rng(T)
    idx = torch.from_numpy(rng.integers(0, 8, (T, 2)).astype(np.int32)).cuda()
    x = torch.from_numpy(rng.standard_normal((T, 1, 1, 512)).astype(np.float32)).cuda().to(torch.bfloat16)
    m(x, idx)
    torch.cuda.synchronize()
    c0 = _lib.launch_count()
    y = m(x, idx)
    torch.cuda.synchronize()
    assert _lib.launch_count() - c0 == launches
    s = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    b.record(s)
    torch.cuda.synchronize()
    _lib.time_next_kernel(a, b)
    y2 = m(x, idx)
    torch.cuda.synchronize()
    assert a.elapsed_time(b) > 0.0
    assert torch.equal(y, y2)
    # the timer is one-shot: a further call leaves the events alone
    t = a.elapsed_time(b)
    m(x, idx)
    torch.cuda.synchronize()
    assert a.elapsed_time(b) == t


def test_switch_path_query_names_the_kernel():
    """vqb_switch_path reports the family the call runs: the forced paths, and
    AUTO's choice for a d8/K16384 layer (the GEMM at any batch)."""
    L, m = _layer()
    from vqlab_b200.vq_switch import make_options
    m.options = make_options(path=1)
    assert m.kernel_path(600, 2) == "decode"
    m.options = make_options(path=2)
    assert m.kernel_path(4, 2) == "gemm"
    big = make_layer(E=4, OUT=128, IN=512, D=8, K=16384, G=64, seed=6)
    codes, cb, sc = to_torch(big)
    mb = VQSwitchLinear(codes, cb, sc, group_size=64, pack_bits=big.bits, in_features=512)
    assert mb.kernel_path(1, 10) == "gemm"
    assert mb.kernel_path(8, 10) == "gemm"
    assert m.kernel_path(4, 2) == "gemm"  # forced
    m.options = None
    assert m.kernel_path(4, 2) == "decode"  # K4096 fits shared memory: decode up to 512 pairs
    # the count of launches of one call matches the family: GEMM = route + gather + GEMM (+ the split-K
    # reduction when the call has few tiles); the d8 codebook's halves were built once by the first call
    x = torch.zeros((8, 1, 1, 512), dtype=torch.bfloat16, device="cuda")
    idx = torch.arange(80, device="cuda", dtype=torch.int32).reshape(8, 10) % 4
    mb(x, idx)
    torch.cuda.synchronize()
    c0 = _lib.launch_count()
    mb(x, idx)
    torch.cuda.synchronize()
    assert _lib.launch_count() - c0 in (3, 4)
