"""vqb_switch_forward_static: the expert decode call that allocates nothing.

It exists for callers that cannot give the library device memory (a host
program that only links the C ABI and owns no device allocator, or a serving
loop that forbids device allocation after start-up); its scratch is an
8 MiB array inside the library.  This file is collected last on purpose, and
it must also pass when it runs alone in a fresh process.

The check: through the C ABI, two calls in a row (different inputs, so the
second call runs on scratch the first one left behind) against the regular
workspace entry point, within the tolerance the other decode tests use
(2e-3 * max|ref| + 1 bf16 ULP), and, stored as fp32, against the CPU oracle
(max relative error <= 2e-3).  Three layouts of the scratch are used: x read
in place (16-byte aligned bf16 rows), x narrowed into the array first (a
misaligned x base), and a geometry the tensor-core kernel does not serve
(G = 32: the one-pair-per-CTA kernel, whose status word the call clears in the
array); an oversized call is refused.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vq_cases import make_layer, max_rel, skewed_routing, to_torch, within_tol_bf16
from vqlab_b200 import VQSwitchLinear, _lib

pytestmark = pytest.mark.gpu


def _call_static(m, x2, idx, k, y, y_dtype=_lib.VQB_BF16):
    d = m.desc()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return _lib.lib().vqb_switch_forward_static(
        ctypes.byref(d), ctypes.c_void_p(x2.data_ptr()), _lib.VQB_BF16, x2.shape[0],
        ctypes.c_void_p(idx.data_ptr()), k, ctypes.c_void_p(y.data_ptr()), y_dtype, None, stream)


def _x_rows(T, IN, vals, aligned):
    """bf16 x [T, IN] holding vals; aligned=False puts its base 2 bytes past a
    16-byte boundary (the kernel cannot read it in place)."""
    if aligned:
        return torch.from_numpy(vals).to(torch.bfloat16).cuda()
    buf = torch.empty(T * IN + 8, dtype=torch.bfloat16, device="cuda")
    x = buf[1:1 + T * IN].view(T, IN)
    x.copy_(torch.from_numpy(vals).to(torch.bfloat16))
    assert x.data_ptr() % 16 != 0
    return x


@pytest.mark.parametrize("case", ["aligned", "misaligned_x", "per_pair_kernel"])
def test_static_scratch_matches_workspace_call_twice(case):
    E, OUT, IN, k = 16, 512, 1024, 8
    G = 32 if case == "per_pair_kernel" else 64
    L = make_layer(E=E, OUT=OUT, IN=IN, D=8, K=16384, G=G, seed=5)
    codes, cb, sc = to_torch(L)
    m = VQSwitchLinear(codes, cb, sc, group_size=G, pack_bits=L.bits, in_features=IN)
    rng = np.random.default_rng(6)
    for call, T in enumerate((12, 40)):
        idx_np = skewed_routing(T, k, E, seed=call)
        idx = torch.from_numpy(idx_np.astype(np.int32)).cuda()
        vals = orc.round_bf16(rng.standard_normal((T, IN)).astype(np.float32))
        x = _x_rows(T, IN, vals, aligned=(case != "misaligned_x"))
        ref = m(x.reshape(T, 1, 1, IN), idx).reshape(T * k, OUT)
        y = torch.full((T * k, OUT), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = _call_static(m, x, idx, k, y)
        assert st == _lib.VQB_OK, _lib.status_string(st)
        y32 = torch.full((T * k, OUT), float("nan"), dtype=torch.float32, device="cuda")
        st = _call_static(m, x, idx, k, y32, _lib.VQB_F32)
        assert st == _lib.VQB_OK, _lib.status_string(st)
        torch.cuda.synchronize()
        a = ref.float().cpu().numpy()
        b = y.float().cpu().numpy()
        assert not np.isnan(b).any()
        assert within_tol_bf16(a, b), f"call {call}"
        oracle = orc.round_f16(orc.switch_fused(L.codes, L.cb_bits, L.sc_bits, orc.f16_bits(vals),
                                                idx_np.reshape(-1), k))
        assert max_rel(oracle, y32.cpu().numpy()) <= 2e-3, f"call {call}"


def test_static_scratch_refuses_oversized_calls():
    E, OUT, IN, k = 4, 128, 4096, 8
    L = make_layer(E=E, OUT=OUT, IN=IN, D=8, K=4096, G=64, seed=7)
    codes, cb, sc = to_torch(L)
    m = VQSwitchLinear(codes, cb, sc, group_size=64, pack_bits=L.bits, in_features=IN)
    T = 2048  # 2048 rows x 4096 fp16 = 16 MiB > 8 MiB
    x = torch.zeros((T, IN), dtype=torch.bfloat16, device="cuda")
    idx = torch.zeros((T, k), dtype=torch.int32, device="cuda")
    y = torch.empty((T * k, OUT), dtype=torch.bfloat16, device="cuda")
    assert _call_static(m, x, idx, k, y) == _lib.VQB_WORKSPACE_TOO_SMALL
