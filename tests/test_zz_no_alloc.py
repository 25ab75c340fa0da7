"""vqb_switch_forward_static: the expert decode call that allocates nothing.

It exists for callers that cannot give the library device memory (a host
program that only links the C ABI and owns no device allocator, or a serving
loop that forbids device allocation after start-up); its scratch is an
8 MiB array inside the library.  This file is collected last on purpose, and
it must also pass when it runs alone in a fresh process.

The check: through the C ABI, two calls in a row (different inputs, so the
second call runs on scratch the first one left behind) against the regular
workspace entry point, within the tolerance the other decode tests use
(2e-3 * max|ref| + 1 bf16 ULP); an oversized call is refused.
"""
import ctypes

import numpy as np
import pytest
import torch

from vq_cases import make_layer, skewed_routing, to_torch, within_tol_bf16
from vqlab_b200 import VQSwitchLinear, _lib

pytestmark = pytest.mark.gpu


def _call_static(m, x2, idx, k, y):
    d = m.desc()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return _lib.lib().vqb_switch_forward_static(
        ctypes.byref(d), ctypes.c_void_p(x2.data_ptr()), _lib.VQB_BF16, x2.shape[0],
        ctypes.c_void_p(idx.data_ptr()), k, ctypes.c_void_p(y.data_ptr()), _lib.VQB_BF16, None, stream)


def test_static_scratch_matches_workspace_call_twice():
    E, OUT, IN, k = 16, 512, 1024, 8
    L = make_layer(E=E, OUT=OUT, IN=IN, D=8, K=16384, G=64, seed=5)
    codes, cb, sc = to_torch(L)
    m = VQSwitchLinear(codes, cb, sc, group_size=64, pack_bits=L.bits, in_features=IN)
    rng = np.random.default_rng(6)
    for call, T in enumerate((12, 40)):
        idx = torch.from_numpy(skewed_routing(T, k, E, seed=call).astype(np.int32)).cuda()
        x = torch.from_numpy(rng.standard_normal((T, IN)).astype(np.float32)).to(torch.bfloat16).cuda()
        ref = m(x.reshape(T, 1, 1, IN), idx).reshape(T * k, OUT)
        y = torch.full((T * k, OUT), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = _call_static(m, x, idx, k, y)
        assert st == _lib.VQB_OK, _lib.status_string(st)
        torch.cuda.synchronize()
        a = ref.float().cpu().numpy()
        b = y.float().cpu().numpy()
        assert not np.isnan(b).any()
        assert within_tol_bf16(a, b), f"call {call}"


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
