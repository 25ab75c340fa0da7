"""SKIPZERO row tables (vq_switch.py:5205-5216): a VQSwitchLinear over COMPACT
live rows plus an [E, OUT] row table must be BYTE-EQUAL to the same module over
EXPANDED rows (dead rows = code 0, scale +0) -- the reference's own
correctness claim (tests/test_vq_skipzero.py:83-113) -- at decode N (the
expert-grouped decode kernel and the per-pair kernel) and at prefill N (the
grouped tcgen05 GEMM), with skewed routing, a whole dead expert, a fully live
expert and odd OUT."""
import numpy as np
import pytest
import torch

from oracle import oracle as orc
from vqlab_b200 import VQSwitchLinear
from vqlab_b200.vq_switch import make_options

pytestmark = pytest.mark.gpu


def _mk(E, OUT, IN, K, packed, dead_frac, D, seed=0):
    r = np.random.default_rng(seed)
    G = 64
    codes = r.integers(0, K, (E, OUT, IN // D)).astype(np.uint16 if K > 256 else np.uint8)
    cb = (r.standard_normal((K, D)) * 0.05).astype(np.float16)
    sc = (r.standard_normal((E, OUT, IN // G)) * 0.1 + 1).astype(np.float16)
    live = r.random((E, OUT)) >= dead_frac
    live[1, :] = False   # one whole dead expert
    live[2, :] = True    # one fully live expert
    codes[~live] = 0     # the expanded form
    sc[~live] = 0
    tbl = np.full((E, OUT), -1, np.int32)
    tbl[live] = np.arange(int(live.sum()), dtype=np.int32)
    cbt = torch.from_numpy(cb).cuda()
    if packed:
        bits = int(K - 1).bit_length()
        full = orc.pack(codes, bits).view(np.int32)
        mk = lambda c, s, **kw: VQSwitchLinear(torch.from_numpy(np.ascontiguousarray(c)).cuda(), cbt,  # noqa: E731
                                               torch.from_numpy(np.ascontiguousarray(s)).cuda(), group_size=G,
                                               pack_bits=bits, in_features=IN, **kw)
    else:
        full = codes
        mk = lambda c, s, **kw: VQSwitchLinear(torch.from_numpy(np.ascontiguousarray(c)).cuda(), cbt,  # noqa: E731
                                               torch.from_numpy(np.ascontiguousarray(s)).cuda(), group_size=G, **kw)
    return mk(full, sc), mk(full[live], sc[live], row_table=torch.from_numpy(tbl).cuda())


def _idx(T, top, E, seed=1):
    r = np.random.default_rng(seed)
    p = np.ones(E)
    p[0] = 10
    p /= p.sum()
    idx = r.choice(E, size=(T, top), p=p).astype(np.int32)
    idx[0, 0] = 1  # the dead expert gets traffic
    return torch.from_numpy(idx).cuda()


GEOMS = [("packed11", 4, 2048, True, 512, 96), ("packed8", 4, 256, True, 512, 96),
         ("u8", 4, 256, False, 512, 96),
         ("d8_gateup", 8, 16384, True, 2048, 97), ("d8_down", 8, 16384, True, 1024, 97)]


@pytest.mark.parametrize("name,D,K,packed,IN,OUT", GEOMS)
@pytest.mark.parametrize("T,top", [(1, 8), (2, 10), (3, 10), (52, 10), (100, 8), (700, 8)])
def test_sz_byte_equal_to_expanded(name, D, K, packed, IN, OUT, T, top):
    E = 8
    full, sz = _mk(E, OUT, IN, K, packed, dead_frac=0.4, D=D)
    assert sz.skipzero and not full.skipzero
    assert (sz.num_experts, sz.output_dims, sz.input_dims) == (full.num_experts, full.output_dims, full.input_dims)
    x = torch.from_numpy(np.random.default_rng(2).standard_normal((T, 1, 1, IN)).astype(np.float16)).cuda()
    idx = _idx(T, top, E)
    a, b = full(x, idx), sz(x, idx)
    assert a.shape == b.shape
    assert torch.equal(a.view(torch.int16), b.view(torch.int16)), name


@pytest.mark.parametrize("path,variant", [(1, 1), (2, 0)])
def test_sz_forced_paths(path, variant):
    """The per-pair kernel and the grouped GEMM at a decode-size batch."""
    E = 8
    full, sz = _mk(E, 97, 1024, 16384, True, dead_frac=0.5, D=8, seed=3)
    for m in (full, sz):
        m.options = make_options(path=path, decode_variant=variant)
    x = torch.from_numpy(np.random.default_rng(4).standard_normal((5, 1, 1, 1024)).astype(np.float32)).cuda()
    x = x.to(torch.bfloat16)
    idx = _idx(5, 10, E, seed=5)
    assert torch.equal(full(x, idx).view(torch.int16), sz(x, idx).view(torch.int16))


def test_sz_dead_rows_are_plus_zero_even_for_inf_input():
    """Dead rows read nothing: +0 whatever x holds (the expanded form would give NaN)."""
    E = 8
    _, sz = _mk(E, 96, 512, 4096, True, dead_frac=0.5, D=8, seed=6)
    tbl = sz.row_table.cpu().numpy()
    x = torch.full((3, 1, 1, 512), float("inf"), dtype=torch.float16).cuda()
    for T_idx in (torch.tensor([[1, 1], [1, 3], [4, 1]], dtype=torch.int32).cuda(),):
        y = sz(x, T_idx).float().cpu().numpy().reshape(3, 2, 96)
        for t in range(3):
            for j in range(2):
                e = int(T_idx[t, j])
                dead = tbl[e] < 0
                assert np.all(y[t, j, dead] == 0) and not np.any(np.signbit(y[t, j, dead]))


@pytest.mark.parametrize("name,D,K,packed,IN,OUT", GEOMS)
@pytest.mark.parametrize("T,top", [(1, 8), (3, 10), (100, 8)])
def test_sz_matches_oracle(name, D, K, packed, IN, OUT, T, top):
    """The compact-row module against the oracle's SKIPZERO restatement
    (oracle.switch_fused_rowtable): live rows within max relative error 2e-3
    of the walk accumulators (fp32 output, fp16 output rounding kept), dead
    rows exactly +0.  T = 100 x 8 pairs runs the grouped GEMM."""
    E, G = 8, 64
    r = np.random.default_rng(21)
    codes = r.integers(0, K, (E, OUT, IN // D)).astype(np.uint16)
    cb = (r.standard_normal((K, D)) * 0.05).astype(np.float16)
    sc = (r.standard_normal((E, OUT, IN // G)) * 0.1 + 1).astype(np.float16)
    live = r.random((E, OUT)) >= 0.4
    live[1, :] = False
    live[2, :] = True
    tbl = np.full((E, OUT), -1, np.int32)
    tbl[live] = np.arange(int(live.sum()), dtype=np.int32)
    ccomp, scomp = codes[live], sc[live]
    if packed:
        bits = int(K - 1).bit_length()
        store = orc.pack(ccomp, bits).view(np.int32)
        kw = dict(pack_bits=bits, in_features=IN)
    else:
        store = ccomp.astype(np.uint8 if K <= 256 else np.uint16)
        kw = {}
    sz = VQSwitchLinear(torch.from_numpy(np.ascontiguousarray(store)).cuda(), torch.from_numpy(cb).cuda(),
                        torch.from_numpy(np.ascontiguousarray(scomp)).cuda(), group_size=G,
                        row_table=torch.from_numpy(tbl).cuda(), **kw)
    x = np.random.default_rng(22).standard_normal((T, 1, 1, IN)).astype(np.float16)
    idx = _idx(T, top, E, seed=23)
    y = sz(torch.from_numpy(x).cuda(), idx, out_dtype=torch.float32).cpu().numpy().reshape(T * top, OUT)
    idx_np = idx.cpu().numpy().astype(np.uint32)
    ref = orc.round_f16(orc.switch_fused_rowtable(ccomp, cb.view(np.uint16), scomp.view(np.uint16),
                                                  x.reshape(T, IN).view(np.uint16), idx_np.reshape(-1), top, tbl))
    dead = ~live[idx_np.reshape(-1)]
    assert np.all(y[dead] == 0) and not np.any(np.signbit(y[dead]))
    from vq_cases import max_rel
    assert max_rel(ref, y) <= 2e-3
