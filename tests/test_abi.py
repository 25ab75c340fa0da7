"""The C ABI library loads, exports every function include/vqb.h declares,
and its host-side validation returns the reference's error classes without
touching a GPU (every case below is rejected before any CUDA call)."""
import ctypes
import pathlib
import re

import numpy as np
import pytest
import torch

from vqlab_b200 import _lib
from vqlab_b200 import VQLinear, VQSwitchLinear

HEADER = pathlib.Path(__file__).resolve().parent.parent / "include" / "vqb.h"


def declared_functions():
    src = HEADER.read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(vqb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_function():
    L = _lib.lib()
    names = declared_functions()
    assert names, "no declarations parsed"
    for n in names:
        assert hasattr(L, n), f"libvqb200.so does not export {n}"
    assert set(_lib.exported_symbols()) <= set(names)


def test_version_and_status_strings():
    assert "sm_100a" in _lib.version()
    assert "sharded" in _lib.status_string(_lib.VQB_CODEBOOK_SHARDED)
    assert _lib.status_string(_lib.VQB_OK) == "ok"


def _desc(**kw):
    d = _lib.LinearDesc()
    base = dict(num_experts=4, out_features=64, in_features=512, dim=8, num_codes=4096, group_size=64,
                pack_bits=12, code_bytes=0, expected_num_codes=4096, codes_last_dim=24,
                codes=0x1000, codebook=0x2000, scales=0x3000, row_table=None)
    base.update(kw)
    for k, v in base.items():
        setattr(d, k, v)
    return d


def _switch(d, n_tokens=1, top_k=2):
    L = _lib.lib()
    return L.vqb_switch_forward(ctypes.byref(d), ctypes.c_void_p(0x4000), _lib.VQB_BF16, n_tokens,
                                ctypes.c_void_p(0x5000), top_k, ctypes.c_void_p(0x6000), _lib.VQB_BF16,
                                ctypes.c_void_p(0x7000), 1 << 20, None, None)


@pytest.mark.parametrize("kw,status", [
    (dict(dim=3), _lib.VQB_UNSUPPORTED_GEOMETRY),
    (dict(pack_bits=17), _lib.VQB_UNSUPPORTED_GEOMETRY),
    (dict(codes_last_dim=23), _lib.VQB_BAD_WPR),
    (dict(num_codes=2048), _lib.VQB_CODEBOOK_SHARDED),
    (dict(in_features=500), _lib.VQB_BAD_SHAPE),
    (dict(group_size=60, in_features=480, codes_last_dim=0), _lib.VQB_BAD_SHAPE),
    (dict(pack_bits=10), _lib.VQB_BAD_SHAPE),        # 2^10 < K
    (dict(codes=None), _lib.VQB_NULL_POINTER),
    (dict(row_table=0x8000, num_rows=-1), _lib.VQB_BAD_SHAPE),
    (dict(codebook=0x2008), _lib.VQB_BAD_ALIGNMENT),
    (dict(pack_bits=0, code_bytes=1, num_codes=4096), _lib.VQB_BAD_SHAPE),
    (dict(pack_bits=0, code_bytes=3), _lib.VQB_UNSUPPORTED_GEOMETRY),
])
def test_switch_validation_statuses(kw, status):
    assert _switch(_desc(**kw)) == status


def test_zero_pairs_is_a_noop():
    assert _switch(_desc(), n_tokens=0) == _lib.VQB_OK


def test_workspace_too_small():
    L = _lib.lib()
    d = _desc()
    st = L.vqb_switch_forward(ctypes.byref(d), ctypes.c_void_p(0x4000), _lib.VQB_BF16, 1, ctypes.c_void_p(0x5000),
                              2, ctypes.c_void_p(0x6000), _lib.VQB_BF16, ctypes.c_void_p(0x7000), 8, None, None)
    assert st == _lib.VQB_WORKSPACE_TOO_SMALL


def test_status_to_exception_classes():
    with pytest.raises(ValueError):
        _lib.check(_lib.VQB_BAD_WPR)
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.VQB_UNSUPPORTED_GEOMETRY)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.VQB_CODEBOOK_SHARDED)


def _module(packed=True):
    E, OUT, IN, D, K = 2, 16, 128, 8, 256
    bits = 8
    codes = torch.zeros((E, OUT, (IN // D + 31) // 32 * bits), dtype=torch.int32)
    cb = torch.zeros((K, D), dtype=torch.float16)
    sc = torch.ones((E, OUT, IN // 64), dtype=torch.float16)
    return VQSwitchLinear(codes, cb, sc, group_size=64, pack_bits=bits, in_features=IN)


def test_module_properties_and_from_weights():
    m = _module()
    assert (m.input_dims, m.output_dims, m.num_experts) == (128, 16, 2)
    m2 = VQSwitchLinear.from_weights(m.codes, m.codebook, m.vq_scales)
    assert m2.pack_bits == 8 and m2.input_dims == 128
    with pytest.raises(ValueError):
        VQSwitchLinear(m.codes, m.codebook, m.vq_scales, pack_bits=8)  # no in_features
    with pytest.raises(ValueError, match="compact"):  # SKIPZERO needs compact 2-D codes / scales
        VQSwitchLinear(m.codes, m.codebook, m.vq_scales, pack_bits=8, in_features=128,
                       row_table=torch.zeros((2, 16), dtype=torch.int32))


def test_skipzero_module_properties():
    """SKIPZERO modules take E and OUT from the row table (vq_switch.py:5272-5282)."""
    m = _module()
    tbl = torch.full((2, 16), -1, dtype=torch.int32)
    tbl[0, :5] = torch.arange(5, dtype=torch.int32)
    sz = VQSwitchLinear(m.codes[0, :5].contiguous(), m.codebook, m.vq_scales[0, :5].contiguous(), pack_bits=8,
                        in_features=128, row_table=tbl)
    assert sz.skipzero and not m.skipzero
    assert (sz.input_dims, sz.output_dims, sz.num_experts) == (128, 16, 2)
    d = sz.desc()
    assert d.num_rows == 5 and d.row_table == tbl.data_ptr()
    with pytest.raises(ValueError, match="int32"):
        VQSwitchLinear(m.codes[0, :5].contiguous(), m.codebook, m.vq_scales[0, :5].contiguous(), pack_bits=8,
                       in_features=128, row_table=tbl.long())


def test_module_refuses_cpu_tensors():
    m = _module()
    x = torch.zeros((1, 1, 1, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        m(x, torch.zeros((1, 2), dtype=torch.int32))


def test_module_sharding_guard():
    m = _module()
    m.codebook = m.codebook[:128]
    with pytest.raises(RuntimeError, match="sharded"):
        m(torch.zeros((1, 1, 1, 128), dtype=torch.bfloat16), torch.zeros((1, 2), dtype=torch.int32))


def test_dense_module_properties():
    codes = torch.zeros((32, 64), dtype=torch.uint8)
    lin = VQLinear(codes, torch.zeros((256, 2), dtype=torch.float16), torch.ones((32, 2), dtype=torch.float16))
    assert (lin.input_dims, lin.output_dims) == (128, 32)
    with pytest.raises(ValueError):
        lin(torch.zeros((1, 128), dtype=torch.bfloat16))


def test_measurement_aids_host_side():
    """vqb_launch_count / vqb_time_next_kernel need no GPU for these paths:
    the count is readable, a half-armed timer is refused, NULL/NULL disarms."""
    L = _lib.lib()
    assert L.vqb_launch_count() >= 0
    assert L.vqb_time_next_kernel(ctypes.c_void_p(16), None) == 10  # VQB_NULL_POINTER
    assert L.vqb_time_next_kernel(None, ctypes.c_void_p(16)) == 10
    assert L.vqb_time_next_kernel(None, None) == 0


def test_dense_refuses_row_table():
    """SKIPZERO is a switch-layer format; a dense call with a row table is refused before any launch."""
    L = _lib.lib()
    d = _desc(num_experts=1, row_table=0x8000, num_rows=10)
    st = L.vqb_dense_forward(ctypes.byref(d), ctypes.c_void_p(0x4000), _lib.VQB_BF16, 1, ctypes.c_void_p(0x6000),
                             _lib.VQB_BF16, ctypes.c_void_p(0x7000), 1 << 20, None, None)
    assert st == _lib.VQB_UNSUPPORTED_GEOMETRY


def test_skipzero_row_table_from_mask():
    """Bit-packed live mask (little bit order) -> compact row per (expert, row), -1 dead."""
    from vqlab_b200.vq_switch import skipzero_row_table
    E, OUT = 3, 13
    rng = np.random.default_rng(0)
    live = rng.random((E, OUT)) < 0.6
    live[1] = False
    packed = np.packbits(np.pad(live, ((0, 0), (0, 16 - OUT))), axis=1, bitorder="little")
    tbl = skipzero_row_table(torch.from_numpy(packed), E, OUT).numpy()
    want = np.full((E, OUT), -1, np.int32)
    want[live] = np.arange(int(live.sum()), dtype=np.int32)
    assert tbl.dtype == np.int32 and np.array_equal(tbl, want)


def _ep_layout(**kw):
    base = dict(world=4, rank=1, tokens=16, top_k=4, hidden=512, experts_per_rank=2)
    base.update(kw)
    return _lib.EpLayout(*(base[n] for n, _ in _lib.EpLayout._fields_))


def test_peer_exchange_region_layout():
    """Region = 512-byte control block, then x rows, slots, weights, partials,
    each 256-byte aligned and sized for world * tokens rows."""
    L = _lib.lib()
    offs = (ctypes.c_size_t * 4)()
    n = L.vqb_ep_region_bytes(ctypes.byref(_ep_layout()), offs)
    R = 4 * 16
    assert list(offs) == [512, 512 + R * 512 * 2, 512 + R * 512 * 2 + R * 4 * 4, 512 + R * 512 * 2 + 2 * R * 4 * 4]
    assert n == offs[3] + R * 512 * 4
    assert all(o % 256 == 0 for o in offs)
    assert _lib.VQB_EP_STATUS_OFFSET + 4 <= 512


@pytest.mark.parametrize("kw", [dict(world=0), dict(world=9), dict(rank=4), dict(rank=-1), dict(tokens=0),
                                dict(top_k=0), dict(top_k=257), dict(hidden=12), dict(experts_per_rank=0)])
def test_peer_exchange_rejects_bad_layouts(kw):
    L = _lib.lib()
    lay = _ep_layout(**kw)
    assert L.vqb_ep_region_bytes(ctypes.byref(lay), None) == 0
    regions = (ctypes.c_void_p * 8)(*([256] * 8))
    st = L.vqb_ep_dispatch(ctypes.byref(lay), regions, ctypes.c_void_p(256), _lib.VQB_BF16, 1, ctypes.c_void_p(256),
                           ctypes.c_void_p(256), None, None)
    assert st == _lib.VQB_BAD_SHAPE
    assert L.vqb_ep_combine(ctypes.byref(lay), regions, ctypes.c_void_p(256), _lib.VQB_BF16, None, None) == \
        _lib.VQB_BAD_SHAPE
    assert L.vqb_ep_reduce(ctypes.byref(lay), ctypes.c_void_p(256), ctypes.c_void_p(256), _lib.VQB_BF16, 1,
                           None) == _lib.VQB_BAD_SHAPE


def test_peer_exchange_host_validation():
    """Null or unaligned regions, too many tokens and bad option phases are
    refused before any launch."""
    L = _lib.lib()
    lay = _ep_layout()
    null = (ctypes.c_void_p * 4)(256, None, 256, 256)
    assert L.vqb_ep_dispatch(ctypes.byref(lay), null, ctypes.c_void_p(256), _lib.VQB_BF16, 1, ctypes.c_void_p(256),
                             ctypes.c_void_p(256), None, None) == _lib.VQB_NULL_POINTER
    odd = (ctypes.c_void_p * 4)(256, 256 + 16, 256, 256)
    assert L.vqb_ep_combine(ctypes.byref(lay), odd, ctypes.c_void_p(256), _lib.VQB_BF16, None, None) == \
        _lib.VQB_BAD_ALIGNMENT
    bad_phase = _lib.EpOptions(7, 0)
    ok = (ctypes.c_void_p * 4)(256, 512, 768, 1024)
    assert L.vqb_ep_combine(ctypes.byref(lay), ok, ctypes.c_void_p(256), _lib.VQB_BF16, ctypes.byref(bad_phase),
                            None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_ep_reduce(ctypes.byref(lay), ctypes.c_void_p(256), ctypes.c_void_p(256), _lib.VQB_BF16, 17,
                           None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_ep_reduce(ctypes.byref(lay), ctypes.c_void_p(256), ctypes.c_void_p(256), _lib.VQB_BF16, 0,
                           None) == _lib.VQB_OK
    assert L.vqb_ep_region_alloc(ctypes.byref(lay), None) == _lib.VQB_NULL_POINTER
    assert L.vqb_ep_ipc_handle(None, None) == _lib.VQB_NULL_POINTER
    assert L.vqb_ep_ipc_close(None) == _lib.VQB_OK
    assert L.vqb_ep_region_free(None) == _lib.VQB_OK


def test_ep_block_exchange_argument():
    from vqlab_b200.ep import EPMoEBlock
    with pytest.raises(ValueError):
        EPMoEBlock(None, None, None, 2, num_experts=4, exchange="nvshmem")
    with pytest.raises(ValueError):
        EPMoEBlock(None, None, None, 2, num_experts=4, exchange="p2p")  # needs static_tokens


def test_codebook_halves_validation():
    """vqb_codebook_halves and the desc's codebook_halves field are checked on
    the host: D must be 8, pointers 16-byte aligned and non-null."""
    L = _lib.lib()
    assert L.vqb_codebook_halves(ctypes.c_void_p(256), 0, ctypes.c_void_p(256), None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_codebook_halves(None, 16, ctypes.c_void_p(256), None) == _lib.VQB_NULL_POINTER
    assert L.vqb_codebook_halves(ctypes.c_void_p(264), 16, ctypes.c_void_p(256), None) == _lib.VQB_BAD_ALIGNMENT
    d = _lib.LinearDesc(num_experts=2, out_features=16, in_features=64, dim=4, num_codes=256, group_size=64,
                        pack_bits=8, codes=256, codebook=256, scales=256, codebook_halves=256)
    y = ctypes.c_void_p(256)
    st = L.vqb_switch_forward(ctypes.byref(d), y, _lib.VQB_BF16, 1, y, 1, y, _lib.VQB_BF16, y, 1 << 20, None, None)
    assert st == _lib.VQB_BAD_SHAPE  # halves given for a d4 codebook
    d.dim, d.num_codes, d.codebook_halves = 8, 256, 264
    st = L.vqb_switch_forward(ctypes.byref(d), y, _lib.VQB_BF16, 1, y, 1, y, _lib.VQB_BF16, y, 1 << 20, None, None)
    assert st == _lib.VQB_BAD_ALIGNMENT


def test_router_validation():
    L = _lib.lib()
    p = ctypes.c_void_p(256)
    assert L.vqb_moe_route(p, 4, 512, 0, p, p, None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_route(p, 4, 512, 33, p, p, None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_route(p, 4, 8, 9, p, p, None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_route(p, 4, 9000, 8, p, p, None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_route(p, -1, 512, 8, p, p, None) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_route(None, 4, 512, 8, p, p, None) == _lib.VQB_NULL_POINTER
    assert L.vqb_moe_route(None, 0, 512, 8, None, None, None) == _lib.VQB_OK


def _block_desc(top_k=4, **kw):
    d = _lib.MoeBlockDesc()
    kw.setdefault("codebook_halves", 0x9000)
    d.gate = _desc(out_features=512, in_features=512, codes_last_dim=24, **kw)
    d.up = _desc(out_features=512, in_features=512, codes_last_dim=24, **kw)
    d.down = _desc(out_features=512, in_features=512, codes_last_dim=24, **kw)
    d.top_k = top_k
    return d


def test_moe_block_host_validation():
    """The fused block's shape checks, before any device query."""
    L = _lib.lib()
    d = _block_desc()
    d.down.in_features = 1024
    d.down.codes_last_dim = 48
    assert L.vqb_moe_block_supported(ctypes.byref(d), 4, _lib.VQB_BF16) == _lib.VQB_BAD_SHAPE  # down IN != I
    assert L.vqb_moe_block_supported(ctypes.byref(_block_desc(top_k=0)), 4, _lib.VQB_BF16) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_block_supported(ctypes.byref(_block_desc(top_k=5)), 4, _lib.VQB_BF16) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_block_supported(ctypes.byref(_block_desc()), 0, _lib.VQB_BF16) == _lib.VQB_BAD_SHAPE
    assert L.vqb_moe_block_supported(None, 4, _lib.VQB_BF16) == _lib.VQB_NULL_POINTER
    unsupported = _lib.VQB_UNSUPPORTED_GEOMETRY
    assert L.vqb_moe_block_supported(ctypes.byref(_block_desc()), 4, _lib.VQB_F32) == unsupported
    assert L.vqb_moe_block_supported(ctypes.byref(_block_desc()), 161, _lib.VQB_BF16) == unsupported  # > 640 pairs
    assert L.vqb_moe_block_supported(ctypes.byref(_block_desc(group_size=128)), 4, _lib.VQB_BF16) == unsupported
    assert L.vqb_moe_block_supported(ctypes.byref(_block_desc(codebook_halves=None)), 4, _lib.VQB_BF16) == unsupported
    # workspace: status block + fp32 partial slots + fp16 SwiGLU rows
    n = L.vqb_moe_block_workspace_size(ctypes.byref(_block_desc()), 4)
    assert n >= 256 + (4 * 64 * 512 + 2 * 64 * 512) * 4 + 16 * 512 * 2 + 4 * 512 * 2 + 2 * 16 * 4
