"""The peer-memory exchange (vqb_ep_dispatch / _combine / _reduce) on ONE GPU:
`world` ranks emulated by regions of the same device, every rank's write
phase launched before any rank's wait phase (so no launch waits on a later
one).  Checked against the NCCL fixed-shape path's arithmetic restated in
torch (vqb_moe_combine_partial per rank, rank-order sum, one rounding) --
byte-equal -- and against the single-GPU MoE block holding every expert."""
import numpy as np
import pytest
import torch

from vqlab_b200 import VQSwitchLinear, _lib
from vqlab_b200.ep import PeerExchange, shard_experts
from vqlab_b200.moe import VQMoEBlock, combine_partial, expert_mlp, route

pytestmark = pytest.mark.gpu

E, H, I, K, C = 8, 512, 256, 4, 16


def _layer(seed):
    from oracle import oracle as orc
    rng = np.random.default_rng(seed)

    def proj(out, inn):
        codes = rng.integers(0, 4096, (E, out, inn // 8)).astype(np.uint16)
        return (torch.from_numpy(orc.pack(codes, 12).view(np.int32)),
                torch.from_numpy((rng.standard_normal((4096, 8)) * 0.02).astype(np.float16)),
                torch.from_numpy(rng.uniform(0.5, 1.5, (E, out, inn // 64)).astype(np.float16)))
    return [proj(I, H), proj(I, H), proj(H, I)]


def _vq(codes, cb, sc, inn):
    return VQSwitchLinear(codes.cuda(), cb.cuda(), sc.cuda(), group_size=64, pack_bits=12, in_features=inn)


def _shards(P, r, W):
    out = []
    for (c, cb, sc), inn in zip(P, (H, H, I)):
        cs, ss = shard_experts(c, sc, r, W)
        out.append(_vq(cs, cb, ss, inn))
    return out


def _step(ex, shards, xs, routes):
    W = len(ex)
    for r in range(W):
        ex[r].dispatch(xs[r], *routes[r], phases=1)
    for r in range(W):
        ex[r].dispatch(xs[r], *routes[r], phases=2)
    ds = []
    for r in range(W):
        X = ex[r].x_rows.reshape(W * C, 1, 1, H)
        ds.append(expert_mlp(*shards[r], X, ex[r].slots).reshape(W * C, K, H))
    for r in range(W):
        ex[r].combine(ds[r], phases=1)
    for r in range(W):
        ex[r].combine(ds[r], phases=2)
    ys = [ex[r].reduce(xs[r].shape[0], torch.bfloat16) for r in range(W)]
    parts = [combine_partial(ds[r], ex[r].weights, ex[r].slots) for r in range(W)]
    return ys, ds, parts


@pytest.mark.parametrize("W", [1, 2, 4])
def test_emulated_exchange_matches_nccl_arithmetic_and_single_gpu(W):
    P = _layer(11)
    el = E // W
    shards = [_shards(P, r, W) for r in range(W)]
    full = VQMoEBlock(*(_vq(c, cb, sc, inn) for (c, cb, sc), inn in zip(P, (H, H, I))), K)
    ex = PeerExchange.emulated(W, C, K, H, el)
    try:
        for step in range(3):  # the epoch advances; rows from the step before must not leak
            g = torch.Generator().manual_seed(100 * step + W)
            Ts = [C - (3 * r + step) % C for r in range(W)]
            xs = [torch.randn((T, H), generator=g).to(torch.bfloat16).cuda() for T in Ts]
            lgs = [torch.randn((T, E), generator=g).cuda() for T in Ts]
            lgs[-1][:, 0] += 3.0  # the last rank leans on rank 0's experts
            routes = [route(lg, K) for lg in lgs]
            ys, ds, parts = _step(ex, shards, xs, routes)
            torch.cuda.synchronize()
            for r in range(W):
                assert ex[r].status() == _lib.VQB_OK
                # dispatched slots: rank r holds every rank's pairs, its own experts local, the rest skipped
                for s in range(W):
                    idx, w = routes[s]
                    T = Ts[s]
                    blk = ex[r].slots[s * C:(s + 1) * C].long()
                    mine = (idx.long() >= r * el) & (idx.long() < (r + 1) * el)
                    want = torch.where(mine, idx.long() - r * el, torch.full_like(idx.long(), -1))
                    assert torch.equal(blk[:T], want)
                    assert bool((blk[T:] == -1).all())
                    assert torch.equal(ex[r].weights[s * C:s * C + T], w)
                    rows = mine.any(dim=1)
                    assert torch.equal(ex[r].x_rows[s * C:s * C + T][rows], xs[s][rows])
            for o in range(W):
                acc = parts[0][o * C:(o + 1) * C]
                for r in range(1, W):
                    acc = acc + parts[r][o * C:(o + 1) * C]
                ref = acc[:Ts[o]].to(torch.bfloat16)
                assert torch.equal(ys[o].view(torch.int16), ref.view(torch.int16))
                single = full(xs[o], lgs[o]).float()
                tol = 2e-3 * single.abs().max() + single.abs() * 2.0 ** -7
                assert bool(((ys[o].float() - single).abs() <= tol).all())
    finally:
        ex[0].close()


def test_wait_gives_up_and_reports_timeout():
    """A rank whose peer never signals: the dispatch's wait ends after its
    limit (20 ms here), the status word reads VQB_TIMEOUT, the GPU context
    stays usable."""
    ex = PeerExchange.emulated(2, C, K, H, E // 2, wait_limit_us=20_000)
    try:
        x = torch.randn((C, H), device="cuda").to(torch.bfloat16)
        idx, w = route(torch.randn((C, E), device="cuda"), K)
        ex[0].dispatch(x, idx, w)  # both phases; rank 1 never dispatches
        torch.cuda.synchronize()
        assert ex[0].status() == _lib.VQB_TIMEOUT
        with pytest.raises(_lib.VQBError):
            ex[0].check()
        assert ex[1].status() == _lib.VQB_OK
        assert float((torch.ones(4, device="cuda") * 2).sum()) == 8.0
    finally:
        ex[0].close()
