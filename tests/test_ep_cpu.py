"""Expert-parallel dispatch / combine on CPU: world_size-2 gloo ranks.

The expert compute is a float64 dense SwiGLU per expert (the VQ kernels need
a GPU); what is under test is the host logic of vqlab_b200.ep -- routing,
the stable order by owning rank, the count exchange, both all-to-alls and the
combine -- against the same pairs computed on one process.  With float64
experts the per-pair arithmetic is the same up to BLAS blocking, so the
results agree to ~1e-12.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vqlab_b200.ep import EPMoEBlock, dispatch_plan
from vqlab_b200.moe import route

E, H, I, K = 8, 16, 12, 3


def _weights():
    g = torch.Generator().manual_seed(1234)
    Wg = torch.randn((E, I, H), generator=g, dtype=torch.float64)
    Wu = torch.randn((E, I, H), generator=g, dtype=torch.float64)
    Wd = torch.randn((E, H, I), generator=g, dtype=torch.float64)
    return Wg, Wu, Wd


def _expert_rows(x, e, W):
    """SwiGLU expert e (global ids) on rows x: [R, H] -> [R, H]."""
    Wg, Wu, Wd = W
    g = torch.einsum("rih,rh->ri", Wg[e], x)
    u = torch.einsum("rih,rh->ri", Wu[e], x)
    return torch.einsum("rhi,ri->rh", Wd[e], torch.nn.functional.silu(g) * u)


def _reference(x, logits, W):
    T = x.shape[0]
    idx, w = route(logits, K)
    xp = x.repeat_interleave(K, dim=0)
    yp = _expert_rows(xp, idx.reshape(-1).long(), W).reshape(T, K, H)
    return (yp.float() * w.unsqueeze(-1)).sum(dim=1).to(x.dtype)


def _inputs(rank, T, skew):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn((T, H), generator=g, dtype=torch.float64)
    logits = torch.randn((T, E), generator=g)
    if skew:
        logits[:, : E // 2] += 50.0  # every pair to rank 0's experts
    return x, logits


def _worker(rank, world, port, out_dir, sizes, skew, static=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W = _weights()
        n = E // world

        def experts(xp, local):
            return _expert_rows(xp, local.long() + rank * n, W)

        blk = EPMoEBlock(None, None, None, top_k=K, num_experts=E, experts=experts, static_tokens=static)
        x, logits = _inputs(rank, sizes[rank], skew)
        y = blk(x, logits)
        ref = _reference(x, logits, W)
        try:
            EPMoEBlock(None, None, None, top_k=K, num_experts=E - 1, experts=experts)
            refused = False
        except ValueError:
            refused = True
        torch.save({"y": y, "ref": ref, "refused": refused}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("sizes,skew", [((5, 7), False), ((9, 0), False), ((6, 6), True)])
def test_ep_two_ranks_matches_single_process(tmp_path, sizes, skew):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), sizes, skew), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        d = torch.load(tmp_path / f"r{r}.pt")
        assert d["y"].shape == (sizes[r], H)
        assert torch.allclose(d["y"], d["ref"], rtol=1e-12, atol=1e-12)
        assert d["refused"]  # 7 experts do not split over 2 ranks


@pytest.mark.parametrize("sizes,skew", [((5, 7), False), ((0, 4), False), ((6, 6), True)])
def test_ep_static_path_matches_single_process(tmp_path, sizes, skew):
    """The fixed-shape decode path (all-gather, pairs of other ranks skipped,
    fp32 partial combine returned by one all-to-all): same pairs, the slot
    sums grouped by rank, so agreement is to fp32 rounding."""
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), sizes, skew, 8), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        d = torch.load(tmp_path / f"r{r}.pt")
        assert d["y"].shape == (sizes[r], H)
        tol = 1e-5 * float(d["ref"].abs().max()) if sizes[r] else 0.0
        assert torch.allclose(d["y"], d["ref"], rtol=1e-5, atol=tol)


def test_dispatch_plan_single_rank_orders_stably():
    idx = torch.tensor([[3, 1], [0, 2], [1, 3]], dtype=torch.int32)
    p = dispatch_plan(idx, experts_per_rank=4, world=1)
    assert p.order.tolist() == [0, 1, 2, 3, 4, 5]
    assert p.send_counts == [6] and p.recv_counts == [6]
    # one row per (token, destination): three tokens, each pair points at its token's row
    assert p.row_send == [3] and p.row_tok.tolist() == [0, 1, 2] and p.pair_row.tolist() == [0, 0, 1, 1, 2, 2]
