"""Expert parallelism on two B200s: NCCL all-to-all dispatch/combine around
the rank-local VQ expert shards, checked against the single-GPU MoE block
holding every expert (same weights, same tokens).  Skipped on boxes with one
GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

E, H, I, K, T = 8, 512, 256, 4, 40


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _proj_np(rng, out, inn):
    from oracle import oracle as orc
    codes = rng.integers(0, 4096, (E, out, inn // 8)).astype(np.uint16)
    packed = orc.pack(codes, 12)
    cb = (rng.standard_normal((4096, 8)) * 0.02).astype(np.float16)
    sc = rng.uniform(0.5, 1.5, (E, out, inn // 64)).astype(np.float16)
    return packed, cb, sc


def _worker(rank, world, port, out_dir, static=None, exchange="nccl", tokens=T):
    import datetime
    import torch.distributed as dist
    from vqlab_b200 import VQSwitchLinear
    from vqlab_b200.ep import EPMoEBlock, shard_experts
    from vqlab_b200.moe import VQMoEBlock

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        rng = np.random.default_rng(2024)  # the same layer on every rank
        P = [_proj_np(rng, I, H), _proj_np(rng, I, H), _proj_np(rng, H, I)]

        def full(p, inn):
            c, cb, sc = p
            return VQSwitchLinear(torch.from_numpy(c.view(np.int32)).to(dev), torch.from_numpy(cb).to(dev),
                                  torch.from_numpy(sc).to(dev), group_size=64, pack_bits=12, in_features=inn)

        def shard(p, inn):
            c, cb, sc = p
            cs, ss = shard_experts(torch.from_numpy(c.view(np.int32)), torch.from_numpy(sc), rank, world)
            return VQSwitchLinear(cs.to(dev), torch.from_numpy(cb).to(dev), ss.to(dev), group_size=64, pack_bits=12,
                                  in_features=inn)

        single = VQMoEBlock(full(P[0], H), full(P[1], H), full(P[2], I), K)
        ep = EPMoEBlock(shard(P[0], H), shard(P[1], H), shard(P[2], I), K, num_experts=E, static_tokens=static,
                        exchange=exchange)
        g = torch.Generator().manual_seed(7 + rank)
        x = torch.randn((tokens + 3 * rank, H), generator=g).to(torch.bfloat16).to(dev)
        lg = torch.randn((tokens + 3 * rank, E), generator=g).to(dev)
        lg[:, 0] += 4.0 * rank  # rank 1's tokens lean on rank 0's experts
        y_ep = ep(x, lg)
        y_ref = single(x, lg)
        torch.cuda.synchronize()
        if static:
            # the fixed-shape path has no host synchronisation: it replays from a CUDA graph
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                y_g = ep(x, lg)
            gr.replay()
            torch.cuda.synchronize()
            assert torch.equal(y_g, y_ep)
            del gr
        if exchange == "p2p":
            ep._peer.check()  # no wait gave up
            ep.close()
        torch.save({"ep": y_ep.float().cpu(), "ref": y_ref.float().cpu()}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("static,exchange,tokens", [(None, "nccl", T), (64, "nccl", T), (64, "p2p", T),
                                                   (320, "p2p", 300)])
def test_ep_two_gpus_matches_single_gpu_block(tmp_path, static, exchange, tokens):
    """Every dispatch path: the dynamic one (exact split sizes read on the
    host), the fixed-shape decode path (all-gather, skipped pairs, fp32
    partial combine), which must also replay from a CUDA graph with its NCCL
    calls, and the same fixed-shape step over peer memory (IPC-mapped
    regions, no NCCL on the data path), also replayed from a graph -- at a
    decode batch (the decode kernel) and at a prefill-size batch (300 tokens
    per rank: the grouped GEMM on the gathered pairs, as bench.py's
    multi-GPU prefill leg runs it)."""
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), static, exchange, tokens), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        d = torch.load(tmp_path / f"r{r}.pt")
        ep, ref = d["ep"], d["ref"]
        assert ep.shape == ref.shape
        # same pairs through the same kernels; allow one bf16 ulp of the output for kernel-path differences
        tol = 2e-3 * ref.abs().max() + ref.abs() * 2.0 ** -7
        assert bool(((ep - ref).abs() <= tol).all())
