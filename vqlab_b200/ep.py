"""Expert parallelism for the VQ MoE block: experts sharded across ranks,
tokens dispatched to the rank that owns each routed expert and the expert
outputs combined back, one all-to-all each way per layer.

The reference runs every expert on one device (its multi-node path pipelines
whole layers, it never shards experts); the layer it computes is the
`ref_moe` block (tests/test_qwen3_5_parity.py:180-204): fp32 softmax router,
top-k, renormalised weights, per (token, slot) pair gate/up/down and the
weighted sum over slots.  EPMoEBlock computes the same pairs, only on the
rank that holds the pair's expert:

  rank r holds experts [r * E_local, (r + 1) * E_local)   (E_local = E / world)
  1. route locally: idx [T, k] global expert ids, weights [T, k]
  2. order the T*k pairs by destination rank (stable), exchange the per-rank
     pair and row counts (an all-to-all of 2 * `world` integers), then one
     all-to-all of token rows -- each token's row once per destination rank,
     however many of its slots that rank serves -- and one of the pairs'
     (row, local expert id) records; the receiver expands rows to pairs
  3. gate / up / SwiGLU / down on the received pairs (x given per pair)
  4. the reverse all-to-all returns each pair's output row to the rank that
     owns the token, which restores pair order and sums over the k slots.

The collectives are torch.distributed all_to_all_single (NCCL over NVLink on
B200 ranks; gloo for the CPU tests).  The expert compute is pluggable so the
dispatch/combine logic can be tested without a GPU: `experts(x_pairs [R, H],
local_ids [R]) -> y_pairs [R, H]`; the default runs the three VQSwitchLinear
projections of this rank.

Decode batches (at most `static_tokens` tokens per rank) take a fixed-shape
path with no host synchronisation, so a whole layer can be captured in a CUDA
graph:

  1. every rank pads its tokens to `static_tokens` rows and all-gathers the
     token rows, expert ids and weights (padding rows route nowhere);
  2. the pairs of this rank's experts keep their local id, every other pair
     is marked VQB_SKIP_EXPERT (-1): the projections run on all gathered
     pairs with no compaction and compute only this rank's;
  3. each token's slots on this rank are summed in fp32 (slot order,
     vqb_moe_combine_partial), an all-to-all of equal splits returns each
     token's partial sum to its owner, and the owner adds the ranks'
     partials in rank order and rounds once.

The all-gathered rows are world x static_tokens x H; for a decode batch that
is a few MB over NVLink.  The numerics differ from the single-GPU block only
in the fp32 summation order over slots (grouped by rank).

With exchange="p2p" the fixed-shape path moves the same data without NCCL
(PeerExchange, vqb_ep_* in include/vqb.h): every rank writes its rows, expert
slots and weights straight into the other ranks' exchange regions (CUDA IPC
mappings over NVLink), and writes each token's partial sum straight into the
owner's region, three library kernels per layer with the waits inside them.
The arithmetic is the NCCL path's (same slot sums, same rank-order sum).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib
from .moe import combine, expert_mlp, route
from .vq_switch import _DTYPES, _stream_ptr


@dataclass
class DispatchPlan:
    order: torch.Tensor        # [P] flat pair ids sorted by destination rank (stable)
    dest_counts: torch.Tensor  # [world] pairs this rank sends to each rank
    send_counts: list          # host copy of dest_counts
    recv_counts: list          # pairs this rank receives from each rank
    row_tok: torch.Tensor      # [Rs] token of each sent row (rows grouped by destination, tokens ascending)
    pair_row: torch.Tensor     # [P] row (within its destination's rows) of each sorted pair
    row_send: list             # rows this rank sends to each rank
    row_recv: list             # rows this rank receives from each rank


def dispatch_plan(idx: torch.Tensor, experts_per_rank: int, world: int, group=None) -> DispatchPlan:
    """Stable order of the flat (token, slot) pairs by owning rank, the
    deduplicated rows (one per (token, destination)), and the split sizes of
    the all-to-alls (one small all-to-all of counts, read on the host: the
    data all-to-alls need them as lists)."""
    T, k = idx.shape
    dest = idx.reshape(-1).long() // experts_per_rank
    order = torch.sort(dest, stable=True).indices
    counts = torch.bincount(dest, minlength=world)
    # rows: unique (destination, token), in (destination, token) order
    key = dest * T + torch.arange(T * k, device=idx.device) // k
    uniq, inv = torch.unique(key, sorted=True, return_inverse=True)
    row_dest = uniq // T
    row_counts = torch.bincount(row_dest, minlength=world)
    row_start = torch.cumsum(row_counts, 0) - row_counts
    # a sorted pair's row, numbered inside its destination's block
    pair_row = inv.index_select(0, order) - row_start.index_select(0, dest.index_select(0, order))
    if world > 1:
        # counts and row counts travel as one [world, 2] exchange
        send2 = torch.stack([counts, row_counts], dim=1).contiguous()
        recv2 = torch.empty_like(send2)
        dist.all_to_all_single(recv2, send2, group=group)
        rc, rr = recv2[:, 0], recv2[:, 1]
    else:
        rc, rr = counts, row_counts
    host = torch.cat([counts, row_counts, rc, rr]).tolist()
    return DispatchPlan(order=order, dest_counts=counts, send_counts=host[:world], recv_counts=host[2 * world:3 * world],
                        row_tok=uniq % T, pair_row=pair_row, row_send=host[world:2 * world],
                        row_recv=host[3 * world:])


def _a2a(t: torch.Tensor, out_rows: int, out_split, in_split, group) -> torch.Tensor:
    out = t.new_empty((out_rows,) + tuple(t.shape[1:]))
    dist.all_to_all_single(out, t.contiguous(), output_split_sizes=out_split, input_split_sizes=in_split, group=group)
    return out


class _DeviceBytes:
    """A raw device allocation seen by torch through __cuda_array_interface__
    (zero-copy; the owner keeps the memory alive)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 2, "strides": None}


class PeerExchange:
    """The exchange regions of one rank for the peer-memory fixed-shape path
    (vqb_ep_region_alloc / vqb_ep_ipc_* / vqb_ep_dispatch / _combine / _reduce).

    Set-up is collective over `group` (an all-gather of the 64-byte IPC
    handles and a barrier): every rank constructs its exchange at the same
    point, outside any CUDA graph capture.  `emulated(...)` builds `world`
    exchanges over regions of ONE GPU for single-GPU tests; each step then
    runs every rank's phase 1 before any rank's phase 2 (phases=1 / 2), so
    that no launch waits on a later one.
    """

    def __init__(self, tokens: int, top_k: int, hidden: int, experts_per_rank: int, dtype=torch.bfloat16,
                 device=None, group=None, wait_limit_us: int = 2_000_000, _regions=None, _rank=None, _world=None):
        L = _lib.lib()
        dev = torch.device(device) if device is not None else torch.device("cuda")
        self.device = dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())
        emulated = _regions is not None
        self.world = _world if emulated else (dist.get_world_size(group) if dist.is_initialized() else 1)
        self.rank = _rank if emulated else (dist.get_rank(group) if dist.is_initialized() else 0)
        if self.world > _lib.VQB_EP_MAX_WORLD:
            raise ValueError(f"peer exchange spans at most {_lib.VQB_EP_MAX_WORLD} ranks, got {self.world}")
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("peer exchange rows are bf16 or fp16")
        self.tokens, self.top_k, self.hidden, self.dtype = int(tokens), int(top_k), int(hidden), dtype
        self.group = group
        self.layout = _lib.EpLayout(self.world, self.rank, self.tokens, self.top_k, self.hidden, int(experts_per_rank))
        offs = (ctypes.c_size_t * 4)()
        self.nbytes = int(L.vqb_ep_region_bytes(ctypes.byref(self.layout), offs))
        if self.nbytes == 0:
            raise ValueError("peer exchange: invalid layout (world, tokens, top_k, hidden % 8, experts)")
        self._opened = []
        self._own = None
        if emulated:
            ptrs = list(_regions)
        else:
            own = ctypes.c_void_p()
            _lib.check(L.vqb_ep_region_alloc(ctypes.byref(self.layout), ctypes.byref(own)), "vqb_ep_region_alloc")
            self._own = own.value
            ptrs = [None] * self.world
            ptrs[self.rank] = self._own
            if self.world > 1:
                h = (ctypes.c_ubyte * _lib.VQB_EP_IPC_HANDLE_BYTES)()
                _lib.check(L.vqb_ep_ipc_handle(ctypes.c_void_p(self._own), h), "vqb_ep_ipc_handle")
                mine = torch.tensor(list(h), dtype=torch.uint8, device=self.device)
                every = torch.empty(self.world * mine.numel(), dtype=torch.uint8, device=self.device)
                dist.all_gather_into_tensor(every, mine, group=group)
                every = every.cpu().reshape(self.world, -1).tolist()
                for r in range(self.world):
                    if r == self.rank:
                        continue
                    hr = (ctypes.c_ubyte * _lib.VQB_EP_IPC_HANDLE_BYTES)(*every[r])
                    pr = ctypes.c_void_p()
                    _lib.check(L.vqb_ep_ipc_open(hr, ctypes.byref(pr)), "vqb_ep_ipc_open")
                    self._opened.append(pr.value)
                    ptrs[r] = pr.value
                dist.barrier(group=group)
        self._regions = (ctypes.c_void_p * self.world)(*ptrs)
        self._opts = {ph: _lib.EpOptions(ph, int(wait_limit_us)) for ph in (0, 1, 2, 3)}
        base = torch.as_tensor(_DeviceBytes(ptrs[self.rank], self.nbytes), device=self.device)
        R, k, H = self.world * self.tokens, self.top_k, self.hidden
        self.x_rows = base[offs[0]:offs[0] + R * H * 2].view(dtype).view(R, H)
        self.slots = base[offs[1]:offs[1] + R * k * 4].view(torch.int32).view(R, k)
        self.weights = base[offs[2]:offs[2] + R * k * 4].view(torch.float32).view(R, k)
        self.partials = base[offs[3]:offs[3] + R * H * 4].view(torch.float32).view(self.world, self.tokens, H)
        off = _lib.VQB_EP_STATUS_OFFSET
        self._status = base[off:off + 4].view(torch.int32)

    @classmethod
    def emulated(cls, world: int, tokens: int, top_k: int, hidden: int, experts_per_rank: int, dtype=torch.bfloat16,
                 wait_limit_us: int = 2_000_000):
        """`world` exchanges over regions on the current GPU (tests without peers)."""
        L = _lib.lib()
        lay = _lib.EpLayout(world, 0, tokens, top_k, hidden, experts_per_rank)
        regions = []
        for _ in range(world):
            p = ctypes.c_void_p()
            _lib.check(L.vqb_ep_region_alloc(ctypes.byref(lay), ctypes.byref(p)), "vqb_ep_region_alloc")
            regions.append(p.value)
        ex = [cls(tokens, top_k, hidden, experts_per_rank, dtype, device="cuda", wait_limit_us=wait_limit_us,
                  _regions=regions, _rank=r, _world=world) for r in range(world)]
        ex[0]._emulated_regions = regions
        return ex

    def dispatch(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, phases: int = 0) -> None:
        """x [T, H] (T <= tokens), idx [T, k] global expert ids, w [T, k] -> every rank's region."""
        T, H = x.shape
        if H != self.hidden or x.dtype != self.dtype or T > self.tokens or idx.shape != (T, self.top_k):
            raise ValueError(f"dispatch: x {tuple(x.shape)} {x.dtype}, idx {tuple(idx.shape)} do not fit the exchange "
                             f"(tokens {self.tokens}, hidden {self.hidden}, top_k {self.top_k}, {self.dtype})")
        x = x.contiguous()
        idx = idx.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        _lib.check(_lib.lib().vqb_ep_dispatch(ctypes.byref(self.layout), self._regions, ctypes.c_void_p(x.data_ptr()),
                                              _DTYPES[x.dtype], T, ctypes.c_void_p(idx.data_ptr()),
                                              ctypes.c_void_p(w.data_ptr()), ctypes.byref(self._opts[phases]),
                                              _stream_ptr(x.device)), "vqb_ep_dispatch")

    def combine(self, d: torch.Tensor, phases: int = 0) -> None:
        """d [world * tokens, top_k, hidden]: the projections' output for x_rows / slots."""
        if d.shape != (self.world * self.tokens, self.top_k, self.hidden) or d.dtype not in (torch.bfloat16,
                                                                                              torch.float16):
            raise ValueError(f"combine: expects [{self.world * self.tokens}, {self.top_k}, {self.hidden}] bf16/fp16")
        d = d.contiguous()
        _lib.check(_lib.lib().vqb_ep_combine(ctypes.byref(self.layout), self._regions, ctypes.c_void_p(d.data_ptr()),
                                             _DTYPES[d.dtype], ctypes.byref(self._opts[phases]),
                                             _stream_ptr(d.device)), "vqb_ep_combine")

    def reduce(self, n_tokens: int, dtype=None) -> torch.Tensor:
        """y [n_tokens, hidden]: this rank's tokens, the ranks' partials summed in rank order."""
        dtype = dtype or self.dtype
        y = torch.empty((n_tokens, self.hidden), dtype=dtype, device=self.device)
        _lib.check(_lib.lib().vqb_ep_reduce(ctypes.byref(self.layout), ctypes.c_void_p(self._regions[self.rank]),
                                            ctypes.c_void_p(y.data_ptr()), _DTYPES[dtype], n_tokens,
                                            _stream_ptr(self.device)), "vqb_ep_reduce")
        return y

    def status(self) -> int:
        """VQB_OK, or VQB_TIMEOUT once a wait in this rank's kernels gave up (synchronises)."""
        return int(self._status.item())

    def check(self) -> None:
        _lib.check(self.status(), "peer exchange")

    def close(self) -> None:
        """Collective: every rank stops using the peers' regions before any region is freed."""
        if self._regions is None:
            return
        torch.cuda.synchronize(self.device)
        L = _lib.lib()
        if self._own is not None and self.world > 1:
            dist.barrier(group=self.group)
        for p in self._opened:
            L.vqb_ep_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own is not None:
            if self.world > 1:
                dist.barrier(group=self.group)
            L.vqb_ep_region_free(ctypes.c_void_p(self._own))
            self._own = None
        for p in getattr(self, "_emulated_regions", []):
            L.vqb_ep_region_free(ctypes.c_void_p(p))
        self._emulated_regions = []
        self._regions = None


class EPMoEBlock(torch.nn.Module):
    """One MoE layer with its experts sharded over the ranks of `group`.

    gate_proj / up_proj / down_proj are this rank's VQSwitchLinear shards
    (E_local experts each); num_experts is the global E (E % world == 0).
    """

    def __init__(self, gate_proj, up_proj, down_proj, top_k: int, num_experts: int, group=None,
                 experts: Optional[Callable[[torch.Tensor, torch.Tensor], torch.Tensor]] = None,
                 static_tokens: Optional[int] = None, exchange: str = "nccl"):
        super().__init__()
        self.static_tokens = int(static_tokens) if static_tokens else None
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', not {exchange!r}")
        if exchange == "p2p" and not self.static_tokens:
            raise ValueError("exchange='p2p' serves the fixed-shape path: give static_tokens")
        self.exchange = exchange
        self._peer: Optional[PeerExchange] = None
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj
        self.top_k = int(top_k)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world != 0:
            raise ValueError(f"num_experts={num_experts} is not a multiple of the {self.world} ranks")
        self.num_experts = int(num_experts)
        self.experts_per_rank = self.num_experts // self.world
        if gate_proj is not None and gate_proj.num_experts != self.experts_per_rank:
            raise ValueError(f"rank shard holds {gate_proj.num_experts} experts, expected {self.experts_per_rank}")
        self._experts = experts if experts is not None else self._vq_experts

    def _vq_experts(self, xp: torch.Tensor, local: torch.Tensor) -> torch.Tensor:
        """gate/up/SwiGLU/down of R pairs (x per pair) on this rank's VQ shards."""
        R, H = xp.shape
        if R == 0:
            return xp.new_empty((0, self.down_proj.output_dims))
        ids = local.to(torch.int32).reshape(R, 1)
        return expert_mlp(self.gate_proj, self.up_proj, self.down_proj, xp.reshape(R, 1, 1, H), ids).reshape(R, -1)

    def _all_gather(self, t: torch.Tensor) -> torch.Tensor:
        out = t.new_empty((self.world * t.shape[0],) + tuple(t.shape[1:]))
        if self.world == 1:
            out.copy_(t)
        elif t.is_cuda:
            dist.all_gather_into_tensor(out, t.contiguous(), group=self.group)
        else:
            dist.all_gather(list(out.chunk(self.world)), t.contiguous(), group=self.group)
        return out

    def peer_exchange(self, hidden: int, dtype, device) -> PeerExchange:
        """This rank's PeerExchange (collective on first use, and again when
        static_tokens, the hidden size or the dtype changed: every rank makes
        it together)."""
        p = self._peer
        if p is not None and (p.tokens, p.hidden, p.dtype) != (self.static_tokens, hidden, dtype):
            self.close()
        if self._peer is None:
            self._peer = PeerExchange(self.static_tokens, self.top_k, hidden, self.experts_per_rank, dtype=dtype,
                                      device=device, group=self.group)
        return self._peer

    def close(self) -> None:
        """Release the peer exchange (collective); the NCCL path holds nothing.
        `last_pairs` may be views of the exchange region: dropped here."""
        if getattr(self, "last_pairs", None) is not None and self._peer is not None:
            self.last_pairs = None
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def _forward_p2p(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        C, k, W = self.static_tokens, self.top_k, self.world
        ex = self.peer_exchange(H, x.dtype, x.device)
        ex.dispatch(x, idx, w)
        X = ex.x_rows.reshape(W * C, 1, 1, H)
        self.last_pairs = (X, ex.slots)
        d = expert_mlp(self.gate_proj, self.up_proj, self.down_proj, X, ex.slots)
        ex.combine(d.reshape(W * C, k, -1))
        return ex.reduce(T, x.dtype)

    def forward_static(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """The fixed-shape path (module docstring): T <= static_tokens on every rank."""
        T, H = x.shape
        C, k, W, el = self.static_tokens, self.top_k, self.world, self.experts_per_rank
        if T > C:
            raise ValueError(f"{T} tokens exceed static_tokens={C}")
        idx, w = route(router_logits, k)
        if self.exchange == "p2p" and x.is_cuda and self._experts == self._vq_experts:
            return self._forward_p2p(x, idx, w)
        xp = x.new_zeros((C, H))
        xp[:T] = x
        ip = torch.full((C, k), -1, dtype=torch.int32, device=x.device)
        ip[:T] = idx
        wp = torch.zeros((C, k), dtype=torch.float32, device=x.device)
        wp[:T] = w
        X, I, Wt = self._all_gather(xp), self._all_gather(ip), self._all_gather(wp)
        lo = self.rank * el
        mine = (I >= lo) & (I < lo + el)
        ids = torch.where(mine, I - lo, torch.full_like(I, -1))      # -1 = VQB_SKIP_EXPERT
        self.last_pairs = (X.reshape(W * C, 1, 1, H), ids)          # this rank's pairs (kept for measurement)
        if X.is_cuda and self._experts == self._vq_experts:
            from .moe import combine_partial
            # [W*C, k, 1, H]; rows of skipped pairs are not written
            d = expert_mlp(self.gate_proj, self.up_proj, self.down_proj, X.reshape(W * C, 1, 1, H), ids)
            part = combine_partial(d.reshape(W * C, k, -1), Wt, ids)  # fp32 [W*C, H]
        else:
            # pluggable experts (CPU tests): every gathered pair computed, other ranks' masked out
            yp = self._experts(X.repeat_interleave(k, dim=0), ids.reshape(-1).clamp(min=0)).reshape(W * C, k, -1)
            part = torch.where(mine.unsqueeze(-1), yp.float() * Wt.unsqueeze(-1),
                               torch.zeros((), device=x.device)).sum(1)
        if W > 1:
            back = torch.empty_like(part)
            dist.all_to_all_single(back, part.contiguous(), group=self.group)
        else:
            back = part
        return back.reshape(W, C, -1).sum(0)[:T].to(x.dtype)

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """x [T, H], router_logits [T, E] (this rank's tokens) -> y [T, H] in x's dtype."""
        if self.static_tokens is not None and x.shape[0] <= self.static_tokens:
            return self.forward_static(x, router_logits)
        T, H = x.shape
        k = self.top_k
        idx, w = route(router_logits, k)
        plan = dispatch_plan(idx, self.experts_per_rank, self.world, self.group)
        flat = idx.reshape(-1).long()
        send_rows = x.index_select(0, plan.row_tok)            # one row per (token, destination)
        # per sorted pair: its row inside the destination's block, and its local expert
        send_meta = torch.stack([plan.pair_row, flat.index_select(0, plan.order) % self.experts_per_rank],
                                dim=1).to(torch.int32)
        n_recv = sum(plan.recv_counts)
        if self.world > 1:
            recv_rows = _a2a(send_rows, sum(plan.row_recv), plan.row_recv, plan.row_send, self.group)
            recv_meta = _a2a(send_meta, n_recv, plan.recv_counts, plan.send_counts, self.group)
        else:
            recv_rows, recv_meta = send_rows, send_meta
        # received pairs refer to rows of their source's block: offset by the block starts
        src_row0 = torch.tensor([0] + plan.row_recv[:-1], device=x.device).cumsum(0)
        src_of_pair = torch.repeat_interleave(torch.arange(self.world, device=x.device),
                                              torch.tensor(plan.recv_counts, device=x.device), output_size=n_recv)
        recv_x = recv_rows.index_select(0, recv_meta[:, 0].long() + src_row0.index_select(0, src_of_pair))
        recv_e = recv_meta[:, 1].contiguous()
        self.last_pairs = (recv_x.reshape(-1, 1, 1, H), recv_e.reshape(-1, 1))  # this rank's pairs (measurement)
        y_recv = self._experts(recv_x, recv_e)
        if self.world > 1:
            back = _a2a(y_recv, T * k, plan.send_counts, plan.recv_counts, self.group)
        else:
            back = y_recv
        y_pairs = torch.empty_like(back)
        y_pairs.index_copy_(0, plan.order, back)
        y_pairs = y_pairs.reshape(T, k, y_pairs.shape[1])
        if y_pairs.is_cuda and T > 0:
            return combine(y_pairs, w)
        return (y_pairs.float() * w.unsqueeze(-1)).sum(dim=1).to(x.dtype)


def shard_experts(codes: torch.Tensor, scales: torch.Tensor, rank: int, world: int):
    """This rank's slice [rank*E/world, (rank+1)*E/world) of per-expert codes and scales."""
    E = codes.shape[0]
    if E % world != 0:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    n = E // world
    return codes[rank * n:(rank + 1) * n].contiguous(), scales[rank * n:(rank + 1) * n].contiguous()
