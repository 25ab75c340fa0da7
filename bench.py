"""Benchmark: VQ-MoE decode (and prefill) on B200 through the repo's own API.

Workload (benchmark configuration C2, "one vq_switch MoE layer, decode"): hidden 4096,
512 experts, expert intermediate 1024, top-10 softmax routing from router
logits ~N(0,1), SwiGLU gate/up [1024 x 4096] and down [4096 x 1024], d=8,
K=16384 (14-bit packed codes), one fp16 codebook per projection per layer,
bf16 activations.  Seeded synthetic weights (codes uniform over K, codebook
~N(0, 0.02), scales ~U(0.5, 1.5), G = 64) and inputs (x ~N(0,1)).

A step is one MoE layer forward (router top-k, gate, up, SwiGLU, down,
weighted combine) on the headline batch (64 tokens; 1 and 8 are reported
beside it); on one GPU the layer is the library's fused block (one launch,
vqb_moe_block_forward), `--no-fused` runs it as per-step kernels.  The prefill leg (benchmark configuration C3) runs the same layer on 4096
tokens with top-10 routing drawn from Zipf(1.1) expert popularity and
reports TFLOP/s of the three expert projections.  Several independently seeded layers are rotated so the
weights a step reads are not in L2 from the previous step (the bytes each
step touches, times the rotation, exceed the 126 MB L2).

Multi-GPU (torchrun, one rank per GPU): expert parallelism (benchmark configuration
C5): rank r holds experts [r*E/N, (r+1)*E/N) of every projection, each rank
brings its own batch of tokens (weak scaling), and every layer sends the
(token, slot) pairs to the owning ranks and combines the outputs back
(vqlab_b200.ep: the fixed-shape peer-memory path -- dispatch / combine / reduce
kernels over NVLink, no host synchronisation -- for decode batches and for the
prefill leg alike).  `value` is all ranks' tokens over the max-over-ranks time.
The decode legs replay CUDA graphs.

Other legs in the same JSON line: `batches` (C2 at 1, 8, 64 tokens with each
batch's dominant-kernel roofline: the fused block, or the gate projection's
kernel on the per-step path), `dense` (C4, with the attention and
MLP kernels' rooflines), `c1` (C1: the 4096 x 4096 d8/K4096 matvec),
`prefill` (C3; with N > 1 each rank's expert busy time), `c5` (C5 at its stated
global shapes, 256 decode and 8192 prefill tokens split over the N GPUs).

`--impl reference` times the reference's CPU path (the oracle port of the
reference arithmetic, OpenMP over all host cores) on a bounded sample of the
same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, INTER, E, TOPK, D, K, BITS, G = 4096, 1024, 512, 10, 8, 16384, 14, 64
METRIC = "VQ-MoE decode tokens/s (one MoE layer, C2 shapes)"
UNIT = "tokens/s"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _wpr(nsub):
    return (nsub + 31) // 32 * BITS


def proj_bytes(out, inn):
    """Packed code + scale bytes of one expert's projection."""
    return out * _wpr(inn // D) * 4 + out * (inn // G) * 2


EXPERT_BYTES = {"gate": proj_bytes(INTER, HIDDEN), "up": proj_bytes(INTER, HIDDEN), "down": proj_bytes(HIDDEN, INTER)}
CODEBOOK_BYTES = K * D * 2


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled every 10 ms during
    the timed region, read-only through NVML (the same counters nvidia-smi's
    clocks.sm / clocks_event_reasons.* report); nvidia-smi at its 100 ms
    minimum when NVML is not importable.  The GPU is found by PCI bus id so a
    CUDA_VISIBLE_DEVICES remap cannot point it at another device."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_s: float = 0.01):
        self.gpu = gpu_index
        self.period = period_s
        self.sm, self.mx, self.reasons, self.err = [], None, set(), None
        self.proc = self.f = self.thread = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            p = torch.cuda.get_device_properties(self.gpu)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self.stop = threading.Event()

            def run():
                while True:
                    try:
                        self.sm.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.reasons.update(n for n, b in self.REASONS.items() if bits & b)
                    except Exception as e:  # noqa: BLE001 - reported in the summary
                        self.err = str(e)
                    if self.stop.wait(self.period):
                        return

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            self._start_smi()
        return self

    def _start_smi(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
            t0 = time.time()
            while time.time() - t0 < 3.0 and pathlib.Path(self.f.name).stat().st_size == 0:
                time.sleep(0.02)
            self.skip = len(pathlib.Path(self.f.name).read_text().splitlines())
        except Exception:
            self.proc = None

    def __exit__(self, *a):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.thread is None:
            if self.proc is None or self.f is None:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
            self.f.flush()
            rows = [r.split(",") for r in pathlib.Path(self.f.name).read_text().splitlines()[getattr(self, "skip", 0):]
                    if r.strip()]
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for r in rows:
                r = [c.strip() for c in r]
                if len(r) < 9:
                    continue
                try:
                    self.sm.append(float(r[1]))
                    self.mx = float(r[2])
                except ValueError:
                    continue
                for n, v in zip(names, r[5:9]):
                    if v.lower() == "active":
                        self.reasons.add(n)
        out = {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.mx,
               "reasons": sorted(self.reasons), "samples": len(self.sm),
               "source": "nvml 10 ms" if self.thread is not None else "nvidia-smi 100 ms"}
        if self.err:
            out["sampling_error"] = self.err
        return out


# ------------------------------------------------------------------ GPU arm

def make_layer(torch, dev, seed, rank=0, world=1, exchange="p2p", fused="auto"):
    """One seeded MoE layer; with world > 1 this rank's expert shard of it
    wrapped in the expert-parallel block (codebooks are per layer, so every
    rank builds the same ones)."""
    from vqlab_b200 import VQSwitchLinear
    from vqlab_b200.moe import VQMoEBlock
    from vqlab_b200.ep import EPMoEBlock
    e_local = E // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed * 1009 + rank)
    cgen = torch.Generator(device=dev)
    cgen.manual_seed(seed)

    def proj(out, inn):
        # uniform random words ARE uniform 14-bit codes: K = 2^BITS and NSUB % 32 == 0
        codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (e_local, out, _wpr(inn // D)), dtype=torch.int32, device=dev,
                              generator=gen)
        cb = (torch.randn((K, D), device=dev, generator=cgen) * 0.02).to(torch.float16)
        sc = (torch.rand((e_local, out, inn // G), device=dev, generator=gen) + 0.5).to(torch.float16)
        return VQSwitchLinear(codes, cb, sc, group_size=G, pack_bits=BITS, in_features=inn)

    if world == 1:
        return VQMoEBlock(proj(INTER, HIDDEN), proj(INTER, HIDDEN), proj(HIDDEN, INTER), TOPK, fused=fused)
    # decode batches take the fixed-shape path that CUDA graphs capture (gpu_arm sets
    # static_tokens to the batch it runs; larger batches take the dynamic path)
    return EPMoEBlock(proj(INTER, HIDDEN), proj(INTER, HIDDEN), proj(HIDDEN, INTER), TOPK, num_experts=E,
                      static_tokens=64, exchange=exchange)


def distinct_experts(torch, logits):
    from vqlab_b200.moe import route
    idx, _ = route(logits, TOPK)
    return int(torch.unique(idx).numel())


def layer_bytes(n_distinct, batch):
    per_expert = sum(EXPERT_BYTES.values())
    act = batch * HIDDEN * 2 * 2 + batch * TOPK * INTER * 2 * 3 + batch * TOPK * HIDDEN * 2
    return n_distinct * per_expert + 3 * CODEBOOK_BYTES + act


def fused_layer_bytes(n_distinct, batch):
    """Algorithmic bytes of the one-launch layer: the routed experts' packed
    codes and scales, the three codebooks, router logits, x and y (its
    intermediate partials never need to leave the chip in principle)."""
    return n_distinct * sum(EXPERT_BYTES.values()) + 3 * CODEBOOK_BYTES + batch * (E * 4 + HIDDEN * 2 * 2)


def time_eager_steps(torch, layers, xs, lg, steps, warmup):
    """Eager layer steps (the expert-parallel dispatch reads split sizes on the host)."""
    s = torch.cuda.current_stream()
    n = len(layers)
    for i in range(warmup):
        layers[i % n](xs[i % n], lg[i % n])
    torch.cuda.synchronize()
    torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(steps):
        layers[i % n](xs[i % n], lg[i % n])
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3


def time_graph_steps(torch, graphs, steps, warmup):
    """Replay captured step graphs round-robin; device time of `steps` replays."""
    s = torch.cuda.current_stream()
    for i in range(warmup):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(steps):
        graphs[i % len(graphs)].replay()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3


def kernel_seconds(torch, stream, call, reps):
    """Mean device time of the dominant kernel of `call(i)`: the library
    records two events on the launch stream around that kernel alone.  A
    ~0.1 ms spin kernel queued before each call keeps the stream busy while
    the host prepares the launch, so the interval holds the kernel's device
    time and not the host's launch overhead."""
    from vqlab_b200 import _lib
    pairs = []
    for i in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)  # creates the events
        b.record(stream)
        pairs.append((a, b))
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(pairs):
        torch.cuda._sleep(200_000)
        _lib.time_next_kernel(a, b)
        call(i)
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) for a, b in pairs) / 1e3


def profiled_traffic(kernel, workload):
    """DRAM bytes per launch of `kernel` on `workload` ("c2" / "c3") from the
    committed ncu summaries (profiles/<kernel>_<workload>*.txt, line
    `traffic_bytes_per_launch <kernel> <bytes>`), else None."""
    for f in sorted((ROOT / "profiles").glob(f"{kernel}_{workload}*.txt")):
        for line in f.read_text().splitlines():
            parts = line.split()
            if len(parts) == 3 and parts[0] == "traffic_bytes_per_launch" and parts[1] == kernel:
                return int(float(parts[2]))
    return None


DH, DI, DKV = 5120, 17408, 1024   # benchmark configuration C4: hidden, MLP intermediate, kv width


def make_dense_layer(torch, dev, seed, no_fused=False):
    """One C4 benchmark layer as VQLinear projections: attention q/k/v/o
    with d2/K256 (8-bit codes), MLP gate/up/down with d8/K16384 (14-bit)."""
    from vqlab_b200 import VQLinear
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def lin(out, inn, d, k, bits):
        wpr = (inn // d + 31) // 32 * bits
        codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (out, wpr), dtype=torch.int32, device=dev, generator=g)
        cb = (torch.randn((k, d), device=dev, generator=g) * 0.02).to(torch.float16)
        sc = (torch.rand((out, inn // G), device=dev, generator=g) + 0.5).to(torch.float16)
        return VQLinear(codes, cb, sc, group_size=G, pack_bits=bits, in_features=inn)

    from vqlab_b200.mlp import VQDenseMLP
    attn = [lin(DH, DH, 2, 256, 8), lin(DKV, DH, 2, 256, 8), lin(DKV, DH, 2, 256, 8), lin(DH, DH, 2, 256, 8)]
    mlp = VQDenseMLP(lin(DI, DH, 8, K, BITS), lin(DI, DH, 8, K, BITS), lin(DH, DI, 8, K, BITS),
                     fused="off" if no_fused else "auto")
    return attn, mlp


# packed codes + scales + codebooks of one C4 layer: q, k, v, o (d2/K256, 8-bit) and gate, up, down (d8/K16384)
def _dense_proj_bytes(out, inn, d, k, bits):
    return out * ((inn // d + 31) // 32 * bits) * 4 + out * (inn // G) * 2 + k * d * 2


DENSE_LAYER_BYTES = (2 * _dense_proj_bytes(DH, DH, 2, 256, 8) + 2 * _dense_proj_bytes(DKV, DH, 2, 256, 8) +
                     2 * _dense_proj_bytes(DI, DH, 8, K, BITS) + _dense_proj_bytes(DH, DI, 8, K, BITS))


def dense_step(layer, x):
    """The seven projections of one dense layer (the attention kernel itself is
    outside the VQ runtime: o is applied to q as its stand-in input); the MLP is
    VQDenseMLP (one launch at decode batches, the per-step calls otherwise)."""
    (wq, wk, wv, wo), mlp = layer
    q = wq(x)
    wk(x)
    wv(x)
    h = x + wo(q)
    return h + mlp(h)


def dense_leg(torch, dev, args, peak_gbs, peak_kind):
    """benchmark configuration C4: a 64-layer dense stack at batch 1 and 32 decode
    tokens, timed per layer (4 seeded layers rotated: ~100 MB of packed weights
    each, 400 MB per cycle > 126 MB L2) and scaled to 64 layers; the attention
    (d2/K256, q 5120 x 5120) and MLP (d8/K16384, gate 17408 x 5120)
    projections' dominant kernels are timed alone for their rooflines."""
    layers = [make_dense_layer(torch, dev, 7000 + l, args.no_fused) for l in range(4)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(23)
    out = {}
    for B in (1, 32):
        xs = [torch.randn((B, DH), device=dev, generator=gen).to(torch.bfloat16) for _ in layers]
        for l, L in enumerate(layers):
            dense_step(L, xs[l])
        torch.cuda.synchronize()
        graphs = []
        for l, L in enumerate(layers):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                dense_step(L, xs[l])
            graphs.append(gr)
        steps = max(20, args.steps)
        secs = time_graph_steps(torch, graphs, steps, args.warmup)
        ms = secs * 1e3 / steps
        out[str(B)] = {"ms_per_layer": round(ms, 4), "tokens_per_s_64_layers": round(B / (64 * ms / 1e3), 2),
                       "packed_weight_gbs": round(DENSE_LAYER_BYTES / (ms / 1e3) / 1e9, 1)}
        del graphs
        # dominant kernel of one attention and one MLP projection, timed alone
        s = torch.cuda.current_stream()
        roofs = {}
        mlp_fused = layers[0][1].fused != "off" and B <= 8 and layers[0][1].fused_status(B) == 0
        legs = [("attn_q", lambda L: L[0][0], (DH, DH, 2, 256, 8))]
        if mlp_fused:
            legs.append(("mlp", lambda L: L[1], None))
        else:
            legs.append(("mlp_gate", lambda L: L[1].gate_proj, (DI, DH, 8, K, BITS)))
        for name, pick, geom in legs:
            dur = kernel_seconds(torch, s, lambda i: pick(layers[i % len(layers)])(xs[i % len(layers)]), 8)
            if geom is None:  # the fused MLP: gate, up and down in one launch
                byt = (dense_bytes(DI, DH, 8, K, BITS, n=B) * 2 + dense_bytes(DH, DI, 8, K, BITS, n=B))
            else:
                byt = dense_bytes(*geom, n=B)
            ach = byt / dur / 1e9
            kname = ("dense_lut_kernel" if (name == "attn_q" and B <= 8)
                     else "moe_block_kernel" if name == "mlp" else "vq_prefill_tc_kernel")
            roofs[name] = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak_gbs, "unit": "GB/s",
                           "frac": round(ach / peak_gbs, 4),
                           "traffic": profiled_traffic(kname, f"c4_{name}_n{B}"),
                           "kernel": f"{kname}, timed alone", "algorithmic_bytes_per_launch": byt,
                           "us_per_launch": round(dur * 1e6, 2), "peak_kind": f"{peak_kind} burst copy bandwidth"}
        out[str(B)]["rooflines"] = roofs
    return {"metric": "dense VQ decode, benchmark configuration C4 (64 x [q,k,v,o d2/K256 + gate,up,down d8/K16384])",
            "unit": "tokens/s", "batches": out}


C1_OUT = C1_IN = 4096  # benchmark configuration C1: one dense 4096 x 4096 matvec, d8/K4096 (12-bit codes)


def _vq_linear(torch, dev, gen, out, inn, d, k, bits, g=G):
    from vqlab_b200 import VQLinear
    wpr = (inn // d + 31) // 32 * bits
    # uniform random words are uniform codes when K = 2^bits and NSUB % 32 == 0
    # (every benchmark geometry)
    assert k == 1 << bits and (inn // d) % 32 == 0
    codes = torch.randint(-2 ** 31, 2 ** 31 - 1, (out, wpr), dtype=torch.int32, device=dev, generator=gen)
    cb = (torch.randn((k, d), device=dev, generator=gen) * 0.02).to(torch.float16)
    sc = (torch.rand((out, inn // g), device=dev, generator=gen) + 0.5).to(torch.float16)
    return VQLinear(codes, cb, sc, group_size=g, pack_bits=bits, in_features=inn)


def dense_bytes(out, inn, d, k, bits, g=G, n=1):
    """Algorithmic bytes of one dense VQ projection call: packed codes, scales,
    the codebook, x and y (bf16)."""
    wpr = (inn // d + 31) // 32 * bits
    return out * wpr * 4 + out * (inn // g) * 2 + k * d * 2 + n * (inn + out) * 2


def c1_leg(torch, dev, args, peak_gbs, peak_kind):
    """benchmark configuration C1: the single 4096 x 4096 d8/K4096 vq_dense matvec
    (N = 1, bf16 x).  64 independently seeded layers (3.75 MB each, 240 MB per
    cycle > L2) are called round-robin from a CUDA graph; the dominant kernel
    is also timed alone for the roofline."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(31)
    lins = [_vq_linear(torch, dev, gen, C1_OUT, C1_IN, 8, 4096, 12) for _ in range(64)]
    xs = [torch.randn((1, C1_IN), device=dev, generator=gen).to(torch.bfloat16) for _ in lins]
    for L, x in zip(lins, xs):
        L(x)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for L, x in zip(lins, xs):
            L(x)
    reps = max(5, args.steps // 4)
    secs = time_graph_steps(torch, [g], reps, args.warmup)
    del g
    per_call = secs / (reps * len(lins))
    byt = dense_bytes(C1_OUT, C1_IN, 8, 4096, 12)
    s = torch.cuda.current_stream()
    dur = kernel_seconds(torch, s, lambda i: lins[i % len(lins)](xs[i % len(lins)]), 16)
    ach = byt / dur / 1e9
    return {"metric": "dense VQ matvec, benchmark configuration C1 (4096 x 4096, d8/K4096 12-bit, N = 1, bf16)",
            "us_per_call": round(per_call * 1e6, 2), "calls_per_s": round(1.0 / per_call, 1),
            "packed_weight_gbs": round(byt / per_call / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(ach / peak_gbs, 4), "traffic": profiled_traffic("dense_lut8_kernel", "c1"),
                         "kernel": "dense_lut8_kernel (bf16 weights, whole codebook in shared memory, one launch), "
                                   "timed alone",
                         "algorithmic_bytes_per_launch": byt, "us_per_launch": round(dur * 1e6, 2),
                         "peak_kind": f"{peak_kind} burst copy bandwidth"}}


def zipf_logits(torch, dev, gen, T, alpha=1.1):
    """Router logits whose top-10 is a draw without replacement from Zipf(alpha)
    expert popularity: log(popularity) + Gumbel noise (the Gumbel-top-k trick)."""
    perm = torch.randperm(E, device=dev, generator=gen)
    pop = torch.empty(E, device=dev)
    pop[perm] = 1.0 / torch.arange(1, E + 1, device=dev, dtype=torch.float32) ** alpha
    u = torch.rand((T, E), device=dev, generator=gen).clamp_(1e-12, 1.0 - 1e-7)
    return pop.log()[None, :] - torch.log(-torch.log(u))


def expert_busy_seconds(torch, layer, reps=3):
    """Device time of this rank's expert projections (gate, up, SwiGLU, down)
    on the pairs it served in the layer's last expert-parallel step."""
    from vqlab_b200.moe import expert_mlp
    X, ids = layer.last_pairs
    s = torch.cuda.current_stream()
    expert_mlp(layer.gate_proj, layer.up_proj, layer.down_proj, X, ids)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(reps):
        expert_mlp(layer.gate_proj, layer.up_proj, layer.down_proj, X, ids)
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def gather_floats(torch, dev, v, world):
    """[v of every rank] (an all-gather of one float), or [v] on one GPU."""
    if world == 1:
        return [v]
    t = torch.tensor([v], device=dev)
    out = torch.empty(world, device=dev)
    torch.distributed.all_gather_into_tensor(out, t)
    return [float(a) for a in out.tolist()]


def prefill_leg(torch, dev, args, peak_tf, peak_kind, rank, world, T=4096, seed=5000):
    """benchmark configuration C3: one MoE layer on T tokens per rank, Zipf(1.1)
    routing.  With several ranks the layer takes the fixed-shape peer-memory
    path at T tokens per rank (no host synchronisation: the exchange regions
    hold every rank's T token rows, pairs of other ranks' experts are skipped)."""
    layer = make_layer(torch, dev, seed, rank, world)
    if world > 1:
        layer.static_tokens = T
    gen = torch.Generator(device=dev)
    gen.manual_seed(17 + rank)
    x = torch.randn((T, HIDDEN), device=dev, generator=gen).to(torch.bfloat16)
    lg = zipf_logits(torch, dev, gen, T)
    for _ in range(2):
        layer(x, lg)
    torch.cuda.synchronize()
    steps = max(10, args.steps // 5)
    s = torch.cuda.current_stream()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        e0.record(s)
        for _ in range(steps):
            layer(x, lg)
        e1.record(s)
        torch.cuda.synchronize()
    secs = e0.elapsed_time(e1) / 1e3
    if world > 1:
        t = torch.tensor([secs], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        secs = float(t.item())
    flops = 3 * 2 * INTER * HIDDEN * T * TOPK
    from vqlab_b200.moe import route
    idx, _ = route(lg, TOPK)
    counts = torch.bincount(idx.reshape(-1).long(), minlength=E)
    if world == 1:
        xg, gidx = x[:, None, None, :], idx
    else:
        xg, gidx = layer.last_pairs
    dur = kernel_seconds(torch, s, lambda i: layer.gate_proj(xg, gidx), 5)
    served = int((gidx >= 0).sum())  # this rank's pairs (read before the exchange regions are released)
    kflops = 2 * INTER * HIDDEN * served
    ach = kflops / dur / 1e12
    busy = None
    if world > 1:
        # per-rank expert compute against the layer time: Zipf imbalance vs the exchange
        busy = [round(b * 1e3, 3) for b in gather_floats(torch, dev, expert_busy_seconds(torch, layer), world)]
        del xg, gidx
        layer.close()  # collective; xg / gidx were views of this rank's exchange region
    return {"metric": f"VQ-MoE prefill TFLOP/s (one MoE layer, {T} tokens per GPU, Zipf(1.1) top-10)",
            "value": round(flops * steps * world / secs / 1e12, 2), "unit": "TFLOP/s", "steps": steps,
            "ms_per_layer": round(secs * 1e3 / steps, 3), "tokens_per_s": round(T * steps * world / secs, 1),
            "tokens_per_expert": {"max": int(counts.max()), "median": float(counts.float().median()),
                                  "min": int(counts.min())},
            "flops_per_layer": flops, "clocks": clk.summary(),
            "expert_busy_ms_per_rank": busy,
            "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": round(ach / peak_tf, 4),
                         "traffic": profiled_traffic("vq_prefill_tc_kernel", "c3") if world == 1 else None,
                         "kernel": "vq_prefill_tc_kernel (gate projection, %d pairs on this rank), timed alone" % served,
                         "us_per_launch": round(dur * 1e6, 1), "peak_kind": f"{peak_kind} burst bf16 GEMM"}}


C5_DECODE_TOKENS, C5_PREFILL_TOKENS, C5_LAYERS = 256, 8192, 60


def c5_leg(torch, dev, args, rank, world):
    """benchmark configuration C5 at its stated global shapes: 256 concurrent
    decode tokens and an 8192-token prefill over the box, split evenly over the
    `world` ranks (strong scaling), experts sharded expert-parallel (E / world
    per rank), per layer; the 60-layer figures are 60 x the per-layer time of
    2 independently seeded layers rotated (each rank's weights per layer
    >= 600 MB, far above L2)."""
    B = C5_DECODE_TOKENS // world
    layers = [make_layer(torch, dev, 9000 + l, rank, world) for l in range(2)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(41 + rank)
    if world > 1:
        for L in layers:
            L.static_tokens = B
    xs = [torch.randn((B, HIDDEN), device=dev, generator=gen).to(torch.bfloat16) for _ in layers]
    lg = [torch.randn((B, E), device=dev, generator=gen) for _ in layers]
    outs = [L(x, l) for L, x, l in zip(layers, xs, lg)]
    torch.cuda.synchronize()
    graphs = []
    for i, L in enumerate(layers):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs[i] = L(xs[i], lg[i])
        graphs.append(g)
    if world > 1:
        torch.distributed.barrier()
    steps = max(20, args.steps // 2)
    secs = time_graph_steps(torch, graphs, steps, args.warmup)
    del graphs
    if world > 1:
        t = torch.tensor([secs], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        secs = float(t.item())
        for L in layers:
            L.close()
    del layers
    torch.cuda.synchronize()
    dec_ms = secs * 1e3 / steps
    _, peak_tf, peak_kind = _peaks()
    pre = prefill_leg(torch, dev, args, peak_tf, peak_kind, rank, world, T=C5_PREFILL_TOKENS // world, seed=9500)
    return {"metric": "benchmark configuration C5 at its global shapes: 256 decode tokens and an 8192-token "
                      "prefill split over the GPUs, experts sharded expert-parallel",
            "scaling": "strong", "decode_tokens_per_gpu": B, "prefill_tokens_per_gpu": C5_PREFILL_TOKENS // world,
            "decode_ms_per_layer": round(dec_ms, 4),
            "decode_tokens_per_s": round(C5_DECODE_TOKENS / (dec_ms / 1e3), 1),
            "decode_ms_per_60_layers": round(C5_LAYERS * dec_ms, 3),
            "decode_tokens_per_s_60_layers": round(C5_DECODE_TOKENS / (C5_LAYERS * dec_ms / 1e3), 1),
            "prefill_ms_per_layer": pre["ms_per_layer"], "prefill_tflops": pre["value"],
            "prefill_ms_per_60_layers": round(C5_LAYERS * pre["ms_per_layer"], 2),
            "prefill_expert_busy_ms_per_rank": pre.get("expert_busy_ms_per_rank")}


def gpu_arm(args, rank, world, dev):
    import torch
    torch.cuda.set_device(dev)
    peak_gbs, peak_tf, peak_kind = _peaks()
    batches = sorted(set([args.batch] + [int(b) for b in args.extra_batches.split(",") if b]))
    n_layers = args.layers
    layers = [make_layer(torch, dev, 1000 + l, rank, world, args.exchange, "off" if args.no_fused else "auto")
              for l in range(n_layers)]
    gen = torch.Generator(device=dev)
    gen.manual_seed(7 + rank)
    results = {}
    for B in batches:
        if world > 1:
            for L in layers:
                L.static_tokens = B  # the fixed-shape expert-parallel path pads every rank to this batch
        xs = [torch.randn((B, HIDDEN), device=dev, generator=gen).to(torch.bfloat16) for _ in range(n_layers)]
        lg = [torch.randn((B, E), device=dev, generator=gen) for _ in range(n_layers)]
        outs = [None] * n_layers
        # warm the allocator / library, then capture one graph per layer
        for l in range(n_layers):
            outs[l] = layers[l](xs[l], lg[l])
        torch.cuda.synchronize()
        graphs = []
        graph_note = "cuda graphs"
        try:
            for l in range(n_layers):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    outs[l] = layers[l](xs[l], lg[l])
                graphs.append(g)
        except Exception as e:  # noqa: BLE001 - a capture the backend refuses: eager steps instead
            graphs = []
            graph_note = f"eager steps (graph capture failed: {type(e).__name__})"
            torch.cuda.synchronize()
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        with ClockSampler(dev.index if dev.index is not None else 0) as clk:
            if graphs:
                secs = time_graph_steps(torch, graphs, args.steps, args.warmup)
            else:
                secs = time_eager_steps(torch, layers, xs, lg, args.steps, args.warmup)
        if world > 1:
            t = torch.tensor([secs], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            secs = float(t.item())
        nd = [distinct_experts(torch, lg[l]) for l in range(n_layers)]
        avg_bytes = statistics.mean(layer_bytes(n, B) for n in nd)
        results[B] = {"secs": secs, "ms_per_step": secs * 1e3 / args.steps,
                      "tokens_per_s": B * args.steps * world / secs,
                      # packed weight bytes of the experts a step touches (one GPU holds them all)
                      "hbm_gbs": avg_bytes * args.steps / secs / 1e9 if world == 1 else None,
                      "distinct_experts_mean": statistics.mean(nd), "clocks": clk.summary(), "timing": graph_note}
        del graphs
        torch.cuda.synchronize()
        xs_last, lg_last = xs, lg

    # ---- dominant kernel: the expert decode launch (gate projection), timed
    # alone at every batch (the headline roofline is the one at --batch)
    projs = [layers[l].gate_proj for l in range(n_layers)]
    s = torch.cuda.current_stream()
    roofs = {}
    for Bq in batches:
        if world == 1:
            x = torch.randn((Bq, 1, 1, HIDDEN), device=dev, generator=gen).to(torch.bfloat16)
            lgt = torch.randn((Bq, E), device=dev, generator=gen)
            from vqlab_b200.moe import route
            idx, _ = route(lgt, TOPK)
        elif Bq == batches[-1]:
            # the pairs this rank's experts served in the last expert-parallel step (-1: another rank's)
            x, idx = layers[0].last_pairs
        else:
            continue
        npairs = int((idx >= 0).sum())
        nd = int(torch.unique(idx[idx >= 0]).numel())
        fused = world == 1 and layers[0].fused != "off" and layers[0].fused_status(Bq) == 0
        if fused:
            # the whole layer is one launch (vqb_moe_block_forward): its bytes are
            # the three projections of every routed expert, the codebooks, x and y
            x2, lg2 = x.reshape(Bq, HIDDEN), lgt
            for L_ in layers:
                L_(x2, lg2)
            torch.cuda.synchronize()
            dur = kernel_seconds(torch, s, lambda i: layers[i % n_layers](x2, lg2), max(3, args.steps))
            alg = fused_layer_bytes(nd, Bq)
            kname, what = "moe_block_kernel", "the fused MoE block: router, gate, up, SwiGLU, down, combine"
        else:
            for p_ in projs:
                p_(x, idx)
            torch.cuda.synchronize()
            dur = kernel_seconds(torch, s, lambda i: projs[i % n_layers](x, idx), max(3, args.steps))
            rows = int((idx >= 0).reshape(x.shape[0], -1).any(dim=1).sum())  # token rows the served pairs read
            alg = nd * EXPERT_BYTES["gate"] + CODEBOOK_BYTES + rows * HIDDEN * 2 + npairs * INTER * 2
            kname = ("vq_prefill_tc_kernel" if projs[0].kernel_path(x.shape[0], idx.shape[-1]) == "gemm"
                     else "vq_decode_mma_kernel")
            what = "gate projection"
        achieved = alg / dur / 1e9
        traffic = profiled_traffic(kname, f"c2_b{Bq}") if world == 1 else None
        roofs[Bq] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak_gbs, "unit": "GB/s",
                     "frac": round(achieved / peak_gbs, 4), "traffic": traffic,
                     "kernel": "%s (%s, %d pairs, %d distinct experts), timed alone" % (kname, what, npairs, nd),
                     "algorithmic_bytes_per_launch": alg, "us_per_launch": round(dur * 1e6, 2),
                     "peak_kind": f"{peak_kind} burst copy bandwidth"}
    roof = roofs.get(args.batch)
    B = args.batch

    # ---- e2e through the public API with host buffers: every step copies its
    # inputs from pinned host memory into the layer's input buffers, runs the
    # layer (replaying the graph captured from the same public calls, or
    # eagerly when capture is refused) and reads the result back to the host
    e2e = None
    if not args.skip_e2e:
        xh = torch.randn((B, HIDDEN)).to(torch.bfloat16).pin_memory()
        lh = torch.randn((B, E)).pin_memory()
        yh = torch.empty((B, HIDDEN), dtype=torch.bfloat16).pin_memory()
        xin = [torch.empty((B, HIDDEN), dtype=torch.bfloat16, device=dev) for _ in range(n_layers)]
        lin = [torch.empty((B, E), device=dev) for _ in range(n_layers)]
        for l in range(n_layers):
            xin[l].copy_(xh)
            lin[l].copy_(lh)
        youts = [None] * n_layers
        egraphs = []
        try:
            for l in range(n_layers):
                youts[l] = layers[l](xin[l], lin[l])
            torch.cuda.synchronize()
            for l in range(n_layers):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    youts[l] = layers[l](xin[l], lin[l])
                egraphs.append(g)
        except Exception:  # noqa: BLE001 - capture refused: eager layer calls
            egraphs = []
            torch.cuda.synchronize()

        def e2e_step(i):
            l = i % n_layers
            xin[l].copy_(xh, non_blocking=True)
            lin[l].copy_(lh, non_blocking=True)
            if egraphs:
                egraphs[l].replay()
                y = youts[l]
            else:
                y = layers[l](xin[l], lin[l])
            yh.copy_(y, non_blocking=True)
            s.synchronize()

        for i in range(args.warmup):
            e2e_step(i)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(args.steps):
            e2e_step(i)
        e1.record(s)
        torch.cuda.synchronize()
        secs = e0.elapsed_time(e1) / 1e3
        del egraphs
        if world > 1:
            t = torch.tensor([secs], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            secs = float(t.item())
        e2e = {"value": round(B * args.steps * world / secs, 1), "unit": UNIT,
               "h2d_bytes_per_step": B * HIDDEN * 2 + B * E * 4, "d2h_bytes_per_step": B * HIDDEN * 2,
               "ms_per_step": round(secs * 1e3 / args.steps, 4)}
    # our kernels per step, counted by the library on one eager step
    from vqlab_b200 import _lib
    c0 = _lib.launch_count()
    layers[0](xs_last[0], lg_last[0])
    torch.cuda.synchronize()
    launches = _lib.launch_count() - c0
    if world > 1:
        for L in layers:
            L.close()  # collective: peer regions are released together
    for Bq, r in roofs.items():
        results[Bq]["roofline"] = r
    return results, roof, e2e, launches


# ------------------------------------------------------------------ CPU arms

def cpu_sample(tokens: int, seed: int = 11):
    """Time the oracle port of the reference arithmetic on `tokens` tokens of
    the C2 layer (router, gate/up walk decode, SwiGLU, down, combine) with all
    host threads.  Weights are generated only for the experts those tokens
    touch (same distributions as the GPU arm)."""
    import numpy as np

    from oracle import oracle as orc
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((tokens, HIDDEN)).astype(np.float32)
    lg = rng.standard_normal((tokens, E)).astype(np.float32)
    idx, w = orc.router_topk(lg, TOPK)
    used = np.unique(idx)
    remap = np.zeros(E, dtype=np.uint32)
    remap[used] = np.arange(used.size, dtype=np.uint32)
    lidx = remap[idx].reshape(-1)
    ne = used.size

    def proj(out, inn):
        words = rng.integers(0, 2 ** 32, (ne, out, _wpr(inn // D)), dtype=np.uint64).astype(np.uint32)
        cb = (rng.standard_normal((K, D)) * 0.02).astype(np.float16).view(np.uint16)
        sc = rng.uniform(0.5, 1.5, (ne, out, inn // G)).astype(np.float16).view(np.uint16)
        return words, cb, sc

    P = [proj(INTER, HIDDEN), proj(INTER, HIDDEN), proj(HIDDEN, INTER)]
    xb = orc.round_bf16(x)

    def run():
        xh = orc.f16_bits(xb)
        g = orc.switch_fused(P[0][0], P[0][1], P[0][2], xh, lidx, TOPK, packed_bits=BITS)
        u = orc.switch_fused(P[1][0], P[1][1], P[1][2], xh, lidx, TOPK, packed_bits=BITS)
        h = orc.swiglu_bf16(orc.round_bf16(orc.round_f16(g)), orc.round_bf16(orc.round_f16(u)))
        dn = orc.switch_fused(P[2][0], P[2][1], P[2][2], orc.f16_bits(h), lidx, 1, packed_bits=BITS)
        return orc.combine_bf16(orc.round_bf16(orc.round_f16(dn)).reshape(tokens, TOPK, HIDDEN), w)

    run()
    t0 = time.perf_counter()
    run()
    return time.perf_counter() - t0


def cpu_model() -> str:
    """The host CPU's model name (the first "model name" of /proc/cpuinfo)."""
    try:
        for line in pathlib.Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline_block(tokens):
    from oracle import oracle as orc
    secs = cpu_sample(tokens)
    return {"value": round(tokens / secs, 3), "unit": UNIT, "cores": orc.num_threads(), "cpu_model": cpu_model(),
            "kind": "port",
            "sample": f"{tokens} token(s) of the C2 layer (10 pairs each x gate/up/down, walk-order decode of "
                      f"packed 14-bit codes, SwiGLU, combine) on the oracle port, {secs:.2f} s"}


def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    from oracle import oracle as orc
    tokens = 1
    cpu_sample(tokens)  # warm-up (page-in, thread pool)
    times = []
    for i in range(args.warmup):
        cpu_sample(tokens, seed=100 + i)
    for i in range(args.steps):
        times.append(cpu_sample(tokens, seed=200 + i))
    secs = sum(times)
    value = tokens * args.steps / secs
    cb = {"value": round(value, 3), "unit": UNIT, "cores": orc.num_threads(), "cpu_model": cpu_model(), "kind": "port",
          "sample": f"{tokens} token of the C2 layer per step (router, 3 x 10-pair walk decode, SwiGLU, "
                    f"combine) on the oracle port of the reference arithmetic"}
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(secs * 1e3 / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 accumulate over fp16 (bf16 I/O)",
            "data": "synthetic (seeded)", "impl": "reference",
            "config": dict(_config(args, world),
                           workload="C2 one VQ-MoE layer decode, 1 token per step on the host (oracle port of the "
                                    "reference arithmetic: router, 10-pair walk decode of gate/up/down, SwiGLU, "
                                    "combine; hidden 4096, 512 experts, inter 1024, top-10, d8 K16384 14-bit, G64)",
                           global_batch=1),
            "cpu_baseline": cb,
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def _config(args, world):
    return {"workload": f"C2 one VQ-MoE layer decode, batch {args.batch} tokens/GPU (hidden 4096, 512 experts, "
                        f"inter 1024, top-10, d8 K16384 14-bit, G64)",
            "global_batch": args.batch * world, "experts": E, "top_k": TOPK, "hidden": HIDDEN,
            "intermediate": INTER, "dim": D, "codebook": K, "pack_bits": BITS, "group": G,
            "parallelism": (f"ep{world} (experts sharded; decode batches exchanged " +
                            ("by peer-memory kernels over NVLink, vqb_ep_dispatch/combine/reduce)"
                             if args.exchange == "p2p" else "by NCCL all-gather / all-to-all)")) if world > 1
                           else "single",
            "l2": f"{args.layers} independently seeded layers rotated per step (weights touched per cycle >> 126 MB L2)"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--extra-batches", default="1,8")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="expert-parallel decode exchange (N > 1): peer-memory kernels or NCCL collectives")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--skip-prefill", action="store_true")
    ap.add_argument("--skip-dense", action="store_true")
    ap.add_argument("--skip-c1", action="store_true")
    ap.add_argument("--skip-c5", action="store_true")
    ap.add_argument("--no-fused", action="store_true",
                    help="run the C2 decode layer as per-step kernels instead of the one-launch fused block")
    ap.add_argument("--prefill-only", action="store_true", help="run only the C3 prefill leg (for profiling)")
    ap.add_argument("--only", choices=["c1", "dense", "c5"],
                    help="run one leg alone and print its JSON (profiling runs)")
    ap.add_argument("--cpu-tokens", type=int, default=2048,
                    help="tokens of the CPU baseline sample (~12 s of oracle work on 16 host threads)")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    from vqlab_b200 import _lib
    _lib.lib()
    if args.prefill_only or args.only:
        # one leg alone (profiling runs): its own JSON line
        _, peak_tf, peak_kind = _peaks()
        if args.only == "c1":
            p = c1_leg(torch, dev, args, *_peaks()[::2]) if world == 1 else {}
        elif args.only == "dense":
            p = dense_leg(torch, dev, args, *_peaks()[::2]) if world == 1 else {}
        elif args.only == "c5":
            p = c5_leg(torch, dev, args, rank, world)
        else:
            p = prefill_leg(torch, dev, args, peak_tf, peak_kind, rank, world)
        if rank == 0:
            print(json.dumps(p), flush=True)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return 0
    results, roof, e2e, launches = gpu_arm(args, rank, world, dev)
    dense = None
    if not args.skip_dense and world == 1:
        dense = dense_leg(torch, dev, args, *_peaks()[::2])
    c1 = None
    if not args.skip_c1 and world == 1:
        c1 = c1_leg(torch, dev, args, *_peaks()[::2])
    prefill = None
    if not args.skip_prefill:
        _, peak_tf, peak_kind = _peaks()
        prefill = prefill_leg(torch, dev, args, peak_tf, peak_kind, rank, world)
    c5 = None
    if not args.skip_c5:
        c5 = c5_leg(torch, dev, args, rank, world)
    if rank == 0:
        head = results[args.batch]
        line = {"metric": METRIC, "value": round(head["tokens_per_s"], 1), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(head["ms_per_step"], 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 accumulate over fp16 (bf16 I/O)", "data": "synthetic (seeded)",
                "config": _config(args, world), "clocks": head["clocks"],
                "packed_weight_hbm_gbs": round(head["hbm_gbs"], 1) if head["hbm_gbs"] else None,
                "batches": {str(b): {"tokens_per_s": round(r["tokens_per_s"], 1),
                                     "ms_per_step": round(r["ms_per_step"], 4),
                                     "hbm_gbs": round(r["hbm_gbs"], 1) if r["hbm_gbs"] else None,
                                     "distinct_experts": round(r["distinct_experts_mean"], 1),
                                     "roofline": r.get("roofline")}
                            for b, r in results.items()},
                "roofline": roof, "e2e": e2e, "gpu_launches": launches * args.steps,
                "gpu_launches_per_step": launches}
        if prefill is not None:
            line["prefill"] = prefill
        if dense is not None:
            line["dense"] = dense
        if c1 is not None:
            line["c1"] = c1
        if c5 is not None:
            line["c5"] = c5
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline_block(args.cpu_tokens)
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
