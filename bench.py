"""Benchmark of the A->F->A MoE round trip (one DeepSeek-V3-shape MXFP4 MoE layer) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N = 1: one GPU holds one A rank and one F rank (loopback arenas): T = 16384 tokens, hidden 7168, 256 routed
experts (all on the F rank), top-8 sigmoid routing, intermediate 2048, MXFP4 weights, plus one bf16 shared
expert (intermediate 2048) computed on the A side and added in the combine.
N > 1 (torchrun, one rank per GPU): ranks [0, N/2) are A replicas (T = 16384 each), ranks [N/2, N) F ranks with
a contiguous share of the 256 experts; the data path is P2P stores over NVLink (no collective); gloo carries the
plumbing (endpoint exchange, barriers, the max over ranks of the timed region).

A step is one layer through dispatch -> experts -> combine for every A replica.  value = tokens of all A replicas
per second over exactly K timed steps (CUDA events, barrier + synchronize around, max over ranks); inputs are
larger than L2 (x 235 MB, weights 6 GB).  e2e = the same through AsapMoE.forward with pinned host buffers and the
host<->device copies inside the timed region.  --impl reference times the CPU restatement of the reference's
torch semantics (oracle/, test infrastructure) on a bounded sample of the same workload, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "sgl-afd-plugin_b200"))
sys.path.insert(0, ROOT)

METRIC = "MoE layer tokens/s A->F->A (DeepSeek-V3-shape MXFP4 layer, T=16384 per A replica)"
H, I, E, K_TOP, T_DEFAULT = 7168, 2048, 256, 8, 16384
ROUTING, KIND, SHARED = "sigmoid", "mxfp4", True
LAYERS = {
    # config 2: DeepSeek-V3 shape, MXFP4 experts, top-8 sigmoid, one bf16 shared expert on the A side
    "layer": dict(H=7168, I=2048, E=256, K_TOP=8, T_DEFAULT=16384, ROUTING="sigmoid", KIND="mxfp4", SHARED=True,
                  METRIC=METRIC),
    # config 4: FP8 E4M3 experts with fp32 128x128 block scales, H=8192, I=3584, 64 experts, top-6 softmax
    "fp8-layer": dict(H=8192, I=3584, E=64, K_TOP=6, T_DEFAULT=8192, ROUTING="softmax", KIND="fp8", SHARED=False,
                      METRIC="MoE layer tokens/s A->F->A (FP8 block-scaled layer: H=8192, 64 experts, top-6, I=3584, "
                             "T=8192 per A replica)"),
}
DTYPE = {"mxfp4": "mxfp8 x mxfp4 (fp32 accumulate), bf16 transport",
         "fp8": "e4m3 x e4m3 (fp32 block-scale promotion per 128-deep K block), bf16 transport"}
SWEEP_T = [256, 1024, 4096, 16384]
ZIPF_S = 1.2
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            return json.load(fh), "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 50 ms from before the timed region to after it.  The
    sampler starts on entry (nvidia-smi needs a moment to produce its first line); ``mark_start`` / ``mark_end``
    bracket the timed region and ``summary`` keeps the samples read inside it (or, for a region shorter than the
    sampling period, the samples nearest to it)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []
        self.t_start = self.t_end = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            deadline = time.time() + 3.0
            while not self.lines and time.time() < deadline:  # the first sample, so the region is covered
                time.sleep(0.01)
        except OSError:
            self.proc = None
        self.t_start = time.time()
        return self

    def mark_start(self):
        self.t_start = time.time()

    def mark_end(self):
        self.t_end = time.time()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def __exit__(self, *exc):
        if self.t_end is None:
            self.t_end = time.time()
        if self.proc is not None:
            time.sleep(0.1)  # the sample that covers the end of the region
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        lines = [(t, l) for t, l in self.lines if self.t_start - 0.01 <= t <= self.t_end + 0.06]
        window = "timed region"
        if not lines and self.lines:  # region shorter than the sampling period: the nearest samples
            mid = (self.t_start + self.t_end) / 2
            lines = sorted(self.lines, key=lambda tl: abs(tl[0] - mid))[:2]
            window = "nearest samples (timed region shorter than the 50 ms period)"
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for _, line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "window": window}


# ------------------------------------------------------------------------------------------ workload
def make_routing(T, seed, device):
    """Top-k of N(0,1) router logits: sigmoid scores (config 2) or softmax probabilities (config 4), the selected
    weights renormalised to sum 1."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    logits = torch.randn(T, E, device=device, generator=g)
    scores = torch.sigmoid(logits) if ROUTING == "sigmoid" else torch.softmax(logits, dim=1)
    w, ids = torch.topk(scores, K_TOP, dim=1)
    w = w / w.sum(1, keepdim=True)
    return ids.to(torch.int32).contiguous(), w.float().contiguous()


def zipf_routing(T, seed, device, s=ZIPF_S, perm_seed=1234):
    """Skewed routing: expert popularity p ~ 1/r^s over a seeded permutation of the experts (the same for every
    replica), each token's top-8 drawn without replacement with probabilities p (Gumbel top-k), weights
    sigmoid(N(0,1)) normalised over the 8."""
    import torch

    perm = torch.randperm(E, generator=torch.Generator().manual_seed(perm_seed))
    logp = torch.empty(E)
    logp[perm] = -s * torch.log(torch.arange(1, E + 1, dtype=torch.float32))
    g = torch.Generator(device=device).manual_seed(seed)
    u = torch.rand(T, E, device=device, generator=g).clamp_(1e-12, 1.0 - 1e-7)
    scores = logp.to(device) - torch.log(-torch.log(u))
    ids = torch.topk(scores, K_TOP, dim=1).indices
    w = torch.sigmoid(torch.randn(T, K_TOP, device=device, generator=g))
    w = w / w.sum(1, keepdim=True)
    return ids.to(torch.int32).contiguous(), w.float().contiguous()


def make_experts(P, expert_base, seed, device="cuda"):
    """Seeded synthetic routed experts of the selected layer: MXFP4 (uniform E2M1 codes, E8M0 scales 2^-10..2^-7)
    or FP8 (N(0, 0.02) weights block-quantised to E4M3 with fp32 128x128 scales)."""
    from asap_b200.experts import Fp8Experts, Mxfp4Experts

    if KIND == "fp8":
        return Fp8Experts.random(P, H, I, expert_base=expert_base, seed=seed, device=device)
    return Mxfp4Experts.random(P, H, I, expert_base=expert_base, seed=seed, scale_lo=117, scale_hi=120,
                               device=device)


def bind_numa(gpu: int) -> dict:
    """Run this process on the host cores local to its GPU (from the GPU's PCI device in sysfs), so that the pinned
    host buffers of the e2e leg are allocated on that NUMA node and copied over the GPU's own host link."""
    import torch

    try:
        pr = torch.cuda.get_device_properties(gpu)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as fh:
            spec = fh.read().strip()
        cpus = set()
        for part in spec.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= set(os.sched_getaffinity(0)) or cpus
        os.sched_setaffinity(0, cpus)
        return {"gpu_pci": bus, "cpus": len(cpus)}
    except (OSError, AttributeError, ValueError) as exc:
        return {"unbound": f"{type(exc).__name__}: {exc}"}


def placement(world, n_a, how):
    """(A ranks, F ranks) of a run: 'block' puts the A replicas on ranks [0, n_a); 'interleave' spreads them evenly
    over the box (ranks round(i * world / n_a)), so that their host copies (the e2e leg) use different host links
    and NUMA nodes.  NVLink through NVSwitch is the same between any two GPUs, so the data path does not care.
    Rank 0 is always an A replica (it prints the result line)."""
    a_ranks = list(range(n_a)) if how == "block" else sorted({round(i * world / n_a) for i in range(n_a)})
    if len(a_ranks) != n_a:
        raise SystemExit(f"placement {how} cannot place {n_a} A replicas on {world} GPUs")
    return a_ranks, [r for r in range(world) if r not in a_ranks]


def topology(name, world):
    """(A replicas, F ranks) of a ``world``-GPU run: 'half' = world/2 each (1A1F, 2A2F, 4A4F), '2a6f' on 8 GPUs,
    '2a4f' on 6."""
    if name == "half":
        return world // 2, world - world // 2
    n_a, n_f = int(name[0]), int(name[2])
    if name[1] != "a" or name[3] != "f" or n_a + n_f != world:
        raise SystemExit(f"topology {name} does not fit {world} GPUs")
    return n_a, n_f


class SharedExpert:
    """One bf16 shared expert (SwiGLU, intermediate 2048) on the A side, cuBLAS GEMMs through torch."""

    def __init__(self, device, seed=7):
        import torch

        g = torch.Generator(device=device).manual_seed(seed)
        self.w13 = (torch.randn(2 * I, H, device=device, generator=g) * 0.02).to(torch.bfloat16)
        self.w2 = (torch.randn(H, I, device=device, generator=g) * 0.02).to(torch.bfloat16)

    def __call__(self, x):
        import torch

        gu = x @ self.w13.t()
        return (torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]) @ self.w2.t()


def gemm_flops(pairs):
    return 2.0 * pairs * H * (2 * I), 2.0 * pairs * I * H


NVLINK_NOMINAL_GBS = 900.0  # NVLink 5 per direction per GPU (nominal)
# --serve auto: below this many expected (token, local expert) pairs per message and F rank, the rest of a step's
# messages are answered as one joined job (measured at 4A4F: configs 4 and 5 up to T=4096 gain, config 2's 32768
# pairs per message lose to per-message jobs, whose replies overlap the next job)
FTR_PAIRS = 32768


def first_then_rest(args, n_a, T, p_max):
    """Whether an F rank answers a step of n_a messages of T tokens as first-ready + joined rest (--serve)."""
    if n_a < 2 or args.join_replicas:
        return False
    if args.serve == "auto" and n_a < 3:  # the rest of a step is one message: nothing to join
        return False
    if args.serve != "auto":
        return args.serve == "first-then-rest"
    return T * K_TOP * p_max / E < FTR_PAIRS


def f_job_launches(rows=1):
    """Kernels of one F job: the doorbell wait (any / all rows), the routing count + scan + place, the activation
    quantise + permute, the two GEMMs, the weighted reduce + reply, and for a joined job the gather of its rows."""
    return 1 + 3 + 1 + 2 + 1 + (1 if rows > 1 else 0)


def hbm_kernel_gbs(T, pairs, kernel_ms):
    """Algorithmic GB/s of the two HBM-bound F kernels: quantise+permute reads each token's bf16 row once and
    writes its activation codes + scales into every local pair row; the weighted reduce reads every pair's bf16 row
    and writes each token's reply row."""
    scale_bytes = H // 32 if KIND == "mxfp4" else 4 * (H // 128)
    qp = T * 2 * H + pairs * (H + scale_bytes)
    red = pairs * 2 * H + T * 2 * H
    def gbs(nbytes, ms):
        return round(nbytes / (ms * 1e-3) / 1e9, 1) if ms and ms > 0 else None

    return {"quantise_permute": gbs(qp, kernel_ms.get("quantise_permute")),
            "reduce_reply": gbs(red, kernel_ms.get("reduce_reply")),
            "bytes": {"quantise_permute": qp, "reduce_reply": red}}


def expert_bytes():
    """Weight bytes of one routed expert in the layer's format (codes + scales)."""
    if KIND == "fp8":
        return 3 * H * I + 4 * (3 * (H // 128) * (I // 128))
    return 3 * H * I // 2 + 3 * H * I // 32


def step_roofline(flop_busiest_f, weight_bytes_busiest_f, ms, what):
    """The roofline of a multi-kernel step whose F chain dominates: the busiest F rank's expert GEMM FLOPs at the
    FP8-rate tensor peak (2 x the measured sustained bf16 rate: a step-long timed region) and its weight bytes at
    the measured HBM rate; bound = the larger; achieved = FLOP / measured step time (whole step, so transfers and
    the HBM-bound kernels count against it)."""
    peaks, peak_kind = load_peaks()
    fp8 = 2.0 * peaks["bf16_tflops_sustained"]
    t_flop = flop_busiest_f / (fp8 * 1e12) * 1e3
    t_hbm = weight_bytes_busiest_f / (peaks["hbm_gbs"] * 1e9) * 1e3
    if t_flop >= t_hbm:
        achieved = flop_busiest_f / (ms * 1e-3) / 1e12
        return {"kernel": what, "bound": "tensor", "achieved": round(achieved, 1), "peak": round(fp8, 1),
                "unit": "TFLOP/s", "frac": round(achieved / fp8, 4), "traffic": None,
                "peak_source": f"{peak_kind} bf16_tflops_sustained x 2 (FP8-rate tensor kind)",
                "t_flop_ms": round(t_flop, 4), "t_hbm_ms": round(t_hbm, 4)}
    achieved = weight_bytes_busiest_f / (ms * 1e-3) / 1e9
    return {"kernel": what, "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None, "peak_source": f"{peak_kind} hbm_gbs",
            "t_flop_ms": round(t_flop, 4), "t_hbm_ms": round(t_hbm, 4)}


def layer_roofline(n_a, T, f_rows, bounds, ms, peaks, peak_kind, nvlink_gbs=None):
    """Per-layer roofline of an nA x nF step: for each F rank, the time its inbound rows take over NVLink
    (x bf16 + ids + weights per routed row), its reply rows outbound, its expert GEMMs at the FP8-rate tensor peak
    (pairs expected under uniform routing: every replica's T·k pairs spread over the experts), and its weight +
    activation bytes at the HBM peak.  Bound = the largest of those over F ranks; serial = in + flop + out.
    ``nvlink_gbs``: the link rate measured in the same run (copy-engine peer write), else the nominal 900 GB/s."""
    fp8_tflops = 2.0 * peaks["bf16_tflops_sustained"]
    link_src = "copy-engine peer write measured in this run" if nvlink_gbs else "nominal NVLink 5 per direction"
    nvlink_gbs = nvlink_gbs or NVLINK_NOMINAL_GBS
    per_f = []
    for f, rows in enumerate(f_rows):
        p_f = bounds[f + 1] - bounds[f]
        pairs = n_a * T * K_TOP * p_f / E
        t_in = rows * (2 * H + 8 * K_TOP) / (nvlink_gbs * 1e9) * 1e3
        t_out = rows * 2 * H / (nvlink_gbs * 1e9) * 1e3
        t_flop = pairs * 6.0 * H * I / (fp8_tflops * 1e12) * 1e3
        t_hbm = (p_f * expert_bytes() + rows * (2 * H + 8 * K_TOP) + rows * 2 * H) / (peaks["hbm_gbs"] * 1e9) * 1e3
        per_f.append((t_in, t_out, t_flop, t_hbm))
    worst = max(per_f, key=lambda t: max(t))
    names = ("nvlink_in", "nvlink_out", "tensor", "hbm")
    t_bound = max(max(t) for t in per_f)
    t_serial = max(t[0] + t[1] + t[2] for t in per_f)
    return {"bound": names[worst.index(max(worst))], "t_in_ms": round(worst[0], 4), "t_out_ms": round(worst[1], 4),
            "t_flop_ms": round(worst[2], 4), "t_hbm_ms": round(worst[3], 4), "t_bound_ms": round(t_bound, 4),
            "t_serial_ms": round(t_serial, 4), "measured_ms": round(ms, 4), "frac": round(t_bound / ms, 4),
            "frac_serial": round(t_serial / ms, 4),
            "peaks": {"nvlink_gbs": round(nvlink_gbs, 1), "fp8_tflops": round(fp8_tflops, 1), "hbm_gbs": peaks["hbm_gbs"],
                      "source": f"{peak_kind} MEASURED_PEAKS (FP8 = 2 x bf16 sustained); NVLink: {link_src}"},
            "pairs": "expected under uniform routing"}


class HostPipeline:
    """End-to-end driver of the public API on pinned host buffers: every step copies its inputs host->device and
    its output device->host; step i+1's upload and step i's download run on copy streams while the compute stream
    runs step i (double-buffered device inputs), as a serving loop would."""

    def __init__(self, x, ids, w, dev, forward):
        import torch

        self.dev, self.forward = dev, forward
        self.hx, self.hi, self.hw = x.cpu().pin_memory(), ids.cpu().pin_memory(), w.cpu().pin_memory()
        self.hout = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        self.dx = [torch.empty_like(x) for _ in range(2)]
        self.di = [torch.empty_like(ids) for _ in range(2)]
        self.dw = [torch.empty_like(w) for _ in range(2)]
        self.up, self.down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        self.in_ready = [torch.cuda.Event() for _ in range(2)]
        self.in_free = [torch.cuda.Event() for _ in range(2)]
        self.uploaded = [False, False]
        self.h2d = self.hx.numel() * 2 + self.hi.numel() * self.hi.element_size() + self.hw.numel() * 4
        self.d2h = self.hout[0].numel() * 2
        self.i = 0

    def upload(self, b):
        import torch

        self.up.wait_event(self.in_free[b])
        with torch.cuda.stream(self.up):
            self.dx[b].copy_(self.hx, non_blocking=True)
            self.di[b].copy_(self.hi, non_blocking=True)
            self.dw[b].copy_(self.hw, non_blocking=True)
        self.in_ready[b].record(self.up)

    def run(self, steps):
        """``steps`` more steps; the upload of the step after the last is already issued when this returns."""
        import torch

        compute = torch.cuda.current_stream(self.dev)
        for _ in range(steps):
            b = self.i % 2
            if not self.uploaded[b]:
                self.upload(b)
            self.upload(1 - b)
            self.uploaded[1 - b] = True
            compute.wait_event(self.in_ready[b])
            out = self.forward(self.dx[b], self.di[b], self.dw[b])
            self.uploaded[b] = False
            self.in_free[b].record(compute)
            done = torch.cuda.Event()
            done.record(compute)
            self.down.wait_event(done)
            with torch.cuda.stream(self.down):
                self.hout[b].copy_(out, non_blocking=True)
                out.record_stream(self.down)
            self.i += 1

    def finish(self):
        """Make the compute stream wait for the last download (before a timing event is recorded)."""
        import torch

        torch.cuda.current_stream(self.dev).wait_stream(self.down)


# ------------------------------------------------------------------------------------------ 1 GPU
def run_single(args):
    import torch

    from asap_b200.dispatcher import AsapDispatcher
    from asap_b200.experts import Mxfp4Experts
    from asap_b200.layer import AsapMoE
    from asap_b200.loopback import Loopback
    from asap_b200.sglang_shim import StandardTopKOutput
    from asap_b200 import _native as N
    from asap_b200.transport.layout import Geometry
    import ctypes

    dev = "cuda:0"
    torch.cuda.set_device(0)
    T = args.tokens
    experts = make_experts(E, 0, 1, dev)
    lb = Loopback(Geometry(1, 1, 2, T, H, K_TOP, 1), {0: experts}, timeout_s=30.0)
    lb.install()
    shared = SharedExpert(dev) if SHARED else (lambda _x: None)
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    ids, w = make_routing(T, 3, dev)
    disp = AsapDispatcher(0)
    topk = StandardTopKOutput(w, ids)
    stream = torch.cuda.current_stream()

    def step():
        d = disp.dispatch(x, topk)
        s = shared(x)
        return disp.combine(d, shared=s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    lb.check()
    N.call("asap_ffn_enable_timing", lb.sched.ws_handle, 1)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        torch.cuda.synchronize()
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
    lb.check()
    ms = t0.elapsed_time(t1) / args.steps
    kms = (ctypes.c_float * 5)()
    N.call("asap_ffn_last_timing", lb.sched.ws_handle, kms, 5)
    N.call("asap_ffn_enable_timing", lb.sched.ws_handle, 0)
    kernel_ms = dict(zip(("routing", "quantise_permute", "gemm1", "gemm2", "reduce_reply"), list(kms)))
    pairs = int(lb.sched.debug_tensors()["expert_counts"].sum().item())

    # dispatch / combine kernel times on their own streams (extra measured steps, outside the timed region)
    dsp, cmb = [], []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        buf = lb.buffer
        buf.send_stream.wait_stream(stream)
        e0.record(buf.send_stream)
        d = disp.dispatch(x, topk)
        e1.record(buf.send_stream)
        s = shared(x)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        lb.local.before_combine(d.ticket, stream)
        c0.record(stream)
        disp.combine(d, shared=s)
        c1.record(stream)
        torch.cuda.synchronize()
        dsp.append(e0.elapsed_time(e1))
        cmb.append(c0.elapsed_time(c1))
    lb.check()

    # e2e: the public API (AsapMoE.forward) on pinned host buffers, copies inside the timed region
    e2e = None
    if not args.no_e2e:
        def forward(dx, di, dw):  # the layer as a model runs it: routed experts + shared expert, fused combine
            d = disp.dispatch(dx, StandardTopKOutput(dw, di))
            return disp.combine(d, shared=shared(dx))

        pipe = HostPipeline(x, ids, w, dev, forward)
        pipe.run(args.warmup)
        pipe.finish()
        torch.cuda.synchronize()
        t0.record(stream)
        pipe.run(args.steps)
        pipe.finish()
        t1.record(stream)
        torch.cuda.synchronize()
        lb.check()
        e2e_ms = t0.elapsed_time(t1) / args.steps
        e2e = {"value": round(T / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "h2d_bytes_per_step": pipe.h2d,
               "d2h_bytes_per_step": pipe.d2h, "ms_per_step": round(e2e_ms, 4),
               "path": "AsapDispatcher.dispatch/combine (+ shared expert) per step, H2D of x/ids/w from pinned host "
                       "and D2H of the output overlapped with the previous/next step on copy streams"}

    # parity of the timed configuration: one more step on the same inputs, its buffers against the oracle (the
    # CPU-baseline leg, which then times the reference's torch semantics on the same tokens and weights)
    parity, cpu = None, None
    if not args.no_cpu:
        d = disp.dispatch(x, topk)
        s_out = shared(x)
        out = disp.combine(d, shared=s_out)
        torch.cuda.synchronize()
        lb.check()
        parity, inputs = check_single(x, ids, w, experts, lb.sched, out, s_out, n_experts=args.cpu_experts)
        cpu = cpu_baseline(args.cpu_experts, inputs=inputs, steps=3)

    bar = flashinfer_bar(x, ids, w, args.steps) if KIND == "mxfp4" and not args.no_flashinfer else None

    peaks, peak_kind = load_peaks()
    g1_flops, g2_flops = gemm_flops(pairs)
    fp8_burst = 2.0 * peaks["bf16_tflops"]  # kind::f8f6f4 runs at twice the bf16 rate
    fp8_sustained = 2.0 * peaks["bf16_tflops_sustained"]
    achieved = g1_flops / (kernel_ms["gemm1"] * 1e-3) / 1e12
    traffic = load_traffic("gemm1" if KIND == "mxfp4" else "gemm1_fp8", pairs)
    clk = clocks.summary()
    nvlink_bytes_dispatch = T * (2 * H + 8 * K_TOP)
    workload = (f"1 GPU loopback A+F: config 2 layer (T={T}, H=7168, {E} experts, top-8 sigmoid, I=2048, MXFP4 "
                "weights, 1 bf16 shared expert)" if KIND == "mxfp4" else
                f"1 GPU loopback A+F: config 4 layer (T={T}, H={H}, {E} experts, top-{K_TOP} softmax, I={I}, FP8 E4M3 "
                "weights with fp32 128x128 block scales, no shared expert)")
    line = {
        "metric": METRIC, "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": DTYPE[KIND], "data": "synthetic",
        "config": {"workload": workload, "tokens_per_replica": T,
                   "a_replicas": 1, "f_ranks": 1, "parallelism": "1A1F loopback",
                   "l2": f"inputs larger than L2 (x {T * H * 2 / 1e6:.0f} MB, weights {experts.nbytes / 1e9:.1f} GB), "
                         "no flush"},
        "e2e": e2e,
        # dispatch 2 (route, pack) + the F job + combine 2 (wait, sum); the cuBLAS shared expert is not counted
        "gpu_launches": args.steps * (4 + f_job_launches()),
        "roofline": {"kernel": "moe_gemm_kernel<0> (GEMM1 + SwiGLU + MXFP8 requant)" if KIND == "mxfp4" else
                     "moe_gemm_fp8_kernel<0> (GEMM1, block-scale promotion + SwiGLU + FP8 requant)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": round(fp8_burst, 1), "unit": "TFLOP/s",
                     "frac": round(achieved / fp8_burst, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} bf16_tflops (burst) x 2 (FP8-rate tensor kind)",
                     "frac_of_sustained": round(achieved / fp8_sustained, 4),
                     "frac_of_fp4_dense_nominal" if KIND == "mxfp4" else "frac_of_fp8_dense_nominal":
                         round(achieved / (9000.0 if KIND == "mxfp4" else 4500.0), 4)},
        "kernels_ms": {k: round(v, 4) for k, v in kernel_ms.items()},
        "f_chain_ms": round(sum(kernel_ms.values()), 4),
        "flashinfer_bar": bar,
        "kernels_gbs": hbm_kernel_gbs(T, pairs, kernel_ms),
        "dispatch_ms": round(statistics.median(dsp), 4), "combine_ms": round(statistics.median(cmb), 4),
        "dispatch_gbs_algorithmic": round(nvlink_bytes_dispatch / (statistics.median(dsp) * 1e-3) / 1e9, 1),
        "pairs": pairs, "gemm_tflops_per_step": round((g1_flops + g2_flops) / 1e12, 3),
        "cpu_baseline": cpu, "parity": parity, "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    lb.close()
    experts.release()


def flashinfer_bar(x, ids, w, steps):
    """The reference's expert backend on the same layer, same GPU: FlashInfer's trtllm-gen MXFP4 MoE
    (trtllm_fp4_block_scale_routed_moe, as srt/layers/quantization/mxfp4_flashinfer_trtllm_moe.py:68-99 calls it)
    over this step's tokens and routing with synthetic MXFP4 experts of the same distribution, activations
    pre-quantised to MXFP8.  The call is timed with CUDA events (median over ``steps`` calls after 3 warm-up calls);
    compare with this build's F chain (f_chain_ms: routing + quantise + both GEMMs + reduce).  Test and benchmark
    infrastructure under tests/golden; null-equivalent with the reason when the prebuilt module is absent."""
    import torch

    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    try:
        import flashinfer_ref
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"{type(exc).__name__}: {exc}"}
    why = flashinfer_ref.available()
    if why:
        return {"unavailable": why}
    try:
        weights = flashinfer_ref.random_weights(E, H, I, seed=11)
        xq, xsf = flashinfer_ref.mxfp8_quantize(x)
        out = torch.empty(x.shape[0], H, dtype=torch.bfloat16, device=x.device)
        for _ in range(3):
            flashinfer_ref.run(xq, xsf, ids, w, weights, E, I, out=out)
        torch.cuda.synchronize()
        times = []
        for _ in range(max(steps, 3)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            flashinfer_ref.run(xq, xsf, ids, w, weights, E, I, out=out)
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
        finite = bool(torch.isfinite(out.float()).all().item())
        del weights
        torch.cuda.empty_cache()
        return {"ms": round(ms, 4), "tflops": round(6.0 * H * I * int(ids.numel()) / (ms * 1e-3) / 1e12, 1),
                "output_finite": finite, "calls": len(times),
                "what": "flashinfer trtllm_fp4_block_scale_routed_moe (MXFP8 x MXFP4, SwiGLU, weighted sum), "
                        "same tokens and routing, synthetic experts; excludes the activation quantisation"}
    except Exception as exc:  # noqa: BLE001
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}


def load_traffic(kernel, pairs):
    """DRAM bytes per launch of ``kernel`` from a committed ncu summary, scaled to this launch's pair count."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as fh:
        d = json.load(fh).get(kernel)
    if not d:
        return None
    return int(d["dram_bytes"] * pairs / d["pairs"])


# ------------------------------------------------------------------------------------------ CPU baseline
def _cpu_cores():
    return len(os.sched_getaffinity(0))


def _dequant_first(experts, n_experts, which=None):
    """Dequantised (gate, up, w2) fp32 numpy arrays of local experts [0, n_experts) of device-layout experts, or of
    the local experts listed in ``which`` (in that order)."""
    import torch

    from oracle import moe

    idx = torch.arange(n_experts) if which is None else torch.as_tensor(list(which), dtype=torch.long)
    n = len(idx)

    def rows(t, P):
        return t.view(P, -1).index_select(0, idx.to(t.device)).cpu().numpy()

    if getattr(experts, "kind", "mxfp4") == "fp8":
        return moe.dequant_fp8(experts.w13.index_select(0, idx.to(experts.w13.device)).cpu().numpy(),
                               experts.w13_scale.index_select(0, idx.to(experts.w13.device)).cpu().numpy(),
                               experts.w2.index_select(0, idx.to(experts.w2.device)).cpu().numpy(),
                               experts.w2_scale.index_select(0, idx.to(experts.w2.device)).cpu().numpy())
    P, Hh, Ii = experts.num_local, experts.hidden, experts.inter
    gate, up = moe.dequant_w13(rows(experts.w13, P), rows(experts.w13_sf, P), n, Hh, Ii)
    return gate, up, moe.dequant_w2(rows(experts.w2, P), rows(experts.w2_sf, P), n, Hh, Ii)


def _time_torch_cpu(x, ids, w, weights, n_experts, act, reps):
    """Median seconds of the torch CPU restatement (oracle/torch_cpu.py) over ``reps`` runs: every pair of the
    message that routes to experts [0, n_experts), dequantised weights (dequantisation not timed)."""
    import torch

    from oracle import torch_cpu as tc

    torch.set_num_threads(_cpu_cores())
    gate, up, w2 = (torch.from_numpy(a) for a in weights)
    xt, it, wt = torch.from_numpy(x), torch.from_numpy(ids.astype("int64")), torch.from_numpy(w)
    times = []
    for _ in range(reps):
        t = time.perf_counter()
        tc.reduce_pairs(*tc.ffn_pairs(xt, it, wt, gate, up, w2, 0, range(n_experts), act_quant=act))
        times.append(time.perf_counter() - t)
    return statistics.median(times), torch.get_num_threads()


def cpu_baseline(n_experts=4, seed=0, steps=1, warmup=0, inputs=None):
    """The reference's torch semantics on the host cores (oracle/torch_cpu.py, with the GPU path's activation
    rounding: MXFP8 for config 2, E4M3 per 1x128 for config 4): every (token, slot) pair of the layer that routes
    to experts [0, n_experts).  ``inputs`` = (x bf16 values, ids, w, (gate, up, w2)) as numpy arrays: the
    benchmark's own tokens and dequantised weights; without it, seeded random ones of the same shapes.
    tokens/s counts pairs / top-k."""
    import numpy as np

    from oracle import moe, mx

    rng = np.random.default_rng(seed)
    T = T_DEFAULT
    act = "fp8" if KIND == "fp8" else True
    P = n_experts
    if inputs is None:
        logits = rng.standard_normal((T, E))
        ids, w = moe.topk_routing(logits, K_TOP, ROUTING)
        x = mx.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
        if KIND == "fp8":
            # E4M3 codes with magnitudes 2^-1 .. 2^3 and random signs, one scale per 128x128 block
            sign = lambda shape: rng.integers(0, 2, shape, dtype=np.uint8) << 7  # noqa: E731
            q13 = rng.integers(0x30, 0x50, (P, 2 * I, H), dtype=np.uint8) | sign((P, 2 * I, H))
            q2 = rng.integers(0x30, 0x50, (P, H, I), dtype=np.uint8) | sign((P, H, I))
            s13 = rng.uniform(0.002, 0.01, (P, 2 * I // 128, H // 128)).astype(np.float32)
            s2 = rng.uniform(0.002, 0.01, (P, H // 128, I // 128)).astype(np.float32)
            weights = moe.dequant_fp8(q13, s13, q2, s2)
        else:
            codes13 = rng.integers(0, 256, (P, 2 * I, H // 2), dtype=np.uint8)
            sf13 = rng.integers(117, 121, (P, 2 * I * H // 32), dtype=np.uint8)
            codes2 = rng.integers(0, 256, (P, H, I // 2), dtype=np.uint8)
            sf2 = rng.integers(117, 121, (P, H * I // 32), dtype=np.uint8)
            weights = (*moe.dequant_w13(codes13, sf13, P, H, I), moe.dequant_w2(codes2, sf2, P, H, I))
        source = "seeded random tokens and weights of the layer's shapes"
    else:
        x, ids, w, weights = inputs
        source = "the benchmark's own tokens, routing and dequantised expert weights"
    sel = np.any(ids < n_experts, axis=1)
    pairs = int(np.sum(ids[sel] < n_experts))
    for _ in range(warmup):
        _time_torch_cpu(x[sel], ids[sel], w[sel], weights, P, act, 1)
    dt, threads = _time_torch_cpu(x[sel], ids[sel], w[sel], weights, P, act, max(steps, 1))
    cfg = "config-2" if KIND == "mxfp4" else "config-4"
    return {"value": round(pairs / K_TOP / dt, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"all {pairs} (token, expert) pairs of the T={T} {cfg} layer that route to experts "
                      f"0..{n_experts - 1} ({source}; torch CPU fp32, {'FP8 1x128' if act == 'fp8' else 'MXFP8'} "
                      f"activation emulation, {threads} threads); tokens = pairs / top-k; {dt:.2f} s per sample",
            "config1": cpu_config1()}


def check_single(x, ids, w, experts, sched, out, shared_out, n_experts=4, n_tokens=64, seed=0, busiest=False):
    """Parity of the timed configuration (the CPU-baseline leg's check; oracle/ is the checker): the last step's
    device buffers against the oracle on the benchmark's own inputs.  ``experts`` / ``sched``: one F rank's, or
    lists of them (F ranks of a loopback deployment in F order, contiguous expert ranges from 0).
      * routing: per F rank, the per-local-expert counts and the expert-major position of every pair of the
        tokens sent to it (in token order), bit-exact (all pairs of the step);
      * F rank 0's local experts [0, n_experts) -- or, with ``busiest``, its n_experts experts with the most
        pairs this step (skewed routing can leave the first ones empty): MXFP8 activation codes + scales of their
        pairs bit-exact (MXFP4 layers), and the weighted GEMM2 rows within relative L2 1e-2 of the oracle's
        ffn_pairs;
      * n_tokens sampled tokens: every F rank's reply (fp32 sum of the token's pair rows in slot order) and the
        combined output (+ shared expert) bit-exact from the device's own pair rows.
    -> (parity dict, inputs for cpu_baseline)."""
    import numpy as np
    import torch

    from asap_b200.transport.server import _raw_bytes
    from oracle import moe, mx

    ex_list = list(experts) if isinstance(experts, (list, tuple)) else [experts]
    sc_list = list(sched) if isinstance(sched, (list, tuple)) else [sched]
    dev = x.device
    ids_np, w_np = ids.cpu().numpy(), w.cpu().numpy()
    T, k = ids_np.shape
    ids64 = ids_np.astype(np.int64)
    tables, pairs = True, 0
    per_f = []  # (tokens sent to F f, their compacted index, pair positions, y2 view)
    for e_f, s_f in zip(ex_list, sc_list):
        P, e0 = e_f.num_local, e_f.expert_base
        sent = np.any((ids64 >= e0) & (ids64 < e0 + P), axis=1)
        n_f = int(sent.sum())
        dbg = s_f.debug_tensors()
        pos_ref, _, counts_ref = moe.expert_permutation(ids_np[sent], e0, P)
        counts = dbg["expert_counts"].cpu().numpy()
        pos = dbg["pair_pos"][:n_f].cpu().numpy()
        tables = tables and bool(np.array_equal(counts, counts_ref) and np.array_equal(pos, pos_ref))
        pairs += int(counts_ref.sum())
        rows = int(pos_ref.max()) + 1 if n_f else 1
        y2 = _raw_bytes(dbg["y2"], rows * H * 2, dev.index).view(torch.bfloat16).view(rows, H)
        per_f.append((sent, np.cumsum(sent) - 1, pos_ref, y2, dbg, rows))
    x_np = x.float().cpu().numpy()
    experts0 = ex_list[0]
    e00, P0 = experts0.expert_base, experts0.num_local
    if busiest:
        cnt0 = np.bincount(np.clip(ids64 - e00, -1, P0)[(ids64 >= e00) & (ids64 < e00 + P0)], minlength=P0)
        which = sorted(np.argsort(-cnt0, kind="stable")[:n_experts].tolist())
    else:
        which = list(range(n_experts))
    weights = _dequant_first(experts0, n_experts, which)
    sent0, cidx0, pos0, y2_0, dbg0, rows0 = per_f[0]
    sel = np.any(np.isin(ids64, e00 + np.asarray(which)), axis=1)
    tsel = np.nonzero(sel)[0]
    y_ref, used = moe.ffn_pairs(x_np[sel], ids_np[sel], w_np[sel], *weights, e00, P0, experts=which,
                                act_quant="fp8" if KIND == "fp8" else True)
    tt, jj = np.nonzero(used)
    prow = torch.from_numpy(pos0[cidx0[tsel[tt]], jj].astype(np.int64)).to(dev)
    y_gpu = y2_0.index_select(0, prow).float().cpu().numpy()
    rel = moe.rel_l2(y_gpu, y_ref[tt, jj])
    act_ok = None
    if KIND == "mxfp4":
        xq = _raw_bytes(dbg0["xq"], rows0 * H, dev.index).view(rows0, H).index_select(0, prow).cpu().numpy()
        kb = H // 32
        sfb = _raw_bytes(dbg0["xq_sf"], -(-rows0 // 128) * 128 * kb, dev.index).cpu().numpy()
        pr = prow.cpu().numpy()[:, None]
        sf = sfb[mx.sf_atom_offset(pr, np.arange(kb)[None, :], kb)]
        q_ref, s_ref = mx.mx_quantize(x_np[tsel[tt]])
        act_ok = bool(np.array_equal(xq, q_ref) and np.array_equal(sf, s_ref))
    rng = np.random.default_rng(seed)
    toks = np.sort(rng.choice(T, size=min(n_tokens, T), replace=False))
    replies, row_of = [], []
    for sent, cidx, pos_ref, y2, _, _ in per_f:
        hit = sent[toks]
        tp = np.full((len(toks), k), -1, np.int64)
        if hit.any():
            tp[hit] = pos_ref[cidx[toks[hit]]]
        live = tp >= 0
        gathered = y2.index_select(0, torch.from_numpy(np.where(live, tp, 0).reshape(-1).astype(np.int64)).to(dev))
        replies.append(moe.reduce_pairs(gathered.float().cpu().numpy().reshape(len(toks), k, H), live))
        row_of.append(np.where(hit, np.arange(len(toks)), -1).astype(np.int32))
    shared_rows = shared_out[toks].float().cpu().numpy() if shared_out is not None else None
    want = moe.combine(replies, np.stack(row_of), len(toks), shared_rows)
    got = out[toks].float().cpu().numpy()
    combine_ok = bool(np.array_equal(got, want))
    parity = {"checked": "timed configuration, last step's buffers", "tables_bitexact": tables,
              "f_ranks": len(per_f), "pairs": pairs, "experts_checked": [e00 + e for e in which],
              "pairs_checked": int(len(tt)),
              "rel_l2": round(rel, 6), "tol": 1e-2, "act_codes_bitexact": act_ok,
              "tokens_checked": int(len(toks)), "reply_combine_bitexact": combine_ok,
              "pass": bool(tables and rel < 1e-2 and act_ok is not False and combine_ok)}
    return parity, (x_np, ids_np, w_np, weights)


def cpu_config1(reps=3):
    """Config 1 on the host cores, the benchmark's own CPU case: the oracle's round trip (1 A replica, 2 F ranks
    x 8 experts, T=512, H=1024, top-2 softmax over N(0,1) logits, I=512, fp32 N(0, 0.02) weights, x bf16 N(0,1),
    seed 0, fp32 arithmetic with no activation quantisation)."""
    import numpy as np

    from oracle import moe, mx

    rng = np.random.default_rng(0)
    T1, H1, I1, E1 = 512, 1024, 512, 16
    experts = []
    for _ in range(2):
        w13 = rng.standard_normal((8, 2 * I1, H1)).astype(np.float32) * 0.02
        w2 = rng.standard_normal((8, H1, I1)).astype(np.float32) * 0.02
        experts.append((w13[:, :I1], w13[:, I1:], w2))
    x = mx.bf16_round(rng.standard_normal((T1, H1)).astype(np.float32))
    ids, w = moe.topk_routing(rng.standard_normal((T1, E1)), 2, "softmax")
    times = []
    for _ in range(reps):
        t = time.perf_counter()
        moe.round_trip(x, ids, w, [0, 8, 16], experts, act_quant=False)
        times.append(time.perf_counter() - t)
    dt = statistics.median(times)
    return {"value": round(T1 / dt, 1), "unit": "tokens/s", "ms_per_layer": round(dt * 1e3, 2),
            "sample": "config 1: one layer, T=512, H=1024, 16 experts over 2 F ranks, top-2 softmax, I=512, fp32"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_baseline(args.cpu_experts, steps=1)
    vals = []
    t_all = time.perf_counter()
    last = None
    for _ in range(args.steps):
        last = cpu_baseline(args.cpu_experts, steps=1)
        vals.append(last["value"])
    wall = time.perf_counter() - t_all
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32 (numpy)",
            "data": "synthetic",
            "config": {"workload": f"{'config 2' if KIND == 'mxfp4' else 'config 4'} layer, bounded CPU sample",
                       "tokens_per_replica": T_DEFAULT},
            "cpu_baseline": {**last, "value": v},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------ 1 GPU, Zipf sweep
def run_sweep(args):
    """Routing skew and job size on one GPU: one A rank and 4 F ranks (64 experts each, the 4A4F split) in
    loopback, Zipf(s=1.2) popularity, T in SWEEP_T.  Per T: tokens/s over K timed steps, the per-F row counts and
    their imbalance (max / mean), and from device timestamps (one globaltimer, one GPU) the doorbell latency --
    dispatch released the doorbells -> F rank 0's wait saw its doorbell -- and the F ranks' rows per second of
    busy time."""
    import torch

    import ctypes

    from asap_b200 import _native as N
    from asap_b200.dispatcher import AsapDispatcher
    from asap_b200.experts import Mxfp4Experts
    from asap_b200.loopback import Loopback
    from asap_b200.sglang_shim import StandardTopKOutput
    from asap_b200.transport.layout import Geometry

    dev = "cuda:0"
    torch.cuda.set_device(0)
    n_f = 4
    bounds = expert_bounds(n_f)
    per_f = [{0: Mxfp4Experts.random(bounds[f + 1] - bounds[f], H, I, expert_base=bounds[f], seed=100 + f,
                                     scale_lo=117, scale_hi=120)} for f in range(n_f)]
    T_max = max(SWEEP_T)
    lb = Loopback(Geometry(1, 1, 2, T_max, H, K_TOP, n_f), per_f, timeout_s=30.0, graphs=args.graphs)
    lb.install()
    shared = SharedExpert(dev)
    x_all = torch.randn(T_max, H, device=dev, generator=torch.Generator(device=dev).manual_seed(0)).to(torch.bfloat16)
    disp = AsapDispatcher(0)
    stream = torch.cuda.current_stream()
    for T in SWEEP_T:
        x = x_all[:T]
        ids, w = zipf_routing(T, 3, dev) if args.routing == "zipf" else make_routing(T, 3, dev)
        topk = StandardTopKOutput(w, ids)

        def step():
            d = disp.dispatch(x, topk)
            s_out = shared(x)
            return disp.combine(d, shared=s_out), d.ticket, s_out

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        lb.check()
        if not args.graphs:  # per-stage events are host-side marks: not inside captured graphs
            N.call("asap_ffn_enable_timing", lb.scheds[0].ws_handle, 1)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(0) as clocks:
            torch.cuda.synchronize()
            t0.record(stream)
            for _ in range(args.steps):
                step()
            t1.record(stream)
            torch.cuda.synchronize()
        lb.check()
        ms = t0.elapsed_time(t1) / args.steps
        f0_ms = None
        if not args.graphs:
            kms = (ctypes.c_float * 5)()
            N.call("asap_ffn_last_timing", lb.scheds[0].ws_handle, kms, 5)
            N.call("asap_ffn_enable_timing", lb.scheds[0].ws_handle, 0)
            f0_ms = dict(zip(("routing", "quantise_permute", "gemm1", "gemm2", "reduce_reply"),
                             [round(v, 4) for v in kms]))
        pairs_f = [int(sc.debug_tensors()["expert_counts"].sum().item()) for sc in lb.scheds]
        # the four F ranks share this one GPU: the step's bound is all their pairs' FLOPs or all experts' bytes
        roof = step_roofline(6.0 * H * I * sum(pairs_f), E * expert_bytes(), ms,
                             f"step of all {n_f} F ranks on this GPU ({sum(pairs_f)} pairs, every expert's weights "
                             "read once)")
        lat, busy, rows = [], [], None
        for _ in range(max(args.latency_iters, 1)):
            out, ticket, s_out = step()
            torch.cuda.synchronize()
            info = lb.channel.dispatch_info(ticket.slot, stream.cuda_stream)
            jobs = [sc.job_info(stream.cuda_stream) for sc in lb.scheds]
            rows = info["counts"]
            lat.append((jobs[0]["t_seen_ns"] - info["t_ring_ns"]) * 1e-3)
            busy.append(sum(j["t_reply_ns"] - j["t_seen_ns"] for j in jobs) * 1e-9)
        lb.check()
        # parity of this T on the last step's buffers (every F rank's tables and replies, F rank 0's busiest experts)
        parity, _ = check_single(x, ids, w, [d[0] for d in per_f], lb.scheds, out, s_out, busiest=True)
        mean_f = sum(rows) / n_f
        line = {
            "metric": METRIC, "value": round(T / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "mxfp8 x mxfp4 (fp32 accumulate), bf16 transport",
            "data": "synthetic", "workload_mode": "zipf-sweep",
            "config": {"workload": f"1 GPU loopback 1A{n_f}F: config 2 layer, T={T}, top-8 " + (
                           "Zipf(s=1.2) popularity over a seeded expert permutation" if args.routing == "zipf"
                           else "sigmoid"),
                       "tokens_per_replica": T, "a_replicas": 1, "f_ranks": n_f, "expert_bounds": bounds,
                       "parallelism": f"1A{n_f}F loopback", "routing": args.routing,
                       "f_jobs": "CUDA-graph replays" if args.graphs else "eager launches"},
            "f_rows": rows, "f_imbalance": round(max(rows) / mean_f, 4),
            "doorbell_to_f_start_us_p50": round(statistics.median(lat), 2),
            "f_rows_per_s": round(sum(rows) / statistics.median(busy), 1),
            "f_busy_ms_p50": round(statistics.median(busy) * 1e3, 4), "f0_kernels_ms": f0_ms,
            "weights_gb_read_per_step": round(E * (2 * I * H + H * I) * (0.5 + 1 / 32) / 1e9, 3),
            "e2e": None, "gpu_launches": args.steps * (4 + f_job_launches() * n_f), "roofline": roof,
            "f_pairs": pairs_f, "cpu_baseline": None, "parity": parity,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    lb.close()
    for d in per_f:
        d[0].release()


# ------------------------------------------------------------------------------------------ config 3: layer stack
N_LAYERS = 8


def run_stack(args):
    """Config 3: a stack of N_LAYERS config-2 layers, each A replica's T tokens as two micro-batches of T/2 on
    slots 0 and 1 (two-batch overlap): per layer dispatch(mb0), shared(mb0), dispatch(mb1), shared(mb1),
    combine(mb0), combine(mb1) through the public API (AsapDispatcher per layer), so each micro-batch's shared
    expert runs while its routed experts are away and the F ranks always hold the other slot's job.  The output of
    layer l, RMS-normalised, is the input of layer l+1.  N = 1: loopback (one F rank with all experts of all
    layers); N > 1: the --topology split (2a4f on 6 GPUs is the benchmark's), F jobs enqueued by a feeder
    thread.  value = tokens of all A replicas per second through the whole stack."""
    from datetime import timedelta

    import torch

    from asap_b200.dispatcher import AsapBuffer, AsapDispatcher
    from asap_b200.sglang_shim import StandardTopKOutput
    from asap_b200.transport.layout import Geometry

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    T = args.tokens
    Tmb = T // 2
    L = N_LAYERS
    steps_total = args.warmup + args.steps
    if world == 1:
        from asap_b200.loopback import Loopback

        n_a, n_f, is_a = 1, 1, True
        layers = {l: make_experts(E, 0, 1 + l, dev) for l in range(L)}
        lb = Loopback(Geometry(1, 1, 2, Tmb, H, K_TOP, 1), layers, timeout_s=60.0)
        lb.install()
        bounds = [0, E]
    else:
        import torch.distributed as dist

        from asap_b200.scheduler import FfnScheduler
        from asap_b200.transport.channel import AttnChannel
        from asap_b200.transport.server import FfnServer

        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
        n_a, n_f = topology(args.topology, world)
        a_ranks, f_ranks = placement(world, n_a, args.placement)
        g = Geometry(n_a, 1, 2, Tmb, H, K_TOP, n_f)
        bounds = expert_bounds(n_f)
        is_a = rank in a_ranks
        ep = None
        if not is_a:
            f = f_ranks.index(rank)
            layers = {l: make_experts(bounds[f + 1] - bounds[f], bounds[f], 100 + 10 * l + f, dev) for l in range(L)}
            server = FfnServer(f, g, device=local, run_dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else "/tmp",
                               host="127.0.0.1", port=0).start()
            sched = FfnScheduler(server, layers, timeout_s=120.0)
            ep = ("127.0.0.1", server.port)
        eps = [None] * world
        dist.all_gather_object(eps, ep)
        endpoints = [e for e in eps if e is not None]
        if is_a:
            channel = AttnChannel(a_ranks.index(rank), g, endpoints, device=local, expert_bounds=bounds,
                                  timeout_s=120.0).connect()
            AsapBuffer.attach(channel, local)
        dist.barrier()
        feeder = None
        if not is_a:
            fstream = torch.cuda.Stream(dev)

            def feed():
                torch.cuda.set_device(local)
                for step in range(steps_total + 1):  # + the parity step
                    for l in range(L):
                        for mb in range(2):
                            for a in range(n_a):
                                sched.run_device_wait(a, mb, step * L + l + 1, l, fstream.cuda_stream)

            feeder = threading.Thread(target=feed, daemon=True)
            feeder.start()
    ms = 0.0
    clocks_summary = None
    if is_a:
        a_index = 0 if world == 1 else a_ranks.index(rank)
        shared = SharedExpert(dev)
        gen = torch.Generator(device=dev).manual_seed(a_index)
        x_in = [torch.randn(Tmb, H, device=dev, generator=gen).to(torch.bfloat16) for _ in range(2)]
        topk = [[StandardTopKOutput(*reversed(make_routing(Tmb, 1000 * a_index + 10 * l + mb, dev))) for mb in range(2)]
                for l in range(L)]
        disps = [AsapDispatcher(l) for l in range(L)]

        def norm(t):  # the RMSNorm in front of every DeepSeek MoE block (keeps the stack's activations bounded)
            return torch.nn.functional.rms_norm(t, (H,))

        def step(record=False):
            xs, rec = x_in, None
            for l in range(L):
                d0 = disps[l].dispatch(xs[0], topk[l][0], micro_batch=0)
                s0 = shared(xs[0])
                d1 = disps[l].dispatch(xs[1], topk[l][1], micro_batch=1)
                s1 = shared(xs[1])
                c0 = disps[l].combine(d0, shared=s0)
                n0 = norm(c0)
                c1 = disps[l].combine(d1, shared=s1)
                if record and l == L - 1:  # the last layer's second micro-batch: the F ranks' last job
                    rec = (xs[1], topk[l][1], c1, s1)
                xs = [n0, norm(c1)]
            return (xs, rec) if record else xs

        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if is_a:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            t0.record()
            for _ in range(args.steps):
                out = step()
            t1.record()
            torch.cuda.synchronize()
        clocks_summary = clocks.summary()
        ms = t0.elapsed_time(t1) / args.steps
        finite = bool(torch.isfinite(out[0]).all().item() and torch.isfinite(out[1]).all().item())
        # parity step: one more pass; the last layer's second micro-batch is checked below
        _, rec = step(record=True)
        torch.cuda.synchronize()
    parity = None
    if world > 1:
        mt = torch.tensor([ms])
        dist.all_reduce(mt, op=dist.ReduceOp.MAX)
        ms = float(mt.item())
        if feeder is not None:
            feeder.join()
        torch.cuda.synchronize()
        (sched if not is_a else channel).check()
        dist.barrier()
        mine = None
        if is_a:  # against a 1-GPU loopback twin of the last layer (its experts regenerated from the F seeds)
            xr, tk, cr, sr = rec
            counts = channel.dispatch_info(1, torch.cuda.current_stream().cuda_stream)["counts"]
            mine = twin_check((xr, tk.topk_ids, tk.topk_weights, sr, cr, counts), bounds, dev, local,
                              seed_base=100 + 10 * (L - 1))
        parities = [None] * world
        dist.all_gather_object(parities, mine)
        parities = [p for p in parities if p is not None]
        parity = {"mode": "last layer, micro-batch 1 of the parity step: each A replica's output and per-F row "
                          "counts against a 1-GPU loopback twin of that layer (same experts, same tokens), byte "
                          "for byte", "replicas": len(parities),
                  "output_bitexact": all(p["output_bitexact"] for p in parities),
                  "tables_bitexact": all(p["tables_bitexact"] for p in parities),
                  "counts_match_routing": all(p["counts_match_routing"] for p in parities),
                  "pass": all(p["pass"] for p in parities)}
    else:
        lb.check()
        xr, tk, cr, sr = rec
        parity, _ = check_single(xr, tk.topk_ids, tk.topk_weights, layers[L - 1], lb.sched, cr, sr)
        parity["checked"] = "last layer, micro-batch 1 of the parity step (the F rank's last job)"
    if rank == 0:
        line = {
            "metric": "MoE layer-stack tokens/s A->F->A (8 DeepSeek-V3-shape MXFP4 layers, 2 micro-batches)",
            "value": round(n_a * T / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": DTYPE[KIND], "data": "synthetic", "workload_mode": "stack",
            "config": {"workload": f"config 3: {L} stacked config-2 layers, {n_a}A{n_f}F, T={T} per A replica as "
                                   f"2 micro-batches of {Tmb} on slots 0/1, shared expert between dispatch and "
                                   "combine, uniform (sigmoid top-8) routing", "tokens_per_replica": T,
                       "a_replicas": n_a, "f_ranks": n_f, "layers": L, "parallelism": f"{n_a}A{n_f}F",
                       "expert_bounds": bounds},
            "layer_tokens_per_s": round(n_a * T * L / (ms * 1e-3), 1), "output_finite": finite,
            "e2e": None, "gpu_launches": args.steps * L * 2 * (4 + f_job_launches() * n_f) * n_a,
            "roofline": step_roofline(
                6.0 * H * I * L * n_a * T * K_TOP * max(bounds[f + 1] - bounds[f] for f in range(n_f)) / E,
                L * max(bounds[f + 1] - bounds[f] for f in range(n_f)) * expert_bytes(), ms,
                "stack step of the busiest F rank (uniform routing: its share of every layer's pairs)"),
            "cpu_baseline": None, "parity": parity, "clocks": clocks_summary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if is_a:
            channel.unmap_peers()
        else:
            server.unmap_peers()
        dist.barrier()
        if is_a:
            AsapBuffer.install(None)
            channel.close()
        else:
            sched.close()
            server.close()
            for e in layers.values():
                e.release()
        dist.barrier()
        dist.destroy_process_group()
    else:
        lb.close()
        for e in layers.values():
            e.release()


# ------------------------------------------------------------------------------------------ N GPUs
def expert_bounds(num_f):
    return [(f * E) // num_f for f in range(num_f + 1)]


def twin_check(check, bounds, dev, local, seed_base=100):
    """An A replica's parity-step output against a 1-GPU loopback twin: the same experts (regenerated from the F
    ranks' seeds on this GPU), the same tokens, routing and shared-expert rows, one F scheduler per F rank over the
    same transport.  The kernels are deterministic, so the combined output and the per-F row counts must match
    byte for byte; the counts are also checked against the routing itself (tokens with an expert in each F rank's
    range).  F rank f's experts are regenerated from seed ``seed_base + f``."""
    import torch

    from asap_b200.dispatcher import AsapBuffer, AsapDispatcher
    from asap_b200.loopback import Loopback
    from asap_b200.sglang_shim import StandardTopKOutput
    from asap_b200.transport.layout import Geometry

    x, ids, w, s, out, counts = check
    T, n_f = x.shape[0], len(bounds) - 1
    per_f = [{0: make_experts(bounds[f + 1] - bounds[f], bounds[f], seed_base + f, dev)} for f in range(n_f)]
    lb = Loopback(Geometry(1, 1, 1, T, H, K_TOP, n_f), per_f, device=local, timeout_s=30.0)
    prev = AsapBuffer._buffer
    lb.install()
    try:
        disp = AsapDispatcher(0)
        d = disp.dispatch(x, StandardTopKOutput(w, ids))
        twin = disp.combine(d, shared=s)
        torch.cuda.synchronize()
        lb.check()
        twin_counts = lb.channel.dispatch_info(d.ticket.slot, torch.cuda.current_stream().cuda_stream)["counts"]
        ids64 = ids.long()
        want = [int(((ids64 >= bounds[f]) & (ids64 < bounds[f + 1])).any(dim=1).sum().item()) or 1
                for f in range(n_f)]  # a rank with no token is announced one padding row
        res = {"output_bitexact": bool(torch.equal(out.view(torch.int16), twin.view(torch.int16))),
               "tables_bitexact": list(counts) == list(twin_counts),
               "counts_match_routing": list(counts) == want}
    finally:
        lb.close()
        AsapBuffer.install(prev)
        for dct in per_f:
            dct[0].release()
    res["pass"] = all(res.values())
    return res


def measure_links(args, is_a, channel, sched, stream, send_stream, x_all, a_idx, n_a, n_f, a_ranks, f_ranks, seqs,
                  rank, world, dev, T, rounds=5):
    """NVLink rates of an N-GPU run, measured on the device (CUDA events), max/median over ranks by gather:
      * dispatch: each A rank's algorithmic bytes (x row + ids + weights per routed row, every F rank) / the
        dispatch kernels' time, all replicas sending at once (as in a step);
      * reply: each F rank's reply bytes (one bf16 row per routed row) / its reduce+reply kernel time;
      * ce_peer_write: a 256 MB copy-engine write from each A rank into F rank (a mod F)'s unused slot-1 region,
        the link rate the layer roofline divides by.
    Every rank takes the same collective steps."""
    import ctypes

    import torch
    import torch.distributed as dist

    from asap_b200 import _native as N
    from asap_b200.transport.server import _raw_bytes

    res = {}
    if not is_a:
        sched.enable_timing(True)
        for r in range(rounds):
            for a in range(n_a):
                sched.run_device_wait(a, 0, seqs[a] + 1 + r, 0, stream.cuda_stream)
    dist.barrier()
    if is_a:
        ids_l, w_l = make_routing(T, 10 + a_idx, dev)
        xx = x_all[:T]
        times, nbytes = [], 0
        for r in range(rounds):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            send_stream.wait_stream(stream)
            e0.record(send_stream)
            t = channel.send(0, 0, xx.data_ptr(), ids_l.data_ptr(), w_l.data_ptr(), T, send_stream.cuda_stream)
            e1.record(send_stream)
            out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
            channel.combine(t, out.data_ptr(), stream.cuda_stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        counts = channel.dispatch_info(0, stream.cuda_stream)["counts"]
        nbytes = sum(counts) * (2 * H + 8 * K_TOP)
        res = {"dispatch_ms": statistics.median(times), "dispatch_bytes": nbytes, "counts": counts}
    else:
        torch.cuda.synchronize()
        kms = sched.last_timing()
        sched.enable_timing(False)
        res = {"reply_ms": float(kms[4]) if kms else 0.0}  # mean over this rank's jobs of the rounds
    dist.barrier()
    # copy-engine peer write, each A rank into one F rank's slot-1 region (unused by this benchmark)
    if is_a:
        f = a_idx % n_f
        g = channel.g
        nb = min(256 << 20, g.region_bytes)
        dst = _raw_bytes(channel.recv_bases[f] + g.region_off(a_idx, 1), nb, torch.cuda.current_device())
        src = torch.empty(nb, dtype=torch.uint8, device=dev)
        dst.copy_(src)
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    if is_a:
        c0.record()
        for _ in range(10):
            dst.copy_(src)
        c1.record()
        torch.cuda.synchronize()
        res["ce_write_gbs"] = 10 * nb / (c0.elapsed_time(c1) * 1e-3) / 1e9
    dist.barrier()
    allr = [None] * world
    dist.all_gather_object(allr, res)
    a_res = [allr[r] for r in a_ranks]
    f_res = [allr[r] for r in f_ranks]
    disp = [ar["dispatch_bytes"] / (ar["dispatch_ms"] * 1e-3) / 1e9 for ar in a_res]
    # F rank f's mean reply: one bf16 row per row it received, averaged over the replicas' messages
    rows_f = [statistics.mean(ar["counts"][f] for ar in a_res) for f in range(n_f)]
    reply = [rows_f[f] * 2 * H / (fr["reply_ms"] * 1e-3) / 1e9 if fr["reply_ms"] > 0 else None
             for f, fr in enumerate(f_res)]
    ce = [ar["ce_write_gbs"] for ar in a_res]
    return {"dispatch_gbs_per_a": [round(v, 1) for v in disp],
            "dispatch_ms_per_a": [round(ar["dispatch_ms"], 4) for ar in a_res],
            "reply_gbs_per_f": [round(v, 1) if v else None for v in reply],
            "ce_peer_write_gbs": [round(v, 1) for v in ce], "ce_peer_write_gbs_median": round(statistics.median(ce), 1),
            "nominal_gbs_per_direction": NVLINK_NOMINAL_GBS,
            "note": "dispatch = P2P stores of every replica at once (an F rank's inbound link is shared by all "
                    "replicas); reply = the F rank's reduce+reply kernel, whose stores cross NVLink into the A rank; "
                    "CUDA events on the launching streams, median of the rounds"}


def run_multi(args):
    """N GPUs, one process each: ranks [0, n_a) are A replicas, the rest F ranks (--topology, default half/half).
    Each F rank's jobs are enqueued by a feeder thread (each job starts with a bounded device wait for its
    doorbell), so the main thread stays free for the gloo barriers even when the launch queue is full."""
    import ctypes
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from asap_b200 import _native as N
    from asap_b200.experts import Mxfp4Experts
    from asap_b200.scheduler import FfnScheduler
    from asap_b200.transport.channel import AttnChannel, serve_order
    from asap_b200.transport.layout import Geometry
    from asap_b200.transport.server import FfnServer

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=timedelta(seconds=90))
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    binding = bind_numa(local) if not args.no_numa_bind else {"unbound": "--no-numa-bind"}
    n_a, n_f = topology(args.topology, world)
    sweep = args.workload == "zipf-sweep"
    t_list = SWEEP_T if sweep else [args.tokens]
    T_max = max(t_list)
    g = Geometry(n_a, 1, 2, T_max, H, K_TOP, n_f)
    bounds = expert_bounds(n_f)
    p_max = max(bounds[i + 1] - bounds[i] for i in range(n_f))
    ftr = [first_then_rest(args, n_a, T, p_max) for T in t_list]  # F serving mode per token count of the run
    a_ranks, f_ranks = placement(world, n_a, args.placement)
    is_a = rank in a_ranks
    a_idx = a_ranks.index(rank) if is_a else -1
    lat_iters = args.latency_iters if sweep else 0
    phases = len(t_list) * (1 if sweep else 2)  # timed (+ e2e) per token count
    steps_per_phase = args.warmup + args.steps
    timeout_s = 120.0
    ep = None
    if not is_a:
        f = f_ranks.index(rank)
        experts = make_experts(bounds[f + 1] - bounds[f], bounds[f], 100 + f, dev)
        server = FfnServer(f, g, device=local, run_dir="/dev/shm" if os.access("/dev/shm", os.W_OK) else "/tmp",
                           host="127.0.0.1", port=0).start()
        sched = FfnScheduler(server, {0: experts}, timeout_s=timeout_s,
                             join=n_a if (args.join_replicas or any(ftr)) else 1,
                             overlap_replies=args.overlap_replies if n_a > 1 and not args.graphs else 0)
        ep = ("127.0.0.1", server.port)
    eps = [None] * world
    dist.all_gather_object(eps, ep)
    endpoints = [e for e in eps if e is not None]
    if is_a:
        channel = AttnChannel(a_idx, g, endpoints, device=local, expert_bounds=bounds, timeout_s=timeout_s).connect()
    dist.barrier()
    feeder = None
    if not is_a:
        stream = torch.cuda.Stream(dev)
        queued = phases * steps_per_phase + 1  # + the parity-check step

        def feed():
            torch.cuda.set_device(local)
            for s in range(queued):
                if args.join_replicas:  # one job answers every replica's message of this step
                    msgs = [(a, 0, s + 1) for a in range(n_a)]
                    if args.graphs:
                        sched.run_graph(msgs, 0, stream.cuda_stream)
                    else:
                        sched.run_device_wait_rows(msgs, 0, stream.cuda_stream)
                    continue
                ov = sched.reserve > 0  # every job of the step but its last replies from the side stream
                if ftr[min(s // (steps_per_phase * (1 if sweep else 2)), len(t_list) - 1)]:
                    # the first ready message alone, then the rest of the step together
                    sched.run_device_wait_any([(a, 0) for a in range(n_a)], 0, stream.cuda_stream, overlap=ov)
                    sched.run_device_wait_rest([(a, 0, s + 1) for a in range(n_a)], 0, stream.cuda_stream)
                    continue
                if args.any_order:  # each job answers whichever replica's message is ready first (round robin)
                    for i in range(n_a):
                        sched.run_device_wait_any([(a, 0) for a in range(n_a)], 0, stream.cuda_stream,
                                                  graph=args.graphs, overlap=ov and i < n_a - 1)
                    continue
                # fixed order: answer the A ranks in the order their messages complete here (send_order)
                for a in serve_order(f, n_a, n_f):
                    if args.graphs:
                        sched.run_graph([(a, 0, s + 1)], 0, stream.cuda_stream)
                    else:
                        sched.run_device_wait(a, 0, s + 1, 0, stream.cuda_stream)

        if not args.graphs:  # per-stage CUDA events of every job (host-side marks: not inside captured graphs)
            sched.enable_timing(True)
        feeder = threading.Thread(target=feed, daemon=True)
        feeder.start()
    else:
        shared = SharedExpert(dev) if SHARED else None
        gen = torch.Generator(device=dev).manual_seed(a_idx)
        x_all = torch.randn(T_max, H, device=dev, generator=gen).to(torch.bfloat16)
        send_stream = torch.cuda.Stream(dev)
        stream = torch.cuda.current_stream()

    def timed(fn, finish=None, clocks=None):
        for _ in range(args.warmup):
            fn()
        if is_a:
            torch.cuda.synchronize()
        dist.barrier()
        ms = 0.0
        if clocks is not None:
            clocks.mark_start()
        if is_a:
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(args.steps):
                fn()
            if finish is not None:
                finish()
            t1.record()
            torch.cuda.synchronize()
            ms = t0.elapsed_time(t1) / args.steps
        if clocks is not None:
            clocks.mark_end()
        mt = torch.tensor([ms])
        dist.all_reduce(mt, op=dist.ReduceOp.MAX)
        dist.barrier()
        return float(mt.item())

    results = []
    clock_summary = None
    for T in t_list:
        if is_a:
            x = x_all[:T]
            ids, w = (zipf_routing(T, 10 + a_idx, dev) if args.routing == "zipf" else
                      make_routing(T, 10 + a_idx, dev))

            def step(xx=x, ii=ids, ww=w, TT=T):
                send_stream.wait_stream(stream)
                t = channel.send(0, 0, xx.data_ptr(), ii.data_ptr(), ww.data_ptr(), TT, send_stream.cuda_stream)
                s = shared(xx) if shared is not None else None
                out = torch.empty(TT, H, dtype=torch.bfloat16, device=dev)
                channel.combine(t, out.data_ptr(), stream.cuda_stream, s.data_ptr() if s is not None else 0)
                return out
        with ClockSampler(local) as clocks:
            ms = timed(step if is_a else (lambda: None), clocks=clocks)
        clock_summary = clocks.summary()
        res = {"T": T, "ms": ms}
        if is_a:
            channel.check()
            counts = channel.dispatch_info(0, stream.cuda_stream)["counts"]
        else:
            counts = None
        allc = [None] * world
        dist.all_gather_object(allc, counts)
        per_f = [sum(allc[r][f] for r in a_ranks) for f in range(n_f)]
        res["f_rows"] = per_f
        if not sweep:
            if is_a:
                pipe = HostPipeline(x, ids, w, dev, lambda dx, di, dw: step(dx, di, dw))

                def e2e_step():
                    pipe.run(1)
            res["e2e_ms"] = timed(e2e_step if is_a else (lambda: None), pipe.finish if is_a else None)
        results.append(res)
    # parity step: every replica sends its last message once more; its output is checked against a 1-GPU
    # loopback twin below (after the F ranks have answered everything)
    check = None
    if is_a:
        send_stream.wait_stream(stream)
        s_chk = shared(x) if shared is not None else None
        t_chk = channel.send(0, 0, x.data_ptr(), ids.data_ptr(), w.data_ptr(), T, send_stream.cuda_stream)
        out_chk = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        channel.combine(t_chk, out_chk.data_ptr(), stream.cuda_stream, s_chk.data_ptr() if s_chk is not None else 0)
        torch.cuda.synchronize()
        channel.check()
        check = (x, ids, w, s_chk, out_chk, channel.dispatch_info(0, stream.cuda_stream)["counts"])
    if feeder is not None:
        feeder.join()
    torch.cuda.synchronize()  # F: every queued job has now been answered
    if is_a:
        channel.check()
    else:
        sched.check()
    parity = twin_check(check, bounds, dev, local) if is_a else None
    parities = [None] * world
    dist.all_gather_object(parities, parity)
    parities = [p for p in parities if p is not None]
    # the F ranks' mean per-stage kernel times over their last 64 jobs (the end of the last phase and the parity step)
    fk = None
    if not is_a and not args.graphs:
        fk = sched.last_timing()
        sched.enable_timing(False)
    fks = [None] * world
    dist.all_gather_object(fks, fk)
    fks = [v for v in fks if v is not None]
    f_kernels = None
    if fks:
        stages = ("routing", "quantise_permute", "gemm1", "gemm2", "reduce_reply")
        mean = [statistics.mean(v[i] for v in fks) for i in range(5)]
        f_kernels = {"per_job_ms_mean_over_f": {k: round(v, 4) for k, v in zip(stages, mean)},
                     "per_job_ms_sum": round(sum(mean), 4),
                     "note": "CUDA events per stage inside each F job, mean over each F rank's last 64 jobs (of the "
                             "last token count), then over the F ranks; replies on a side stream: "
                             + (f"every job of a step but its last, on {args.overlap_replies} SMs"
                                if args.overlap_replies and n_a > 1 else "no") + "; jobs per step per F rank: "
                             + ("2 (first ready, then the rest joined)" if ftr[-1] else
                                "1 (joined)" if args.join_replicas else str(n_a))}
    # doorbell latency: one message at a time from A rank 0, F ranks idle and already spinning on their doorbell
    lat = []
    seq_next = phases * steps_per_phase + 2
    for r in range(lat_iters):
        T = t_list[0]
        if not is_a:
            sched.run_device_wait(0, 0, seq_next + r, 0, stream.cuda_stream)
        dist.barrier()
        info = None
        if rank == 0:
            ids, w = zipf_routing(T, 10, dev) if args.routing == "zipf" else make_routing(T, 10, dev)
            step(x_all[:T], ids, w, T)
            torch.cuda.synchronize()
            info = channel.dispatch_info(0, stream.cuda_stream)
        elif not is_a:
            torch.cuda.synchronize()
            info = sched.job_info(stream.cuda_stream)
        infos = [None] * world
        dist.all_gather_object(infos, info)
        if rank == 0:
            a0 = infos[0]
            fi = [infos[r] for r in f_ranks]
            busy = [(i["t_reply_ns"] - i["t_seen_ns"]) * 1e-3 for i in fi]
            rt = (a0["t_replies_ns"] - a0["t_ring_ns"]) * 1e-3
            lat.append({"round_trip_us": rt, "f_busy_us": busy, "signal_us": rt - max(busy)})
    if is_a:
        channel.check()
    else:
        sched.check()
    dist.barrier()
    # NVLink rates, at the largest token count of the run: every replica sends one message at a time (all replicas
    # at once, F ranks idle and already waiting), CUDA events around each A rank's dispatch and the F ranks'
    # per-stage timing of their replies; then a copy-engine write of 256 MB from each A rank into one F rank's
    # unused slot-1 region (the link rate the roofline uses)
    seq_a = phases * steps_per_phase + 1 + (lat_iters if a_idx == 0 else 0)  # the replica's last message
    seqs = [None] * world
    dist.all_gather_object(seqs, seq_a if is_a else None)
    seqs = [seqs[r] for r in a_ranks]
    link = measure_links(args, is_a, channel if is_a else None, sched if not is_a else None,
                         stream, send_stream if is_a else None, x_all if is_a else None, a_idx, n_a, n_f, a_ranks,
                         f_ranks, seqs, rank, world, dev, T_max)
    if is_a:
        channel.check()
    else:
        sched.check()
    dist.barrier()
    if rank == 0:
        h2d = T_max * H * 2 + T_max * K_TOP * 8
        base = {
            "metric": METRIC, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": DTYPE[KIND], "data": "synthetic",
            "gpu_launches": args.steps * (4 * n_a +
                                          (f_job_launches(n_a) if args.join_replicas else
                                           f_job_launches() + f_job_launches(n_a)
                                           if first_then_rest(args, n_a, T, p_max)
                                           else f_job_launches() * n_a) * n_f), "roofline": None,  # set per line below
            "cpu_baseline": None,
            "clocks": clock_summary,
        }
        for res in results:
            T, ms = res["T"], res["ms"]
            mean_f = sum(res["f_rows"]) / n_f
            line = dict(base, value=round(n_a * T / (ms * 1e-3), 1), ms_per_step=round(ms, 4))
            line["config"] = {
                "workload": (f"{n_a}A{n_f}F: config 2 layer per A replica (T={T}, H=7168, 256 experts, "
                             f"top-8 {'Zipf(s=1.2) popularity' if args.routing == 'zipf' else 'sigmoid'}, I=2048, "
                             "MXFP4, 1 bf16 shared expert)") if KIND == "mxfp4" else
                            (f"{n_a}A{n_f}F: config 4 layer per A replica (T={T}, H={H}, {E} experts, top-{K_TOP} "
                             f"softmax, I={I}, FP8 E4M3 with fp32 128x128 block scales)"),
                "tokens_per_replica": T, "a_replicas": n_a, "f_ranks": n_f, "parallelism": f"{n_a}A{n_f}F",
                "expert_bounds": bounds, "routing": args.routing,
                "placement": args.placement, "a_ranks": a_ranks,
                "f_jobs": ("one joined job per step (all replicas' messages)" if args.join_replicas else
                           "two jobs per step: the first ready message alone, then the step's other messages joined"
                           if first_then_rest(args, n_a, T, p_max) else
                           "one job per message" + (", first ready replica first (round robin on the device)"
                                                    if args.any_order else ""))
                          + (", CUDA-graph replays" if args.graphs else ""), "host_binding": binding,
                "dispatch": "one pass, F ranks filled in turn from a*F/A (each doorbell rung when its rows are stored)",
                "l2": "inputs larger than L2, no flush"
                if T >= 4096 else "x smaller than L2 (weights 6 GB are not)"}
            line["f_rows"] = res["f_rows"]
            line["f_imbalance"] = round(max(res["f_rows"]) / mean_f, 4) if mean_f else None
            p_max = max(bounds[f + 1] - bounds[f] for f in range(n_f))
            line["roofline"] = step_roofline(6.0 * H * I * n_a * T * K_TOP * p_max / E, p_max * expert_bytes(), ms,
                                             "layer step of the busiest F rank (expected pairs of uniform routing)")
            if args.routing != "zipf":
                line["layer_roofline"] = layer_roofline(n_a, T, res["f_rows"], bounds, ms, *load_peaks(),
                                                        nvlink_gbs=link["ce_peer_write_gbs_median"])
            line["parity"] = {"mode": "each A replica's parity-step output and per-F row counts against a 1-GPU "
                                      "loopback twin (same experts, same tokens), byte for byte, and the row counts "
                                      "against the routing", "tokens_per_replica": t_list[-1],
                              "replicas": len(parities),
                              "output_bitexact": all(p["output_bitexact"] for p in parities),
                              "tables_bitexact": all(p["tables_bitexact"] for p in parities),
                              "counts_match_routing": all(p["counts_match_routing"] for p in parities),
                              "pass": all(p["pass"] for p in parities)}
            line["nvlink"] = link
            if res is results[-1] and f_kernels is not None:
                line["f_kernels_ms"] = f_kernels
            if "e2e_ms" in res:
                e = res["e2e_ms"]
                line["e2e"] = {"value": round(n_a * T / (e * 1e-3), 1), "unit": "tokens/s",
                               "h2d_bytes_per_step": n_a * h2d, "d2h_bytes_per_step": n_a * T * H * 2,
                               "ms_per_step": round(e, 4)}
            else:
                line["e2e"] = None
            if sweep:
                line["workload_mode"] = "zipf-sweep"
            print(json.dumps(line), flush=True)
        if lat:
            print(json.dumps({"workload_mode": "doorbell-latency", "n_gpus": world, "parallelism": f"{n_a}A{n_f}F",
                              "tokens": t_list[0], "iters": len(lat),
                              "round_trip_us_p50": round(statistics.median(l["round_trip_us"] for l in lat), 2),
                              "signal_us_p50": round(statistics.median(l["signal_us"] for l in lat), 2),
                              "f_busy_us_p50": round(statistics.median(max(l["f_busy_us"]) for l in lat), 2),
                              "note": "signal = A round trip (doorbell release -> combine saw every done flag, A "
                                      "clock) - slowest F's busy time (doorbell seen -> done flag released, F clock): "
                                      "one doorbell plus one done-flag hop; no cross-GPU clock needed"}), flush=True)
    # orderly shutdown: every process unmaps its peers' memory before any process frees its own
    dist.barrier()
    if is_a:
        channel.unmap_peers()
    else:
        server.unmap_peers()
    dist.barrier()
    if is_a:
        channel.close()
    else:
        sched.close()
        server.close()
        experts.release()
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--tokens", type=int, default=None, help="tokens per A replica (default: the layer's T)")
    ap.add_argument("--experts", type=int, default=None, help="routed experts (small profiling cases)")
    ap.add_argument("--cpu-experts", type=int, default=4)
    ap.add_argument("--no-e2e", action="store_true", help="skip the e2e leg (profiling runs)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-flashinfer", action="store_true", help="skip the FlashInfer expert-backend bar")
    ap.add_argument("--workload", choices=("layer", "fp8-layer", "zipf-sweep", "stack"), default="layer",
                    help="layer: config 2 (MXFP4); fp8-layer: config 4 (FP8 block-scaled); zipf-sweep: config 5, "
                         "T in 256/1024/4096/16384 with skewed routing, one line per T; stack: config 3, 8 layers "
                         "x 2 micro-batches")
    ap.add_argument("--routing", choices=("sigmoid", "zipf"), default=None,
                    help="default: sigmoid for the layer workload, zipf for the sweep")
    ap.add_argument("--topology", default="half", help="N>1: half (NA/NF), 2a6f (8 GPUs), 2a4f (6 GPUs)")
    ap.add_argument("--latency-iters", type=int, default=10, help="zipf-sweep: single-message latency samples")
    ap.add_argument("--graphs", action="store_true",
                    help="F jobs as CUDA-graph replays (FfnScheduler.run_graph; zipf-sweep and N>1)")
    ap.add_argument("--placement", choices=("block", "interleave"), default="interleave",
                    help="N>1: which ranks are A replicas: interleave (default) = spread over the box, so that their "
                         "host copies use different host links; block = the first N_A")
    ap.add_argument("--fixed-order", action="store_true",
                    help="N>1: F ranks answer the replicas in a fixed order (default: each F job answers the first "
                         "ready replica's message, round robin, asap_ffn_wait_any -- the reference's poll order)")
    ap.add_argument("--no-numa-bind", action="store_true", help="N>1: do not bind ranks to their GPU's NUMA node")
    ap.add_argument("--join-replicas", action="store_true",
                    help="N>1: each F rank answers all A replicas' messages of a step with one joined job")
    ap.add_argument("--overlap-replies", type=int, default=0,
                    help="N>1: SMs left to the F ranks' replies, which then run on a side stream while the step's "
                         "next job computes (every job of a step but its last; 0 = each reply in its job's order)")
    ap.add_argument("--serve", choices=("auto", "per-message", "first-then-rest"), default="auto",
                    help="N>1, several A replicas: per-message = one F job per message; first-then-rest = the first "
                         "ready message of a step alone (asap_ffn_wait_any), then the step's other messages as one "
                         "joined job (asap_ffn_wait_rest); auto = first-then-rest with three or more replicas when a "
                         f"message brings an F rank fewer than {FTR_PAIRS} expected pairs (small jobs: fewer chains), "
                         "else per-message (the replies of earlier jobs overlap later jobs' compute)")
    args = ap.parse_args()
    layer = LAYERS["fp8-layer" if args.workload == "fp8-layer" else "layer"]
    globals().update(layer)
    if args.tokens is None:
        args.tokens = T_DEFAULT
    if args.experts is not None:
        globals()["E"] = args.experts
    if args.warmup < 3:
        args.warmup = 3
    if args.routing is None:
        args.routing = "zipf" if args.workload == "zipf-sweep" else ROUTING
    args.any_order = not args.fixed_order
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "stack":
        run_stack(args)
    elif int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_multi(args)
    elif args.workload == "zipf-sweep":
        run_sweep(args)
    else:
        run_single(args)


if __name__ == "__main__":
    main()
