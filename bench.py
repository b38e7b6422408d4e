"""Benchmark of the Mamba-3 SISO scan path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--what ...]

Headline (BASELINE.json ``configs[1]``): the chunked-scan forward at B=8 H=32 L=8192
N=128 P=64 chunk=128, bf16 operands / fp32 state, through the fused raw boundary
(preprocess in-kernel).  One "step" is one forward over the whole batch; ``value`` is
tokens/s over all ranks, device-timed with CUDA events (max over ranks), inputs resident
in HBM and larger than L2 (nothing is cached between steps).  The same line carries

* ``e2e``       -- the same metric through the public API with pinned host buffers:
                   every step copies the inputs host->device and y device->host;
* ``roofline``  -- the forward kernel against the measured HBM / bf16 peaks;
* ``fwd_bwd``   -- forward + backward tokens/s at the same shapes;
* ``decode``    -- the 24-layer LM decode step at B=256: us/token, plus
                   the decode kernel's own HBM roofline;
* ``cpu_baseline`` -- the CPU oracle restatement of the reference (``oracle/``) timed on
                   this host's cores on a bounded sample of the forward workload;
* ``torch_ref_baseline`` -- beside it, the reference's own plain-torch recurrent
                   reference (``torch_ref.mamba3_siso_ref``, from baseline/_ref when installed).

Multi-GPU (torchrun): strong scaling.  configs[1]'s batch of 8 sequences x 32 heads is
split over the ranks by batch (B / N per rank, all heads), configs[3]'s decode batch of
256 likewise, and configs[4]'s global training batch of 64; the (b, h) pairs of the scan
are independent, so there is no collective on the scan's data path.  ``value`` is the
global problem's tokens over the slowest rank's device time.
``--impl reference`` times the reference's CPU path (the oracle port; JAX is absent, so
the reference's own Pallas-interpret / reference.py path cannot run) on rank 0, and the
reference's ``torch_ref.py`` beside it.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mamba3-siso-tpu_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "fwd & fwd+bwd tok/s @B8 H32 L8192 N128 P64 bf16; decode µs/token @B=256"
CFG2 = dict(B=8, H=32, L=8192, N=128, P=64, Nr=64, chunk=128)
FWD_FLOP_PER_TOKEN_HEAD = 2 * (128 * 128 + 128 * 64 + 2 * 128 * 64)          # 81,920 at C=128
BWD_FLOP_PER_TOKEN_HEAD = 2 * (128 * (2 * 64 + 3 * 128) + 4 * 64 * 128)      # 196,608


def fwd_bytes_per_token_head(c):
    """Algorithmic HBM bytes of the fused forward per (token, head): v, z in and y out
    (bf16, P each), head-shared q/k (bf16, N each, shared by H heads), the raw dt/A/trap
    streams (f32) and the head-shared raw angles (f32, Nr, shared by H heads)."""
    return 3 * c["P"] * 2 + 2 * c["N"] * 2 / c["H"] + 3 * 4 + c["Nr"] * 4 / c["H"]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


TRAFFIC_SOURCES = ("m3_fwd_ws.cuh", "m3_chunk_common.cuh", "m3_umma.cuh", "m3_fwd.cu", "m3_common.cuh")


def kernel_source_hash(files=TRAFFIC_SOURCES):
    """Short sha256 over the forward kernel's source files (what a traffic capture is tied to)."""
    h = hashlib.sha256()
    for f in files:
        h.update(open(os.path.join(ROOT, "mamba3-siso-tpu_b200", "csrc", f), "rb").read())
    return h.hexdigest()[:16]


def load_traffic():
    """Per-launch DRAM bytes of the profiled kernels (from one ncu capture), keyed by kernel.

    A line reads `<kernel> <bytes> src=<hash>`: the hash of the kernel sources the capture was
    taken with.  A figure whose hash differs from the sources being benched is stale and is
    returned as None, so the bench line never carries traffic of another build."""
    p = os.path.join(ROOT, "profiles", "traffic.txt")
    out = {}
    if not os.path.exists(p):
        return out
    cur = kernel_source_hash()
    for line in open(p):
        parts = line.split()
        if len(parts) >= 2 and not line.startswith("#"):
            try:
                val = float(parts[1])
            except ValueError:
                continue
            src = next((x[4:] for x in parts[2:] if x.startswith("src=")), None)
            out[parts[0]] = {"bytes": val if src == cur else None, "src": src,
                             "status": "current" if src == cur else "stale (kernel sources changed since the capture)"}
    return out


# ----------------------------------------------------------------------------------------
# clocks sampling during the timed region
# ----------------------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.idx = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[2:6]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------


def bind_to_gpu_cpus(dev_index: int) -> None:
    """Run this process on the host CPUs local to its GPU (NVML's CPU affinity), so the pinned
    host buffers of the end-to-end section are allocated on the GPU's NUMA node (first
    touch) and each rank's copies take its own socket's path.  Best effort: unchanged when
    NVML or the affinity call is unavailable."""
    try:
        import pynvml

        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(dev_index)
            if hasattr(pr, "pci_bus_id"):  # CUDA and NVML may number the GPUs differently
                bus = "{:08x}:{:02x}:{:02x}.0".format(pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            else:
                h = pynvml.nvmlDeviceGetHandleByIndex(dev_index)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
            cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1}
            cpus &= set(range(os.cpu_count()))
            if cpus:
                os.sched_setaffinity(0, cpus)
                print(f"bench: GPU {dev_index} -> {len(cpus)} local CPUs", file=sys.stderr)
        finally:
            pynvml.nvmlShutdown()
    except Exception:
        pass


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(fn, steps, warmup, world, stream=None):
    """Device time (ms) of ``steps`` calls, barrier + synchronize on both sides, max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s = stream or torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    barrier(world)
    ms = e0.elapsed_time(e1)
    return max_over_ranks(ms, world)


L2_BYTES = 126 * 2 ** 20
_FLUSH = {}


def graph_of(fn):
    """`fn` (a sequence of stream-ordered launches) captured once as a CUDA graph, after two
    eager calls on a side stream (allocator warm-up); returns the replay callable."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g.replay


def timed_steps(fn, steps, warmup, world, flush: bool):
    """Device time (ms) of ``steps`` calls of ``fn`` (barrier + synchronize on both sides,
    max over ranks), each bracketed by its own CUDA events; with ``flush`` a 256 MB buffer
    is written before every step, outside the events, so no step finds the previous one's
    data in the 126 MB L2."""
    for _ in range(warmup):
        fn()
    buf = None
    if flush:
        dev = torch.cuda.current_device()
        buf = _FLUSH.get(dev)
        if buf is None:
            buf = _FLUSH[dev] = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device="cuda")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    for e0, e1 in ev:
        if buf is not None:
            buf.zero_()
        e0.record()
        fn()
        e1.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev)
    return max_over_ranks(ms, world)


def per_rank_stream_bytes(c):
    """HBM bytes one rank's forward streams (v, z, y bf16; q, k bf16; raw scalars and angles f32)."""
    B, L, H, N, P, Nr = c["B"], c["L"], c["H"], c["N"], c["P"], c["Nr"]
    return B * L * (3 * H * P * 2 + 2 * N * 2 + 3 * H * 4 + Nr * 4)


# ----------------------------------------------------------------------------------------
# config 2 inputs
# ----------------------------------------------------------------------------------------


def make_cfg2_inputs(c, seed, device="cuda"):
    """Seeded synthetic operands with configs[1]'s distributions: x, z ~ N(0,1) (B,L,H,P);
    head-shared q, k ~ N(0, 1/N) (B,L,N); dt = softplus(b_h + N(0, 0.5)) with exp(b_h)
    log-uniform in [1e-3, 0.1]; A_h = -exp(U(0, ln 16)) (a_raw = |A_h| - 1, so the heavy-
    tail activation returns |A_h|); rotary rate tanh(angles) pi ~ U(-pi, pi), head-shared,
    Nr = N/2; lambda = sigmoid(N(0,1)); D ~ N(0,1); q/k biases 0.1 N(0,1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    B, H, L, N, P, Nr = c["B"], c["H"], c["L"], c["N"], c["P"], c["Nr"]
    bf = torch.bfloat16
    kw = dict(device=device, generator=g)
    d = {}
    d["x"] = torch.randn(B, L, H, P, **kw).to(bf)
    d["z"] = torch.randn(B, L, H, P, **kw).to(bf)
    d["q"] = (torch.randn(B, L, N, **kw) / math.sqrt(N)).to(bf)
    d["k"] = (torch.randn(B, L, N, **kw) / math.sqrt(N)).to(bf)
    u = torch.rand(H, **kw)
    d["dt_bias"] = u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)
    d["dt_raw"] = torch.randn(B, L, H, **kw) * 0.5
    A = -torch.exp(torch.rand(H, **kw) * math.log(16.0))
    d["a_raw"] = (-A - 1.0).expand(B, L, H).contiguous()
    d["angles"] = torch.atanh(torch.rand(B, L, Nr, **kw) * 2 * (1 - 1e-6) - (1 - 1e-6))
    d["trap_raw"] = torch.randn(B, L, H, **kw)
    d["d_skip"] = torch.randn(H, **kw)
    d["q_bias"] = torch.randn(H, N, **kw) * 0.1
    d["k_bias"] = torch.randn(H, N, **kw) * 0.1
    d["dy"] = torch.randn(B, L, H, P, **kw).to(bf)
    return d


def fwd_call(d, c):
    from mamba3_b200 import kernel_fwd as KF

    return KF.siso_forward_raw(d["q"], d["k"], d["x"].permute(0, 2, 1, 3), d["dt_raw"], d["a_raw"], d["trap_raw"],
                               d["angles"], d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"],
                               z=d["z"].permute(0, 2, 1, 3), chunk=c["chunk"], dtype_policy="bf16")


# ----------------------------------------------------------------------------------------
# sections
# ----------------------------------------------------------------------------------------


def rank_slice(c, world):
    """This rank's share of configs[1]'s batch (strong scaling: B / world sequences)."""
    if c["B"] % world:
        raise SystemExit(f"--gpus {world} does not divide the batch of {c['B']}")
    return dict(c, B=c["B"] // world)


def bench_fwd(c, steps, warmup, world, rank, peaks):
    from mamba3_b200 import kernel_fwd as KF

    cl = rank_slice(c, world)
    d = make_cfg2_inputs(cl, seed=1000 + rank)
    tokens = c["B"] * c["L"]  # the global batch
    # replayed as a CUDA graph (at one batch row per GPU the length split's host-side calls
    # would otherwise outlast the 0.2 ms of device work); L2 flushed when the inputs fit in it
    step = graph_of(lambda: fwd_call(d, cl))
    ms = timed_steps(step, steps, warmup, world, flush=per_rank_stream_bytes(cl) < 2 * L2_BYTES)
    per_step = ms / steps
    th = cl["B"] * cl["L"] * cl["H"]  # one rank's launch
    flops = FWD_FLOP_PER_TOKEN_HEAD * th
    byts = fwd_bytes_per_token_head(c) * th
    return {
        "tok_s": tokens / (per_step / 1e3),
        "ms_per_step": per_step,
        "kernel_ms": per_step,
        "flops": flops,
        "bytes": byts,
        "tflops": flops / (per_step / 1e3) / 1e12,
        "gbs": byts / (per_step / 1e3) / 1e9,
        # the head-shared rotary-rate pass + the forward kernel (+ the length split's kernels
        # when the per-GPU batch is too small to fill the SMs)
        "launches": steps * KF.forward_launches(d["q"], d["x"].permute(0, 2, 1, 3), d["angles"], cl["chunk"]),
    }, d


def bench_e2e(c, steps, warmup, world, rank):
    """Public API with pinned host buffers: H2D of every input, the forward, D2H of y, each
    step (`siso.siso_segment_streamed`)."""
    from mamba3_b200 import siso as S

    glob = c
    c = rank_slice(c, world)
    d = make_cfg2_inputs(c, seed=2000 + rank)
    names = ["q", "k", "x", "z", "dt_raw", "a_raw", "trap_raw", "angles"]
    host = {n: d[n].cpu().pin_memory() for n in names}
    small = {n: d[n] for n in ("dt_bias", "q_bias", "k_bias", "d_skip")}
    y_host = torch.empty(c["B"], c["L"], c["H"], c["P"], dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = y_host.numel() * y_host.element_size()

    def step():
        # host -> device, the scan and device -> host overlap over 8 segments of L
        S.siso_segment_streamed(host["q"], host["k"], host["x"], host["dt_raw"], host["a_raw"], host["trap_raw"],
                                host["angles"], small["dt_bias"], small["q_bias"], small["k_bias"], small["d_skip"],
                                host["z"], chunk=c["chunk"], policy_name="bf16", segments=8, y_out=y_host)

    with torch.no_grad():
        ms = timed(step, steps, warmup, world)
    per = ms / steps
    return {"value": glob["B"] * glob["L"] / (per / 1e3), "unit": "tok/s", "ms_per_step": per,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}


def bench_fwd_bwd(c, steps, warmup, world, rank):
    from mamba3_b200 import kernel_bwd as KB

    glob = c
    c = rank_slice(c, world)
    d = make_cfg2_inputs(c, seed=3000 + rank)
    ws = torch.empty(KB.workspace_bytes(c["B"], c["L"], c["H"], c["N"], c["P"], c["Nr"], c["chunk"]),
                     dtype=torch.uint8, device="cuda")
    v = d["x"].permute(0, 2, 1, 3)
    z = d["z"].permute(0, 2, 1, 3)
    dy = d["dy"].permute(0, 2, 1, 3)

    from mamba3_b200 import kernel_fwd as KF

    def step():  # the forward saves the chunk-start states into the backward's workspace
        _, saved = KF.siso_forward_raw(d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                                       d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z,
                                       chunk=c["chunk"], dtype_policy="bf16", bwd_states=ws, return_saved=True)
        KB.siso_backward_raw(dy, d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                             d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z, chunk=c["chunk"],
                             dtype_policy="bf16", workspace=ws, states_ready=saved)
        return saved

    def step_recompute():  # kernel_bwd.py's scheme: nothing kept from the forward, the sweep recomputes
        KF.siso_forward_raw(d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                            d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z,
                            chunk=c["chunk"], dtype_policy="bf16")
        KB.siso_backward_raw(dy, d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                             d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z, chunk=c["chunk"],
                             dtype_policy="bf16", workspace=ws, states_ready=False)

    saved = step()
    flush = per_rank_stream_bytes(c) < 2 * L2_BYTES
    ms = timed_steps(graph_of(step), steps, warmup, world, flush)
    per = ms / steps
    per_rc = timed_steps(graph_of(step_recompute), steps, warmup, world, flush) / steps
    th = c["B"] * c["L"] * c["H"]
    flops = (FWD_FLOP_PER_TOKEN_HEAD + BWD_FLOP_PER_TOKEN_HEAD) * th
    kept = c["B"] * c["H"] * (c["L"] // c["chunk"] + 1) * (c["N"] * c["P"] * 2 + c["Nr"] * 4)
    return {"tok_s": glob["B"] * glob["L"] / (per / 1e3), "ms_per_step": per,
            "tflops": flops / (per / 1e3) / 1e12,
            # fwd (rates + scan, saving the states) + bwd; the recompute path adds the sweep's two
            "launches_per_step": 3 if saved else 5,
            "states": "saved by the forward" if saved else "recomputed",
            "saved_state_bytes": kept if saved else 0,
            "recompute": {"tok_s": glob["B"] * glob["L"] / (per_rc / 1e3), "ms_per_step": per_rc,
                          "tflops": flops / (per_rc / 1e3) / 1e12, "launches_per_step": 5,
                          "saved_state_bytes": 0,
                          "note": "forward keeps nothing; the backward's states-only sweep recomputes the "
                                  "chunk-start states (the reference's scheme, kernel_bwd.py:103-355)"}}


def bench_layer_cfg0(steps, warmup, world):
    """one Mamba-3 SISO layer forward in fp32 (d_model 256, N 32, P 32, H 16,
    Nr 8, chunk 64) on u (2, 512, 256) ~ N(0, 1), parameters from `init_params(seed 0)`.
    Parity with the reference is a test (tests/test_model_gpu.py); this is the wall time."""
    from mamba3_b200 import layer as LY

    cfg = LY.SISOConfig(d_model=256, d_state=32, headdim=32, expand=2, rope_fraction=0.5, chunk=64,
                        policy_name="fp32")
    params = LY.init_params(cfg, key=0, dtype=torch.float32)
    u = torch.randn(2, 512, 256, generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        ms = timed(lambda: LY.mamba3_siso_layer(params, u, cfg), steps, warmup, world)
    return {"ms_per_forward": ms / steps, "shape": "u (2, 512, 256), fp32 policy", "kernel": "generic (fp32)"}


def markov3_tokens(batch, length, seed, device="cuda", vocab=256, alpha=0.1):
    """Seeded order-3 Markov source over 256 symbols with Dirichlet(alpha) transition rows
    (configs[4]'s stand-in for a byte corpus).  The 256^3 rows are never materialised: the
    row of context c is the normalised Gamma(alpha) draws of a counter-based hash of
    (seed, c, symbol), and the next symbol is drawn by Gumbel-max over its logarithms."""
    M64 = (1 << 63) - 1

    def mix(x):  # splitmix-style integer hash on int64 (arithmetic wraps)
        x = (x ^ (x >> 31)) * 0x5851F42D4C957F2D
        x = (x ^ (x >> 29)) * 0x14057B7EF767814F
        return (x ^ (x >> 32)) & M64

    def unif(x):
        return ((mix(x) >> 11).double() + 0.5) / float(1 << 52)

    sym = torch.arange(vocab, device=device, dtype=torch.int64)
    g = torch.Generator(device=device).manual_seed(seed)
    toks = torch.empty(batch, length, dtype=torch.int64, device=device)
    ctx = torch.randint(0, vocab ** 3, (batch,), device=device, generator=g)
    for t in range(length):
        key = (ctx[:, None] * vocab + sym[None, :]) * 0x9E3779B97F4A7C15 + seed
        # Gamma(alpha) draw for alpha < 1 via U^(1/alpha) * Gamma(1 + alpha) ~ U^(1/alpha) * Exp(1)
        logw = torch.log(unif(key)) / alpha + torch.log(-torch.log(unif(key + 0x632BE59BD9B4E019)))
        gumbel = -torch.log(-torch.log(torch.rand(batch, vocab, device=device, generator=g, dtype=torch.float64)))
        nxt = torch.argmax(logw + gumbel, dim=1)
        toks[:, t] = nxt
        ctx = (ctx * vocab + nxt) % (vocab ** 3)
    return toks


def bench_train(steps, warmup, world, rank, global_batch=64, seq_len=8192):
    """data-parallel training of the 8-layer byte-level LM (d_model 512, N 128,
    P 64, H 16, Nr 32, chunk 128, tied head, no MLP), bf16 compute on fp32 master weights,
    AdamW lr 1e-3, NCCL all-reduce of bucketed gradients.  The global batch of 64 x 8192 is
    split over the ranks (strong scaling); tokens come from `markov3_tokens`."""
    from mamba3_b200 import layer as LY
    from mamba3_b200 import model as M
    from mamba3_b200 import train as T

    per = max(1, global_batch // world)
    scfg = LY.SISOConfig(d_model=512, d_state=128, headdim=64, expand=2, rope_fraction=0.5, chunk=128,
                         policy_name="bf16")
    cfg = M.LMConfig(vocab_size=256, n_layers=8, siso=scfg, d_intermediate=0)
    params = M.init_lm(cfg, key=0, dtype=torch.float32)
    step = T.make_step(cfg, params, lr=1e-3)
    toks = markov3_tokens(per, seq_len + 1, seed=5000 + rank)
    xs, ys = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
    ms = timed(lambda: step(xs, ys), steps, warmup, world)
    t = ms / steps
    loss = float(step(xs, ys))
    return {"tok_s": per * world * seq_len / (t / 1e3), "ms_per_step": t, "global_batch": per * world,
            "seq_len": seq_len, "params": cfg.param_count(), "loss": loss, "scaling": "strong (global batch 64)",
            "data": "synthetic order-3 Markov bytes, Dirichlet(0.1) rows"}


def bench_decode(steps, warmup, world, rank, peaks, global_batch=256):
    """24-layer LM, d_model 2048, N 128, P 64, H 64, Nr 32, MLP 4096,
    vocab 128256, bf16 weights, global B=256 split over the ranks, state pre-filled by a
    512-token prefill.  µs/token = the slowest rank's step time / 256."""
    from mamba3_b200 import kernel_decode as KD
    from mamba3_b200 import layer as LY
    from mamba3_b200 import model as M

    scfg = LY.SISOConfig(d_model=2048, d_state=128, headdim=64, expand=2, rope_fraction=0.5, chunk=128,
                         policy_name="bf16")
    cfg = M.LMConfig(vocab_size=128256, n_layers=24, siso=scfg, d_intermediate=4096)
    params = M.init_lm(cfg, key=0, dtype=torch.bfloat16)
    batch = global_batch // world
    g = torch.Generator(device="cuda").manual_seed(4000 + rank)
    prompt = torch.randint(0, cfg.vocab_size, (batch, 512), device="cuda", generator=g)
    states = M.zero_states(cfg, batch)
    with torch.no_grad():
        _, states = M.lm_forward(params, prompt, cfg, states=states, logits="none")
    tok = torch.randint(0, cfg.vocab_size, (batch,), device="cuda", generator=g)
    runner = M.DecodeGraph(params, cfg, states, batch)
    ms = timed(lambda: runner.step(tok), steps, warmup, world)
    per = ms / steps
    # decode kernel alone, one layer's state (bandwidth roofline, 67,724 B per (b, h))
    H, P, N, Nr = scfg.nheads, scfg.headdim, scfg.d_state, scfg.n_angles
    st = states[0]
    q = torch.randn(batch, N, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(batch, N, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(batch, H, P, device="cuda", dtype=torch.bfloat16)
    z = torch.randn(batch, H, P, device="cuda", dtype=torch.bfloat16)
    raw = torch.randn(batch, 3, H, device="cuda") * 0.1
    ang = torch.randn(batch, Nr, device="cuda")
    p0 = params.blocks[0].siso
    byts = batch * H * (2 * P * N * 4 + 2 * (N + P) * 4 + 2 * Nr * 4 + 3 * P * 2 + 3 * 4)
    # one launch per CUDA-graph replay with its own events, so that the host-side cost of the
    # Python call does not hide a short kernel (a few rows per rank); L2 flushed between
    # launches when one layer's state would fit twice in it
    call = graph_of(lambda: KD.siso_decode_raw(q, k, v, raw[:, 0], raw[:, 1], raw[:, 2], ang, p0.dt_bias,
                                               p0.c_bias, p0.b_bias, st, d_skip=p0.d_skip, z=z,
                                               dtype_policy="bf16"))
    kms = timed_steps(call, steps * 4, warmup, world, byts < 2 * L2_BYTES)
    kper = kms / (steps * 4)
    gbs = byts / (kper / 1e3) / 1e9
    gen = bench_generate(params, cfg, rank)
    return {"us_per_token": per * 1e3 / global_batch, "ms_per_step": per, "batch_per_gpu": batch,
            "kernel_ms_per_layer": kper, "kernel_gbs": gbs, "kernel_hbm_frac": gbs / peaks["hbm_gbs"],
            "kernel_bytes_per_layer": byts, "launches_per_step": cfg.n_layers, "generate_b1": gen}


def bench_generate(params, cfg, rank, n_short=32, n_long=160, reps=3):
    """`train.generate` at B = 1 on the configs[3] model (``train.py:503-582``): a 129-token
    prompt (128 prefilled in one chunk), sampling on the device.  Per-token cost = the
    difference of two generation lengths (best of ``reps`` each), so prefill and set-up
    cancel; device loop (one replayed CUDA graph per token, host sync every 32 tokens) and
    eager launches.  ``graph_step_ms`` is the device time of one replay (CUDA events)."""
    from mamba3_b200 import model as M
    from mamba3_b200 import train as TR
    from mamba3_b200.sampling import TokenSampler

    g = torch.Generator().manual_seed(5000 + rank)
    prompt = torch.randint(0, cfg.vocab_size, (129,), generator=g).tolist()
    res = {}
    for name, dl in (("device_loop", True), ("eager", False)):
        times = {}
        for n in (n_short, n_long):
            best = float("inf")
            for _ in range(reps):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                TR.generate(params, cfg, 1, prompt, n_tokens=n, device_loop=dl)
                torch.cuda.synchronize()
                best = min(best, time.perf_counter() - t0)
            times[n] = best
        res[name + "_us_per_token"] = (times[n_long] - times[n_short]) / (n_long - n_short) * 1e6
    states = M.zero_states(cfg, 1)
    smp = TokenSampler(1, cfg.vocab_size, "cuda")
    smp.reset([prompt])
    graph = TR._GenerateGraph(params, cfg, states, smp, None)
    res["graph_step_ms"] = timed(graph.replay, 32, 3, 1) / 32
    res["timing"] = "host wall clock around whole generate calls (host syncs included); graph_step_ms by CUDA events"
    return res


def bench_seqpar(c, steps, warmup, world, rank):
    """Sequence-parallel prefill of configs[1]'s batch: rank r scans the r-th L / world
    slice (`siso.siso_segment_seq_parallel`, two scans + two all-gathers).  The forward
    section's ms_per_step is one GPU scanning the same B x L."""
    from mamba3_b200 import siso as SISO

    L = c["L"]
    per = L // world
    d = make_cfg2_inputs(c, seed=7000)  # the same sequences on every rank
    lo, hi = rank * per, (rank + 1) * per
    args = (d["q"][:, lo:hi], d["k"][:, lo:hi], d["x"][:, lo:hi].permute(0, 2, 1, 3), d["dt_raw"][:, lo:hi],
            d["a_raw"][:, lo:hi], d["trap_raw"][:, lo:hi], d["angles"][:, lo:hi], d["dt_bias"], d["q_bias"],
            d["k_bias"], d["d_skip"], d["z"][:, lo:hi].permute(0, 2, 1, 3))
    ms = timed(lambda: SISO.siso_segment_seq_parallel(*args, chunk=c["chunk"], policy_name="bf16"),
               steps, warmup, world)
    tok = c["B"] * L
    return {"tok_s": tok / (ms / steps / 1e3), "ms_per_step": ms / steps, "slice_len": per,
            "note": "one batch of B sequences split along L over the ranks (strong scaling of one prefill)"}


def cpu_baseline_sample(threads=None, seconds=10.0):
    """The oracle restatement (``oracle/``) on a bounded slice of configs[1]'s forward: all
    32 heads, N=128 P=64 Nr=64 chunk=128, L=256 tokens, float32, on the host cores."""
    from oracle import siso_oracle as O

    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    c = dict(CFG2, B=1, L=1024)
    g = torch.Generator().manual_seed(0)
    B, H, L, N, P, Nr = c["B"], c["H"], c["L"], c["N"], c["P"], c["Nr"]
    f = torch.float32
    q = torch.randn(B, L, N, generator=g, dtype=f) / math.sqrt(N)
    k = torch.randn(B, L, N, generator=g, dtype=f) / math.sqrt(N)
    v = torch.randn(B, H, L, P, generator=g, dtype=f)
    z = torch.randn(B, H, L, P, generator=g, dtype=f)
    dt_raw = torch.randn(B, L, H, generator=g, dtype=f) * 0.5
    a_raw = torch.rand(B, L, H, generator=g, dtype=f) * 15
    trap = torch.randn(B, L, H, generator=g, dtype=f)
    ang = torch.randn(B, L, Nr, generator=g, dtype=f)
    dtb = torch.randn(H, generator=g, dtype=f) - 4
    qb = torch.randn(H, N, generator=g, dtype=f) * 0.1
    kb = torch.randn(H, N, generator=g, dtype=f) * 0.1
    dsk = torch.randn(H, generator=g, dtype=f)

    def run():
        with torch.no_grad():
            O.siso_segment(q, k, v, dt_raw, a_raw, trap, ang, dtb, qb, kb, dsk, z, chunk=128)

    run()
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el > seconds:
            break
    return {"value": B * L * n / el, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"oracle siso_segment fp32, B=1 H=32 L=1024 N=128 P=64 Nr=64 chunk=128, {n} runs in {el:.1f}s"}


REF_TORCH = os.path.join(ROOT, "baseline", "_ref", "mamba3_pallas", "torch_ref.py")


def ref_torch_sample(threads=None, seconds=10.0, L=256):
    """The reference's own CPU code for the path: ``mamba3_siso_ref`` of the installed
    reference's ``torch_ref.py`` (plain torch; the package's ``__init__`` needs JAX, so the
    file is loaded on its own), unmodified, on a bounded slice of configs[1]'s forward: all
    32 heads, N=128 P=64 Nr=64, B=1, ``L`` tokens, float32, with gate and skip."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_ref_torch_ref", REF_TORCH)
    tr = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tr)
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    B, H, N, P, Nr = 1, CFG2["H"], CFG2["N"], CFG2["P"], CFG2["Nr"]
    g = torch.Generator().manual_seed(0)
    f = torch.float32
    # head-shared q / k and angles (as the layer produces them), expanded to the per-head
    # layout the reference function takes
    Q = (torch.randn(B, L, 1, N, generator=g, dtype=f) / math.sqrt(N)).expand(B, L, H, N).contiguous()
    K = (torch.randn(B, L, 1, N, generator=g, dtype=f) / math.sqrt(N)).expand(B, L, H, N).contiguous()
    V = torch.randn(B, L, H, P, generator=g, dtype=f)
    Z = torch.randn(B, L, H, P, generator=g, dtype=f)
    dt = torch.exp(torch.rand(B, H, L, generator=g, dtype=f) * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3))
    adt = -(1.0 + 3.0 * torch.rand(H, generator=g, dtype=f))[None, :, None] * dt
    trap = torch.randn(B, H, L, generator=g, dtype=f)
    ang = (0.5 * torch.randn(B, L, 1, Nr, generator=g, dtype=f)).expand(B, L, H, Nr).contiguous()
    qb = 0.1 * torch.randn(H, N, generator=g, dtype=f)
    kb = 0.1 * torch.randn(H, N, generator=g, dtype=f)
    dsk = torch.randn(H, generator=g, dtype=f)

    def run():
        with torch.no_grad():
            tr.mamba3_siso_ref(Q, K, V, adt, dt, trap, qb, kb, ang, D=dsk, Z=Z)

    run()
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el > seconds:
            break
    return {"value": B * L * n / el, "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"reference torch_ref.mamba3_siso_ref fp32 (baseline/_ref, unmodified), B=1 H=32 L={L} "
                      f"N=128 P=64 Nr=64, gate and skip, {n} runs in {el:.1f}s"}


# ----------------------------------------------------------------------------------------


def run_reference(args, world, rank):
    """The reference arm, on the host cores, each step a bounded sample of configs[1]'s forward.
    Its value is the reference's chunked CPU algorithm (``reference.py``) through the oracle
    restatement, since JAX is absent; beside it, the reference's own plain-torch code for the
    path (``torch_ref.mamba3_siso_ref`` from the installed reference in baseline/_ref, the
    recurrent form it pins parity with) is timed unmodified when the install is present."""
    if rank != 0:
        return 0
    cb = None
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline_sample(seconds=4.0)
        if i >= args.warmup:
            vals.append(r["value"])
        cb = r
    v = statistics.median(vals)
    cb["value"] = v
    tref = ref_torch_sample(seconds=8.0) if os.path.exists(REF_TORCH) else None
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 65536 / v * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "configs[1] kernel fwd B8 H32 L8192 N128 P64 chunk128 (CPU sample)",
                       "sample": cb["sample"]},
            "impl": "reference", "cpu_baseline": cb,
            "torch_ref_baseline": tref,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "JAX is absent here and on the GPU image, so reference.py / interpret-mode Pallas cannot run; "
                    "the reference's chunked CPU path is timed through its restatement in oracle/, and the "
                    "reference's own torch_ref.py (recurrent, plain torch) beside it as torch_ref_baseline"}
    print(json.dumps(line), flush=True)
    return 0


def run_profile_case(which):
    """Three launches of one path on a case small enough for a full ncu capture.  Its inputs
    (v, z, y 67 MB each at L = 2048) are still larger than L2."""
    torch.cuda.set_device(0)
    if which == "trainstep":  # configs[4]: one optimizer step at 1/8 of the global batch, inside an NVTX range
        from mamba3_b200 import layer as LY
        from mamba3_b200 import model as M
        from mamba3_b200 import train as T

        scfg = LY.SISOConfig(d_model=512, d_state=128, headdim=64, expand=2, rope_fraction=0.5, chunk=128,
                             policy_name="bf16")
        cfg = M.LMConfig(vocab_size=256, n_layers=8, siso=scfg, d_intermediate=0)
        params = M.init_lm(cfg, key=0, dtype=torch.float32)
        step = T.make_step(cfg, params, lr=1e-3)
        toks = torch.randint(0, 256, (8, 8193), device="cuda")
        xs, ys = toks[:, :-1].contiguous(), toks[:, 1:].contiguous()
        for i in range(3):
            if i == 2:  # the backward runs on autograd's own thread: bracket by profiler start/stop
                torch.cuda.synchronize()
                torch.cuda.profiler.start()
                torch.cuda.nvtx.range_push("train_step")
            step(xs, ys)
            if i == 2:
                torch.cuda.synchronize()
                torch.cuda.nvtx.range_pop()
                torch.cuda.profiler.stop()
        torch.cuda.synchronize()
        return 0
    if which == "generate":  # configs[3] model, B = 1: one decode step + sampling, eager, in an NVTX range
        from mamba3_b200 import layer as LY
        from mamba3_b200 import model as M
        from mamba3_b200.sampling import TokenSampler

        scfg = LY.SISOConfig(d_model=2048, d_state=128, headdim=64, expand=2, rope_fraction=0.5, chunk=128,
                             policy_name="bf16")
        cfg = M.LMConfig(vocab_size=128256, n_layers=24, siso=scfg, d_intermediate=4096)
        params = M.init_lm(cfg, key=0, dtype=torch.bfloat16)
        states = M.zero_states(cfg, 1)
        smp = TokenSampler(1, cfg.vocab_size, "cuda")
        smp.reset([[1, 2, 3]])
        with torch.no_grad():
            for i in range(3):
                if i == 2:
                    torch.cuda.nvtx.range_push("generate_token")
                lg, _ = M.lm_decode_step(params, smp.token, states, cfg)
                smp.pick(lg)
                if i == 2:
                    torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        return 0
    if which == "decodestep":  # configs[3]: one 24-layer decode step, eager, inside an NVTX range
        from mamba3_b200 import layer as LY
        from mamba3_b200 import model as M

        scfg = LY.SISOConfig(d_model=2048, d_state=128, headdim=64, expand=2, rope_fraction=0.5, chunk=128,
                             policy_name="bf16")
        cfg = M.LMConfig(vocab_size=128256, n_layers=24, siso=scfg, d_intermediate=4096)
        params = M.init_lm(cfg, key=0, dtype=torch.bfloat16)
        states = M.zero_states(cfg, 256)
        tok = torch.randint(0, cfg.vocab_size, (256,), device="cuda")
        with torch.no_grad():
            for i in range(3):
                if i == 2:
                    torch.cuda.nvtx.range_push("decode_step")
                M.lm_decode_step(params, tok, states, cfg)
                if i == 2:
                    torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        return 0
    if which == "decode":
        from mamba3_b200 import kernel_decode as KD
        from mamba3_b200.state import SISOState
        B, H, P, N, Nr = 256, 64, 64, 128, 32
        g = torch.Generator(device="cuda").manual_seed(7)
        r = lambda *sh, dt=torch.float32: torch.randn(*sh, device="cuda", generator=g).to(dt)
        st = SISOState(ssm=r(B, H, P, N), k=r(B, H, N), v=r(B, H, P), phi=r(B, H, Nr))
        raw = r(B, 3, H) * 0.1
        for _ in range(3):
            KD.siso_decode_raw(r(B, N, dt=torch.bfloat16), r(B, N, dt=torch.bfloat16), r(B, H, P, dt=torch.bfloat16),
                               raw[:, 0], raw[:, 1], raw[:, 2], r(B, Nr), r(H), r(H, N), r(H, N), st,
                               d_skip=r(H), z=r(B, H, P, dt=torch.bfloat16), dtype_policy="bf16")
        torch.cuda.synchronize()
        return 0
    if which == "fwdphases":  # needs a library built with -DM3_WS_TIMING (diagnostic)
        import ctypes
        from mamba3_b200 import _capi as C
        lib = C.lib()
        if not hasattr(lib, "m3_debug_ws_timing"):
            raise SystemExit("fwdphases: rebuild with build.build(force=True, extra=['-DM3_WS_TIMING'])")
        lib.m3_debug_ws_timing.argtypes = [ctypes.POINTER(ctypes.c_ulonglong), ctypes.c_int]
        from mamba3_b200 import kernel_fwd as KF
        c = dict(CFG2)
        d = make_cfg2_inputs(c, 0)
        v, z = d["x"].permute(0, 2, 1, 3), d["z"].permute(0, 2, 1, 3)
        for so in (False, True):  # the full forward, then its states-only mode
            def call():
                return KF.siso_forward_raw(d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                                           d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z,
                                           chunk=c["chunk"], dtype_policy="bf16", lsplit=1, states_only=so)
            for _ in range(3):
                call()
            torch.cuda.synchronize()
            buf = (ctypes.c_ulonglong * 256)()
            lib.m3_debug_ws_timing(buf, 1)
            call()
            torch.cuda.synchronize()
            lib.m3_debug_ws_timing(buf, 1)
            print("states-only" if so else "full")
            for code in range(128):  # per code: cycles per call (a wait site or a phase of one role)
                if buf[128 + code]:
                    print(f"code {code:3d}: {buf[code] / buf[128 + code]:9.1f} cycles over {buf[128 + code]} calls")
        return 0
    if which == "bwdphases":  # needs a library built with -DM3_TC_TIMING (diagnostic)
        import ctypes
        from mamba3_b200 import _capi as C
        from mamba3_b200 import kernel_bwd as KB
        from mamba3_b200 import kernel_fwd as KF
        lib = C.lib()
        if not hasattr(lib, "m3_debug_tc_timing"):
            raise SystemExit("bwdphases: rebuild with build.build(force=True, extra=['-DM3_TC_TIMING'])")
        lib.m3_debug_tc_timing.argtypes = [ctypes.POINTER(ctypes.c_ulonglong), ctypes.c_int]
        c = dict(CFG2)
        d = make_cfg2_inputs(c, 0)
        ws = torch.empty(KB.workspace_bytes(c["B"], c["L"], c["H"], c["N"], c["P"], c["Nr"], c["chunk"]),
                         dtype=torch.uint8, device="cuda")
        v, z, dy = (d[n].permute(0, 2, 1, 3) for n in ("x", "z", "dy"))

        def step():
            _, saved = KF.siso_forward_raw(d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                                           d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z,
                                           chunk=c["chunk"], dtype_policy="bf16", bwd_states=ws, return_saved=True)
            KB.siso_backward_raw(dy, d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                                 d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z, chunk=c["chunk"],
                                 dtype_policy="bf16", workspace=ws, states_ready=saved)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        buf = (ctypes.c_ulonglong * 24)()
        lib.m3_debug_tc_timing(buf, 1)
        step()
        torch.cuda.synchronize()
        lib.m3_debug_tc_timing(buf, 1)
        marks = c["B"] * c["H"] * (c["L"] // c["chunk"])  # thread 0 of each CTA, once per chunk
        for i in range(24):
            if buf[i]:
                print(f"phase {i:2d}: {buf[i] / marks:9.0f} cycles per chunk")
        return 0
    if which == "fwdsplit":  # one rank's share at --gpus 8: B = 1, full L, the length split
        c = dict(CFG2, B=1)
        d = make_cfg2_inputs(c, 0)
        for _ in range(3):
            fwd_call(d, c)
        torch.cuda.synchronize()
        return 0
    c = dict(CFG2, L=2048)
    d = make_cfg2_inputs(c, 0)
    if which == "fwd":
        for _ in range(3):
            fwd_call(d, c)
    else:
        from mamba3_b200 import kernel_bwd as KB
        ws = torch.empty(KB.workspace_bytes(c["B"], c["L"], c["H"], c["N"], c["P"], c["Nr"], c["chunk"]),
                         dtype=torch.uint8, device="cuda")
        v, z, dy = (d[n].permute(0, 2, 1, 3) for n in ("x", "z", "dy"))
        for _ in range(3):
            fwd_call(d, c)
            KB.siso_backward_raw(dy, d["q"], d["k"], v, d["dt_raw"], d["a_raw"], d["trap_raw"], d["angles"],
                                 d["dt_bias"], d["q_bias"], d["k_bias"], d_skip=d["d_skip"], z=z, chunk=c["chunk"],
                                 dtype_policy="bf16", workspace=ws)
    torch.cuda.synchronize()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--what", default="all",
                    help="comma list of fwd,e2e,fwdbwd,decode,train,layer,cpu,seqpar (N > 1) or all")
    ap.add_argument("--profile", choices=["fwd", "fwdsplit", "fwdphases", "fwdbwd", "bwdphases", "decode",
                                          "decodestep", "trainstep", "generate"],
                    help="run the small profiling case (configs[1] shapes at L=2048, or one decode layer "
                         "at configs[3]) three times and exit; for ncu captures, prints no bench line")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile:
        return run_profile_case(args.profile)

    world, rank, local = dist_setup() if args.impl == "ours" else (
        int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0)
    if args.impl == "reference":
        return run_reference(args, world, rank)

    what = set(["fwd", "e2e", "fwdbwd", "decode", "train", "layer", "cpu", "seqpar"] if args.what == "all"
               else args.what.split(","))
    peaks = load_peaks()
    traffic = load_traffic()
    c = dict(CFG2)
    torch.backends.cuda.matmul.allow_tf32 = False
    out = {}
    # the CPU baseline first, on an idle host and before any GPU work, the way the reference
    # arm (a fresh process) takes it
    cpu = cpu_baseline_sample() if ("cpu" in what and rank == 0 and world == 1) else None
    tref = (ref_torch_sample(seconds=5.0) if ("cpu" in what and rank == 0 and world == 1
                                              and os.path.exists(REF_TORCH)) else None)
    # then the host side of every section on the CPUs local to this rank's GPU
    bind_to_gpu_cpus(torch.cuda.current_device())
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    with ClockSampler(torch.cuda.current_device()) as clk:
        fwd, _ = bench_fwd(c, args.steps, args.warmup, world, rank, peaks)
        if "e2e" in what:
            out["e2e"] = bench_e2e(c, max(2, args.steps // 2), args.warmup, world, rank)
        if "fwdbwd" in what:
            out["fwd_bwd"] = bench_fwd_bwd(c, max(2, args.steps // 2), args.warmup, world, rank)
        if "decode" in what:
            out["decode"] = bench_decode(args.steps, args.warmup, world, rank, peaks)
        if "train" in what:
            out["train"] = bench_train(max(2, args.steps // 3), args.warmup, world, rank)
        if "layer" in what:
            out["layer_cfg0"] = bench_layer_cfg0(args.steps, args.warmup, world)
        if "seqpar" in what and world > 1:
            out["seqpar"] = bench_seqpar(c, max(2, args.steps // 2), args.warmup, world, rank)
    clocks = clk.summary()

    if rank != 0:
        return 0
    kname = "m3_fwd"
    hbm_frac = fwd["gbs"] / peaks["hbm_gbs"]
    line = {
        "metric": METRIC,
        "value": fwd["tok_s"],
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": fwd["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "configs[1]: kernel-level chunked-scan forward, fused raw boundary",
                   "global_batch": c["B"], "batch_per_gpu": c["B"] // world, "nheads": c["H"], "seq_len": c["L"],
                   "d_state": c["N"],
                   "headdim": c["P"], "n_angles": c["Nr"], "chunk": c["chunk"], "policy": "bf16",
                   "parallelism": f"bh-sharded x{world} (strong: batch split)",
                   "timing": "CUDA-graph replay of the forward call, per-step CUDA events",
                   "l2": ("inputs larger than L2 ({:.0f} MB streamed per rank per step)".format(
                       per_rank_stream_bytes(dict(c, B=c["B"] // world)) / 1e6)
                          if per_rank_stream_bytes(dict(c, B=c["B"] // world)) >= 2 * L2_BYTES
                          else "L2 flushed (256 MB write) before every step, outside the timed events")},
        "roofline": {"bound": "hbm", "achieved": fwd["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": hbm_frac, "traffic": (traffic.get(kname) or {}).get("bytes"),
                     "traffic_capture": (traffic.get(kname) or {}).get("status", "no capture"),
                     "peak_src": peaks["src"],
                     "algorithmic_bytes_per_launch": fwd["bytes"],
                     "tensor": {"achieved_tflops": fwd["tflops"], "peak_tflops": peaks["bf16_tflops"],
                                "frac": fwd["tflops"] / peaks["bf16_tflops"],
                                "flops_per_launch": fwd["flops"]}},
        "gpu_launches": fwd["launches"],
        "clocks": dict(clocks, sampled="whole timed run (fwd, e2e, fwd+bwd, decode sections)"),
    }
    if "e2e" in out:
        e = out["e2e"]
        line["e2e"] = {"value": e["value"], "unit": "tok/s", "h2d_bytes_per_step": e["h2d_bytes_per_step"],
                       "d2h_bytes_per_step": e["d2h_bytes_per_step"], "ms_per_step": e["ms_per_step"]}
    if "fwd_bwd" in out:
        line["fwd_bwd"] = out["fwd_bwd"]
    if "decode" in out:
        line["decode"] = out["decode"]
    if "train" in out:
        line["train"] = out["train"]
    if "layer_cfg0" in out:
        line["layer_cfg0"] = out["layer_cfg0"]
    if "seqpar" in out:
        line["seqpar_prefill"] = out["seqpar"]
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if tref is not None:
        line["torch_ref_baseline"] = tref
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
