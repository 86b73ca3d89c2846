"""Benchmark of the B200 Hyena-mixer hot path (evo2_flash mixers) on its
BASELINE configurations, printing one JSON line.

Workloads (synthetic, seeded; no checkpoint or dataset is used):
  prefill  config 2: one HCS + HCM + HCL mixer triple at the 7B shape (H=4096,
           fp8 e4m3 in_proj 4096->12288 with per-tensor scales, bf16 out_proj),
           batch 8 x 8192 uniform-random ACGT tokens embedded through a seeded
           N(0,1) 512xH table and Evo2RMSNorm.  One step = the triple over the
           batch.  `value` = prefill tokens/s of the whole job.
  decode   config 3: 128 sequences, prompts of U[256, 4096] random ACGT prefilled
           into paged state, then single-token decode steps through the triple,
           replayed as one CUDA graph per step.
Multi-GPU (torchrun, one rank per GPU): every rank runs the same per-rank
workload on its own sequences (independent replicas, weak scaling); only the
timing reduction crosses ranks.
  --workload tp40b  config 5: the 40B-shape triple (H=8192, fp8 in_proj
           8192->24576) channel-sharded over the ranks (tensor parallel, strong
           scaling), one 262144-token sequence prefilled in chunks whose
           all-reduces overlap the next chunks' kernels, then batch-1 decode
           steps.  `value` = prefill tokens/s of the whole job.
  --workload cp40b  config 5 with context parallelism instead: every rank runs
           the full-width triple on its contiguous slice of the 262144-token
           sequence (FIR layers with a K+1-row halo, the LI layer in two passes
           around one all-gather of (H, 16) slice states); strong scaling.
  --workload hcm256  config 1: one HCM block at H=256 (GPU path + CPU port).
  --workload model7b config 4: the full random-init 7B model scoring a bounded
           sample of the Markov sequences (prefill tok/s, mean NLL).

`--impl reference` times the reference algorithm's CPU implementation (the
oracle port in oracle/, all host threads) on a bounded sample of the same
workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path
from types import SimpleNamespace

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

H = 4096
PREFILL_B, PREFILL_L = 8, 8192
DECODE_B = 128
METRIC = "Hyena-mixer prefill+decode tok/s/GPU at 7B shape; % HBM / fp8 tensor roofline"
L2_BYTES = 126 * 2 ** 20
# DRAM bytes (read + write) of one in_proj GEMM launch (the SM-pair kernel) per
# token, from an ncu capture of the T = 16384 case (dram__bytes_read.sum +
# dram__bytes_write.sum = 446.2 + 376.3 MB), scaled by T
IN_PROJ_DRAM_BYTES_PER_TOKEN = (446246400 + 376256768) / 16384


# ---------------------------------------------------------------- synthetic model
def rmsnorm(x, eps=1e-6):
    """Evo2RMSNorm with unit weight: x / (||x||_2 H^-0.5 + eps) (model.py:47-74)."""
    xf = x.float()
    return (xf / (xf.norm(2, dim=-1, keepdim=True) * xf.shape[-1] ** -0.5 + eps)).to(torch.bfloat16)


def acgt_tokens(n, gen):
    lut = torch.tensor([65, 67, 71, 84])
    return lut[torch.randint(0, 4, (n,), generator=gen)]


def embed_norm(tokens, table, device):
    return rmsnorm(table[tokens.to(table.device)].to(device))


def layer_params(kind, k, seed, device):
    """BASELINE recipes (evo2_flash_b200.synthetic.mixer_tensors): projections
    N(0, 0.02) with in_proj quantised to e4m3 under a per-tensor scale, short
    filter N(0,1)/sqrt(3), FIR w[:, K-1-lag] = N(0,1)/sqrt(K) exp(-0.05 lag),
    log-poles -exp(U(-6,0)), residues N(0,1)/16, D N(0, 0.02), out_proj bias 0."""
    from evo2_flash_b200.synthetic import mixer_tensors

    return mixer_tensors(kind, H, k, seed, fp8=True, device=device)


TRIPLE = (("hcs", 7), ("hcm", 128), ("hcl", 16))


def build_triple(device, input_scale, num_blocks, num_spec=0, params=None):
    """The config-2/3 triple (params: reuse the (m, p) list of another triple's
    weights; num_spec > 0: speculative layout with 1 + num_spec verifier slots)."""
    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer

    cfg = SimpleNamespace(hidden_size=H, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=True)
    layers = []
    for i, (kind, k) in enumerate(TRIPLE):
        if params is None:
            p = layer_params(kind, k, 100 + i, "cpu")
            p["in_proj.input_scale"] = input_scale.reshape(1)
        else:
            p = params[i][1]
        kw = dict(num_spec=num_spec, device=device)
        if kind == "hcl":
            m = HyenaIIRMixer(cfg, i, prefix=f"triple.{i}", **kw)
        else:
            m = HyenaFIRMixer(cfg, i, prefix=f"triple.{i}", k_inner=k, **kw)
        m.load_full_weights({kk: v.to(device) for kk, v in p.items()})
        m.allocate_state(num_blocks, device)
        layers.append((m, p))
    return layers


def prefill_meta(lengths, blocks, device, init=None):
    qsl = [0]
    for n in lengths:
        qsl.append(qsl[-1] + n)
    n = len(lengths)
    return SimpleNamespace(
        num_decodes=0, num_decode_tokens=0, num_prefills=n, num_prefill_tokens=qsl[-1],
        query_start_loc_p=torch.tensor(qsl, dtype=torch.int32, device=device),
        has_initial_states_p=torch.tensor(init or [False] * n, dtype=torch.bool, device=device),
        state_indices_tensor_p=torch.tensor(blocks, dtype=torch.int32, device=device),
        state_indices_tensor_d=torch.zeros(0, dtype=torch.int32, device=device),
        query_start_loc_d=None, num_accepted_tokens=None,
        seq_lens=torch.tensor(lengths, dtype=torch.int32, device=device))


def decode_meta(blocks, device):
    n = len(blocks)
    return SimpleNamespace(
        num_decodes=n, num_decode_tokens=n, num_prefills=0, num_prefill_tokens=0,
        query_start_loc_p=torch.zeros(1, dtype=torch.int32, device=device),
        has_initial_states_p=torch.zeros(0, dtype=torch.bool, device=device),
        state_indices_tensor_p=torch.zeros(0, dtype=torch.int32, device=device),
        state_indices_tensor_d=torch.tensor(blocks, dtype=torch.int32, device=device),
        query_start_loc_d=None, num_accepted_tokens=None,
        seq_lens=torch.zeros(n, dtype=torch.int32, device=device))


# ---------------------------------------------------------------- measurement
class Clocks:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return None
        rows = [r.split(",") for r in self.path.read_text().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            try:
                s = float(r[1]); mx = float(r[2]); pw = float(r[3])
            except (ValueError, IndexError):
                continue
            if pw > 300:  # under load
                sm.append(s)
            for nm, v in zip(names, r[5:9]):
                if v.strip() == "Active":
                    reasons.add(nm)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples_under_load": len(sm)}


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def fp8_peak_tflops(device, sustain_s=2.0):
    """Dense e4m3 GEMM throughput of cuBLAS (torch._scaled_mm, 8192^3) measured
    in this run, the tensor roofline for the fp8 in_proj: (burst = best of 10
    single launches, sustained = mean over back-to-back launches for
    `sustain_s` seconds, i.e. under the power cap like a kernel inside a long
    step).  MEASURED_PEAKS.json carries no fp8 figure."""
    n = 8192
    a = torch.randn(n, n, device=device).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=device).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=device)
    for _ in range(3):
        torch._scaled_mm(a, b, one, one, out_dtype=torch.bfloat16)
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._scaled_mm(a, b, one, one, out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    flop = 2 * n ** 3
    reps = max(1, int(sustain_s / (best * 1e-3)))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        torch._scaled_mm(a, b, one, one, out_dtype=torch.bfloat16)
    e1.record()
    torch.cuda.synchronize()
    sustained = flop * reps / (e0.elapsed_time(e1) * 1e-3) / 1e12
    return flop / (best * 1e-3) / 1e12, sustained


class KernelTimer:
    """CUDA events around every call of one op on the launching (current) stream."""

    def __init__(self, module, name):
        self.module, self.name = module, name
        self.orig = getattr(module, name)
        self.events = []
        self.active = False

    def __enter__(self):
        def wrapped(*a, **kw):
            if not self.active:
                return self.orig(*a, **kw)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            r = self.orig(*a, **kw)
            e1.record()
            self.events.append((e0, e1))
            return r

        setattr(self.module, self.name, wrapped)
        return self

    def __exit__(self, *a):
        setattr(self.module, self.name, self.orig)

    def mean_ms(self):
        ts = [a.elapsed_time(b) for a, b in self.events]
        return sum(ts) / len(ts) if ts else None


# ---------------------------------------------------------------- workloads
def run_prefill(layers, x, meta, steps, warmup, dist_ok, device, gemm_timer):
    from evo2_flash_b200 import set_forward_metadata

    def step():
        with set_forward_metadata(meta):
            for m, _ in layers:
                m(x)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if dist_ok:
        torch.distributed.barrier()
    times = []
    gemm_timer.active = True
    idx = torch.cuda.current_device()
    with Clocks(idx) as clk:
        for _ in range(steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            times.append((e0, e1))
        torch.cuda.synchronize()
    gemm_timer.active = False
    ms = sum(a.elapsed_time(b) for a, b in times)
    return ms, clk.summary()


class LocalNumaAlloc:
    """Restricts this process to the CPUs of the GPU's NUMA node while pinned
    host buffers are allocated (their pages land on the node whose memory
    controller the GPU's PCIe link hangs off), then restores the affinity.
    No-op where sysfs does not say."""

    def __init__(self, device):
        self.saved = None
        try:
            pr = torch.cuda.get_device_properties(device)
            bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            node = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text())
            cpus = set()
            for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
            self.cpus = cpus if node >= 0 else None
        except (OSError, ValueError, AttributeError, RuntimeError):
            self.cpus = None

    def __enter__(self):
        if self.cpus:
            self.saved = os.sched_getaffinity(0)
            os.sched_setaffinity(0, self.cpus & self.saved or self.saved)
        return self

    def __exit__(self, *a):
        if self.saved is not None:
            os.sched_setaffinity(0, self.saved)


def run_e2e(layers, x_host, meta, steps, device):
    """Public-API end to end: every step copies the hidden states from pinned host
    memory to the device, runs the triple, and copies the last layer's output
    back to pinned host memory.  The copies run on their own streams (one per
    direction), double-buffered, so step i+1's upload and step i-1's download
    overlap step i's kernels; the timed region spans the first upload to the last
    download."""
    from evo2_flash_b200 import set_forward_metadata

    comp = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    xbuf = [torch.empty(x_host.shape, dtype=x_host.dtype, device=device) for _ in range(2)]
    with LocalNumaAlloc(device):
        out_host = [torch.empty_like(x_host, pin_memory=True).fill_(0) for _ in range(2)]
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(up)
    with torch.cuda.stream(up):
        xbuf[0].copy_(x_host, non_blocking=True)
        uploaded[0].record(up)
    for i in range(steps):
        b = i % 2
        comp.wait_event(uploaded[b])
        with set_forward_metadata(meta):
            for m, _ in layers:
                y = m(xbuf[b])
        computed[b].record(comp)
        if i + 1 < steps:
            with torch.cuda.stream(up):
                if i >= 1:
                    up.wait_event(computed[1 - b])  # step i-1 no longer reads that buffer
                xbuf[1 - b].copy_(x_host, non_blocking=True)
                uploaded[1 - b].record(up)
        with torch.cuda.stream(down):
            down.wait_event(computed[b])
            y.record_stream(down)
            out_host[b].copy_(y, non_blocking=True)
    down.wait_stream(up)
    e1.record(down)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1), x_host.numel() * x_host.element_size(), out_host[0].numel() * 2


def run_decode(layers, table, device, steps, warmup, gen):
    """Config 3: 128 ragged prompts prefilled into paged state, then decode steps
    of the triple replayed from one CUDA graph."""
    from evo2_flash_b200 import set_forward_metadata

    lengths = torch.randint(256, 4097, (DECODE_B,), generator=gen).tolist()
    blocks = list(range(1, DECODE_B + 1))
    toks = acgt_tokens(sum(lengths), gen)
    x = embed_norm(toks, table, device)
    meta = prefill_meta(lengths, blocks, device)
    with set_forward_metadata(meta):
        for m, _ in layers:
            m(x)
    del x
    nsteps = warmup + steps
    xs = embed_norm(acgt_tokens(DECODE_B * nsteps, gen), table, device).view(nsteps, DECODE_B, H)
    dmeta = decode_meta(blocks, device)
    x_static = torch.empty(DECODE_B, H, dtype=torch.bfloat16, device=device)

    def step():
        with set_forward_metadata(dmeta):
            for m, _ in layers:
                m(x_static)

    x_static.copy_(xs[0])
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm the caching allocator outside capture
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for i in range(warmup):
        x_static.copy_(xs[i])
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, nsteps):
        x_static.copy_(xs[i])
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del graph
    return ms / steps, lengths


def run_verify(layers, table, device, steps, warmup, gen, q=4):
    """Config 3's speculative verify: the same 128 ragged prompts prefilled into
    a speculative-layout triple (1 + 3 verifier slots per request), then steps
    of q = 4 positions per request (anchor + 3 drafts of random ACGT) whose
    accepted counts are drawn uniformly from 1..4 and resolved from the state's
    position stamps, replayed from one CUDA graph."""
    from evo2_flash_b200 import set_forward_metadata

    spec = build_triple(device, None, 1 + DECODE_B * q, num_spec=q - 1, params=layers)
    lengths = torch.randint(256, 4097, (DECODE_B,), generator=gen).tolist()
    slots = torch.arange(1, 1 + DECODE_B * q, dtype=torch.int32).view(DECODE_B, q)
    x = embed_norm(acgt_tokens(sum(lengths), gen), table, device)
    with set_forward_metadata(prefill_meta(lengths, slots[:, 0].tolist(), device)):
        for m, _ in spec:
            m(x)
    del x
    nsteps = warmup + steps
    xs = embed_norm(acgt_tokens(DECODE_B * q * nsteps, gen), table, device).view(nsteps, DECODE_B * q, H)
    acc = torch.randint(1, q + 1, (nsteps, DECODE_B), generator=gen).to(device)
    computed = torch.tensor(lengths, dtype=torch.int32, device=device)
    meta = SimpleNamespace(
        num_decodes=DECODE_B, num_decode_tokens=DECODE_B * q, num_prefills=0,
        num_prefill_tokens=0,
        query_start_loc_p=torch.zeros(1, dtype=torch.int32, device=device),
        has_initial_states_p=torch.zeros(0, dtype=torch.bool, device=device),
        state_indices_tensor_p=torch.zeros(0, dtype=torch.int32, device=device),
        state_indices_tensor_d=slots.to(device),
        query_start_loc_d=torch.arange(0, DECODE_B * q + 1, q, dtype=torch.int32, device=device),
        num_accepted_tokens=None, num_computed_tokens_d=computed,
        seq_lens=torch.zeros(DECODE_B, dtype=torch.int32, device=device))
    x_static = torch.empty(DECODE_B * q, H, dtype=torch.bfloat16, device=device)

    def step():
        with set_forward_metadata(meta):
            for m, _ in spec:
                m(x_static)

    def advance(i):  # the previous step accepted acc[i] tokens per request
        x_static.copy_(xs[i])
        computed.add_(acc[i].to(torch.int32))

    x_static.copy_(xs[0])  # first step: accepted = 1 (stamp = prompt length)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for i in range(warmup):
        advance(i)
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(warmup, nsteps):
        advance(i)
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del graph, spec
    return ms


def verify_bytes_per_step(q=4):
    """Algorithmic HBM bytes of one verify step of the triple at B=128: weights
    once, per request and layer the accepted snapshot read and q snapshots
    written (S1 6 / 127 columns for HCS / HCM, S2 16 modes for HCL), the S0
    window (2 + q - 1 columns) read and written, activations in and out."""
    w_in = 3 * (3 * H * H)
    w_out = 3 * (H * H * 2 + H * 2)
    per_req = 3 * (2 * (2 + q - 1) * 3 * H * 2)
    per_req += (1 + q) * (6 * H * 4 + 127 * H * 4 + 17 * H * 4)
    act = 3 * DECODE_B * q * (H * 2 + 3 * H * 2 * 2 + H * 2 * 2 + H * 2)
    return w_in + w_out + DECODE_B * per_req + act


def decode_bytes_per_step():
    """Algorithmic HBM bytes of one decode step of the triple at B=128 (weights read
    once, every state slice read and written once, activations in/out)."""
    w_in = 3 * (3 * H * H)            # e4m3
    w_out = 3 * (H * H * 2 + H * 2)   # bf16 + bias
    filt = 3 * H * 3 * 2 * 3 + H * 7 * 2 + H * 128 * 2 + 2 * H * 16 * 4 + 3 * H * 2
    per_req = 3 * (2 * 2 * 3 * H * 2)            # S0 r+w, three layers
    per_req += 2 * 6 * H * 4 + 2 * 127 * H * 4 + 2 * 16 * H * 4   # S1 (HCS, HCM), S2
    act = 3 * DECODE_B * (H * 2 + 3 * H * 2 * 2 + H * 2 * 2 + H * 2)  # x, z w+r, g w+r, out
    return w_in + w_out + filt + DECODE_B * per_req + act


def prefill_flops_bytes(T):
    """Per-kernel algorithmic FLOPs / HBM bytes of one prefill step of the triple."""
    f_in = 2 * T * H * 3 * H           # per layer, fp8
    f_out = 2 * T * H * H              # per layer, bf16
    b_in = T * H * 1 + 3 * H * H + T * 3 * H * 2      # xq read, W8, z write
    b_out = T * H * 2 + H * H * 2 + T * H * 2         # g read, W, out write
    b_quant = T * H * 2 + T * H
    b_core = T * 3 * H * 2 + T * H * 2                # z read, g write
    return f_in, f_out, b_in, b_out, b_quant, b_core


def cpu_baseline_sample(tokens_per_step, steps, warmup):
    """The reference algorithm on the host cores (oracle port, all threads):
    the triple over one sequence of `tokens_per_step` tokens."""
    from oracle import hyena_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    table = torch.randn(512, H, generator=gen)
    x = embed_norm(acgt_tokens(tokens_per_step, gen), table, "cpu")
    sx = (x.float().abs().amax() / 448.0).reshape(1)
    params = []
    for i, (kind, k) in enumerate(TRIPLE):
        p = layer_params(kind, k, 100 + i, "cpu")
        w_deq = (p["in_proj.weight"].float() * p["in_proj.weight_scale"]).to(torch.bfloat16)
        params.append(O.MixerParams(
            H=H, kind="iir" if kind == "hcl" else "fir", k_inner=k, short_filter=p["short_filter"],
            conv=p.get("conv"), D=p.get("D"), log_poles=p.get("log_poles"),
            residues=p.get("residues"), in_proj_weight=w_deq, in_proj_scales=None,
            out_proj_weight=p["out_proj.weight"], out_proj_bias=p["out_proj.bias"]))
    meta = prefill_meta([tokens_per_step], [1], "cpu")

    def step():
        for p in params:
            states = [torch.zeros(2, 2, 3 * H, dtype=torch.bfloat16), torch.zeros(2, 127, H),
                      torch.zeros(2, H, 16)]
            O.mixer_forward(x, p, meta, states)

    for _ in range(warmup):
        step()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    med = statistics.median(ts)
    return tokens_per_step / med, threads, med



# ---------------------------------------------------------------- config 5 (TP)
H40 = 8192
TP_TOKENS = 262144


def collective_used(layers):
    """Which all-reduce the channel-sharded out_proj of these layers ran."""
    from evo2_flash_b200 import parallel

    red = [r for r in parallel._REDUCERS.values() if r]
    if layers[0].tp_collective == "nccl" or not red:
        return "nccl all-reduce"
    return f"in-switch NVLS all-reduce kernel ({red[0].num_ctas} CTAs, collective stream)"


def run_tp40b(args, world, rank, device, dist_ok, quiet=False):
    """40B-shape triple, channel-sharded over `world` ranks; chunked prefill with
    the row-parallel all-reduces in flight under the following chunks, then
    batch-1 decode steps (eager, one all-reduce per layer).  Returns the JSON
    line (printed by rank 0 unless `quiet`)."""
    import torch.distributed as dist

    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer, set_forward_metadata
    from evo2_flash_b200.synthetic import mixer_tensors

    from evo2_flash_b200 import ops

    group = dist.group.WORLD if dist_ok else None
    reserve = args.tp_reserve_sms if world > 1 else 0
    if world > 1 and not args.tp_chaining:
        ops.set_launch_chaining(False)
    if reserve:
        props = torch.cuda.get_device_properties(device)
        ops.set_gemm_max_ctas(props.multi_processor_count - reserve)
    cfg = SimpleNamespace(hidden_size=H40, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=True)
    # identical (seeded, on-device) full tensors on every rank; each keeps its shard
    gen = torch.Generator(device=device).manual_seed(5)
    table = torch.randn(512, H40, generator=gen, device=device)
    lut = torch.tensor([65, 67, 71, 84], device=device)
    toks = lut[torch.randint(0, 4, (TP_TOKENS,), generator=gen, device=device)]
    x = rmsnorm(table[toks])
    sx = (x[:4096].float().abs().amax() / 448.0).reshape(1)
    layers = []
    for i, (kind, k) in enumerate(TRIPLE):
        t = mixer_tensors(kind, H40, k, 200 + i, fp8=True, device=device)
        t["in_proj.input_scale"] = sx
        kw = dict(tp_rank=rank, tp_size=world, tp_group=group, device=device,
                  tp_collective=args.tp_collective)
        m = (HyenaIIRMixer(cfg, i, prefix=f"tp.{i}", **kw) if kind == "hcl"
             else HyenaFIRMixer(cfg, i, prefix=f"tp.{i}", k_inner=k, **kw))
        m.load_full_weights(t)
        del t
        m.allocate_state(2, device)
        layers.append(m)
    chunk = args.tp_chunk
    nchunks = TP_TOKENS // chunk
    metas = [prefill_meta([chunk], [1], device, init=[c > 0]) for c in range(nchunks)]

    def prefill_step():
        pend = []
        for c in range(nchunks):
            xc = x[c * chunk:(c + 1) * chunk]
            with set_forward_metadata(metas[c]):
                for m in layers:
                    pend.append(m.forward_async(xc))
        for p in pend:
            p.wait()

    for _ in range(args.warmup):
        prefill_step()
    torch.cuda.synchronize()
    if dist_ok:
        dist.barrier()
    with Clocks(torch.cuda.current_device()) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            prefill_step()
        e1.record()
        torch.cuda.synchronize()
    t_step = e0.elapsed_time(e1) / args.steps
    if dist_ok:
        tt = torch.tensor([t_step], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_step = float(tt.item())

    # batch-1 decode after the prefill (state continues from the last chunk)
    dmeta = decode_meta([1], device)
    xd = rmsnorm(table[lut[torch.randint(0, 4, (args.tp_decode_steps + args.warmup,),
                                         generator=gen, device=device)]])

    def decode_step(i):
        with set_forward_metadata(dmeta):
            for m in layers:
                m(xd[i:i + 1])

    for i in range(args.warmup):
        decode_step(i)
    torch.cuda.synchronize()
    if dist_ok:
        dist.barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    for i in range(args.tp_decode_steps):
        decode_step(args.warmup + i)
    d1.record()
    torch.cuda.synchronize()
    d_ms = d0.elapsed_time(d1) / args.tp_decode_steps
    if dist_ok:
        tt = torch.tensor([d_ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        d_ms = float(tt.item())

    f_gemm = 3 * (2 * TP_TOKENS * H40 * 3 * H40 + 2 * TP_TOKENS * H40 * H40)  # whole job
    value = TP_TOKENS / (t_step * 1e-3)
    line = {
        "metric": METRIC + " (config 5: 40B-shape triple, tensor parallel)",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "e4m3/bf16",
        "data": "synthetic (seeded ACGT, random-init weights)",
        "config": {"workload": "config5: HCS+HCM+HCL mixer triple, 40B shape (H=8192), "
                               "channel-sharded (column-parallel in_proj, row-parallel out_proj "
                               "+ one all-reduce per layer)",
                   "hidden": H40, "global_batch": 1, "seq_len": TP_TOKENS,
                   "parallelism": f"tp{world}", "prefill_chunk": chunk,
                   "gemm_sms_left_to_collectives": reserve,
                   "collective": collective_used(layers) if world > 1 else None,
                   "launch_chaining": bool(args.tp_chaining) or world == 1,
                   "l2": "inputs larger than L2 (x 4.3 GB)"},
        "tok_per_s_per_gpu": value / world,
        "projection_tflops_per_gpu": f_gemm / world / (t_step * 1e-3) / 1e12,
        "decode": {"batch": 1, "ms_per_step": d_ms, "tok_per_s": 1e3 / d_ms,
                   "steps": args.tp_decode_steps, "graph": False},
        "clocks": clk.summary(),
    }
    if rank == 0 and not quiet:
        print(json.dumps(line))
    return line



def run_cp40b(args, world, rank, device, dist_ok, quiet=False):
    """40B-shape triple, one 262144-token sequence split into `world`
    contiguous slices (context parallel); per layer the only collective is the
    LI layer's all-gather of (H, 16) slice states.  Returns the JSON line
    (printed by rank 0 unless `quiet`)."""
    from evo2_flash_b200 import HyenaFIRMixer, HyenaIIRMixer
    from evo2_flash_b200.context_parallel import cp_prefill, dist_gather, halo_rows
    from evo2_flash_b200.synthetic import mixer_tensors

    cfg = SimpleNamespace(hidden_size=H40, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=True)
    gen = torch.Generator(device=device).manual_seed(5)
    table = torch.randn(512, H40, generator=gen, device=device)
    lut = torch.tensor([65, 67, 71, 84], device=device)
    toks = lut[torch.randint(0, 4, (TP_TOKENS,), generator=gen, device=device)]
    L = TP_TOKENS // world
    lo = rank * L
    halo = 136  # >= every layer's halo_rows (129 for K = 128)
    x_src = table[toks[max(0, lo - halo):lo + L]]
    x_all = rmsnorm(x_src)
    x_local = x_all[x_all.shape[0] - L:]
    x_halo = None if rank == 0 else x_all[:x_all.shape[0] - L]
    calib = rmsnorm(table[toks[:4096]])
    sx = (calib.float().abs().amax() / 448.0).reshape(1)
    layers = []
    for i, (kind, k) in enumerate(TRIPLE):
        t = mixer_tensors(kind, H40, k, 200 + i, fp8=True, device=device)
        t["in_proj.input_scale"] = sx
        m = (HyenaIIRMixer(cfg, i, prefix=f"cp.{i}", device=device) if kind == "hcl"
             else HyenaFIRMixer(cfg, i, prefix=f"cp.{i}", k_inner=k, device=device))
        m.load_full_weights(t)
        del t
        m.allocate_state(2, device)
        assert halo >= halo_rows(m)
        layers.append(m)
    if dist_ok:
        gather = dist_gather()
    else:
        gather = lambda t: t[None]  # noqa: E731

    def step():
        for m in layers:
            cp_prefill(m, x_local, x_halo, rank, gather)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if dist_ok:
        torch.distributed.barrier()
    with Clocks(torch.cuda.current_device()) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    t_step = e0.elapsed_time(e1) / args.steps
    if dist_ok:
        tt = torch.tensor([t_step], device=device)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_step = float(tt.item())
    value = TP_TOKENS / (t_step * 1e-3)
    line = {
        "metric": METRIC + " (config 5: 40B-shape triple, context parallel)",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "e4m3/bf16",
        "data": "synthetic (seeded ACGT, random-init weights)",
        "config": {"workload": "config5: HCS+HCM+HCL mixer triple, 40B shape (H=8192), one "
                               "sequence split into contiguous per-rank slices (FIR halo rows, "
                               "LI slice states all-gathered)",
                   "hidden": H40, "global_batch": 1, "seq_len": TP_TOKENS,
                   "parallelism": f"cp{world}", "slice_tokens": L, "halo_rows": halo,
                   "l2": "inputs larger than L2"},
        "tok_per_s_per_gpu": value / world,
        "clocks": clk.summary(),
    }
    if rank == 0 and not quiet:
        print(json.dumps(line))
    return line



def run_hcm256(args, device):
    """Config 1: one HCM mixer block at H = 256 (bf16 in_proj), 2 x 1024 uniform
    ACGT tokens through an N(0,1) 512 x 256 table; the B200 path, with the
    reference algorithm's CPU port timed beside it (cpu_baseline)."""
    from evo2_flash_b200 import HyenaFIRMixer, set_forward_metadata
    from evo2_flash_b200.synthetic import mixer_tensors

    Hs, B, L = 256, 2, 1024
    cfg = SimpleNamespace(hidden_size=Hs, short_filter_length=3, hcm_filter_length=128,
                          state_size=16, use_fp8_input_projections=False)
    t = mixer_tensors("hcm", Hs, 128, 0, fp8=False)
    m = HyenaFIRMixer(cfg, 0, prefix="cfg1", k_inner=128, device=device)
    m.load_full_weights({k: v.to(device) for k, v in t.items()})
    m.allocate_state(B + 1, device)
    table = torch.randn(512, Hs, generator=torch.Generator().manual_seed(1))
    toks = acgt_tokens(B * L, torch.Generator().manual_seed(0))
    x = rmsnorm(table[toks]).to(device)
    meta = prefill_meta([L] * B, list(range(1, B + 1)), device)

    def step():
        with set_forward_metadata(meta):
            m(x)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps

    from oracle import hyena_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    po = O.MixerParams(H=Hs, kind="fir", k_inner=128, short_filter=t["short_filter"], conv=t["conv"],
                       D=t["D"], log_poles=None, residues=None, in_proj_weight=t["in_proj.weight"],
                       in_proj_scales=None, out_proj_weight=t["out_proj.weight"],
                       out_proj_bias=t["out_proj.bias"])
    xc, mc = x.cpu(), prefill_meta([L] * B, list(range(1, B + 1)), "cpu")
    ts = []
    for i in range(4):
        states = [torch.zeros(B + 1, 2, 3 * Hs, dtype=torch.bfloat16), torch.zeros(B + 1, 127, Hs),
                  torch.zeros(B + 1, Hs, 16)]
        t0 = time.perf_counter()
        O.mixer_forward(xc, po, mc, states)
        if i:
            ts.append(time.perf_counter() - t0)
    cpu = B * L / statistics.median(ts)
    line = {
        "metric": METRIC + " (config 1: one HCM block, H=256)", "value": B * L / (ms * 1e-3),
        "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded uniform ACGT, random-init weights)",
        "config": {"workload": "config1: HCM mixer block, H=256, bf16, 2 x 1024 tokens",
                   "hidden": Hs, "global_batch": B, "seq_len": L,
                   "l2": "fits in L2 (launch-bound case)"},
        "cpu_baseline": {"value": cpu, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": "the whole config (2 x 1024 tokens), median of 3"},
    }
    print(json.dumps(line))


def run_model7b(args, device, quiet=False):
    """Config 4: the full random-init StripedHyena2 7B (32 blocks, attention at
    3/10/17/24/31, fp8 Hyena in_proj) scoring a bounded sample of the 64
    order-3-Markov ACGT sequences (lengths U[1k, 32k], seeded): prefill tok/s
    and mean per-token NLL (parity with the all-reference arm is a test)."""
    from evo2_flash_b200.model import StripedHyena2, StripedHyena2Config
    from evo2_flash_b200.synthetic import markov_acgt

    lens = torch.randint(1024, 32769, (64,), generator=torch.Generator().manual_seed(3)).tolist()
    seqs = markov_acgt(lens[:args.model_seqs], seed=3)
    model = StripedHyena2(StripedHyena2Config.evo2_7b(), device=device)
    model.load_tensors(model.random_tensors(0, gen_device=device))
    ntok = sum(len(s) for s in seqs)
    for _ in range(max(1, args.warmup - 2)):
        model.score(seqs[:1], max_tokens_per_step=args.model_step_tokens)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    nll = model.score(seqs, max_tokens_per_step=args.model_step_tokens)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    line = {
        "metric": METRIC + " (config 4: full random-init 7B, scoring prefill)",
        "value": ntok / (ms * 1e-3), "unit": "tok/s", "n_gpus": 1, "steps": 1,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3/bf16",
        "data": "synthetic (seeded order-3 Markov ACGT, random-init weights)",
        "config": {"workload": "config4: StripedHyena2 7B scoring", "sequences": len(seqs),
                   "tokens": ntok, "max_tokens_per_step": args.model_step_tokens,
                   "attention": "torch SDPA (outside the mixer path)"},
        "mean_nll": sum(nll) / len(nll),
    }
    if not quiet:
        print(json.dumps(line))
    return line


def sharded_40b_record(args, world, rank, device, dist_ok):
    """Config 5 inside the default run, so that every N of a scaling run records
    the channel-sharded design: t1 = the unsharded 40B-shape triple on rank 0
    alone (the same 32768-token chunks), then the tensor-parallel and the
    context-parallel prefill over all `world` ranks, each with its parallel
    efficiency t1 / (N t_N)."""
    sub = SimpleNamespace(**vars(args))
    sub.steps = 3
    if world == 1:
        tp = run_tp40b(sub, 1, 0, device, False, quiet=True)
        t1 = tp["ms_per_step"]
    else:
        t1 = 0.0
        if rank == 0:
            t1 = run_tp40b(sub, 1, 0, device, False, quiet=True)["ms_per_step"]
        torch.cuda.empty_cache()
        torch.distributed.barrier()
        tp = run_tp40b(sub, world, rank, device, True, quiet=True)
    tp_error = collective_error(world, device)
    torch.cuda.empty_cache()
    cp = run_cp40b(sub, world, rank, device, dist_ok, quiet=True)
    torch.cuda.empty_cache()

    def part(line):
        t = line["ms_per_step"]
        return {"ms_per_step": t, "tok_per_s": line["value"],
                "tok_per_s_per_gpu": line["value"] / world,
                "efficiency": t1 / (world * t), "parallelism": line["config"]["parallelism"],
                "steps": sub.steps, "clocks": line.get("clocks")}

    rec = {"workload": "config5: HCS+HCM+HCL triple at the 40B shape (H=8192, fp8 in_proj "
                       "8192->24576), one 262144-token sequence",
           "t1_ms": t1, "t1_source": "rank 0 alone, unsharded, same chunking as tp",
           "tp": part(tp), "cp": part(cp)}
    rec["tp"]["decode_ms_per_step"] = tp["decode"]["ms_per_step"]
    rec["tp"]["decode_steps"] = tp["decode"]["steps"]
    rec["tp"]["collective"] = tp["config"].get("collective")
    if tp_error:
        rec["tp"]["error"] = "a cross-rank wait of the in-switch all-reduce expired"
    return rec


def collective_error(world, device) -> bool:
    """True when an in-switch reducer of any rank reports an expired cross-rank
    wait (agreed over the ranks, so that all take the same path)."""
    from evo2_flash_b200 import parallel

    err = 0
    for red in parallel._REDUCERS.values():
        if red:
            red.stream.synchronize()
            err |= int(red.error.item())
            red.error.zero_()
    if world > 1:
        t = torch.tensor([err], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        err = int(t.item())
    return bool(err)


def release_reducers():
    """Checks every in-switch reducer's error word (a cross-rank wait that
    expired) and frees their symmetric buffers, before the process group goes."""
    from evo2_flash_b200 import parallel

    for red in parallel._REDUCERS.values():
        if red:
            red.check()
    parallel._REDUCERS.clear()
    torch.cuda.synchronize()


def config2(world, batch):
    """The `config` of the default line (config 2), shared by both arms."""
    return {"workload": "config2: HCS+HCM+HCL mixer triple prefill, 7B shape",
            "model": "StripedHyena2-7B mixer triple (random init)", "hidden": H,
            "global_batch": batch * world, "seq_len": PREFILL_L,
            "parallelism": f"replicas x{world}",
            "l2": "inputs larger than L2 (x 512 MiB, z 1.5 GiB per layer)"}


# ---------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--decode-steps", type=int, default=500)
    ap.add_argument("--cpu-tokens", type=int, default=512)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-40b", action="store_true",
                    help="skip the config-5 (sharded 40B) record of the default run")
    ap.add_argument("--no-model7b", action="store_true",
                    help="skip the config-4 (full 7B model) record of the default run")
    ap.add_argument("--only", choices=["prefill", "decode"], default=None,
                    help="run one workload (small profiling cases)")
    ap.add_argument("--batch", type=int, default=PREFILL_B, help="prefill sequences per rank")
    ap.add_argument("--workload", choices=["triple", "tp40b", "cp40b", "hcm256", "model7b"],
                    default="triple")
    ap.add_argument("--model-seqs", type=int, default=8, help="model7b: sequences scored")
    ap.add_argument("--model-step-tokens", type=int, default=65536,
                    help="model7b: packed tokens per prefill step")
    ap.add_argument("--tp-chunk", type=int, default=32768, help="tp40b prefill chunk (tokens)")
    ap.add_argument("--tp-decode-steps", type=int, default=256)
    ap.add_argument("--tp-reserve-sms", type=int, default=0,
                    help="tp40b with N > 1: SMs the projection GEMMs leave to the all-reduces")
    ap.add_argument("--tp-collective", choices=["auto", "nvls", "nccl"], default="auto",
                    help="tp40b: the out_proj all-reduce (in-switch kernel or NCCL)")
    ap.add_argument("--tp-chaining", type=int, default=1,
                    help="tp40b with N > 1: programmatic dependent launch between kernels (1/0)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        tps, threads, med = cpu_baseline_sample(args.cpu_tokens, args.steps, 1)
        line = {
            "metric": METRIC, "value": tps, "unit": "tok/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": med * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config2(args.gpus, args.batch),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"1 x {args.cpu_tokens} ACGT tokens through the triple "
                                       "per step (a bounded sample of the workload above)"},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line))
        return

    import torch.distributed as dist

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist_ok = world > 1
    if dist_ok:
        from datetime import timedelta

        kw = {}
        if args.workload in ("tp40b", "triple"):  # collectives overlap compute: their CTAs first
            opts = dist.ProcessGroupNCCL.Options()
            opts.is_high_priority_stream = True
            kw["pg_options"] = opts
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device, **kw)

    if args.workload in ("hcm256", "model7b"):
        if rank == 0:
            (run_hcm256 if args.workload == "hcm256" else run_model7b)(args, device)
        if dist_ok:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.workload in ("tp40b", "cp40b"):
        (run_tp40b if args.workload == "tp40b" else run_cp40b)(args, world, rank, device, dist_ok)
        release_reducers()
        if dist_ok:
            dist.barrier()
            dist.destroy_process_group()
        return

    from evo2_flash_b200 import ops as ops_mod

    gen = torch.Generator().manual_seed(1234 + rank)
    table = torch.randn(512, H, generator=torch.Generator().manual_seed(1))
    T = args.batch * PREFILL_L
    x = embed_norm(acgt_tokens(T, gen), table, device)
    calib = embed_norm(acgt_tokens(4096, torch.Generator().manual_seed(9)), table, device)
    input_scale = (calib.float().abs().amax() / 448.0).reshape(1).cpu()
    layers = build_triple(device, input_scale, num_blocks=DECODE_B + 2)
    meta = prefill_meta([PREFILL_L] * args.batch, list(range(1, args.batch + 1)), device)

    if args.only == "decode":  # decode-only profiling case
        dgen = torch.Generator().manual_seed(2 + rank)
        d_ms, _ = run_decode(layers, table, device, args.decode_steps, args.warmup, dgen)
        v_ms = run_verify(layers, table, device, max(10, args.decode_steps // 4), args.warmup,
                          torch.Generator().manual_seed(4 + rank))
        if rank == 0:
            print(json.dumps({"decode_ms_per_step": d_ms, "decode_tok_per_s": DECODE_B / d_ms * 1e3,
                              "verify_ms_per_step": v_ms}))
        return

    with KernelTimer(ops_mod, "gemm_e4m3") as gt:
        ms, clocks = run_prefill(layers, x, meta, args.steps, args.warmup, dist_ok, device, gt)
    t_step = ms / args.steps
    if dist_ok:
        tt = torch.tensor([t_step], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_step = float(tt.item())
    value = world * T / (t_step * 1e-3)

    peaks = measured_peaks()
    fp8_burst, fp8_peak = fp8_peak_tflops(device)
    gemm_ms = gt.mean_ms()
    f_in, f_out, b_in, b_out, b_quant, b_core = prefill_flops_bytes(T)
    achieved = f_in / (gemm_ms * 1e-3) / 1e12
    # the in_proj / out_proj are timed inside a long step: sustained peaks
    bf16_peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops", 1590.0))
    hbm = peaks.get("hbm_gbs", 6650.0)
    t_roof = 3 * (max(f_in / (fp8_peak * 1e12), b_in / (hbm * 1e9))
                  + max(f_out / (bf16_peak * 1e12), b_out / (hbm * 1e9))
                  + b_quant / (hbm * 1e9) + b_core / (hbm * 1e9))

    decode = None
    if args.only != "prefill" and not os.environ.get("HYENA_BENCH_NO_DECODE"):
        dgen = torch.Generator().manual_seed(2 + rank)
        d_ms, lengths = run_decode(layers, table, device, args.decode_steps, args.warmup, dgen)
        if dist_ok:
            tt = torch.tensor([d_ms], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            d_ms = float(tt.item())
        dbytes = decode_bytes_per_step()
        decode = {"tok_per_s": world * DECODE_B / (d_ms * 1e-3), "ms_per_step": d_ms,
                  "batch": DECODE_B, "steps": args.decode_steps, "graph": True,
                  "hbm_gbs": dbytes / (d_ms * 1e-3) / 1e9,
                  "hbm_frac": dbytes / (d_ms * 1e-3) / 1e9 / hbm,
                  "bytes_per_step": dbytes,
                  "prompt_tokens": int(sum(lengths))}
        v_ms = run_verify(layers, table, device, max(10, args.decode_steps // 4), args.warmup,
                          torch.Generator().manual_seed(4 + rank))
        if dist_ok:
            tt = torch.tensor([v_ms], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            v_ms = float(tt.item())
        vbytes = verify_bytes_per_step()
        decode["verify"] = {"q": 4, "ms_per_step": v_ms, "positions_per_s": world * DECODE_B * 4 / (v_ms * 1e-3),
                            "accepted": "uniform 1..4, resolved from position stamps",
                            "hbm_gbs": vbytes / (v_ms * 1e-3) / 1e9,
                            "hbm_frac": vbytes / (v_ms * 1e-3) / 1e9 / hbm,
                            "bytes_per_step": vbytes, "graph": True}

    e2e = None
    if not args.no_e2e:
        with LocalNumaAlloc(device):
            x_host = x.cpu().pin_memory()
        e_steps = max(3, args.steps)
        e_ms, h2d, d2h = run_e2e(layers, x_host, meta, e_steps, device)
        e_step = e_ms / e_steps
        if dist_ok:
            tt = torch.tensor([e_step], device=device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_step = float(tt.item())
        e2e = {"value": world * T / (e_step * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e_step}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, threads, med = cpu_baseline_sample(args.cpu_tokens, 3, 1)
        cpu = {"value": tps, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"1 x {args.cpu_tokens} ACGT tokens through the triple (oracle port, "
                         f"in_proj as bf16 GEMM on dequantised e4m3 weights), median of 3"}

    model7b = None
    if rank == 0 and world == 1 and not args.no_model7b and args.only is None:
        ml = run_model7b(args, device, quiet=True)
        model7b = {"workload": ml["config"]["workload"], "tok_per_s": ml["value"],
                   "mean_nll": ml["mean_nll"], "ms": ml["ms_per_step"],
                   "sequences": ml["config"]["sequences"], "tokens": ml["config"]["tokens"]}
        torch.cuda.empty_cache()

    sharded = None
    if not args.no_40b and args.only is None:
        del layers
        torch.cuda.empty_cache()
        sharded = sharded_40b_record(args, world, rank, device, dist_ok)

    launches_per_step = 5 + 5 + 8  # quant+gemm+core(2 or 5)+gemm per layer
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e4m3/bf16",
        "data": "synthetic (seeded ACGT, random-init weights)",
        "config": config2(world, args.batch),
        "roofline": {"bound": "tensor", "kernel": "hyena_gemm_e4m3 (in_proj, tcgen05)",
                     "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
                     "frac": achieved / fp8_peak,
                     "traffic": IN_PROJ_DRAM_BYTES_PER_TOKEN * T,
                     "traffic_algorithmic": b_in,
                     "peak_source": "measured in this run: cuBLAS e4m3 8192^3, sustained "
                                    "(back-to-back for 2 s, under the power cap); "
                                    "the kernel is timed inside a long step",
                     "peak_burst": fp8_burst, "frac_of_burst": achieved / fp8_burst,
                     "triple_peaks": {"fp8_tflops": fp8_peak,
                                      "bf16_tflops": bf16_peak, "hbm_gbs": hbm},
                     "triple_t_roof_ms": t_roof * 1e3, "triple_frac": t_roof * 1e3 / t_step},
        "decode": decode,
        "config4": model7b,
        "sharded_40b": sharded,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line))
    release_reducers()
    if dist_ok:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
