"""Benchmark of the redistribute collectives (BASELINE.json metric: redistribute bus GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--op OP] [--sweep]

N = 1: the reference's same-device mode -- every rank of the group on one GPU, one kernel does the whole
       collective (HBM-bound: the rank-order reduce reads n partials and writes one result).
N > 1: launched by torchrun, one process per GPU; each process is one rank of a dt_comm whose peers are
       IPC-mapped, and the kernels move data through peer HBM over NVLink.

The default workload is BASELINE configs[1]: all-reduce Partial->Replicate, bf16 (8192, 8192), rank r's
partial N(0,1) from seed + r, fp32 accumulation in rank order. `--op` selects the other configs.

`value` is the whole-job aggregate bus bandwidth: the nccl-tests bus bandwidth of one rank (algorithm
bandwidth times 2(n-1)/n for all-reduce, (n-1)/n for the others) times the number of GPUs. `bus_gbs_per_rank`
is the per-rank figure and `pct_nvlink_peak` compares it with 900 GB/s per direction.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
os.environ.setdefault("DTORCH_COMM_TIMEOUT_SECOND", "60")

import numpy as np  # noqa: E402
import torch  # noqa: E402

NVLINK_NOMINAL_GBS = 900.0      # NVLink 5, per direction per GPU
NVLINK_P2P_CEILING_GBS = 709.0  # SM stores to a peer, both directions at once (profiles/nvlink_p2p_ceiling_probe.md)
FALLBACK_HBM_GBS = 6650.0

# ---------------------------------------------------------------------------------------------------------
# Workloads
# ---------------------------------------------------------------------------------------------------------
CONFIGS = {
    "all_gather": dict(name="C1 all-gather Shard(0)->Replicate fp32 (4096,4096)", dtype=torch.float32,
                       global_shape=(4096, 4096), dist="rand", emul_n=2),
    "all_reduce": dict(name="C2 all-reduce Partial->Replicate bf16 (8192,8192)", dtype=torch.bfloat16,
                       shape=(8192, 8192), dist="randn", emul_n=8),
    "reduce_scatter": dict(name="C3 reduce-scatter Partial->Shard(0) bf16 (16384,8192)", dtype=torch.bfloat16,
                           shape=(16384, 8192), dist="randn", emul_n=8),
    "all_to_all": dict(name="C4 Ulysses all-to-all Shard(1)->Shard(2) bf16 (1,65536,64,128)", dtype=torch.bfloat16,
                       global_shape=(1, 65536, 64, 128), dist="randn", emul_n=8, src_dim=1, dst_dim=2),
}
DT_NAME = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}


def shard_sizes(length, n):
    return [length // n + (1 if i < length % n else 0) for i in range(n)]


def bus_factor(op, n):
    return 2.0 * (n - 1) / n if op == "all_reduce" else (n - 1) / n


def gen(shape, dtype, seed, dist, device):
    g = torch.Generator(device=device).manual_seed(seed)
    if dist == "rand":
        t = torch.rand(*shape, generator=g, device=device)
    elif dist == "uniform":
        t = torch.rand(*shape, generator=g, device=device) * 2 - 1
    else:
        t = torch.randn(*shape, generator=g, device=device)
    return t.to(dtype)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": FALLBACK_HBM_GBS}, "fallback"


def profile_traffic(key):
    """DRAM bytes per launch of the dominant kernel, from the committed ncu summary (profiles/traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get(key)
    except Exception:
        return None


# ---------------------------------------------------------------------------------------------------------
# Clock sampling during the timed region (NVML; nvidia-smi as fallback)
# ---------------------------------------------------------------------------------------------------------
_SAMPLER = r"""
import sys, time
import pynvml as nv
nv.nvmlInit()
h = nv.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
period = float(sys.argv[2])
print("max", nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM), flush=True)
while True:
    try:
        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
    except Exception:
        r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
    print(time.time(), nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), int(r), flush=True)
    time.sleep(period)
"""


class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML in a separate process (a sampling thread would
    compete for the GIL with the launch loop) during the timed region."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.dev = device_index
        self.period = period_s
        self.proc = None
        self.max_mhz = None
        self.samples = []
        self.t0 = self.t1 = 0.0

    def __enter__(self):
        import subprocess

        try:
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, str(self.dev), str(self.period)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            first = self.proc.stdout.readline().split()
            self.max_mhz = int(first[1]) if len(first) == 2 and first[0] == "max" else None
            self.proc.stdout.readline()  # one sample taken: the sampler is running
        except Exception:
            self.proc = None
        self.t0 = time.time()
        return self

    def __exit__(self, *a):
        self.t1 = time.time()
        if self.proc is None:
            return
        time.sleep(2 * self.period)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        for line in out.splitlines():
            f = line.split()
            if len(f) == 3:
                self.samples.append((float(f[0]), int(f[1]), int(f[2])))

    def summary(self):
        if self.proc is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        inside = [s for s in self.samples if self.t0 <= s[0] <= self.t1]
        if not inside:  # region shorter than one period: the first sample after it
            after = [s for s in self.samples if s[0] > self.t1]
            inside = after[:1] or self.samples[-1:]
        reasons = 0
        for s in inside:
            reasons |= s[2]
        names = [k for k, v in self.REASONS.items() if reasons & v and k != "gpu_idle"]
        return {"sm_mhz": statistics.median([s[1] for s in inside]), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(inside), "region_s": round(self.t1 - self.t0, 4)}


# ---------------------------------------------------------------------------------------------------------
# NVLink traffic counters (NVML field values, read-only): payload bytes this GPU sent and received over all of
# its NVLinks. Read before and after the timed steps, they give the traffic of the collective per launch.
# ---------------------------------------------------------------------------------------------------------
class NvLinkCounter:
    FI_TX, FI_RX = 138, 139  # NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX / _RX, in KiB
    MAX_LINKS = 18

    def __init__(self, cuda_index: int):
        self.h = None
        self.scope = None
        try:
            import pynvml as nv

            nv.nvmlInit()
            self.nv = nv
            try:
                p = torch.cuda.get_device_properties(cuda_index)
                bus = "%08x:%02x:%02x.0" % (p.pci_domain_id, p.pci_bus_id, p.pci_device_id)
                self.h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = nv.nvmlDeviceGetHandleByIndex(cuda_index)
            # aggregate over links if the driver offers it, else the sum of the per-link counters
            for scope in ([0xFFFFFFFF], list(range(self.MAX_LINKS))):
                if self._read(scope) is not None:
                    self.scope = scope
                    break
        except Exception:
            self.h = None

    def _read(self, scopes):
        try:
            ids = [(f, sc) for f in (self.FI_TX, self.FI_RX) for sc in scopes]
            vals = self.nv.nvmlDeviceGetFieldValues(self.h, ids)
        except Exception:
            return None
        tx = rx = 0
        good = 0
        for (f, _), v in zip(ids, vals):
            if v.nvmlReturn != 0:
                continue
            good += 1
            x = int(v.value.ullVal) * 1024
            if f == self.FI_TX:
                tx += x
            else:
                rx += x
        return (tx, rx) if good else None

    def read(self):
        if self.h is None or self.scope is None:
            return None
        return self._read(self.scope)


# ---------------------------------------------------------------------------------------------------------
# 1-GPU (same-device) workloads
# ---------------------------------------------------------------------------------------------------------
class LocalWorkload:
    """n emulated ranks on cuda:0; one same-device kernel per step."""

    def __init__(self, op, cfg, stream):
        from dtorch_b200 import capi

        self.capi = capi
        self.op = op
        self.cfg = cfg
        self.n = cfg["emul_n"]
        self.stream = stream
        self.dtype = cfg["dtype"]
        self.es = torch.tensor([], dtype=self.dtype).element_size()
        dev = "cuda:0"
        n = self.n
        if op in ("all_reduce", "reduce_scatter"):
            self.ins = [gen(cfg["shape"], self.dtype, r, cfg["dist"], dev).reshape(-1) for r in range(n)]
            self.msg_bytes = self.ins[0].numel() * self.es  # per-rank buffer (AR) / per-rank input (RS)
            if op == "all_reduce":
                self.outs = [torch.empty_like(self.ins[0])]
            else:
                self.outs = [torch.empty(self.ins[0].numel() // n, dtype=self.dtype, device=dev) for _ in range(n)]
            self.hbm_bytes = (n + 1) * self.msg_bytes if op == "all_reduce" else (n + 1) * self.msg_bytes // 1
            if op == "reduce_scatter":
                self.hbm_bytes = n * self.msg_bytes + self.msg_bytes  # read n inputs, write n chunks of S/n
        elif op == "all_gather":
            gs = cfg["global_shape"]
            lens = shard_sizes(gs[0], n)
            full = gen(gs, self.dtype, 0, cfg["dist"], dev)
            self.ins = [t.contiguous() for t in torch.split(full, lens, 0)]
            self.lens = lens
            self.inner = int(np.prod(gs[1:])) * self.es
            self.outs = [torch.empty(gs, dtype=self.dtype, device=dev)]
            self.msg_bytes = full.numel() * self.es  # S = output size
            self.hbm_bytes = 2 * self.msg_bytes
        else:  # all_to_all
            gs = list(cfg["global_shape"])
            sd, dd = cfg["src_dim"], cfg["dst_dim"]
            full = gen(gs, self.dtype, 0, cfg["dist"], dev)
            self.src_lens = shard_sizes(gs[sd], n)
            self.ins = [t.contiguous() for t in torch.split(full, self.src_lens, sd)]
            split = shard_sizes(gs[dd], n)
            self.outs = []
            for k in range(n):
                shp = list(gs)
                shp[dd] = split[k]
                self.outs.append(torch.empty(shp, dtype=self.dtype, device=dev))
            self.in_shape = list(self.ins[0].shape)
            self.msg_bytes = self.ins[0].numel() * self.es  # per-rank buffer
            self.hbm_bytes = 2 * full.numel() * self.es
        self.in_ptrs = [t.data_ptr() for t in self.ins]
        self.out_ptrs = [t.data_ptr() for t in self.outs]
        # pinned host copies for the end-to-end leg, on the GPU's own NUMA node
        from dtorch_b200.multiprocess import near_device

        with near_device(torch.device(dev).index or 0):
            self.h_ins = [t.cpu().pin_memory() for t in self.ins]
            self.h_outs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in self.outs]
        self.h2d = sum(t.numel() * self.es for t in self.ins)
        self.d2h = sum(t.numel() * self.es for t in self.outs)

    def step(self):
        c = self.capi
        s = self.stream.cuda_stream
        if self.op == "all_reduce":
            code = c.dtype_code(self.dtype)
            c.local_all_reduce(self.in_ptrs, self.out_ptrs[0], self.ins[0].numel(), code, 0, s)
        elif self.op == "reduce_scatter":
            code = c.dtype_code(self.dtype)
            c.local_reduce_scatter(self.in_ptrs, self.out_ptrs, self.outs[0].numel(), code, 0, s)
        elif self.op == "all_gather":
            c.local_all_gather(self.in_ptrs, self.out_ptrs[0], 1, self.lens, self.inner, s)
        else:
            c.local_all_to_all(self.in_ptrs, self.out_ptrs, self.in_shape, self.cfg["src_dim"], self.cfg["dst_dim"],
                               self.src_lens, self.es, s)

    def e2e_step(self):
        if self.op == "all_reduce":
            # the host-buffer entry point: chunked H2D, reduction and D2H overlapping inside one call
            c = self.capi
            c.local_all_reduce_host([h.data_ptr() for h in self.h_ins], self.in_ptrs, self.out_ptrs[0],
                                    self.h_outs[0].data_ptr(), self.ins[0].numel(), c.dtype_code(self.dtype), 0, 0,
                                    self.stream.cuda_stream)
            return
        with torch.cuda.stream(self.stream):
            for d, h in zip(self.ins, self.h_ins):
                d.copy_(h, non_blocking=True)
            self.step()
            for h, d in zip(self.h_outs, self.outs):
                h.copy_(d, non_blocking=True)


def time_steps(fn, steps, stream):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps  # ms per step


def l2_plan(in_bytes, device, l2_bytes=None):
    """How the timed steps keep L2 from serving the inputs: (flush, l2 bytes, description). Inputs larger than
    L2 are not flushed; smaller ones get an L2 flush between timed steps (time_steps_flushed). `l2_bytes`
    defaults to the device's L2 size."""
    l2 = int(l2_bytes if l2_bytes is not None else torch.cuda.get_device_properties(device).L2_cache_size)
    mib = lambda b: f"{b / 2**20:.0f} MiB"  # noqa: E731
    if in_bytes > l2:
        return False, l2, f"inputs on this GPU ({mib(in_bytes)}) larger than L2 ({mib(l2)}); no flush"
    return True, l2, (f"inputs on this GPU ({mib(in_bytes)}) fit in L2 ({mib(l2)}): L2 flushed between timed "
                      f"steps (a {mib(2 * l2)} write, then a read of it, outside each step's events)")


def time_steps_flushed(fn, steps, stream, l2_bytes, align=None):
    """ms per step with L2 flushed before every step: a write of twice L2 on `stream`, then a read of the same
    buffer (so L2 is left holding clean lines and the step pays for no write-back of the flush), then the step
    between its own pair of events; the steps' event times are summed. `align` (N > 1: a device barrier of the
    ranks) runs after the flush, outside the events, so a rank's step does not time the other ranks' flushes."""
    scratch = torch.empty(2 * l2_bytes // 4, dtype=torch.float32, device=stream.device)
    sink = torch.empty((), dtype=torch.float32, device=stream.device)
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i, (a, b) in enumerate(pairs):
            scratch.fill_(float(i))
            torch.amax(scratch, dim=0, out=sink)
            if align is not None:
                align()
            a.record(stream)
            fn()
            b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in pairs) / steps


# ---------------------------------------------------------------------------------------------------------
# CPU baseline: the reference's own thread-group code (oracle/_ref) on this host's cores
# ---------------------------------------------------------------------------------------------------------
def cpu_inputs(op, cfg, n):
    """Seeded host inputs of the workload as raw numpy storage (uint16 bits for bf16). Generated on the GPU
    when one is present (much faster than the CPU generator), then copied to host memory."""
    dtype = cfg["dtype"]
    gdev = "cuda" if torch.cuda.is_available() else "cpu"

    def raw(t):
        t = t.contiguous()
        return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)

    if op in ("all_reduce", "reduce_scatter"):
        return [raw(gen(cfg["shape"], dtype, r, cfg["dist"], gdev).reshape(-1).cpu()) for r in range(n)]
    gs = cfg["global_shape"]
    full = gen(gs, dtype, 0, cfg["dist"], gdev).cpu()
    dim = 0 if op == "all_gather" else cfg["src_dim"]
    return [raw(t) for t in torch.split(full, shard_sizes(gs[dim], n), dim)]


def sample_inputs(op, cfg, ins, frac):
    """A leading fraction of the workload with the same layout (rows of dim 0 of the global tensor)."""
    if frac >= 1.0:
        return ins
    n = len(ins)
    if op in ("all_reduce", "reduce_scatter"):
        m = max(n, int(ins[0].size * frac) // n * n)
        return [a[:m] for a in ins]
    if op == "all_gather":
        return [a[: max(1, int(a.shape[0] * frac))] for a in ins]
    # all-to-all: cut the source-dim shards (Ulysses sequence) proportionally
    sd = cfg["src_dim"]
    return [np.ascontiguousarray(np.take(a, range(max(1, int(a.shape[sd] * frac))), axis=sd)) for a in ins]


def cpu_reference_run(op, cfg, ins, reps, threads):
    """Time the reference's CPU DeviceMesh path on `ins`; returns (per-rep seconds list, kind)."""
    from oracle.oracle import Reference, Restatement

    code = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[cfg["dtype"]]
    if Reference.available():
        ref = Reference()
        if op == "all_reduce":
            _, s = ref.all_reduce(ins, code, iters=reps, threads=threads)
        elif op == "reduce_scatter":
            _, s = ref.reduce_scatter(ins, code, iters=reps, threads=threads)
        elif op == "all_gather":
            _, s = ref.all_gather(ins, code, 0, iters=reps, threads=threads)
        else:
            _, s = ref.all_to_all(ins, code, cfg["src_dim"], cfg["dst_dim"], iters=reps, threads=threads)
        return [float(v) for v in s], "reference"
    R = Restatement()
    out = []
    for _ in range(reps):
        t0 = time.perf_counter()
        if op == "all_reduce":
            R.fold_sum(ins, code, True)
        elif op == "reduce_scatter":
            R.reduce_scatter(ins, code, True)
        elif op == "all_gather":
            R.all_gather(ins, 0)
        else:
            R.all_to_all(ins, cfg["src_dim"], cfg["dst_dim"])
        out.append(time.perf_counter() - t0)
    return out, "port"


def msg_bytes_of(op, ins):
    """Per-rank message size S of the nccl-tests formulas for host inputs `ins`."""
    if op in ("all_reduce", "reduce_scatter", "all_to_all"):
        return ins[0].nbytes
    return sum(a.nbytes for a in ins)  # all-gather: S = output size


def cpu_baseline(op, cfg, n, budget_s=20.0):
    """Bounded CPU baseline: one probe repetition on a sample, then as many repetitions as fit the budget."""
    cores = os.cpu_count() or 1
    full = cpu_inputs(op, cfg, n)
    frac = 1.0
    ins = full
    probe, kind = cpu_reference_run(op, cfg, ins, 1, cores)
    if probe[0] > budget_s / 3:
        frac = max(1.0 / 64, budget_s / 3 / probe[0])
        ins = sample_inputs(op, cfg, full, frac)
    reps = 3
    secs, kind = cpu_reference_run(op, cfg, ins, reps, cores)
    t = statistics.median(secs)
    msg = msg_bytes_of(op, ins)
    threads = cores if kind == "reference" else 1
    sample = (f"{'full workload' if frac >= 1 else f'{frac:.3f} of the workload (leading rows)'}, median of {reps} "
              f"repetitions, n={n} rank threads on a CPU DeviceMesh, torch intra-op threads={threads}, "
              f"the reference's pre-collective Barrier included" if kind == "reference" else
              f"C restatement (single thread), {frac:.3f} of the workload")
    return t, msg, {"kind": kind, "cores": threads, "sample": sample}


# ---------------------------------------------------------------------------------------------------------
# Parity of the timed collective (outside the timed region): its outputs against the C restatement of the
# reference's algorithm (oracle/dt_oracle.c) on the same seeded inputs. Copies must be bit-exact; the
# rank-order reductions bit-exact against the fp32-accumulate fold; the NVLS reduction (switch order) within
# the north-star tolerance, allclose(rtol=2e-2, atol=2e-2 * rms) for bf16/fp16 and rtol 1e-6 for fp32.
# ---------------------------------------------------------------------------------------------------------
DT_CODE = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
RTOL = {torch.float32: 1e-6, torch.bfloat16: 2e-2, torch.float16: 2e-2}


def raw_np(t):
    """Raw storage of a tensor on the host: float32, or the uint16 bit patterns of bf16 / fp16."""
    t = t.detach().contiguous().cpu()
    return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)


def raw_to_f32(a, code):
    if code == 0:
        return a.astype(np.float32)
    if code == 1:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float16).astype(np.float32)


class Parity:
    """Accumulates output-vs-oracle comparisons into the line's `parity` object."""

    def __init__(self, dtype, tolerance):
        self.code = DT_CODE.get(dtype, 0)
        self.rtol = RTOL.get(dtype, 0.0)
        self.tolerance = tolerance  # False: bit-exact required
        self.bit_exact = True
        self.within = True
        self.max_abs = 0.0
        self.elements = 0
        self.cases = 0

    def compare(self, got, want):
        got = np.asarray(got).reshape(-1)
        want = np.asarray(want).reshape(-1)
        self.cases += 1
        self.elements += int(want.size)
        if got.shape != want.shape:
            self.bit_exact = self.within = False
            self.max_abs = float("inf")
            return
        if np.array_equal(got, want):
            return
        self.bit_exact = False
        g = raw_to_f32(got, self.code).astype(np.float64)
        w = raw_to_f32(want, self.code).astype(np.float64)
        err = np.abs(g - w)
        self.max_abs = max(self.max_abs, float(np.nanmax(err)) if err.size else 0.0)
        rms = float(np.sqrt(np.mean(w * w))) if w.size else 0.0
        ok = bool(np.all(err <= self.rtol * rms + self.rtol * np.abs(w)))
        self.within = self.within and ok and self.tolerance

    @property
    def ok(self):
        return self.bit_exact or (self.tolerance and self.within)

    def summary(self, what):
        return {"checked": True, "ok": self.ok, "bit_exact": self.bit_exact, "max_abs_err": self.max_abs,
                "elements": self.elements, "outputs": self.cases, "against": what,
                "rule": ("within allclose(rtol, atol=rtol*rms), rtol=%g" % self.rtol) if self.tolerance
                else "bit-exact"}


def local_parity(w, par):
    """Outputs of the same-device workload `w` against the restatement."""
    from oracle.oracle import Restatement

    R = Restatement()
    host = [raw_np(t) for t in w.ins]
    if w.op == "all_reduce":
        want = [R.fold_sum(host, par.code, storage_round=False)]
    elif w.op == "reduce_scatter":
        want = R.reduce_scatter(host, par.code, storage_round=False)
    elif w.op == "all_gather":
        want = [R.all_gather(host, 0)]
    else:
        want = R.all_to_all(host, w.cfg["src_dim"], w.cfg["dst_dim"])
    for got, wt in zip(w.outs, want):
        par.compare(raw_np(got), wt)
    return want


# ---------------------------------------------------------------------------------------------------------
# Arms
# ---------------------------------------------------------------------------------------------------------
def run_ours_single(args):
    from dtorch_b200 import capi

    op = args.op
    cfg = CONFIGS[op]
    torch.cuda.set_device(0)
    stream = torch.cuda.Stream(device=0)
    w = LocalWorkload(op, cfg, stream)
    n = w.n
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            w.step()
    torch.cuda.synchronize()
    flush, l2_bytes, l2_note = l2_plan(sum(t.numel() for t in w.ins) * w.es, 0)
    l0 = capi.launch_count()
    with ClockSampler(0) as clk:
        with torch.cuda.stream(stream):
            ms = (time_steps_flushed(w.step, args.steps, stream, l2_bytes) if flush
                  else time_steps(w.step, args.steps, stream))
    launches = capi.launch_count() - l0
    # parity of what the timed steps wrote, against the restatement (outside the timed region)
    par = Parity(cfg["dtype"], tolerance=False)
    want = local_parity(w, par)
    # end to end: pinned host -> device, collective, device -> pinned host, every step
    e2e_par = Parity(cfg["dtype"], tolerance=False)
    if args.skip_e2e:
        e2e_ms = float("nan")
    else:
        for h in w.h_outs:
            h.zero_()
        for _ in range(max(1, args.warmup // 2)):
            w.e2e_step()
        torch.cuda.synchronize()
        e2e_ms = time_steps(w.e2e_step, args.steps, stream)
        for h, wt in zip(w.h_outs, want):
            e2e_par.compare(raw_np(h), wt)
    t = ms / 1e3
    bus = w.msg_bytes * bus_factor(op, n) / t / 1e9
    e2e_bus = w.msg_bytes * bus_factor(op, n) / (e2e_ms / 1e3) / 1e9
    peaks, peak_src = measured_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    achieved = w.hbm_bytes / t / 1e9
    # CPU baseline on this host: the reference's own CPU thread-group path, same workload
    if args.skip_cpu:
        cpu_t, cpu_msg, cpu_info = float("nan"), w.msg_bytes, {"kind": "skipped", "cores": 0, "sample": "--skip-cpu"}
    else:
        cpu_t, cpu_msg, cpu_info = cpu_baseline(op, cfg, n)
    cpu_bus = cpu_msg * bus_factor(op, n) / cpu_t / 1e9
    line = {
        "metric": "redistribute bus GB/s",
        "value": round(bus, 2),
        "unit": "GB/s",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": DT_NAME[cfg["dtype"]],
        "data": "synthetic (seeded, BASELINE.json distribution)",
        "config": {"workload": cfg["name"] + f", same-device group of {n} ranks on 1 GPU (reference same-device "
                   "mode), one kernel per step", "op": op, "group_ranks": n, "msg_bytes_per_rank": w.msg_bytes,
                   "accumulate": "fp32, rank order" if op in ("all_reduce", "reduce_scatter") else "copy",
                   "l2": l2_note, "parallelism": "same-device"},
        "bus_gbs_per_rank": round(bus, 2),
        "pct_nvlink_peak": None,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": profile_traffic(f"local_{op}"),
                     "algorithmic_bytes_per_launch": w.hbm_bytes, "peak_source": f"{peak_src} hbm_gbs"},
        "cpu_baseline": {"value": round(cpu_bus, 4), "unit": "GB/s", "cores": cpu_info["cores"],
                         "kind": cpu_info["kind"], "sample": cpu_info["sample"], "seconds_per_op": round(cpu_t, 4)},
        "e2e": {"value": round(e2e_bus, 3), "unit": "GB/s", "h2d_bytes_per_step": w.h2d, "d2h_bytes_per_step": w.d2h,
                "ms_per_step": round(e2e_ms, 4),
                "path": ("C ABI dt_local_all_reduce_host: pinned host partials in, pinned host sum out, chunked "
                         "H2D / reduction / D2H overlapping" if op == "all_reduce"
                         else "C ABI (dt_local_*) with pinned host buffers")},
        "gpu_launches": launches,
        "clocks": clk.summary(),
        "parity": dict(par.summary("C restatement of the reference's fold / concat / split (oracle/dt_oracle.c), "
                                   "fp32 accumulation in rank order; every output of the timed steps"),
                       e2e_ok=e2e_par.ok if not args.skip_e2e else None),
    }
    print(json.dumps(line), flush=True)
    if not (par.ok and (args.skip_e2e or e2e_par.ok)):
        print("parity check failed: the timed collective's output differs from the oracle", file=sys.stderr)
        sys.exit(3)


def run_reference(args, rank, world):
    """The reference's own CPU thread-group implementation on this host's cores, same config and metric.
    Under torchrun only rank 0 runs it (the CPU mesh lives in one process); the other ranks exit."""
    op = args.op
    cfg = CONFIGS[op]
    n = world if world > 1 else cfg["emul_n"]
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    full = cpu_inputs(op, cfg, n)
    probe, kind = cpu_reference_run(op, cfg, full, 1, cores)
    # each step is a bounded sample so the whole run stays within a few minutes
    budget = 150.0
    frac = min(1.0, max(1.0 / 64, budget / max(1, args.warmup + args.steps) / max(probe[0], 1e-6)))
    ins = sample_inputs(op, cfg, full, frac)
    secs, kind = cpu_reference_run(op, cfg, ins, args.warmup + args.steps, cores)
    t = statistics.median(secs[args.warmup:])
    msg = msg_bytes_of(op, ins)
    bus = msg * bus_factor(op, n) / t / 1e9
    # same basis as our arm: at N > 1 the whole-job aggregate is the per-rank bus bandwidth times the ranks
    value = bus * (n if world > 1 else 1)
    threads = cores if kind == "reference" else 1
    sample = (f"{'full workload' if frac >= 1 else f'{frac:.3f} of the workload (leading rows)'} per step, "
              f"n={n} rank threads, torch intra-op threads={threads}")
    line = {
        "metric": "redistribute bus GB/s", "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": DT_NAME[cfg["dtype"]],
        "data": "synthetic (seeded, BASELINE.json distribution)", "impl": "reference",
        "config": {"workload": cfg["name"] + f", reference CPU DeviceMesh path (ThreadGroupSameDeviceBackend), "
                   f"group of {n} rank threads", "op": op, "group_ranks": n, "msg_bytes_per_rank": msg},
        "bus_gbs_per_rank": round(bus, 4),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def multi_expected(op, cfg, n, rank, dev):
    """This rank's expected output of the workload, from the restatement on the same seeded inputs (every rank
    regenerates the inputs it needs on its own GPU, copies them to the host, and runs the C oracle)."""
    from oracle.oracle import Restatement

    R = Restatement()
    dtype = cfg["dtype"]
    code = DT_CODE[dtype]
    if op == "all_reduce":
        host = [raw_np(gen(cfg["shape"], dtype, r, cfg["dist"], dev).reshape(-1)) for r in range(n)]
        return R.fold_sum(host, code, storage_round=False)
    if op == "reduce_scatter":
        numel = int(np.prod(cfg["shape"]))
        lo, hi = numel // n * rank, numel // n * (rank + 1)
        host = [raw_np(gen(cfg["shape"], dtype, r, cfg["dist"], dev).reshape(-1)[lo:hi]) for r in range(n)]
        return R.fold_sum(host, code, storage_round=False)  # chunk `rank` of the fold = this rank's output
    gs = cfg["global_shape"]
    full = gen(gs, dtype, 0, cfg["dist"], dev)
    if op == "all_gather":
        shards = [raw_np(t) for t in torch.split(full, shard_sizes(gs[0], n), 0)]
        return R.all_gather(shards, 0)
    sd, dd = cfg["src_dim"], cfg["dst_dim"]
    shards = [raw_np(t) for t in torch.split(full, shard_sizes(gs[sd], n), sd)]
    del full
    return R.all_to_all(shards, sd, dd, only=rank)[rank]


def run_api_leg(op, cfg, n, steps, warmup):
    """The same collective through the reference-facing Python API in ONE process driving all n GPUs -- the
    reference's single-controller model: DTensor.redistribute on a 1-D DeviceMesh, the C++ executor's
    kernel-stream threads and ThreadGroup, locals and outputs in the group's symmetric pool. Device time = max
    over the GPUs of CUDA events on each GPU's current stream around `steps` redistribute calls; parity of the
    last result against the restatement."""
    import dtorch_b200 as dtb
    from oracle.oracle import Restatement

    R = Restatement()
    dtype = cfg["dtype"]
    code = DT_CODE[dtype]
    es = torch.tensor([], dtype=dtype).element_size()
    devs = list(range(n))
    mesh = dtb.DeviceMesh("cuda", devs)
    if op in ("all_reduce", "reduce_scatter"):
        shape = tuple(cfg["shape"])
        msg = int(np.prod(shape)) * es
        out_bytes = msg if op == "all_reduce" else msg // n
    else:
        shape = tuple(cfg["global_shape"])
        msg = int(np.prod(shape)) * es if op == "all_gather" else int(np.prod(shape)) * es // n
        out_bytes = int(np.prod(shape)) * es if op == "all_gather" else msg
    # room for the input and several generations of outputs per GPU, so the host can run ahead of the GPUs
    # while earlier outputs wait to be reclaimed
    dtb.set_pool_bytes(((msg + 8 * out_bytes) >> 20) + 64 << 20)
    dtb.clear()
    try:
        if op in ("all_reduce", "reduce_scatter"):
            x = dtb.DTensor.empty({d: shape for d in devs}, dtype, mesh, [dtb.Partial()], shape)
            host = []
            for d in devs:
                t = gen(shape, dtype, d, cfg["dist"], f"cuda:{d}")
                x.local(d).copy_(t)
                host.append(raw_np(t.reshape(-1)))
            target = [dtb.Replicate()] if op == "all_reduce" else [dtb.Shard(0)]
        else:
            full = gen(shape, dtype, 0, cfg["dist"], "cuda:0").cpu()
            src = [dtb.Shard(0)] if op == "all_gather" else [dtb.Shard(cfg["src_dim"])]
            x = dtb.DTensor.from_torch(full, mesh, src)
            target = [dtb.Replicate()] if op == "all_gather" else [dtb.Shard(cfg["dst_dim"])]
        for d in devs:
            torch.cuda.synchronize(d)
        info = dtb.dtensor._host.pool_info(devs, 0)
        in_pool = all(dtb.dtensor._host.in_pool(devs, d, x.local(d)) for d in devs)
        y = None
        for _ in range(warmup):
            y = x.redistribute(placements=target)
        for d in devs:
            torch.cuda.synchronize(d)
        ev = {d: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for d in devs}
        for d in devs:
            ev[d][0].record(torch.cuda.current_stream(d))
        t0 = time.perf_counter()
        for _ in range(steps):
            y = x.redistribute(placements=target)
        host_s = (time.perf_counter() - t0) / steps
        for d in devs:
            ev[d][1].record(torch.cuda.current_stream(d))
        for d in devs:
            torch.cuda.synchronize(d)
        ms = max(ev[d][0].elapsed_time(ev[d][1]) for d in devs) / steps
        out_in_pool = all(dtb.dtensor._host.in_pool(devs, d, y.local(d)) for d in devs)
        nvls = bool(info["nvls"]) and op == "all_reduce" and n >= 6 and msg >= (8 << 20)
        par = Parity(dtype, tolerance=nvls)
        if op == "all_reduce":
            want = R.fold_sum(host, code, storage_round=False)
            for d in devs:
                par.compare(raw_np(y.local(d)), want)
        elif op == "reduce_scatter":
            rows = shape[0] // n
            want = R.reduce_scatter([h.reshape(shape) for h in host], code, storage_round=False)
            for d in devs:
                par.compare(raw_np(y.local(d)), want[d].reshape(rows, *shape[1:]))
        elif op == "all_gather":
            par.compare(raw_np(y.local(0)), raw_np(full))
            for d in devs[1:]:
                par.compare(raw_np(y.local(d)), raw_np(full))
        else:
            sd, dd = cfg["src_dim"], cfg["dst_dim"]
            shards = [raw_np(t) for t in torch.split(full, shard_sizes(shape[sd], n), sd)]
            want = R.all_to_all(shards, sd, dd)
            for d in devs:
                par.compare(raw_np(y.local(d)), want[d])
        bus = msg * bus_factor(op, n) / (ms / 1e3) / 1e9
        return {"bus_gbs_per_rank": round(bus, 2), "value": round(bus * n, 2), "ms_per_step": round(ms, 5),
                "host_ms_per_call": round(host_s * 1e3, 4),
                "path": "one process, DTensor.redistribute on DeviceMesh('cuda', range(n)) -> C++ executor -> "
                        "ThreadGroup -> C ABI; locals and outputs in the group's symmetric pool",
                "pool": {"bytes": int(info["bytes"]), "nvls": bool(info["nvls"]), "inputs_in_pool": in_pool,
                         "outputs_in_pool": out_in_pool},
                "algorithm": "nvls (in-switch reduction)" if nvls else "rank-order P2P kernels",
                "parity": par.summary("C restatement (oracle/dt_oracle.c) on every GPU's output")}
    finally:
        dtb.clear()
        dtb.set_pool_bytes(0)


def heap_tensor(base, offset, numel, dtype, device):
    from dtorch_b200.multiprocess import device_view

    return device_view(base + offset, numel, dtype, device)


def run_ours_multi(args, rank, world, local_rank):
    """One rank per process; peers IPC-mapped through the communicator's symmetric heap."""
    import datetime

    import torch.distributed as dist

    from dtorch_b200 import capi

    op = args.op
    cfg = CONFIGS[op]
    n = world
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    # host-only group: the other ranks wait on it while rank 0 drives every GPU in the API leg, so no NCCL
    # kernel sits on their GPUs meanwhile
    cpu_group = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=900))
    dtype = cfg["dtype"]
    es = torch.tensor([], dtype=dtype).element_size()
    # per-rank buffers
    if op in ("all_reduce", "reduce_scatter"):
        in_numel = int(np.prod(cfg["shape"]))
        out_numel = in_numel if op == "all_reduce" else in_numel // n
        msg = in_numel * es
    elif op == "all_gather":
        gs = cfg["global_shape"]
        lens = shard_sizes(gs[0], n)
        inner = int(np.prod(gs[1:]))
        in_numel = lens[rank] * inner
        out_numel = gs[0] * inner
        msg = out_numel * es
    else:
        gs = list(cfg["global_shape"])
        sd, dd = cfg["src_dim"], cfg["dst_dim"]
        src_lens = shard_sizes(gs[sd], n)
        split = shard_sizes(gs[dd], n)
        in_shape = list(gs)
        in_shape[sd] = src_lens[rank]
        in_numel = int(np.prod(in_shape))
        out_numel = int(np.prod(gs)) // gs[sd] * gs[sd] // gs[dd] * split[rank]
        msg = in_numel * es
    align = 1 << 20
    in_bytes = (in_numel * es + align - 1) // align * align
    out_bytes = (out_numel * es + align - 1) // align * align
    from dtorch_b200.multiprocess import create_rank_comm, setup_nvls

    comm = create_rank_comm(in_bytes + out_bytes, local_rank)
    base, _ = comm.heap(rank)
    x = heap_tensor(base, 0, in_numel, dtype, dev)
    y = heap_tensor(base, in_bytes, out_numel, dtype, dev)
    if op in ("all_reduce", "reduce_scatter"):
        x.copy_(gen(cfg["shape"], dtype, rank, cfg["dist"], dev).reshape(-1))
    elif op == "all_gather":
        x.copy_(gen(gs, dtype, 0, cfg["dist"], dev)[sum(lens[:rank]):sum(lens[:rank + 1])].reshape(-1))
    else:
        full = gen(gs, dtype, 0, cfg["dist"], dev)
        x.copy_(torch.split(full, src_lens, sd)[rank].reshape(-1))
        del full
    stream = torch.cuda.current_stream(dev)
    code = capi.dtype_code(dtype) if dtype in (torch.float32, torch.bfloat16, torch.float16) else 0
    # all-reduce: the two-shot P2P kernel (rank-order fold) on the heap buffers, and -- where the switch
    # supports it and it is faster (n >= 6) -- the NVLS kernel on buffers bound to a multicast object
    algo = {"all_reduce": "p2p two-shot (rank-order fp32 fold)",
            "reduce_scatter": "p2p pull-reduce (rank-order fp32 fold)",
            "all_gather": "p2p push (peer stores at the concat offset)",
            "all_to_all": "p2p push (pack fused into the peer stores)"}[op]
    ar_flags = 0
    xp, yp = x, y
    if op == "all_reduce" and args.algo != "p2p" and (n >= 6 or args.algo == "nvls"):
        if setup_nvls(comm, 2 * in_bytes):
            nb, _ = comm.nvls_buffer(rank)
            xn = heap_tensor(nb, 0, in_numel, dtype, dev)
            yn = heap_tensor(nb, in_bytes, out_numel, dtype, dev)
            xn.copy_(x)
            x, y = xn, yn
            algo = "nvls (in-switch reduction, fp32 accumulate)"
            ar_flags = capi.DT_ALGO_NVLS

    def step():
        s = stream.cuda_stream
        if op == "all_reduce":
            comm.all_reduce(rank, x.data_ptr(), y.data_ptr(), in_numel, code, ar_flags, s)
        elif op == "reduce_scatter":
            comm.reduce_scatter(rank, x.data_ptr(), y.data_ptr(), out_numel, code, 0, s)
        elif op == "all_gather":
            comm.all_gather(rank, x.data_ptr(), y.data_ptr(), 1, lens, inner * es, s)
        else:
            comm.all_to_all(rank, x.data_ptr(), y.data_ptr(), in_shape, sd, dd, src_lens, es, s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    flush, l2_bytes, l2_note = l2_plan(in_numel * es, dev)
    if flush:
        l2_note += "; then the ranks meet in a device barrier (dt_barrier, untimed) before each step's start event"
    nvl = NvLinkCounter(local_rank)
    l0 = capi.launch_count()
    with ClockSampler(local_rank) as clk:
        # ranks start their samplers at different times: line them up after, right before the timed steps
        dist.barrier()
        torch.cuda.synchronize()
        c0 = nvl.read()
        ms = (time_steps_flushed(step, args.steps, stream, l2_bytes,
                                 align=lambda: comm.barrier(rank, stream.cuda_stream)) if flush
              else time_steps(step, args.steps, stream))
    launches = capi.launch_count() - l0 - (args.steps if flush else 0)  # the aligning barriers are untimed
    time.sleep(0.05)
    c1 = nvl.read()
    dist.barrier()
    t_max = torch.tensor([ms], device=dev)
    dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    err = comm.error(rank)
    # NVLink payload bytes this GPU sent / received per launch (NVML counters around the timed steps)
    nvl_tx = nvl_rx = None
    if c0 is not None and c1 is not None:
        nvl_tx = (c1[0] - c0[0]) / args.steps
        nvl_rx = (c1[1] - c0[1]) / args.steps
    # parity of the timed output against the restatement (every rank, outside the timed region)
    want = multi_expected(op, cfg, n, rank, dev)
    par = Parity(dtype, tolerance=(ar_flags == capi.DT_ALGO_NVLS))
    par.compare(raw_np(y), want)
    p2p_bus = None
    p2p_par = None
    if xp is not x:  # the rank-order P2P kernel on the same message, for comparison
        def pstep():
            comm.all_reduce(rank, xp.data_ptr(), yp.data_ptr(), in_numel, code, capi.DT_ALGO_TWOSHOT, stream.cuda_stream)

        for _ in range(3):
            pstep()
        torch.cuda.synchronize()
        dist.barrier()
        pms = time_steps(pstep, args.steps, stream)
        t_max = torch.tensor([pms], device=dev)
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        p2p_bus = msg * bus_factor(op, n) / (float(t_max.item()) / 1e3) / 1e9
        p2p_par = Parity(dtype, tolerance=False)
        p2p_par.compare(raw_np(yp), want)
    # every rank's verdict, gathered on rank 0: [not ok, not bit-exact, max |err|, p2p leg not ok]
    pv = torch.tensor([0.0 if par.ok else 1.0, 0.0 if par.bit_exact else 1.0, par.max_abs,
                       0.0 if (p2p_par is None or p2p_par.ok) else 1.0], device=dev, dtype=torch.float64)
    dist.all_reduce(pv, op=dist.ReduceOp.MAX)
    # end to end: pinned host input -> heap, collective, heap output -> pinned host
    # pinned host buffers on this GPU's NUMA node: with every GPU of the box copying at once, buffers on the
    # other socket would send their DMA over the socket interconnect
    from dtorch_b200.multiprocess import near_device

    with near_device(local_rank) as numa_cpus:
        h_in = x.cpu().pin_memory()
        h_out = torch.empty(out_numel, dtype=dtype).pin_memory()
    e2e_path = "C ABI (dt_* on a multi-process dt_comm) with pinned host buffers, copy - collective - copy"

    def e2e_step():
        x.copy_(h_in, non_blocking=True)
        step()
        h_out.copy_(y, non_blocking=True)

    if op == "all_reduce":
        # the all-reduce chunk by chunk (every rank the same chunks), so the H2D of chunk i+1, the collective on
        # chunk i and the D2H of chunk i-1 overlap -- what dt_local_all_reduce_host does inside the library at N = 1
        per = 16 // es
        step_elems = max(per, ((16 << 20) // es) // per * per)
        chunks = [(lo, min(in_numel, lo + step_elems)) for lo in range(0, in_numel, step_elems)]
        h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_start, ev_end = torch.cuda.Event(), torch.cuda.Event()
        ev_in, ev_red = torch.cuda.Event(), torch.cuda.Event()
        e2e_path = ("C ABI dt_all_reduce per 16 MiB chunk on a multi-process dt_comm, pinned host buffers; H2D, "
                    "collective and D2H of consecutive chunks overlapping")

        def e2e_step():  # noqa: F811 (the chunked variant for the all-reduce)
            ev_start.record(stream)
            h2d_s.wait_event(ev_start)
            d2h_s.wait_event(ev_start)
            for lo, hi in chunks:
                with torch.cuda.stream(h2d_s):
                    x[lo:hi].copy_(h_in[lo:hi], non_blocking=True)
                ev_in.record(h2d_s)
                stream.wait_event(ev_in)
                comm.all_reduce(rank, x.data_ptr() + lo * es, y.data_ptr() + lo * es, hi - lo, code, ar_flags,
                                stream.cuda_stream)
                ev_red.record(stream)
                d2h_s.wait_event(ev_red)
                with torch.cuda.stream(d2h_s):
                    h_out[lo:hi].copy_(y[lo:hi], non_blocking=True)
            ev_end.record(d2h_s)
            stream.wait_event(ev_end)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    e2e_ms = time_steps(e2e_step, args.steps, stream)
    dist.barrier()
    t_max = torch.tensor([e2e_ms], device=dev)
    dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    e2e_ms = float(t_max.item())
    # the host result of the last end-to-end step against the same expected output
    e2e_par = Parity(dtype, tolerance=(ar_flags == capi.DT_ALGO_NVLS))
    e2e_par.compare(raw_np(h_out), want)
    ev2 = torch.tensor([0.0 if e2e_par.ok else 1.0], device=dev, dtype=torch.float64)
    dist.all_reduce(ev2, op=dist.ReduceOp.MAX)
    e2e_ok = ev2.item() == 0.0
    del want
    # NCCL on the same message, for the algorithm table (not the product path)
    nccl_bus = None
    if op in ("all_reduce", "all_gather", "reduce_scatter"):
        a = torch.empty(in_numel, dtype=dtype, device=dev).copy_(x)
        o = torch.empty(out_numel, dtype=dtype, device=dev)

        def nstep():
            if op == "all_reduce":
                dist.all_reduce(a)
            elif op == "reduce_scatter":
                dist.reduce_scatter_tensor(o, a)
            else:
                dist.all_gather_into_tensor(o, a) if len(set(lens)) == 1 else None

        for _ in range(3):
            nstep()
        torch.cuda.synchronize()
        dist.barrier()
        nms = time_steps(nstep, max(5, args.steps // 2), stream)
        t_max = torch.tensor([nms], device=dev)
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        nccl_bus = msg * bus_factor(op, n) / (float(t_max.item()) / 1e3) / 1e9
    bus = msg * bus_factor(op, n) / (ms / 1e3) / 1e9
    e2e_bus = msg * bus_factor(op, n) / (e2e_ms / 1e3) / 1e9
    # free this process's communicator before rank 0 drives every GPU from one process
    del x, y, xp, yp
    torch.cuda.synchronize()
    dist.barrier()
    comm.destroy()
    torch.cuda.synchronize()
    dist.barrier(group=cpu_group)
    api = None
    if rank == 0 and not args.skip_api:
        try:
            api = run_api_leg(op, cfg, n, args.steps, args.warmup)
        except Exception as e:  # reported in the line; the C-ABI figures above stand on their own
            api = {"error": repr(e)[:400]}
    dist.barrier(group=cpu_group)
    if rank == 0:
        line = {
            "metric": "redistribute bus GB/s",
            "value": round(bus * n, 2),
            "unit": "GB/s",
            "n_gpus": n,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": DT_NAME[dtype],
            "data": "synthetic (seeded, BASELINE.json distribution)",
            "config": {"workload": cfg["name"] + f" on {n} GPUs, one rank per GPU, P2P kernels over NVLink",
                       "op": op, "group_ranks": n, "msg_bytes_per_rank": msg,
                       "l2": l2_note, "parallelism": f"group{n}"},
            "bus_gbs_per_rank": round(bus, 2),
            "pct_nvlink_peak": round(bus / NVLINK_NOMINAL_GBS, 4),
            "nccl_bus_gbs_per_rank": None if nccl_bus is None else round(nccl_bus, 2),
            "algorithm": algo,
            "p2p_bus_gbs_per_rank": None if p2p_bus is None else round(p2p_bus, 2),
            "roofline": {"bound": "nvlink", "achieved": round(bus, 1), "peak": NVLINK_NOMINAL_GBS, "unit": "GB/s",
                         "frac": round(bus / NVLINK_NOMINAL_GBS, 4),
                         "traffic": None if nvl_tx is None else int(nvl_tx),
                         "traffic_rx": None if nvl_rx is None else int(nvl_rx),
                         "algorithmic_bytes_per_launch": int(msg * bus_factor(op, n)),
                         "traffic_source": "NVML NVLink data counters (TX / RX payload bytes of rank 0's GPU) around "
                                           "the timed steps, per launch",
                         "peak_source": "NVLink 5 nominal, 900 GB/s per direction per GPU",
                         "frac_of_p2p_ceiling": round(bus / NVLINK_P2P_CEILING_GBS, 4),
                         "p2p_ceiling_source": "store ceiling measured both ways at once on one GPU pair "
                                               "(profiles/nvlink_p2p_ceiling_probe.md)"},
            "parity": {"checked": True, "ok": pv[0].item() == 0.0 and pv[3].item() == 0.0,
                       "bit_exact": pv[1].item() == 0.0, "max_abs_err": float(pv[2].item()), "ranks": n,
                       "rule": par.summary("")["rule"], "p2p_leg_ok": None if p2p_par is None else pv[3].item() == 0.0,
                       "e2e_ok": e2e_ok,
                       "against": "C restatement of the reference's algorithm (oracle/dt_oracle.c), fp32 "
                                  "accumulation in rank order, on every rank's full output"},
            "e2e": {"value": round(e2e_bus * n, 3), "unit": "GB/s", "h2d_bytes_per_step": in_numel * es,
                    "d2h_bytes_per_step": out_numel * es, "ms_per_step": round(e2e_ms, 4),
                    "path": e2e_path, "host_buffers_numa_local": numa_cpus is not None},
            "gpu_launches": launches,
            "device_error": err,
            "clocks": clk.summary(),
            "api": api,
        }
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    api_bad = rank == 0 and isinstance(api, dict) and "parity" in api and not api["parity"]["ok"]
    if pv[0].item() != 0.0 or pv[3].item() != 0.0 or not e2e_ok or api_bad:
        if rank == 0:
            print("parity check failed: the timed collective's output differs from the oracle", file=sys.stderr)
        sys.exit(3)


# ---------------------------------------------------------------------------------------------------------
# C5: message-size sweep (one JSON line per op / dtype / size; not the driver's single-line contract)
# ---------------------------------------------------------------------------------------------------------
def sweep_sizes(lo, hi):
    return [1 << k for k in range(lo, hi + 1)]


def a2a_shape(elems, n):
    """Per-rank (a, n*b) Shard(0)->Shard(1) with a*b*n = elems and 1024-element rows per (row, destination)."""
    b = max(1, min(1024, elems // n))
    a = max(1, elems // (n * b))
    return a, b


def run_sweep_multi(args, rank, world, local_rank):
    import datetime

    import torch.distributed as dist

    from dtorch_b200 import capi

    n = world
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    max_bytes = 1 << args.sweep_hi
    from dtorch_b200.multiprocess import create_rank_comm, setup_nvls

    comm = create_rank_comm(2 * max_bytes + (4 << 20), local_rank)
    base, _ = comm.heap(rank)
    # a side stream made current for the whole sweep: our calls, NCCL's and the CUDA-graph captures
    # (which cannot run on the default stream) all order on it
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    ops = args.sweep_ops.split(",")
    nvls_base = 0
    if "all_reduce" in ops and args.algo != "p2p" and (n >= 4 or args.algo == "nvls"):  # sweep: compare at 4 too
        if setup_nvls(comm, 2 * max_bytes + (4 << 20)):
            nvls_base, _ = comm.nvls_buffer(rank)
    for op in ops:
        for dtype in ([torch.bfloat16, torch.float32] if op in ("all_reduce", "reduce_scatter") else [torch.bfloat16]):
            es = torch.tensor([], dtype=dtype).element_size()
            code = capi.dtype_code(dtype)
            for S in sweep_sizes(args.sweep_lo, args.sweep_hi):
                E = S // es
                if op == "all_reduce":
                    in_n, out_n = E, E
                elif op == "reduce_scatter":
                    E = E // n * n
                    in_n, out_n = E, E // n
                elif op == "all_gather":
                    E = E // n * n
                    in_n, out_n = E // n, E
                else:
                    a, b = a2a_shape(E, n)
                    in_n = out_n = a * n * b
                if in_n == 0 or out_n == 0:
                    continue
                x = heap_tensor(base, 0, in_n, dtype, dev)
                y = heap_tensor(base, max_bytes + (2 << 20), out_n, dtype, dev)
                g = torch.Generator(device=dev).manual_seed(rank)
                x.copy_((torch.rand(in_n, generator=g, device=dev) * 2 - 1).to(dtype))

                def ours():
                    st = stream.cuda_stream
                    if op == "all_reduce":
                        comm.all_reduce(rank, x.data_ptr(), y.data_ptr(), in_n, code, args.sweep_flags, st)
                    elif op == "reduce_scatter":
                        comm.reduce_scatter(rank, x.data_ptr(), y.data_ptr(), out_n, code, args.sweep_flags, st)
                    elif op == "all_gather":
                        comm.all_gather(rank, x.data_ptr(), y.data_ptr(), 1, [in_n] * n, es, st)
                    else:
                        comm.all_to_all(rank, x.data_ptr(), y.data_ptr(), [a, n * b], 0, 1, [a] * n, es, st)

                xa = torch.empty(in_n, dtype=dtype, device=dev).copy_(x)
                ya = torch.empty(out_n, dtype=dtype, device=dev)

                def nccl():
                    if op == "all_reduce":
                        dist.all_reduce(xa)
                    elif op == "reduce_scatter":
                        dist.reduce_scatter_tensor(ya, xa)
                    elif op == "all_gather":
                        dist.all_gather_into_tensor(ya, xa)
                    else:
                        dist.all_to_all_single(ya, xa)

                impls = [("ours", ours)] + ([] if args.sweep_no_nccl else [("nccl", nccl)])
                if op == "all_reduce" and nvls_base and (in_n * es) % 16 == 0:
                    xn = heap_tensor(nvls_base, 0, in_n, dtype, dev)
                    yn = heap_tensor(nvls_base, max_bytes + (2 << 20), out_n, dtype, dev)
                    xn.copy_(x)

                    def ours_nvls():
                        comm.all_reduce(rank, xn.data_ptr(), yn.data_ptr(), in_n, code, capi.DT_ALGO_NVLS,
                                        stream.cuda_stream)

                    impls.append(("nvls", ours_nvls))
                res = {}
                for name, fn in impls:
                    for _ in range(3):
                        fn()
                    torch.cuda.synchronize()
                    dist.barrier()
                    t0 = time.perf_counter()
                    fn()
                    torch.cuda.synchronize()
                    one = time.perf_counter() - t0
                    # every rank must issue the same number of collectives: agree on the max
                    it_t = torch.tensor([int(min(200, max(5, 0.02 / max(one, 1e-6))))], device=dev)
                    dist.all_reduce(it_t, op=dist.ReduceOp.MAX)
                    iters = int(it_t.item())
                    dist.barrier()
                    ms = time_steps(fn, iters, stream)
                    tm = torch.tensor([ms], device=dev)
                    dist.all_reduce(tm, op=dist.ReduceOp.MAX)
                    res[name] = float(tm.item())
                    if args.sweep_graph and name != "nccl":
                        # the same calls captured once into a CUDA graph and replayed: device time without the
                        # host's launch gaps (every rank captures and replays the same sequence)
                        g = torch.cuda.CUDAGraph()
                        dist.barrier()
                        torch.cuda.synchronize()
                        with torch.cuda.graph(g, stream=stream, capture_error_mode="thread_local"):
                            for _ in range(iters):
                                fn()
                        torch.cuda.synchronize()
                        dist.barrier()
                        with torch.cuda.stream(stream):
                            g.replay()
                        torch.cuda.synchronize()
                        dist.barrier()
                        def replay():
                            with torch.cuda.stream(stream):
                                g.replay()

                        gms = time_steps(replay, 1, stream) / iters
                        tm = torch.tensor([gms], device=dev)
                        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
                        res[name + "_graph"] = float(tm.item())
                        del g
                busf = bus_factor(op, n)
                msg = in_n * es if op != "all_gather" else out_n * es
                if rank == 0:
                    nccl_ms = res.get("nccl", float("nan"))
                    line = {"sweep": op, "n_gpus": n, "dtype": DT_NAME[dtype], "bytes": msg,
                            "ours_ms": round(res["ours"], 5), "nccl_ms": round(nccl_ms, 5),
                            "ours_bus_gbs": round(msg * busf / res["ours"] / 1e6, 2),
                            "nccl_bus_gbs": round(msg * busf / nccl_ms / 1e6, 2),
                            "device_error": comm.error(rank)}
                    if "nvls" in res:
                        line["nvls_ms"] = round(res["nvls"], 5)
                        line["nvls_bus_gbs"] = round(msg * busf / res["nvls"] / 1e6, 2)
                    for key in [k for k in res if k.endswith("_graph")]:
                        line[key + "_ms"] = round(res[key], 5)
                        line[key + "_bus_gbs"] = round(msg * busf / res[key] / 1e6, 2)
                    print(json.dumps(line), flush=True)
                del xa, ya
    dist.barrier()
    comm.destroy()
    dist.destroy_process_group()


def run_sweep_single_process(args):
    """All-reduce sweep in the reference's process model: one process drives every visible GPU, one host thread
    per rank, ordinary (torch-allocated) buffers. Per size: the default choice (NCCL at 8 ranks from 256 MiB,
    the rank-order two-shot kernel otherwise), DT_RANK_ORDER (always the two-shot kernel) and DT_ALGO_NCCL,
    timed with CUDA events on every rank's stream, max over ranks; how many of this library's kernels the
    default choice launched (0 = NCCL ran it); and the default result checked against the rank-order one
    with every rank's copy equal."""
    import threading

    from dtorch_b200 import capi

    n = torch.cuda.device_count() if args.gpus <= 1 else args.gpus
    comm = capi.Comm(list(range(n)))
    variants = (("auto", 0), ("rank_order", capi.DT_RANK_ORDER), ("nccl", capi.DT_ALGO_NCCL))
    try:
        for dtype in (torch.bfloat16,):
            es = torch.tensor([], dtype=dtype).element_size()
            code = capi.dtype_code(dtype)
            for S in sweep_sizes(args.sweep_lo, args.sweep_hi):
                count = S // es
                gens = [torch.Generator(device=f"cuda:{r}").manual_seed(r) for r in range(n)]
                xs = [torch.randn(count, device=f"cuda:{r}", generator=gens[r]).to(dtype) for r in range(n)]
                outs = {name: [torch.empty_like(x) for x in xs] for name, _ in variants}
                row = {"sweep": "all_reduce_single_process", "n_gpus": n, "dtype": DT_NAME[dtype], "bytes": S}
                for name, flags in variants:
                    times, launched = [0.0] * n, {}
                    bar = threading.Barrier(n)
                    ys = outs[name]

                    def fn(r):
                        with torch.cuda.device(r):
                            st = torch.cuda.current_stream(r)
                            for _ in range(3):
                                comm.all_reduce(r, xs[r].data_ptr(), ys[r].data_ptr(), count, code, flags, st.cuda_stream)
                            st.synchronize()
                            bar.wait(timeout=300)
                            if r == 0:
                                launched["a"] = capi.launch_count()
                            bar.wait(timeout=300)
                            e0 = torch.cuda.Event(enable_timing=True)
                            e1 = torch.cuda.Event(enable_timing=True)
                            e0.record(st)
                            for _ in range(args.steps):
                                comm.all_reduce(r, xs[r].data_ptr(), ys[r].data_ptr(), count, code, flags, st.cuda_stream)
                            e1.record(st)
                            e1.synchronize()
                            times[r] = e0.elapsed_time(e1) / args.steps
                            bar.wait(timeout=300)
                            if r == 0:
                                launched["b"] = capi.launch_count()

                    ts = [threading.Thread(target=fn, args=(r,)) for r in range(n)]
                    for t in ts:
                        t.start()
                    for t in ts:
                        t.join()
                    ms = max(times)
                    row[f"{name}_ms"] = round(ms, 5)
                    row[f"{name}_bus_gbs"] = round(S * bus_factor("all_reduce", n) / ms / 1e6, 2)
                    row[f"{name}_our_launches_per_call"] = (launched["b"] - launched["a"]) / args.steps / n
                ref = outs["rank_order"][0].float()
                rms = float(ref.pow(2).mean().sqrt())
                ok = all(torch.equal(outs["rank_order"][r].to("cuda:0"), outs["rank_order"][0]) and
                         torch.equal(outs["auto"][r].to("cuda:0"), outs["auto"][0]) for r in range(n))
                ok = ok and bool(torch.allclose(outs["auto"][0].float(), ref, rtol=2e-2, atol=2e-2 * rms))
                row["auto_within_tolerance_of_rank_order"] = ok
                print(json.dumps(row), flush=True)
                del xs, outs
    finally:
        comm.destroy()


def run_sweep_single(args):
    """1 GPU: the same-device kernels for a group of `emul_n` ranks against HBM."""
    from dtorch_b200 import capi

    torch.cuda.set_device(0)
    stream = torch.cuda.Stream(device=0)
    n = 8
    peaks, _ = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    for op in args.sweep_ops.split(","):
        for dtype in ([torch.bfloat16, torch.float32] if op in ("all_reduce", "reduce_scatter") else [torch.bfloat16]):
            es = torch.tensor([], dtype=dtype).element_size()
            code = capi.dtype_code(dtype)
            for S in sweep_sizes(args.sweep_lo, min(args.sweep_hi, 29)):
                E = S // es // n * n
                if E == 0:
                    continue
                if op in ("all_reduce", "reduce_scatter"):
                    ins = [(torch.rand(E, device="cuda:0") * 2 - 1).to(dtype) for _ in range(n)]
                    outs = [torch.empty(E if op == "all_reduce" else E // n, dtype=dtype, device="cuda:0")
                            for _ in range(1 if op == "all_reduce" else n)]
                    hbm_bytes = (n + 1) * E * es
                    msg = E * es
                elif op == "all_gather":
                    ins = [torch.rand(E // n, device="cuda:0").to(dtype) for _ in range(n)]
                    outs = [torch.empty(E, dtype=dtype, device="cuda:0")]
                    hbm_bytes = 2 * E * es
                    msg = E * es
                else:
                    a, b = a2a_shape(E, n)
                    ins = [torch.rand(a * n * b, device="cuda:0").to(dtype) for _ in range(n)]
                    outs = [torch.empty(a * n * b, dtype=dtype, device="cuda:0") for _ in range(n)]
                    hbm_bytes = 2 * n * a * n * b * es
                    msg = a * n * b * es
                ip = [t.data_ptr() for t in ins]
                op_ = [t.data_ptr() for t in outs]

                def fn():
                    st = stream.cuda_stream
                    if op == "all_reduce":
                        capi.local_all_reduce(ip, op_[0], E, code, 0, st)
                    elif op == "reduce_scatter":
                        capi.local_reduce_scatter(ip, op_, E // n, code, 0, st)
                    elif op == "all_gather":
                        capi.local_all_gather(ip, op_[0], 1, [E // n] * n, es, st)
                    else:
                        capi.local_all_to_all(ip, op_, [a, n * b], 0, 1, [a] * n, es, st)

                with torch.cuda.stream(stream):
                    for _ in range(3):
                        fn()
                    ms = time_steps(fn, 20, stream)
                print(json.dumps({"sweep": op, "n_gpus": 1, "group_ranks": n, "dtype": DT_NAME[dtype], "bytes": msg,
                                  "ours_ms": round(ms, 5),
                                  "ours_bus_gbs": round(msg * bus_factor(op, n) / ms / 1e6, 2),
                                  "hbm_gbs": round(hbm_bytes / ms / 1e6, 1),
                                  "hbm_frac": round(hbm_bytes / ms / 1e6 / hbm, 4)}), flush=True)
                del ins, outs


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--op", choices=list(CONFIGS), default="all_reduce")
    p.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline (profiling runs)")
    p.add_argument("--skip-e2e", action="store_true", help="omit the end-to-end leg (profiling runs)")
    p.add_argument("--skip-api", action="store_true", help="N > 1: omit the single-process DTensor API leg")
    p.add_argument("--algo", choices=["auto", "p2p", "nvls"], default="auto",
                   help="all-reduce algorithm at N > 1: auto = NVLS where supported and n >= 6, else P2P two-shot")
    p.add_argument("--sweep", action="store_true", help="C5 message-size sweep, one JSON line per point")
    p.add_argument("--sweep-lo", type=int, default=10, help="smallest size, log2 bytes")
    p.add_argument("--sweep-hi", type=int, default=30, help="largest size, log2 bytes")
    p.add_argument("--sweep-ops", default="all_reduce,all_gather,reduce_scatter,all_to_all")
    p.add_argument("--sweep-no-nccl", action="store_true", help="sweep without the NCCL comparison")
    p.add_argument("--sweep-graph", action="store_true", help="sweep: also time our calls replayed from a CUDA graph")
    p.add_argument("--sweep-single-process", action="store_true",
                   help="all-reduce sweep with one process driving every GPU (default choice, DT_RANK_ORDER, NCCL)")
    p.add_argument("--sweep-flags", type=int, default=0, help="sweep: reduction flags of our all-reduce / reduce-scatter (e.g. 0x20 forces the two-shot kernel)")
    args = p.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.sweep_single_process:
        run_sweep_single_process(args)
    elif args.sweep:
        run_sweep_multi(args, rank, world, local_rank) if world > 1 else run_sweep_single(args)
    elif world > 1:
        run_ours_multi(args, rank, world, local_rank)
    else:
        run_ours_single(args)


if __name__ == "__main__":
    main()
