#!/usr/bin/env python
"""Sampler benchmark: sampled tokens/s at B=4096, V=50257 on 1..8 B200.

Workload (the benchmark's full-vocabulary nucleus stress case): per GPU
B=4096 rows of V=50257 fp32 logits, N(0,1) with a +15 spike in 25% of the
rows and flat N(0, 0.1) in another 25%; knobs top_k=0, top_p=0.95, min_p=0,
temp=1, penalty=1, no history; one uniform per row from the reference
XorShift64* stream.  Synthetic data, generated on the device.  The 823 MB of
logits per step exceed the 126 MB L2, so no flush is needed between steps.

  python bench.py [--gpus N --steps K --warmup W]         this library
  python bench.py --impl reference [...]                 the reference's own
                                                         C sampler on the host
For N > 1 launch one rank per GPU with torch.distributed.run; each rank
samples its own 4096 rows (weak scaling, no collective on the data path).
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "bitmamba.c_b200", "python")]

METRIC = "sampled tokens/s at B=4096,V=50257"
UNIT = "tokens/s"
KNOBS = dict(temp=1.0, penalty=1.0, min_p=0.0, top_p=0.95, top_k=0)
RNG_SEED = 42
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) per row of the c3 workload, from one ncu capture
# of sample_kernel on B = 1024 rows (dram__bytes_read.sum 206.07 MB +
# dram__bytes_write.sum 4.32 MB, profiles/sample_kernel_c3.md); traffic grows
# with the rows processed (each row is read once), so a launch of B rows moves
# about B times this.
DRAM_BYTES_PER_ROW_C3 = (206.067968e6 + 4.322304e6) / 1024


def workload_config(B, V):
    return {
        "workload": "c3 full-vocabulary nucleus stress (B rows/GPU of N(0,1) fp32 logits, "
                    "25% rows +15 spike, 25% rows flat N(0,0.1); top_k=0 top_p=0.95 "
                    "min_p=0 temp=1 penalty=1; no history)",
        "B_per_gpu": B, "V": V,
        "uniforms": f"reference XorShift64* rng_float stream, seed {RNG_SEED}",
        "l2": "inputs (B*V*4 bytes per GPU) larger than the 126 MB L2; no flush",
    }


def make_logits(torch, B, V, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    z = torch.randn(B, V, generator=g, device=device, dtype=torch.float32)
    kind = torch.arange(B, device=device) % 4
    z[kind == 1] *= 0.1
    spike_rows = torch.nonzero(kind == 0).squeeze(1)
    spike_ids = torch.randint(0, V, (spike_rows.numel(),), generator=g, device=device)
    z[spike_rows, spike_ids] += 15.0
    return z.contiguous()


def shard_rows(total, world, rank):
    """Rows [start, start + count) of a global batch of `total` rows owned by
    `rank` (even split, the remainder to the first ranks).  Rows are
    independent, so sharding needs no collective."""
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


def max_over_ranks(dist, x, device=None):
    """The maximum of a per-rank time over all ranks (identity on 1 rank)."""
    if dist is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def ref_uniforms(B, seed=RNG_SEED):
    """rng_float() stream of the reference (src/utils.c:117-140)."""
    s = seed if seed else 0x853C49E6748FEA9B
    m = (1 << 64) - 1
    out = np.empty(B, np.float32)
    for i in range(B):
        s ^= s >> 12
        s ^= (s << 25) & m
        s ^= s >> 27
        v = (s * 0x2545F4914F6CDD1D) & m
        out[i] = np.float32(float(v >> 11)) * np.float32(1.0 / 9007199254740992.0)
    return out


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.t = None
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=5)

    def summary(self):
        rows = self.rows
        if self.window and rows:
            a, b = self.window
            inside = [r for r in rows if a - 0.15 <= r[0] <= b + 0.15]
            rows = inside or [min(rows, key=lambda r: abs(r[0] - (a + b) / 2))]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1][1]) for r in rows if num(r[1][1]) is not None]
        mx = [num(r[1][2]) for r in rows if num(r[1][2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if len(r[1]) > 5 + i and r[1][5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def peak_hbm():
    try:
        d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(d["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured copy, burst)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback 6650 GB/s (pool measurement)"


def oracle_batch(logits_host):
    """The workload rows as an oracle batch (knobs broadcast)."""
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")]
    import synth
    B = logits_host.shape[0]
    return synth.Batch(logits_host, np.zeros(0, np.int32), np.zeros(B + 1, np.int64),
                       np.full(B, KNOBS["temp"], np.float32),
                       np.full(B, KNOBS["penalty"], np.float32),
                       np.full(B, KNOBS["min_p"], np.float32),
                       np.full(B, KNOBS["top_p"], np.float32),
                       np.full(B, KNOBS["top_k"], np.int32))


def cpu_leg(b, u, threads, kind_pref="reference"):
    """Time the reference's C sampler (oracle/_ref, else the oracle port) on
    the rows of synth.Batch b.  Returns (ids, seconds, kind)."""
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")]
    import oracle
    if kind_pref == "reference" and oracle.has_ref():
        t = time.perf_counter()
        ids = oracle.ref_sample_batch_mt(b, u, threads)
        return ids, time.perf_counter() - t, "reference"
    oracle.lib()
    t = time.perf_counter()
    ids, _, _ = oracle.sample_batch(b, u, threads=threads, with_results=False)
    return ids, time.perf_counter() - t, "port"


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    """The reference arm: the reference's own sampler on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    import torch
    B, V = args.B, args.V
    threads = host_threads()
    # the whole B-row workload (the same generator and distribution as the
    # GPU arm's), of which every step samples a bounded share: a different
    # slice of one fixed permutation of the rows per step, sized so warmup +
    # steps stay within about two minutes on this host
    logits = make_logits(torch, B, V, 1234, "cpu").numpy()
    u = ref_uniforms(B)
    perm = np.random.default_rng(RNG_SEED).permutation(B)
    per_row_s = 0.006  # measured scale of the full-sort rows on one core
    budget = 120.0
    rows_per_step = int(max(threads, min(B, budget / (args.steps + args.warmup)
                                         * threads / per_row_s)))
    rows_per_step = max(1, min(B, rows_per_step))
    kind = None

    def step_rows(k):
        return perm[(k * rows_per_step + np.arange(rows_per_step)) % B]

    for w in range(args.warmup):
        sel = step_rows(w)
        _, _, kind = cpu_leg(oracle_batch(np.ascontiguousarray(logits[sel])), u[sel], threads)
    total = 0.0
    for k in range(args.steps):
        sel = step_rows(args.warmup + k)
        _, dt, kind = cpu_leg(oracle_batch(np.ascontiguousarray(logits[sel])), u[sel], threads)
        total += dt
    value = rows_per_step * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(B, V), "impl": "reference",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": kind,
                         "sample": f"{rows_per_step} rows of the {B}-row workload per step "
                                   f"(a different slice of one permutation each step), "
                                   f"row-parallel pthreads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)
    return 0


class Workload:
    """One rank's inputs: device tensors, host copies and the oracle view."""


def slice_batch(b, n):
    """The first n rows of a synth.Batch (CSR histories re-based)."""
    sys.path[:0] = [os.path.join(ROOT, "tests", "golden")]
    import synth
    off = b.hist_off[:n + 1] - b.hist_off[0]
    return synth.Batch(b.logits[:n], b.hist[b.hist_off[0]:b.hist_off[n]], off, b.temp[:n],
                       b.penalty[:n], b.min_p[:n], b.top_p[:n], b.top_k[:n])


def build_workload(args, torch, bm, dev, rank, world):
    """c3 (the benchmark): generated on the device, knobs broadcast, no
    history.  c1, c2, c4: the configs' seeded generators (histories, per-row
    knobs for c4), built on the host and copied once."""
    w = Workload()
    B, V = args.B, args.V
    w.name, w.B, w.V = args.workload, B, V
    start, count = shard_rows(world * B, world, rank)
    # this rank's slice of the global uniform stream
    w.u_host = ref_uniforms(world * B)[start:start + count]
    if args.workload == "c3":
        w.logits = make_logits(torch, B, V, 1234 + rank, dev)
        w.knobs = bm.knobs_array(KNOBS["temp"], KNOBS["penalty"], KNOBS["min_p"],
                                 KNOBS["top_p"], KNOBS["top_k"])
        w.knob_stride = 0
        w.hist_h = w.off_h = None
        w.batch = lambda h, n: oracle_batch(h)
        w.desc = workload_config(B, V)
    else:
        sys.path[:0] = [os.path.join(ROOT, "tests", "golden")]
        import synth
        b = synth.MAKERS[args.workload](1000 + rank, B, V=V)
        w.logits = torch.from_numpy(b.logits).to(dev)
        w.knobs = bm.knobs_array(b.temp, b.penalty, b.min_p, b.top_p, b.top_k)
        w.knob_stride = 1
        w.hist_h, w.off_h = b.hist, b.hist_off
        w.batch = lambda h, n, b=b: slice_batch(b, n)
        w.desc = {"workload": f"{args.workload}: " + CONFIG_DESC[args.workload],
                  "B_per_gpu": B, "V": V, "history_ids": int(b.hist.size),
                  "uniforms": "reference XorShift64* rng_float stream, seed 42",
                  "l2": "inputs larger than the 126 MB L2 when B*V*4 > 126 MB"}
    w.knobs_d = torch.from_numpy(w.knobs.view(np.uint8).copy()).to(dev)
    w.hist_d = torch.from_numpy(w.hist_h).to(dev) if w.hist_h is not None else None
    w.off_d = torch.from_numpy(w.off_h).to(dev) if w.off_h is not None else None
    H = 0 if w.hist_h is None else int(w.hist_h.size)
    w.alg_bytes = (B * (4 * V + 4 + 4) + 4 * H + (8 * (B + 1) if H else 0) +
                   32 * (B if w.knob_stride else 1))
    w.h2d_bytes = B * V * 4 + B * 4 + 4 * H + (8 * (B + 1) if H else 0) + w.knobs.nbytes
    return w


CONFIG_DESC = {
    "c1": "fp32 logits N(0, 2.5^2) with 8 ids +8, 400-id uniform history, "
          "temp 0.8 penalty 1.15 min_p 0.05 top_p 0.9 top_k 40",
    "c2": "fp32 logits 3*Gumbel(0,1), 1024-id Zipf(1.1) history, default knobs",
    "c4": "fp32 logits N(0, 2^2), per-row knobs (temp U[0,1.5] 10% greedy, top_k in "
          "{0,1,40,200}, top_p U[.5,1], min_p U[0,.2], penalty U[1,1.5]), histories "
          "of U[0,2048] ids",
}


def run_ours(args):
    import torch
    import bmsampler as bm

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (no CPU fallback)")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    B, V = args.B, args.V
    dev = torch.device("cuda", local)
    ctx = bm.Context(local)
    # this rank's rows of the global batch (weak scaling: B rows per rank)
    wl = build_workload(args, torch, bm, dev, rank, world)
    logits, knobs, knobs_d, u_host = wl.logits, wl.knobs, wl.knobs_d, wl.u_host
    hist_ptr = wl.hist_d.data_ptr() if wl.hist_d is not None else 0
    off_ptr = wl.off_d.data_ptr() if wl.off_d is not None else 0
    u_d = torch.from_numpy(u_host).to(dev)
    out_d = torch.empty(B, dtype=torch.int32, device=dev)
    # a dedicated stream: torch's legacy default stream has handle 0, which the
    # library reads as "use the context stream"
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)

    def launch():
        ctx.sample_device(logits.data_ptr(), B, V, V, hist_ptr, off_ptr, knobs_d.data_ptr(),
                          wl.knob_stride, u_d.data_ptr(), out_d.data_ptr(), None, None,
                          stream.cuda_stream)

    def barrier():
        if dist is not None:
            dist.barrier()

    # ---- device-resident throughput -------------------------------------
    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize(dev)
    ctx.check()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    t_a = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        launch()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t_b = time.time()
    barrier()
    clocks.window = (t_a, t_b)
    time.sleep(0.25)
    clocks.stop()
    ctx.check()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(dist, ms, dev)
    value = world * B * args.steps / (ms_max / 1e3)
    kernel_ms = ms / args.steps
    alg_bytes = wl.alg_bytes  # logits, histories, uniform, id, knobs
    achieved = alg_bytes / (kernel_ms / 1e3) / 1e9
    peak, peak_src = peak_hbm()
    ids_dev = out_d.cpu().numpy()

    # ---- end to end through the host-buffer API -----------------------------
    e2e = None
    if not args.no_e2e:
        h_logits = logits.cpu().pin_memory()
        h_u = torch.from_numpy(u_host).pin_memory()
        h_ids = torch.empty(B, dtype=torch.int32).pin_memory()
        h_knobs = torch.from_numpy(knobs.view(np.uint8).copy()).pin_memory()
        h_hist = torch.from_numpy(wl.hist_h).pin_memory() if wl.hist_h is not None else None
        h_off = torch.from_numpy(wl.off_h).pin_memory() if wl.off_h is not None else None
        L = bm.lib()
        c = bm.ctypes.c_void_p

        def call():
            bm.check(L.bm_sample_batch_host(ctx.handle, c(h_logits.data_ptr()), B, V, V,
                                            c(h_hist.data_ptr()) if h_hist is not None else None,
                                            c(h_off.data_ptr()) if h_off is not None else None,
                                            c(h_knobs.data_ptr()), wl.knob_stride,
                                            c(h_u.data_ptr()), c(h_ids.data_ptr()), None,
                                            None))
        n_e2e = max(3, min(args.steps, 20))
        for _ in range(min(3, args.warmup)):
            call()
        cs = torch.cuda.ExternalStream(ctx.stream(), device=dev)
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        barrier()
        f0.record(cs)
        for _ in range(n_e2e):
            call()
        f1.record(cs)
        torch.cuda.synchronize(dev)
        barrier()
        e_ms = max_over_ranks(dist, f0.elapsed_time(f1), dev)
        if not np.array_equal(h_ids.numpy(), ids_dev):
            raise SystemExit("e2e ids differ from the device-resident run")
        e2e = {"value": world * B * n_e2e / (e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": B * 4,
               "steps": n_e2e, "ms_per_step": e_ms / n_e2e}

    # ---- CPU baseline on a bounded sample (rank 0, N=1 only) ----------------
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n = min(B, args.cpu_rows)
        threads = host_threads()
        h = logits[:n].cpu().numpy()
        rb = wl.batch(h, n)
        ids_cpu, dt, kind = cpu_leg(rb, u_host[:n], threads)
        cpu = {"value": n / dt, "unit": UNIT, "cores": threads, "kind": kind,
               "sample": f"first {n} rows of the workload, row-parallel pthreads"}
        # the reference's native form: one thread, as model_forward_step calls
        # its sampler once per decode step (src/model.c:1268-1307)
        n1 = min(n, args.cpu_rows_single)
        _, dt1, kind1 = cpu_leg(wl.batch(h[:n1], n1), u_host[:n1], 1)
        cpu["single_thread"] = {"value": n1 / dt1, "unit": UNIT, "cores": 1, "kind": kind1,
                                "sample": f"first {n1} rows of the workload, one thread"}
        same = int((ids_cpu == ids_dev[:n]).sum())
        parity = {"rows": n, "identical_ids": same}
        if same < n:
            # classify the differing rows with the oracle's CDF margins: a row
            # whose draw or cut lies within 1e-5 of a boundary is exempt
            sys.path[:0] = [os.path.join(ROOT, "tests")]
            import oracle
            import parity as parity_rule
            _, _, res = oracle.sample_batch(rb, u_host[:n], threads=threads)
            rep = parity_rule.compare(ids_dev[:n], None, ids_cpu, None, res)
            parity.update({"exempt_mismatch": rep["exempt_mismatch"], "bad": rep["bad"],
                           "rule": "ids identical except draws/cuts within 1e-5 of a CDF "
                                   "boundary"})

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    traffic = DRAM_BYTES_PER_ROW_C3 * B if wl.name == "c3" else None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": wl.desc,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "algorithmic_bytes_per_launch": alg_bytes, "peak_source": peak_src,
                     "kernel": "sample_kernel", "kernel_ms": kernel_ms},
        "cpu_baseline": cpu, "e2e": e2e, "clocks": clocks.summary(),
        "gpu_launches": args.steps, "parity_sample": parity,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_lmhead(args):
    """Configs c5 / c6: the fused decode step for B rows per GPU of
    d_model=2048 hidden states, V=50257, default knobs, 256-id Zipf histories.
    c5: final RMSNorm + bf16 lm_head GEMM on the tensor cores + the sampler.
    c6: the reference's own producer, final RMSNorm + BitLinear RMSNorm +
    int8 quantisation + ternary lm_head (int8 tensor cores, exact int32
    accumulation) + the sampler.  Reports rows/s of the whole step and the
    GEMM's tensor roofline."""
    import torch
    import bmsampler as bm

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (no CPU fallback)")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    sys.path[:0] = [os.path.join(ROOT, "tests", "golden")]
    import synth
    B, V, d = args.B, args.V, args.d_model
    tern = args.workload == "c6"
    dev = torch.device("cuda", local)
    ctx = bm.Context(local)
    g = torch.Generator(device=dev)
    g.manual_seed(4321 + rank)
    hidden = torch.randn(B, d, generator=g, device=dev, dtype=torch.float32)
    norm_w = 1.0 + 0.02 * torch.randn(d, generator=g, device=dev, dtype=torch.float32)
    if tern:
        # c6: the reference's ternary lm_head; 2-bit codes with P(0) = 1/2
        # (a random code 3 becomes 1), decoded to int8 once (weight setup)
        lmh_norm = 1.0 + 0.02 * torch.randn(d, generator=g, device=dev, dtype=torch.float32)
        pk = torch.randint(0, 256, (V, d // 4), generator=g, device=dev, dtype=torch.int32)
        pk = pk & ~((pk & (pk >> 1) & 0x55) << 1)
        packed = pk.to(torch.uint8).contiguous()
        del pk
        w_scale = 16.0
        W = torch.empty((V, d), dtype=torch.int8, device=dev)
        ctx.ternary_unpack(packed.data_ptr(), V, d, W.data_ptr())
        torch.cuda.synchronize(dev)
    else:
        W = (0.02 * torch.randn(V, d, generator=g, device=dev, dtype=torch.float32)).to(
            torch.bfloat16).view(torch.int16).contiguous()
    hists = [synth.ids_zipf(77 + rank, 6000 + r, 256, V) for r in range(B)]
    hist_h = np.concatenate(hists).astype(np.int32)
    off_h = np.arange(0, 256 * (B + 1), 256, dtype=np.int64)
    k = synth.DEFAULT_KNOBS
    knobs = bm.knobs_array(k["temp"], k["penalty"], k["min_p"], k["top_p"], k["top_k"])
    knobs_d = torch.from_numpy(knobs.view(np.uint8).copy()).to(dev)
    hist_d = torch.from_numpy(hist_h).to(dev)
    off_d = torch.from_numpy(off_h).to(dev)
    start, _ = shard_rows(world * B, world, rank)
    u_host = ref_uniforms(world * B)[start:start + B]
    u_d = torch.from_numpy(u_host).to(dev)
    out_d = torch.empty(B, dtype=torch.int32, device=dev)
    ld = (V + 3) // 4 * 4
    logits = torch.empty((B, ld), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)

    def fused():
        if tern:
            ctx.ternary_sample(hidden.data_ptr(), B, d, norm_w.data_ptr(), lmh_norm.data_ptr(),
                               W.data_ptr(), w_scale, V, hist_d.data_ptr(), off_d.data_ptr(),
                               knobs_d.data_ptr(), 0, u_d.data_ptr(), out_d.data_ptr(), None,
                               None, stream.cuda_stream)
        else:
            ctx.lmhead_sample(hidden.data_ptr(), B, d, norm_w.data_ptr(), W.data_ptr(), V,
                              hist_d.data_ptr(), off_d.data_ptr(), knobs_d.data_ptr(), 0,
                              u_d.data_ptr(), out_d.data_ptr(), None, None, stream.cuda_stream)

    def gemm_only():
        if tern:
            ctx.ternary_logits(hidden.data_ptr(), B, d, norm_w.data_ptr(), lmh_norm.data_ptr(),
                               W.data_ptr(), w_scale, V, logits.data_ptr(), ld,
                               stream.cuda_stream)
        else:
            ctx.lmhead_logits(hidden.data_ptr(), B, d, norm_w.data_ptr(), W.data_ptr(), V,
                              logits.data_ptr(), ld, stream.cuda_stream)

    def sampler_only():
        ctx.sample_device(logits.data_ptr(), B, V, ld, hist_d.data_ptr(), off_d.data_ptr(),
                          knobs_d.data_ptr(), 0, u_d.data_ptr(), out_d.data_ptr(), None, None,
                          stream.cuda_stream)

    def timed(fn, steps):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        return max_over_ranks(dist, e0.elapsed_time(e1), dev) / steps

    for fn in (fused, gemm_only, sampler_only):
        for _ in range(args.warmup):
            fn()
    torch.cuda.synchronize(dev)
    ctx.check()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    t_a = time.time()
    ms = timed(fused, args.steps)
    t_b = time.time()
    clocks.window = (t_a, t_b)
    gemm_ms = timed(gemm_only, max(3, args.steps // 2))
    samp_ms = timed(sampler_only, max(3, args.steps // 2))
    time.sleep(0.25)
    clocks.stop()
    ctx.check()
    flops = 2.0 * B * V * d
    tflops = flops / (gemm_ms / 1e3) / 1e12
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    if tern:
        # no int8 figure is measured on this pool: the dense int8 tensor rate
        # of B200 is twice its bf16 rate, so the denominator is twice the
        # measured sustained bf16 figure
        peak = 2.0 * float(peaks.get("bf16_tflops_sustained", 1400.0))
        peak_src = "2 x MEASURED_PEAKS.json bf16_tflops_sustained (int8 dense = 2 x bf16)"
    else:
        peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
        peak_src = "MEASURED_PEAKS.json bf16_tflops_sustained"
    ids_dev = out_d.cpu().numpy()
    fused()
    fb_sampled, fb_computed = ctx.fused_fallback_rows()

    # CPU leg on a bounded sample: the oracle's RMSNorm + float64 product of
    # the same bf16 operands and the sampler oracle on the GPU's own logits
    cpu = parity = None
    if tern and rank == 0 and world == 1 and not args.no_cpu:
        cpu, parity = ternary_cpu_leg(args, hidden, norm_w, lmh_norm, packed, w_scale, logits,
                                      hist_h, off_h, u_host, ids_dev, B, V, d)
    elif rank == 0 and world == 1 and not args.no_cpu:
        sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
        import lmhead_oracle as lo
        import oracle
        import parity as parity_rule
        n = min(B, 16)
        hx = hidden[:n].cpu().numpy()
        wn = norm_w.cpu().numpy()
        wb = W.cpu().numpy().view(np.uint16)
        t0 = time.time()
        ref_logits = lo.lmhead_logits(lo.rmsnorm_bf16(hx, wn), wb)
        dt_gemm = time.time() - t0
        gpu_l = logits[:n, :V].cpu().numpy()
        max_err = float(np.abs(gpu_l - ref_logits).max())
        rb = synth.Batch(gpu_l, hist_h[:256 * n], off_h[:n + 1], np.full(n, k["temp"]),
                         np.full(n, k["penalty"]), np.full(n, k["min_p"]),
                         np.full(n, k["top_p"]), np.full(n, k["top_k"]))
        t0 = time.time()
        rids, _, res = oracle.sample_batch(rb, u_host[:n])
        dt_samp = time.time() - t0
        rep = parity_rule.compare(ids_dev[:n], None, rids, None, res)
        cpu = {"value": n / (dt_gemm + dt_samp), "unit": UNIT, "cores": 1, "kind": "port",
               "sample": f"first {n} rows: numpy RMSNorm + float64 GEMM of the bf16 operands, "
                         f"then the sampler oracle"}
        parity = {"rows": n, "identical_ids": rep["exact"], "bad": rep["bad"],
                  "max_abs_logit_err_vs_float64": max_err}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    if tern:
        metric = "sampled tokens/s, final RMSNorm + ternary BitLinear lm_head + sampler (c6)"
        dtype = "int8 x ternary GEMM (exact int32 accumulate), f32 sampler"
        workload = ("c6 reference lm_head + sampler: hidden N(0,1), final-norm and "
                    "BitLinear-norm weights 1+N(0,.02), ternary W [V x d] (P(0)=1/2, scale "
                    "16) decoded to int8 once, default knobs, 256-id Zipf histories")
        l2 = "W (103 MB int8) and the logits (B*V*4 bytes) exceed the 126 MB L2 together"
        kern = "gemm_kernel<int8> (+ternary_prep)"
        unit_t = "TOP/s"
    else:
        metric = "sampled tokens/s, fused RMSNorm + bf16 lm_head + sampler (c5)"
        dtype = "bf16 GEMM (fp32 accumulate), f32 sampler"
        workload = ("c5 fused lm_head + sampler: hidden N(0,1), RMSNorm weight "
                    "1+N(0,.02), W [V x d] N(0,.02) bf16, default knobs, 256-id "
                    "Zipf histories")
        l2 = "W (206 MB) and the logits (B*V*4 bytes) exceed the 126 MB L2"
        kern = "gemm_kernel (+rmsnorm)"
        unit_t = "TFLOP/s"
    line = {
        "metric": metric,
        "value": world * B / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": dtype,
        "data": "synthetic",
        "config": {"workload": workload, "B_per_gpu": B, "V": V, "d_model": d, "l2": l2},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": unit_t,
                     "frac": tflops / peak, "traffic": None, "kernel": kern,
                     "kernel_ms": gemm_ms, "flops_per_launch": flops,
                     "peak_source": peak_src},
        "parts_ms": {"norm_plus_gemm": gemm_ms, "sampler": samp_ms, "fused_step": ms},
        "fused_rows_from_logits": {"sampled": fb_sampled, "recomputed": fb_computed,
                                   "note": "rows the per-tile lists could not decide (the "
                                           "rest never had logits in HBM)"},
        "cpu_baseline": cpu, "e2e": None, "clocks": clocks.summary(),
        # per fused step: RMSNorm (or the ternary prep), history bits, the
        # summary GEMM, the merge, the fallback gather, the fallback GEMM and
        # the fallback sampler (the last three find empty row lists and return)
        "gpu_launches": 7 * args.steps, "parity_sample": parity,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_decode(args):
    """Config c7: the device-resident decode loop (bm_decode_ternary_step):
    B rows per GPU, K steps per timed iteration, each step the reference's
    final RMSNorm + ternary lm_head + sampler with the 256-id history windows,
    then the loop state update (push, stop checks) on the GPU.  The hidden
    state is held fixed (the model's layers are out of scope), so each step
    differs only through the windows.  Reported against the same steps with a
    host round trip per step (ids copied to the host and the stream
    synchronised), which a host-side loop needs."""
    import torch
    import bmsampler as bm

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (no CPU fallback)")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    sys.path[:0] = [os.path.join(ROOT, "tests", "golden")]
    import synth
    B, V, d, K = args.B, args.V, args.d_model, args.decode_steps
    dev = torch.device("cuda", local)
    ctx = bm.Context(local)
    g = torch.Generator(device=dev)
    g.manual_seed(777 + rank)
    hidden = torch.randn(B, d, generator=g, device=dev, dtype=torch.float32)
    nf = 1.0 + 0.02 * torch.randn(d, generator=g, device=dev, dtype=torch.float32)
    nl = 1.0 + 0.02 * torch.randn(d, generator=g, device=dev, dtype=torch.float32)
    pk = torch.randint(0, 256, (V, d // 4), generator=g, device=dev, dtype=torch.int32)
    packed = (pk & ~((pk & (pk >> 1) & 0x55) << 1)).to(torch.uint8).contiguous()
    del pk
    W = torch.empty((V, d), dtype=torch.int8, device=dev)
    ctx.ternary_unpack(packed.data_ptr(), V, d, W.data_ptr())
    k = synth.DEFAULT_KNOBS
    knobs = bm.knobs_array(k["temp"], k["penalty"], k["min_p"], k["top_p"], k["top_k"])
    knobs_d = torch.from_numpy(knobs.view(np.uint8).copy()).to(dev)
    steps_total = (args.warmup + args.steps) * K
    u_d = torch.rand(steps_total * B, generator=g, device=dev, dtype=torch.float32)
    ids_d = torch.empty(B, dtype=torch.int32, device=dev)
    ids_h = torch.empty(B, dtype=torch.int32).pin_memory()
    prompts = [synth.ids_zipf(31 + rank, 7000 + r, 64, V) for r in range(B)]
    dec = bm.Decode(ctx, B, max_tokens=0, stop_ids=[])
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize(dev)
    st = [0]

    def step(host_round_trip):
        u = u_d[st[0] * B:(st[0] + 1) * B]
        st[0] += 1
        dec.ternary_step(hidden.data_ptr(), d, nf.data_ptr(), nl.data_ptr(), W.data_ptr(), 16.0,
                         V, knobs_d.data_ptr(), 0, u.data_ptr(), ids_d.data_ptr(),
                         stream.cuda_stream)
        if host_round_trip:
            with torch.cuda.stream(stream):
                ids_h.copy_(ids_d, non_blocking=True)
            stream.synchronize()

    def run(host_round_trip, iters):
        dec.reset(prompts)
        st[0] = 0
        for _ in range(args.warmup * K):
            step(host_round_trip)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters * K):
            step(host_round_trip)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        return max_over_ranks(dist, e0.elapsed_time(e1), dev) / (iters * K)

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    t_a = time.time()
    ms = run(False, args.steps)
    t_b = time.time()
    clocks.window = (t_a, t_b)
    ms_rt = run(True, args.steps)
    time.sleep(0.25)
    clocks.stop()
    ctx.check()
    active = dec.active()
    dec.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": "sampled tokens/s, device-resident decode loop (c7: ternary lm_head + "
                  "sampler + history / stop state per step)",
        "value": world * B / (ms / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 x ternary GEMM (exact int32), f32 sampler",
        "data": "synthetic",
        "config": {"workload": "c7 decode loop: c6 inputs held fixed, 64-id Zipf prompts, "
                               "default knobs, no stop tokens", "B_per_gpu": B, "V": V,
                   "d_model": d, "decode_steps_per_iteration": K},
        "host_round_trip": {"ms_per_step": ms_rt, "tokens_per_s": world * B / (ms_rt / 1e3),
                            "note": "the same steps with the ids copied to pinned host memory "
                                    "and the stream synchronised after each step"},
        "rows_active_at_end": active, "cpu_baseline": None, "e2e": None,
        "clocks": clocks.summary(), "gpu_launches": 4 * K * args.steps,
    }
    print(json.dumps(line), flush=True)
    return 0


def ternary_cpu_leg(args, hidden, norm_f, lmh_norm, packed, w_scale, logits, hist_h, off_h,
                    u_host, ids_dev, B, V, d):
    """c6's CPU leg on a bounded sample: the reference's own final RMSNorm +
    ternary lm_head (oracle/_ref, its AVX2 kernels, its thread pool over all
    host cores) and the sampler oracle on the GPU's logits; parity of the
    logits is bit for bit."""
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    import oracle
    import parity as parity_rule
    import synth
    import ternary
    if not oracle.has_ref():
        return None, None
    k = synth.DEFAULT_KNOBS
    n = min(B, 64)
    hx = hidden[:n].cpu().numpy()
    nf = norm_f.cpu().numpy()
    nl = lmh_norm.cpu().numpy()
    pk = packed.cpu().numpy()
    cores = os.cpu_count() or 1
    ternary.ref_logits(hx[:1], nf, nl, pk, w_scale, threads=cores)   # pool start-up
    t0 = time.time()
    ref_l, ks = ternary.ref_logits(hx, nf, nl, pk, w_scale, threads=cores)
    dt = time.time() - t0
    gpu_l = np.ascontiguousarray(logits[:n, :V].cpu().numpy())
    diff = int((gpu_l.view(np.uint32) != ref_l.view(np.uint32)).sum())
    rb = synth.Batch(gpu_l, hist_h[:256 * n], off_h[:n + 1], np.full(n, k["temp"]),
                     np.full(n, k["penalty"]), np.full(n, k["min_p"]),
                     np.full(n, k["top_p"]), np.full(n, k["top_k"]))
    rids, _, res = oracle.sample_batch(rb, u_host[:n])
    rep = parity_rule.compare(ids_dev[:n], None, rids, None, res)
    cpu = {"value": n / dt, "unit": UNIT, "cores": cores, "kind": "reference",
           "sample": f"first {n} rows: the reference's final RMSNorm + ternary lm_head "
                     f"({ks} kernels, {cores} threads), logits only"}
    par = {"rows": n, "logits_bit_identical_to_reference": diff == 0,
           "logits_differing": diff, "identical_ids": rep["exact"], "bad": rep["bad"]}
    return cpu, par


def run_row_latency(args):
    """c1 as the reference's decode loop calls its sampler: one row per step
    through bm_sample_row, the drop-in for the tail of model_forward_step
    (src/model.c:1268-1307): host logits and history, the global XorShift64*
    stream, the id returned.  Each call is synchronous and includes its
    host-to-device and device-to-host copies, so it is timed on the host
    clock (time.perf_counter around the ctypes call).  Beside it the
    reference's own sampler (oracle/_ref, else the oracle port) runs on one
    host thread over the same rows and uniforms, as the reference's CLI runs
    it; the ids of the two are compared."""
    import torch  # noqa: F401  (the library makes its own context on device 0)
    import bmsampler as bm
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")]
    import synth
    V, n = args.V, 256
    b = synth.MAKERS["c1"](1000, n, V=V)
    rows = [np.ascontiguousarray(b.logits[r]) for r in range(n)]
    hists = [np.ascontiguousarray(b.hist[b.hist_off[r]:b.hist_off[r + 1]]) for r in range(n)]
    knobs = [(float(b.penalty[r]), float(b.temp[r]), float(b.min_p[r]), float(b.top_p[r]),
              int(b.top_k[r])) for r in range(n)]

    def call(r):
        return bm.sample_row(rows[r], hists[r], *knobs[r])

    for w in range(args.warmup):
        call(w % n)
    steps = args.steps
    bm.rng_seed(RNG_SEED)
    ids = np.empty(steps, np.int32)
    lat = np.empty(steps)
    for s in range(steps):
        t = time.perf_counter()
        ids[s] = call(s % n)
        lat[s] = time.perf_counter() - t
    # the uniforms those calls drew (every c1 row draws: temp 0.8)
    bm.rng_seed(RNG_SEED)
    u = np.array([bm.rng_float() for _ in range(n)], np.float32)
    best = None
    for _ in range(3):
        ref_ids, dt, kind = cpu_leg(b, u, 1)
        best = dt if best is None else min(best, dt)
    m = min(n, steps)
    same = int((ref_ids[:m] == ids[:m]).sum())
    line = {
        "metric": "bm_sample_row latency, one row per call (c1 row, host buffers)",
        "value": float(np.median(lat) * 1e6), "unit": "us", "n_gpus": 1, "steps": steps,
        "warmup": args.warmup, "higher_is_better": False, "dtype": "f32",
        "data": "synthetic", "p99_us": float(np.percentile(lat, 99) * 1e6),
        "mean_us": float(lat.mean() * 1e6),
        "config": {"workload": "c1row: " + CONFIG_DESC["c1"] + "; one row per call through "
                               "bm_sample_row, rows cycled from a pool of 256",
                   "V": V, "history_ids": 400},
        "cpu_baseline": {"value": best / n * 1e6, "unit": "us per row", "cores": 1,
                         "kind": kind, "sample": f"the pool's {n} rows, best of 3 passes"},
        "identical_ids": f"{same}/{m}",
        "gpu_launches": steps,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--B", type=int, default=4096)
    ap.add_argument("--V", type=int, default=50257)
    ap.add_argument("--cpu-rows", type=int, default=2048)
    ap.add_argument("--cpu-rows-single", type=int, default=256)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload",
                    choices=["c1", "c2", "c3", "c4", "c5", "c6", "c7", "c1row"],
                    default="c3",
                    help="c3 is the benchmark; the others report the other configs "
                         "(c5: the fused bf16 lm_head + sampler step; c6: the reference's "
                         "ternary lm_head + sampler; c7: the device-resident decode "
                         "loop; c1row: per-call latency of bm_sample_row on one c1 row "
                         "beside the reference's sampler on one thread)")
    ap.add_argument("--d-model", type=int, default=2048)
    ap.add_argument("--decode-steps", type=int, default=16,
                    help="c7: decode steps per timed iteration")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload in ("c5", "c6"):
        return run_lmhead(args)
    if args.workload == "c7":
        return run_decode(args)
    if args.workload == "c1row":
        return run_row_latency(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
