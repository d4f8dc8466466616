"""Benchmark of the batched sampler: sampled rows/s and HBM GB/s against the measured peak.

Workload (the metric point): B=256 rows per GPU, V=151,936, float32 logits with config 3's
distribution (Gumbel background + Zipf-ranked head) and parameters (T 0.7, top-p 0.95,
min-p 0.05, repetition 1.1, frequency 0.3, presence 0.2, 2,048-id histories), seeded per rank.
A step is one ``lss_sample`` over the batch (K1 streaming pass, K2 per-row history pairs and
resolve, K3 deferred rows), replayed as one CUDA graph.  With N GPUs (one process per GPU) each
rank samples its own rows and every step ends with the row mode's exchange, one NCCL
all-gather of the int32 token ids, inside the timed region; the time is the maximum over
ranks.  By default every rank has its own 256 rows (weak scaling); ``--strong`` splits the
one 256-row batch over the ranks instead.  ``--workload`` selects another configuration:
configs 1-4 in the same row mode (config 4 always splits its 1,024 rows over the ranks),
config 5 vocabulary-sharded (shard records, one all-gather, merge and draw on every rank).

``--impl reference`` times the reference's CPU implementation of the same path (the
``oracle.torch_port`` restatement of ``sample_next_token``, per-row loop, all host threads)
on a bounded sample of the same rows per step, and reports the measured time of those steps.

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sampled rows/s & HBM GB/s vs peak at B=256 V=151936; 1/2/4/8 GPU"
B_PER_GPU = 256
V = 151_936
L2_BYTES = 126e6
TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
DT_CODE = {"f32": 0, "bf16": 1, "f16": 2}
WORKLOADS = ("headline", "cfg1", "cfg2", "cfg3", "cfg4", "cfg5", "greedy")
DESC = {
    "headline": "headline: B=256 rows/GPU, V=151936 f32 logits, T0.7 p0.95 mp0.05 rep1.1 freq0.3 pres0.2, H=2048",
    "cfg1": "config 1: B=8 rows/GPU, V=151936 f32, 2 greedy + 6 T0.8/k50/p0.9",
    "cfg2": "config 2: B=64 rows/GPU, V=151936 bf16, per-row T/k/p/min-p, rep1.1, H=512",
    "cfg3": "config 3: B=256 rows/GPU, V=128256 f32, T0.7 p0.95 mp0.05 rep1.1 freq0.3 pres0.2, H=2048",
    "cfg4": "config 4: B=1024 rows split over the GPUs, V=151936 bf16, every feature on",
    "cfg5": "config 5: B=128, V=256000 f32 split by columns over the GPUs, T1.0 top-k 64 (records) p0.9",
    "greedy": "greedy seam: B=256 rows/GPU, V=151936 f32 logits (headline rows), argmax of every row",
}


def n_buffers(buf_bytes: float) -> int:
    """Rotating input buffers: enough that one pass over them exceeds twice the L2, so every
    step reads its logits from HBM."""
    return int(min(64, max(4, -(-2 * L2_BYTES // buf_bytes))))


def algorithmic_bytes(w) -> int:
    """Bytes one call must move: logits once, history ids and offsets, params, uniform, token."""
    esize = 4 if w.dtype == "f32" else 2
    return int(w.B * w.V * esize + w.hist_ids.size * 4 + (w.B + 1) * 4 + w.B * (7 * 4 + 4 + 4))


def measured_traffic(key: str, scale: float = 1.0):
    """DRAM bytes (read + write) per launch of a kernel, from one ncu capture recorded in
    profiles/traffic.json, scaled by this launch's units (rows or shard columns) over the
    captured launch's; None when no capture is recorded."""
    tp = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        rec = json.load(open(tp)).get(key)
    except (OSError, ValueError):
        return None
    return None if rec is None else int(round(rec["bytes_per_launch"] * scale))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock and throttle-reason samples taken while the timed region runs: NVML polled every
    2 ms from a thread (``nvidia-smi -lms 100`` when NVML is unavailable)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.thread = None
        self.nv = None
        self.handle = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = None
            try:  # the NVML device of this CUDA device, by PCI bus
                prop = torch.cuda.get_device_properties(gpu_index)
                bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
                h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = nv.nvmlDeviceGetHandleByIndex(gpu_index)
            self.nv, self.handle = nv, h
        except Exception:
            self.nv = None

    def _poll(self):
        nv, h = self.nv, self.handle
        bits = {"hw_slowdown": nv.nvmlClocksThrottleReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksThrottleReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksThrottleReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksThrottleReasonSwPowerCap}
        while not self.stop_flag:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.samples.append((float(sm), float(mx), {n for n, b in bits.items() if r & b}))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.nv is not None:
            import threading
            self.samples, self.stop_flag = [], False
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict:
        sm, mx, reasons = [], [], set()
        if self.thread is not None:
            self.stop_flag = True
            self.thread.join()
            for a, b, r in self.samples:
                sm.append(a)
                mx.append(b)
                reasons |= r
            src = "nvml, 2 ms"
        elif self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for line in out.strip().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    mx.append(float(f[2]))
                except ValueError:
                    continue
                for n, v in zip(self.NAMES, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
            src = "nvidia-smi, 100 ms"
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source"]}
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": src}


def cpu_reference_rate(w, seconds: float = 12.0, min_rows: int = 8):
    """Rows/s of the reference's per-row CPU sampler on this host (bounded sample)."""
    from oracle import torch_port as TP
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(0)
    TP.sample_workload_rows(w, [0], gen)  # warm-up
    t0 = time.perf_counter()
    n = 0
    while n < min_rows or (time.perf_counter() - t0 < seconds and n < w.B):
        TP.sample_workload_rows(w, [n % w.B], gen)
        n += 1
    dt = time.perf_counter() - t0
    return n / dt, threads, n, dt


def _row_block(w, start: int, stop: int):
    """Rows [start, stop) of a workload, histories re-based."""
    import copy
    b = copy.copy(w)
    o = w.hist_offsets
    b.logits = w.logits[start:stop]
    for f in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty", "frequency_penalty",
              "presence_penalty", "uniforms"):
        setattr(b, f, getattr(w, f)[start:stop])
    b.hist_ids = w.hist_ids[o[start]:o[stop]]
    b.hist_offsets = (o[start:stop + 1] - o[start]).astype(np.int32)
    return b


def is_strong(args) -> bool:
    return args.workload == "cfg4" or (args.workload == "headline" and args.strong)


def make_workload(rank: int, world: int = 1, name: str = "headline", strong: bool = False):
    """The rank's rows of a row-mode workload; config 4's 1,024 rows (and with ``strong`` the
    headline's 256) are split over the ranks (strong scaling), every other workload gives each
    rank its own batch (weak scaling)."""
    from localstrm_b200 import workloads as wl
    from localstrm_b200.distributed import shard_rows
    if name == "headline":
        if strong:
            full = wl.headline(seed=0, B=B_PER_GPU, V=V)
            a, b = shard_rows(full.B, world, rank)
            return _row_block(full, a, b)
        return wl.headline(seed=rank, B=B_PER_GPU, V=V)
    if name == "greedy":
        w = wl.headline(seed=rank, B=B_PER_GPU, V=V)
        w.temperature[:] = 0.0
        return w
    if name == "cfg4":
        full = wl.config4(seed=0)
        a, b = shard_rows(full.B, world, rank)
        return _row_block(full, a, b)
    return {"cfg1": wl.config1, "cfg2": wl.config2, "cfg3": wl.config3}[name](seed=rank)


def row_config(args, w, world: int) -> dict:
    """The ``config`` of a row-mode line (both arms print the same one)."""
    esize = 4 if w.dtype == "f32" else 2
    buf = w.B * w.V * esize
    desc = DESC[args.workload]
    if is_strong(args) and args.workload == "headline":
        desc = desc.replace("B=256 rows/GPU", "B=256 rows split over the GPUs")
    return {"workload": desc,
            "global_batch": w.B * world if not is_strong(args) else
            {"cfg4": 1024, "headline": B_PER_GPU}[args.workload],
            "rows_per_gpu": w.B, "vocab": w.V,
            "parallelism": f"rows{world}" if world > 1 else "single",
            "l2": f"{n_buffers(buf)} rotating input buffers of {buf / 1e6:.1f} MB (together > 2 x 126 MB L2)",
            "inner_reps": max(1, args.inner)}


def vocab_config(args, w, world: int) -> dict:
    from localstrm_b200.distributed import shard_vocab
    off, end = shard_vocab(w.V, world, 0)
    buf = w.B * (end - off) * 4
    return {"workload": DESC["cfg5"], "global_batch": w.B, "vocab": w.V, "vocab_per_gpu": end - off,
            "parallelism": f"vocab{world}",
            "l2": f"{n_buffers(buf)} rotating shard buffers of {buf / 1e6:.1f} MB (together > 2 x 126 MB L2)"}


def run_reference(args, rank: int, world: int):
    """The reference's per-row CPU path on rank 0's rows: each step samples a bounded number
    of rows (sized from the warm-up so that the timed steps take about ``--ref-seconds``);
    ``ms_per_step`` is the measured time of those steps."""
    if rank != 0:
        return
    from oracle import torch_port as TP
    if args.workload == "cfg5":
        w = _cfg5_full()
        config = vocab_config(args, w, world)
    else:
        w = make_workload(0, world, args.workload, is_strong(args))
        config = row_config(args, w, world)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    gen = torch.Generator().manual_seed(0)
    nxt = 0

    def sample(n):
        nonlocal nxt
        t0 = time.perf_counter()
        for _ in range(n):
            TP.sample_workload_rows(w, [nxt % w.B], gen)
            nxt += 1
        return time.perf_counter() - t0

    per_row = []
    for _ in range(args.warmup):
        per_row.append(sample(2) / 2)
    t_row = statistics.median(per_row)
    rows_per_step = int(max(1, min(w.B, round(args.ref_seconds / max(args.steps, 1) / t_row))))
    step_s = [sample(rows_per_step) for _ in range(args.steps)]
    total = sum(step_s)
    value = rows_per_step * args.steps / total
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / args.steps, "higher_is_better": True,
        "scaling": "strong" if (is_strong(args) or args.workload == "cfg5") else "weak",
        "vs_baseline": None, "dtype": w.dtype, "data": "synthetic (seeded)", "config": config,
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": cores, "kind": "port",
                         "sample": f"{rows_per_step} rows of rank 0's batch per step ({args.steps} steps, "
                                   f"{total:.1f} s): per-row sample_next_token restated in torch CPU ops "
                                   "(oracle/torch_port.py), all host threads"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch.distributed as dist
    from localstrm_b200 import _lib
    from localstrm_b200.sampling import BatchSampler, RowParams

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    w = make_workload(rank, world, args.workload, is_strong(args))
    B = w.B
    DTC = DT_CODE[w.dtype]
    logits_host = torch.from_numpy(w.logits).to(TORCH_DT[w.dtype]).pin_memory()
    NBUF = n_buffers(logits_host.numel() * logits_host.element_size())
    bufs = [logits_host.to(dev) for _ in range(NBUF)]
    prm = RowParams.from_arrays(dev, temperature=w.temperature, top_k=w.top_k, top_p=w.top_p,
                                min_p=w.min_p, repetition_penalty=w.repetition_penalty,
                                frequency_penalty=w.frequency_penalty, presence_penalty=w.presence_penalty)
    h_off = torch.from_numpy(w.hist_offsets.astype(np.int32)).to(dev)
    h_ids = torch.from_numpy(w.hist_ids.astype(np.int32)).to(dev)
    H = int(h_ids.numel())
    uni = torch.from_numpy(w.uniforms).to(dev)
    tokens = torch.empty(B, dtype=torch.int32, device=dev)
    gathered = torch.empty(B * world, dtype=torch.int32, device=dev)
    s = BatchSampler(dev)
    ws = s.workspace(B, w.V, H)
    stream = torch.cuda.current_stream(dev)
    P = lambda t: t.data_ptr()

    def prepare(sp):
        _lib.check("lss_sample_prepare", lib.lss_sample_prepare(
            B, w.V, P(prm.temperature), P(prm.top_k), P(prm.min_p), P(prm.repetition_penalty),
            P(prm.frequency_penalty), P(prm.presence_penalty), P(h_off), P(h_ids), H, P(ws),
            ws.numel(), sp))

    def rows(x, sp, scan_only=False):
        args_ = (P(x), DTC, B, w.V, x.stride(0), P(prm.temperature), P(prm.top_k), P(prm.top_p),
                 P(prm.min_p), P(prm.repetition_penalty), P(prm.frequency_penalty),
                 P(prm.presence_penalty), P(h_off), P(h_ids), H, P(uni), P(tokens))
        if scan_only:
            _lib.check("lss_scan_pass", lib.lss_scan_pass(*args_, P(ws), ws.numel(), sp))
        else:
            _lib.check("lss_sample_rows", lib.lss_sample_rows(*args_, None, None, P(ws), ws.numel(), sp))

    def gather():
        # The row mode's exchange step (RowShardSampler): every rank's token ids to every
        # rank, one NCCL all-gather of B int32 per rank on the step's stream.
        if world > 1:
            dist.all_gather_into_tensor(gathered, tokens)

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (also configures the kernels before capture)
    for i in range(args.warmup):
        prepare(stream.cuda_stream)
        rows(bufs[i % NBUF], stream.cuda_stream)
        gather()
    torch.cuda.synchronize()

    # One CUDA graph per input buffer: a step (prepare + rows: three kernels chained by
    # programmatic dependent launch) is one graph launch, as a decode loop would replay it.
    graphs, scan_graphs = [], []
    for i in range(NBUF):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            sp_cap = torch.cuda.current_stream().cuda_stream
            prepare(sp_cap)
            rows(bufs[i], sp_cap)
        graphs.append(g)
        gs = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gs):
            rows(bufs[i], torch.cuda.current_stream().cuda_stream, scan_only=True)
        scan_graphs.append(gs)
    for g in graphs:
        g.replay()
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    # The timed steps run back to back, as a decode loop replays them: two events bracket the
    # whole run, none sits between the steps.
    reps = max(1, args.inner)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        for r in range(reps):
            graphs[(i * reps + r) % NBUF].replay()
            gather()
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    clk = clocks.stop()
    # Per-step durations (for the median only): a second pass with events around each step.
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    for i in range(args.steps):
        ev[i][0].record(stream)
        graphs[i % NBUF].replay()
        ev[i][1].record(stream)
        gather()
    torch.cuda.synchronize()
    step_ms_each = [e[0].elapsed_time(e[1]) for e in ev]
    n_steps_total = args.steps * reps
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / n_steps_total
    value = B * world * n_steps_total / (elapsed_ms / 1000.0)

    # The streaming pass (K1) alone, timed with events around each replay of its graph.
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.steps):
        kev[i][0].record(stream)
        scan_graphs[i % NBUF].replay()
        kev[i][1].record(stream)
    torch.cuda.synchronize()
    kern_ms = [e[0].elapsed_time(e[1]) for e in kev]
    # Re-run the full step once so the row paths and flags read below are this workload's.
    graphs[0].replay()
    torch.cuda.synchronize()

    # roofline of the dominant kernel (the streaming pass, lss_stream_kernel)
    alg = algorithmic_bytes(w)
    kern_avg_ms = statistics.mean(kern_ms)
    achieved = alg / (kern_avg_ms / 1000.0) / 1e9
    peak, peak_kind = peaks()
    traffic = None
    if args.workload == "headline":
        traffic = measured_traffic("lss_stream_kernel_headline", w.B / B_PER_GPU)
    elif args.workload == "cfg4":
        traffic = measured_traffic("lss_stream_kernel_cfg4", w.B / 1024)

    # end to end through the public API with host buffers (pinned), copies inside the timing
    e2e = None
    if args.e2e_steps > 0:
        from localstrm_b200.sampling import sample_batch  # noqa: F401  (public API module)
        host_u = torch.from_numpy(w.uniforms).pin_memory()
        host_off = torch.from_numpy(w.hist_offsets.astype(np.int32)).pin_memory()
        host_ids = torch.from_numpy(w.hist_ids.astype(np.int32)).pin_memory()
        host_prm = {k: torch.from_numpy(np.asarray(getattr(w, k))).pin_memory()
                    for k in ("temperature", "top_k", "top_p", "min_p", "repetition_penalty",
                              "frequency_penalty", "presence_penalty")}
        dev_x = torch.empty_like(bufs[0])
        tok_host = torch.empty(B, dtype=torch.int32).pin_memory()
        h2d = logits_host.numel() * logits_host.element_size() + host_u.numel() * 4 + host_off.numel() * 4 + \
            host_ids.numel() * 4 + sum(t.numel() * 4 for t in host_prm.values())
        d2h = B * 4

        def e2e_step():
            dev_x.copy_(logits_host, non_blocking=True)
            for k, t in host_prm.items():
                getattr(prm, k).copy_(t, non_blocking=True)
            h_off.copy_(host_off, non_blocking=True)
            h_ids.copy_(host_ids, non_blocking=True)
            uni.copy_(host_u, non_blocking=True)
            s.sample(dev_x, prm, h_off, h_ids, uni, tokens_out=tokens)
            tok_host[:B].copy_(tokens, non_blocking=True)  # each rank reads back its own rows

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        a1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = a0.elapsed_time(a1)
        if world > 1:
            t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": B * world * args.e2e_steps / (e2e_ms / 1000.0), "unit": "rows/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "ms_per_step": e2e_ms / args.e2e_steps}

    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        rate, cores, n, dt = cpu_reference_rate(w, seconds=args.cpu_seconds)
        cpu = {"value": rate, "unit": "rows/s", "cores": cores, "kind": "port",
               "sample": f"{n} rows of the same workload (~{dt:.1f} s): per-row sample_next_token "
                         f"restated in torch CPU ops (oracle/torch_port.py)"}

    paths = s.row_paths(B)
    flags = s.status()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong" if is_strong(args) else "weak",
            "vs_baseline": None, "dtype": w.dtype,
            "data": "synthetic (seeded; " + ("config 3 distribution at V=151,936)" if args.workload == "headline"
                                             else f"{args.workload})"),
            "config": row_config(args, w, world),
            "exchange": "NCCL all-gather of the token ids after every step, inside the timed region"
                        if world > 1 else None,
            "hbm_gbs": alg * world * n_steps_total / (elapsed_ms / 1000.0) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": "lss_stream_kernel", "peak_source": peak_kind,
                         "algorithmic_bytes_per_launch": alg, "kernel_ms": kern_avg_ms},
            "step_ms_median": statistics.median(step_ms_each),
            "clocks": clk, "e2e": e2e, "cpu_baseline": cpu,
            "gpu_launches": 3 * n_steps_total,
            "row_paths": {str(k): int((paths == k).sum()) for k in np.unique(paths)},
            "device_flags": flags,
        }
        print(json.dumps(line), flush=True)


def _cfg5_full():
    from localstrm_b200 import workloads as wl
    return wl.config5(seed=0)


def run_vocab(args, rank: int, world: int, local_rank: int):
    """Config 5, vocabulary-sharded: every rank holds a column block of all 128 rows; a step is
    the shard records (lss_shard_topk), one all-gather of the records, and the merge and draw
    (lss_shard_merge) on every rank.  Timed eagerly with events (the collective is not captured)."""
    import torch.distributed as dist
    from localstrm_b200 import _lib
    from localstrm_b200.distributed import shard_vocab
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    w = _cfg5_full()
    B, Vt, K = w.B, w.V, 64
    off, end = shard_vocab(Vt, world, rank)
    Vs = end - off
    shard_host = torch.from_numpy(np.ascontiguousarray(w.logits[:, off:end])).pin_memory()
    nbuf = n_buffers(shard_host.numel() * 4)
    bufs = [shard_host.to(dev) for _ in range(nbuf)]
    T = torch.from_numpy(w.temperature).to(dev)
    tp = torch.from_numpy(w.top_p).to(dev)
    u = torch.from_numpy(w.uniforms).to(dev)
    rb = int(lib.lss_shard_record_bytes(K))
    rec = torch.empty(B * rb, dtype=torch.uint8, device=dev)
    gathered = torch.empty(world * B * rb, dtype=torch.uint8, device=dev)
    mws = torch.empty(int(lib.lss_shard_merge_workspace_bytes(B)), dtype=torch.uint8, device=dev)
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream(dev)

    def records(x):
        _lib.check("lss_shard_topk", lib.lss_shard_topk(x.data_ptr(), 0, B, Vs, x.stride(0), off, T.data_ptr(),
                                                        K, rec.data_ptr(), st.cuda_stream))

    def step(i):
        records(bufs[i % nbuf])
        if world > 1:
            dist.all_gather_into_tensor(gathered, rec)
            src = gathered
        else:
            src = rec
        _lib.check("lss_shard_merge", lib.lss_shard_merge(src.data_ptr(), world, B, K, Vt, T.data_ptr(),
                                                          tp.data_ptr(), u.data_ptr(), tok.data_ptr(), None, None,
                                                          mws.data_ptr(), mws.numel(), st.cuda_stream))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        step(i)
    e1.record(st)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # the shard kernel alone (the dominant kernel), events around each launch
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        kev[i][0].record(st)
        records(bufs[i % nbuf])
        kev[i][1].record(st)
    torch.cuda.synchronize()
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    alg = B * Vs * 4 + B * rb
    peak, peak_kind = peaks()
    achieved = alg / (kern_ms / 1000.0) / 1e9
    cpu = None
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        rate, cores, n, dt = cpu_reference_rate(w, seconds=args.cpu_seconds)
        cpu = {"value": rate, "unit": "rows/s", "cores": cores, "kind": "port",
               "sample": f"{n} whole rows (~{dt:.1f} s): per-row sample_next_token with top-k 64, top-p 0.9 "
                         f"restated in torch CPU ops (oracle/torch_port.py)"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": B * args.steps / (ms / 1000.0), "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; cfg5)",
            "config": vocab_config(args, w, world), "records_bytes_per_rank": B * rb,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": measured_traffic("lss_shard_cluster_kernel_cfg5", Vs / Vt),
                         "kernel": "lss_shard_cluster_kernel",
                         "peak_source": peak_kind, "algorithmic_bytes_per_launch": alg, "kernel_ms": kern_ms},
            "clocks": clk, "e2e": None, "cpu_baseline": cpu, "gpu_launches": 2 * args.steps,
        }
        print(json.dumps(line), flush=True)


def run_greedy(args, rank: int, world: int, local_rank: int):
    """The engine's all-greedy seam (llm_engine.py:1139-1141, torch.argmax of the batch): one
    lss_argmax per step over each rank's own 256 headline rows, timed with events."""
    from localstrm_b200 import _lib
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    w = make_workload(rank, world, "headline")
    B = w.B
    host = torch.from_numpy(w.logits).pin_memory()
    nbuf = n_buffers(host.numel() * 4)
    bufs = [host.to(dev) for _ in range(nbuf)]
    tok = torch.empty(B, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream(dev)

    def step(i):
        x = bufs[i % nbuf]
        _lib.check("lss_argmax", lib.lss_argmax(x.data_ptr(), 0, B, w.V, x.stride(0), tok.data_ptr(),
                                                st.cuda_stream))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(args.steps):
        step(i)
    e1.record(st)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    got = tok.cpu().numpy()
    ref = np.argmax(w.logits[:, :], axis=1)  # no NaN in these rows
    assert np.array_equal(got, ref.astype(np.int32)), "argmax mismatch"
    alg = B * w.V * 4 + B * 4
    peak, peak_kind = peaks()
    achieved = alg / (ms / args.steps / 1000.0) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": B * world * args.steps / (ms / 1000.0), "unit": "rows/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; config 3 distribution at V=151,936)",
            "config": {"workload": DESC["greedy"], "global_batch": B * world, "rows_per_gpu": B, "vocab": w.V,
                       "parallelism": f"rows{world}" if world > 1 else "single",
                       "l2": f"{nbuf} rotating input buffers of {host.numel() * 4 / 1e6:.1f} MB"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "kernel": "lss_argmax_kernel",
                         "peak_source": peak_kind, "algorithmic_bytes_per_launch": alg,
                         "kernel_ms": ms / args.steps},
            "clocks": clk, "e2e": None, "cpu_baseline": None, "gpu_launches": args.steps,
        }
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--inner", type=int, default=1, help="calls per timed step")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--workload", default="headline", choices=WORKLOADS,
                    help="headline (the metric point) or one of the other configurations")
    ap.add_argument("--strong", action="store_true",
                    help="headline: split one 256-row batch over the GPUs instead of 256 rows per GPU")
    ap.add_argument("--ref-seconds", type=float, default=40.0,
                    help="--impl reference: CPU time of the timed steps together")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world == 1 and args.gpus > 1:
        print(json.dumps({"error": "run N>1 under torch.distributed.run"}), file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank, world)  # CPU only; ranks other than 0 exit without work
        return
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "cfg5":
            run_vocab(args, rank, world, local_rank)
        elif args.workload == "greedy":
            run_greedy(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
