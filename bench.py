"""Benchmark of the primitive path on B200: transformReduce (sum of squares over 2^30 fp32), sharded over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU, NCCL)

A step is one pass of the hot path over the workload: every rank reduces its contiguous shard of the 2^30 seeded
fp32 values in one kernel launch through the C ABI; for N > 1 that same kernel stores its unrounded partial into every
peer's mapped slot buffer over NVLink and combines the world's partials in rank order (a3b_transform_reduce_allranks;
`--collective nccl` uses an NCCL all-reduce after the kernel instead, and the fused run also reports that variant's
time). `value` is the whole-job throughput (4 * 2^30 bytes per step / max-over-ranks step time) with the inputs
resident in HBM; `e2e` is the same step through the C ABI from pinned HOST memory (host->device copy of each rank's
shard and device->host read of the result inside the timed region). The line also carries `parts`: the other
kernels the metric names (BabelStream copy/mul/add/triad and dot at 2^25 fp64, exclusive scan of 2^30 int32,
inclusive scan of 2^28 uint64, nBody, heat, HACCmk), each device-timed the same way, on one GPU at N = 1 and sharded
over the same ranks at N > 1, and a `parity` block (small-size checks of every sharded path). On several ranks every
timed region starts at a device-side start line (align_ranks), after the host barrier. The inputs (>= 268 MB per
array) exceed the 126 MB L2 in every case.

`--impl reference` times alpaka3's own OpenMP host backend (oracle/_ref, compiled from the reference headers) on the
host cores for the same metric and workload; under torchrun only rank 0 runs it.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "triad/dot/reduce/scan HBM GB/s (fraction of ~8 TB/s) at 1/2/4/8 B200"
N_SUMSQ = 1 << 30
SEED = 0x5EED0001
# the same string in both arms; how each arm splits the work is in config.parallelism
WORKLOAD = ("transformReduce sum of squares (std::plus, x*x) over 2^30 fp32 uniform[-1,1) from a seeded Philox "
            "stream")
FP32_PEAK = 148 * 128 * 2 * 1.965e9  # FP32 lanes x 2 flop x boost clock, nominal (not driver-measured)


def host_threads():
    """Host threads this process may run on (the OpenMP thread count of the CPU arms; launchers such as torchrun set
    OMP_NUM_THREADS=1, which must not decide the reference's core count)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def use_all_host_threads():
    """Before the OpenMP runtime of the CPU arms is loaded: alpaka3's host queue runs its kernels on a worker thread of
    its own, whose OpenMP thread count comes from OMP_NUM_THREADS when the runtime starts (a later omp_set_num_threads
    on this thread does not reach it)."""
    os.environ["OMP_NUM_THREADS"] = str(host_threads())


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU through NVML while the timed region runs."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, pci_bus_id, period_s=0.002):
        self.period = period_s
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByPciBusId(pci_bus_id)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for name, bit in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)
        except Exception:  # noqa: BLE001
            pass

    def start(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self.nv and self._t:
            self._stop.set()
            self._t.join()
            self._sample()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def gpu_local_cpus(torch, ordinal):
    """CPUs attached to the GPU's PCIe root (sysfs local_cpulist of its PCI device), or None."""
    try:
        bdf = pci_bus_id(torch, ordinal).lower()[4:]  # dddd:bb:dd.f
        with open(f"/sys/bus/pci/devices/{bdf}/local_cpulist") as f:
            text = f.read().strip()
        cpus = set()
        for part in text.split(","):
            if "-" in part:
                a, b = part.split("-")
                cpus.update(range(int(a), int(b) + 1))
            elif part:
                cpus.add(int(part))
        return cpus & set(os.sched_getaffinity(0)) or None
    except (OSError, ValueError, AttributeError):
        return None


def pci_bus_id(torch, ordinal):
    p = torch.cuda.get_device_properties(ordinal)
    return "%08X:%02X:%02X.0" % (getattr(p, "pci_domain_id", 0), p.pci_bus_id, p.pci_device_id)


# ------------------------------------------------------------------------------------------------ device timing
def time_steps(torch, dist_on, step, steps, warmup, kernel_events=True):
    """W untimed steps, then K steps between barrier+sync on both sides; returns (ms per step, average ms between
    the per-step kernel events that `step` records, or None when kernel_events is False)."""
    for _ in range(warmup):
        step(None)
    torch.cuda.synchronize()
    if dist_on:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    if dist_on:
        align_ranks(torch, s)
    t0.record(s)
    for k in range(steps):
        step(ev[k] if kernel_events else None)
    t1.record(s)
    torch.cuda.synchronize()
    if dist_on:
        import torch.distributed as dist
        dist.barrier()
    total = t0.elapsed_time(t1)
    kern = statistics.mean(a.elapsed_time(b) for a, b in ev) if kernel_events else None
    return total / steps, kern


ALIGN_SPIN_CYCLES = 4_000_000  # ~2 ms at 1.965 GHz


def align_ranks(torch, s):
    """Untimed device-side start line of a timed region on several ranks. The host processes leave the barrier tens
    of microseconds apart, and the ranks' timed kernels wait for one another (peer exchanges, NCCL), so without this
    every rank's first event would include the slowest host's lag. Each rank's stream first spins ~2 ms on its GPU
    (long enough for the host to queue the timed steps behind it), then passes a one-element all-reduce, which the
    ranks' streams leave within a few microseconds of each other; the start event is recorded right after it."""
    import torch.distributed as dist
    spin = getattr(torch.cuda, "_sleep", None)  # torch's clock-spin kernel; without it only the all-reduce aligns
    if spin is not None:
        spin(ALIGN_SPIN_CYCLES)
    t = torch.zeros(1, device=s.device)
    dist.all_reduce(t)


def max_over_ranks(torch, dist_on, v):
    if not dist_on:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def run_b200(args):
    import torch
    from alpaka3_b200 import algo, capi, dist as adist

    world, rank, local = adist.init()
    dist_on = world > 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    capi.lib()
    # nothing on this stream signals its dependents early, so consecutive reductions may overlap
    algo.set_early_start(True)
    peak, peak_kind = peaks()

    # ---------------------------------------------------------------- headline: sum of squares, 2^30 fp32
    b, e = adist.shard_range(N_SUMSQ, rank, world)
    n_local = e - b
    x = torch.empty(n_local, dtype=torch.float32, device=dev)
    algo.random_f32(x, SEED, -1.0, 1.0, start=b)
    out = torch.empty(1, dtype=torch.float32, device=dev)
    partial = torch.empty(1, dtype=torch.float64, device=dev)
    s = torch.cuda.current_stream()
    launches = [0]

    group = adist.PeerGroup() if dist_on and args.collective == "fused" else None

    def step(ev):
        if ev:
            ev[0].record(s)
        if group is not None:
            group.transform_reduce(0.0, "plus", "square", x, out=out)  # one launch: reduce + all-reduce
        elif dist_on:
            algo.transform_reduce_partial("plus", "square", x, partial=partial)
        else:
            algo.transform_reduce(0.0, out, "plus", "square", x)
        if ev:
            ev[1].record(s)
            launches[0] += 1
        if dist_on and group is None:
            adist.allreduce_partial(partial, "plus")

    def nccl_step(ev):
        algo.transform_reduce_partial("plus", "square", x, partial=partial)
        adist.allreduce_partial(partial, "plus")

    sampler = ClockSampler(pci_bus_id(torch, local))
    sampler.start()
    # value: K steps back to back between two events. A step is one launch of the reduce kernel (N = 1, or the fused
    # reduce + all-reduce for N > 1), so the roofline's launch duration is the timed region's average per launch;
    # consecutive launches overlap (early start), which an event pair around every launch would prevent, so the
    # second pass with such pairs is reported beside it as the isolated launch time
    ms, _ = time_steps(torch, dist_on, step, args.steps, args.warmup, kernel_events=False)
    _, iso_ms = time_steps(torch, dist_on, step, args.steps, args.warmup)
    sampler.stop()
    ms = max_over_ranks(torch, dist_on, ms)
    iso_ms = max_over_ranks(torch, dist_on, iso_ms)
    # with the NCCL all-reduce after the kernel a step is more than one launch: the kernel's own time is the pair's
    one_launch_steps = not (dist_on and group is None)
    kern_ms = ms if one_launch_steps else iso_ms
    nccl_ms = None
    if group is not None:
        nccl_ms, _ = time_steps(torch, dist_on, nccl_step, args.steps, args.warmup, kernel_events=False)
        nccl_ms = max_over_ranks(torch, dist_on, nccl_ms)
    total_bytes = 4.0 * N_SUMSQ
    value = total_bytes / (ms * 1e-3) / 1e9
    kern_gbs = 4.0 * n_local / (kern_ms * 1e-3) / 1e9
    result = float(out.item()) if (group is not None or not dist_on) else float(partial.item())

    # ---------------------------------------------------------------- e2e: host buffers through the C ABI
    e2e = None
    if not args.no_e2e:
        # pinned pages land on the NUMA node of the allocating thread: allocate (and touch) them from CPUs next to
        # this rank's GPU, so the host->device copies do not cross the socket interconnect
        local_cpus = gpu_local_cpus(torch, local)
        saved_affinity = os.sched_getaffinity(0)
        if local_cpus:
            os.sched_setaffinity(0, local_cpus)
        host = torch.empty(n_local, dtype=torch.float32, pin_memory=True)
        host.copy_(x.cpu())
        res_host = torch.empty(1, dtype=torch.float64 if (dist_on and group is None) else torch.float32,
                               pin_memory=True)
        sh = algo.stream_handle()
        import ctypes

        def e2e_step(ev):
            capi.call("a3b_memcpy_async", ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(host.data_ptr()),
                      4 * n_local, sh)
            if group is not None:
                group.transform_reduce(0.0, "plus", "square", x, out=out)
                src = out
            elif dist_on:
                algo.transform_reduce_partial("plus", "square", x, partial=partial)
                adist.allreduce_partial(partial, "plus")
                src = partial
            else:
                algo.transform_reduce(0.0, out, "plus", "square", x)
                src = out
            capi.call("a3b_memcpy_async", ctypes.c_void_p(res_host.data_ptr()), ctypes.c_void_p(src.data_ptr()),
                      src.element_size(), sh)

        e_steps = max(1, min(args.steps, 10))
        e_ms, _ = time_steps(torch, dist_on, e2e_step, e_steps, 1, kernel_events=False)
        e_ms = max_over_ranks(torch, dist_on, e_ms)

        def h2d_step(ev):
            capi.call("a3b_memcpy_async", ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(host.data_ptr()),
                      4 * n_local, sh)

        h_ms, _ = time_steps(torch, dist_on, h2d_step, e_steps, 1, kernel_events=False)
        h_worst = max_over_ranks(torch, dist_on, h_ms)
        e2e = {"value": total_bytes / (e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 4 * N_SUMSQ,
               "d2h_bytes_per_step": res_host.element_size() * world, "steps": e_steps,
               "path": "a3b_memcpy_async(H2D, pinned) + a3b_transform_reduce + a3b_memcpy_async(D2H)",
               "h2d_only_GBps_all_ranks": round(total_bytes / (h_worst * 1e-3) / 1e9, 1),
               "host_buffer": "pinned, allocated from the CPUs local to each rank's GPU" if local_cpus
               else "pinned (GPU-local CPUs unknown)"}
        del host
        os.sched_setaffinity(0, saved_affinity)

    # ---------------------------------------------------------------- other kernels of the metric
    del x
    torch.cuda.empty_cache()
    parts = None
    if not args.no_parts:
        if world == 1:
            parts = bench_parts(torch, algo, dev, args, peak)
        else:
            parts = bench_parts_multi(torch, algo, adist, world, rank, dev, args, peak, peak_kind)

    # ---------------------------------------------------------------- parity of every sharded path (small sizes)
    parity = None if args.no_parity else parity_checks(torch, algo, adist, world, rank, dev)

    # ---------------------------------------------------------------- CPU baseline: alpaka3's OpenMP backend
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu:
        cpu = cpu_baseline(budget_s=args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Philox4x32-10, uniform [-1,1))",
            "config": {"workload": WORKLOAD, "n": N_SUMSQ, "bytes_per_step": int(total_bytes),
                       "per_rank_elements": n_local, "l2": "inputs larger than L2 (4.29 GB total, >= 537 MB per GPU)",
                       "parallelism": (f"contiguous shards on {world} GPUs, fp64 partials combined by a fused peer "
                                       "all-reduce" if group is not None else
                                       f"contiguous shards on {world} GPUs, fp64 partials combined by NCCL all-reduce")
                       if dist_on else "single GPU",
                       "early_start": "consecutive reductions overlap (a3b_set_early_start on the bench stream)"},
            "result": result,
            "roofline": {"bound": "hbm", "achieved": round(kern_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(kern_gbs / peak, 4), "peak_kind": peak_kind,
                         "traffic": SUMSQ_TRAFFIC_PER_LAUNCH(n_local),
                         "kernel": ("reduceAllRanksKernel<float, 8 per pack, plus, square> "
                                    "(a3b_transform_reduce_allranks)" if group is not None else
                                    "reduceKernel<float, 8 per pack, plus, square> (a3b_transform_reduce_partial)"
                                    if dist_on else
                                    "reduceKernel<float, 8 per pack, plus, square> (a3b_transform_reduce)"),
                         "kernel_ms": round(kern_ms, 5), "isolated_kernel_ms": round(iso_ms, 5),
                         "duration": ("average launch over the timed region (K back-to-back launches, overlapping)"
                                      if one_launch_steps else "event pair around every kernel launch")},
            "e2e": e2e, "gpu_launches": launches[0], "clocks": sampler.summary(),
        }
        if nccl_ms is not None:
            line["nccl_allreduce_ms_per_step"] = round(nccl_ms, 5)
        if cpu:
            line["cpu_baseline"] = cpu
        if parts:
            line["parts"] = parts
        if parity is not None:
            line["parity"] = parity
        print(json.dumps(line), flush=True)
    if dist_on:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()
        if group is not None:
            group.close()
        dist.barrier()
        dist.destroy_process_group()


def SUMSQ_TRAFFIC_PER_LAUNCH(n_local):
    """DRAM bytes per launch from the committed ncu capture (profiles/), scaled by elements; None if not captured."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            t = json.load(f)["sumsq_f32_bytes_per_element"]
        return int(t * n_local)
    except (OSError, KeyError, ValueError):
        return None


def bench_parts(torch, algo, dev, args, peak):
    parts = {}
    steps = max(args.steps, 20)

    def measure(name, step, bytes_per_step, extra=None):
        # K calls back to back between two events (no event pair per call), as the reference comparator times them
        ms, _ = time_steps(torch, False, lambda ev: step(), steps, max(args.warmup, 3), kernel_events=False)
        gbs = bytes_per_step / (ms * 1e-3) / 1e9
        d = {"GB/s": round(gbs, 1), "frac": round(gbs / peak, 4), "ms_per_call": round(ms, 5),
             "bytes_per_step": int(bytes_per_step)}
        if extra:
            d.update(extra)
        parts[name] = d

    n = 1 << 25
    a, b, c = (torch.empty(n, dtype=torch.float64, device=dev) for _ in range(3))
    algo.babelstream("init", a, b, c)
    # BabelStream byte accounting (babelStreamCommon.hpp:440-463): copy/mul/dot move 2 arrays, add/triad 3
    measure("copy_f64_2^25", lambda: algo.babelstream("copy", a, b, c), 2 * 8 * n)
    measure("mul_f64_2^25", lambda: algo.babelstream("mul", a, b, c), 2 * 8 * n)
    measure("add_f64_2^25", lambda: algo.babelstream("add", a, b, c), 3 * 8 * n)
    measure("triad_f64_2^25", lambda: algo.babelstream("triad", a, b, c), 3 * 8 * n)
    out = torch.empty(1, dtype=torch.float64, device=dev)
    measure("dot_f64_2^25", lambda: algo.transform_reduce(0.0, out, "plus", "product", a, b), 2 * 8 * n)
    del a, b, c
    n = 1 << 30
    xi = torch.empty(n, dtype=torch.int32, device=dev)
    algo.random_u32(xi, SEED, shift=28)
    yi = torch.empty_like(xi)
    measure("exclusive_scan_i32_2^30", lambda: algo.exclusive_scan(yi, xi), 2 * 4 * n)
    del xi, yi
    n = 1 << 28
    xu = torch.empty(n, dtype=torch.int64, device=dev)
    algo.random_u64(xu, SEED)
    yu = torch.empty_like(xu)
    measure("inclusive_scan_u64_2^28", lambda: algo.inclusive_scan(yu, xu), 2 * 8 * n)
    del xu, yu

    # nBody, 262144 bodies, one step = kick + drift; 20 flop per pair (example/nBody/src/common.hpp:21-30)
    nb = 262144
    m, px, py, pz = (torch.empty(nb, dtype=torch.float32, device=dev) for _ in range(4))
    algo.random_f32(m, SEED + 1, 0.5, 1.0)
    for k, t in enumerate((px, py, pz)):
        algo.random_f32(t, SEED + 2 + k, 0.0, 1.0)
    v = [torch.zeros(nb, dtype=torch.float32, device=dev) for _ in range(3)]
    flops = 20.0 * nb * nb + 6.0 * nb
    ms_nb, kern_nb = time_steps(torch, False, lambda ev: _wrap(torch, ev, lambda: algo.nbody_step(
        m, px, py, pz, *v, 1e-3, 1e-3)), 10, 2)
    fp32_peak = 148 * 128 * 2 * 1.965e9
    parts["nbody_262144_step"] = {"GFLOP/s": round(flops / (kern_nb * 1e-3) / 1e9, 1),
                                  "frac_fp32_fma": round(flops / (kern_nb * 1e-3) / fp32_peak, 4),
                                  "kernel_ms": round(kern_nb, 4), "flop_per_step": flops, "steps": 10,
                                  "peak": "148 SMs x 128 FP32 lanes x 2 x 1.965 GHz = 74.4 TFLOP/s (nominal)"}
    del m, px, py, pz, v

    # HACCmk short-range force at the benchmark's defaults (15000 particles, 784 active; benchmark/HACCmk/src/misc.hpp:
    # 24-25): the benchmark reports the average kernel time
    n2, n1 = 15000, 784
    hx, hy, hz, hm = (torch.empty(n2, dtype=torch.float32, device=dev) for _ in range(4))
    d1 = (1.0 / n2, 2.0 / n2, 3.0 / n2)
    idx = torch.arange(n2, dtype=torch.float64, device=dev)
    for t, d in zip((hx, hy, hz), d1):
        t.copy_((idx * d).float())  # stand-in positions of the same spread (timing only; parity is in the tests)
    hm.copy_((idx * 0.01).float() + hx)
    hv = [torch.zeros(n1, dtype=torch.float32, device=dev) for _ in range(3)]
    ms_h, _ = time_steps(torch, False, lambda ev: algo.haccmk_step10(hx, hy, hz, hm, *hv, n1, 0.5, 0.03, 0.23),
                         max(args.steps, 20), max(args.warmup, 3), kernel_events=False)
    parts["haccmk_15000x784_step10"] = {"us_per_call": round(ms_h * 1e3, 2),
                                        "pairs_per_s": round(float(n1) * n2 / (ms_h * 1e-3), 1)}
    del hx, hy, hz, hm, hv, idx

    # heat, 32768 x 32768 interior fp64 (8.6 GB per field), dt/dx^2 = 0.2
    side = 32768
    u = torch.empty((side + 2, side + 2), dtype=torch.float64, device=dev)
    dx = 1.0 / (side + 1)
    algo.heat_init(u, dx, dx)
    w = u.clone()
    cells = float(side) * side
    state = [u, w]

    def heat_step():
        algo.heat_step(state[0], state[1], 0.2, 0.2)
        state[0], state[1] = state[1], state[0]

    measure("heat_32768^2_step", heat_step, 16.0 * cells)
    del u, w, state
    torch.cuda.synchronize()
    return parts


def _wrap(torch, ev, fn):
    s = torch.cuda.current_stream()
    if ev:
        ev[0].record(s)
    fn()
    if ev:
        ev[1].record(s)


def cpu_baseline(budget_s=8.0, n=1 << 28):
    """alpaka3's own transformReduce on exec::cpuOmpBlocks over a 2^28 fp32 sample (1.07 GB), repeated for about
    budget_s seconds; GB/s of input read."""
    use_all_host_threads()
    try:
        from oracle.oracle import Port, Ref
        ref, port = Ref(), Port()
    except Exception as e:  # noqa: BLE001
        return {"value": None, "unit": "GB/s", "kind": "reference", "unavailable": str(e)}
    ref.set_num_threads(host_threads())
    x = port.gen_f32(n, -1.0, 1.0, seed=SEED)
    ref.sumsq(x)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        ref.sumsq(x)
        times.append(time.perf_counter() - t0)
    best = min(times)
    return {"value": round(4.0 * n / best / 1e9, 2), "unit": "GB/s", "cores": ref.num_threads(), "kind": "reference",
            "sample": f"alpaka3 onHost::transformReduce(exec::cpuOmpBlocks) over 2^28 fp32 (first 2^28 elements of the "
                      f"workload's stream), best of {len(times)} runs in {budget_s:.0f} s",
            "median_GB/s": round(4.0 * n / statistics.median(times) / 1e9, 2)}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    use_all_host_threads()
    try:
        from oracle.oracle import Port, Ref
        ref, port = Ref(), Port()
    except Exception as e:  # noqa: BLE001
        print(json.dumps({"impl": "reference", "unavailable": f"alpaka3 host backend not built: {e}"}), flush=True)
        return
    ref.set_num_threads(host_threads())
    x = port.gen_f32(N_SUMSQ, -1.0, 1.0, seed=SEED)
    for _ in range(args.warmup):
        ref.sumsq(x)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        r = ref.sumsq(x)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    value = 4.0 * N_SUMSQ / (ms * 1e-3) / 1e9
    cores = ref.num_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Philox4x32-10, uniform [-1,1))",
        "config": {"workload": WORKLOAD, "n": N_SUMSQ, "bytes_per_step": 4 * N_SUMSQ,
                   "parallelism": f"alpaka3 exec::cpuOmpBlocks, {cores} OpenMP threads, whole input in host memory"},
        "result": float(r),
        "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": cores, "kind": "reference",
                         "sample": "alpaka3 onHost::transformReduce(exec::cpuOmpBlocks) over the full 2^30 fp32 "
                                   "workload per step"},
        "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_profile_case(args):
    """One kernel at a chosen size, W + K launches, for ncu captures (`-k regex:<kernel>`); not a bench line."""
    import torch
    from alpaka3_b200 import algo
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    case, lg = args.profile_case, args.log2n
    if case == "sumsq":
        n = 1 << (lg or 28)
        x = torch.empty(n, dtype=torch.float32, device=dev)
        algo.random_f32(x, SEED, -1.0, 1.0)
        out = torch.empty(1, dtype=torch.float32, device=dev)
        fn, nbytes = (lambda: algo.transform_reduce(0.0, out, "plus", "square", x)), 4 * n
    elif case in ("triad", "copy", "dot"):
        n = 1 << (lg or 25)
        a, b, c = (torch.empty(n, dtype=torch.float64, device=dev) for _ in range(3))
        algo.babelstream("init", a, b, c)
        out = torch.empty(1, dtype=torch.float64, device=dev)
        if case == "dot":
            fn, nbytes = (lambda: algo.transform_reduce(0.0, out, "plus", "product", a, b)), 16 * n
        else:
            fn, nbytes = (lambda: algo.babelstream(case, a, b, c)), (24 if case == "triad" else 16) * n
    elif case == "scan_i32":
        n = 1 << (lg or 28)
        x = torch.empty(n, dtype=torch.int32, device=dev)
        algo.random_u32(x, SEED, shift=28)
        y = torch.empty_like(x)
        fn, nbytes = (lambda: algo.exclusive_scan(y, x)), 8 * n
    elif case == "scan_u64":
        n = 1 << (lg or 27)
        x = torch.empty(n, dtype=torch.int64, device=dev)
        algo.random_u64(x, SEED)
        y = torch.empty_like(x)
        fn, nbytes = (lambda: algo.inclusive_scan(y, x)), 16 * n
    elif case == "nbody":
        n = 1 << (lg or 16)
        m, px, py, pz = (torch.empty(n, dtype=torch.float32, device=dev) for _ in range(4))
        algo.random_f32(m, SEED + 1, 0.5, 1.0)
        for k, t in enumerate((px, py, pz)):
            algo.random_f32(t, SEED + 2 + k, 0.0, 1.0)
        v = [torch.zeros(n, dtype=torch.float32, device=dev) for _ in range(3)]
        fn, nbytes = (lambda: algo.nbody_step(m, px, py, pz, *v, 1e-3, 1e-3)), 20 * n * n
    else:
        side = 1 << ((lg or 26) // 2)
        u = torch.empty((side + 2, side + 2), dtype=torch.float64, device=dev)
        dx = 1.0 / (side + 1)
        algo.heat_init(u, dx, dx)
        w = u.clone()
        fn, nbytes = (lambda: algo.heat_step(u, w, 0.2, 0.2)), 16 * side * side
    ms, kern = time_steps(torch, False, lambda ev: _wrap(torch, ev, fn), args.steps, args.warmup)
    print(json.dumps({"profile_case": case, "n_log2": lg, "kernel_ms": kern, "units_per_s": nbytes / (kern * 1e-3)}))


def setup_workload(torch, algo, adist, wl, world, rank, dev, collective="fused"):
    """One of the metric's other configurations on N ranks: returns a namespace with the step function, this rank's
    and the whole job's units per step, a description and a close() for its peer resources.
    triad / dot: BabelStream fp64, 2^25 elements per array PER GPU (weak scaling, every rank's arrays exceed L2);
    scan_i32 / scan_u64: exclusive scan of 2^30 int32 / inclusive scan of 2^28 uint64 split across ranks (one fused
    launch for the shard total and the carry over lower ranks via peer slots, then the carried single-pass scan);
    nbody: 262144 bodies split across ranks, positions all-gathered every step; heat: 32768^2 fp64 in row slabs, one
    halo row exchanged with each neighbour per step inside the stencil kernel (or by NCCL)."""
    import types
    dist_on = world > 1
    W = types.SimpleNamespace(name=wl, scaling="strong", unit="GB/s", close=lambda: None)
    if wl in ("triad", "dot"):
        n = 1 << 25
        a, b, c = (torch.empty(n, dtype=torch.float64, device=dev) for _ in range(3))
        algo.babelstream("init", a, b, c)
        out = torch.empty(1, dtype=torch.float64, device=dev)
        W.scaling, W.dtype = "weak", "f64"
        if wl == "triad":
            W.fn, W.unit_bytes = (lambda: algo.babelstream("triad", a, b, c)), 24.0 * n
        else:
            group = adist.PeerGroup() if dist_on else None
            W.fn = (lambda: group.transform_reduce(0.0, "plus", "product", a, b, out=out)) if group else (
                lambda: algo.transform_reduce(0.0, out, "plus", "product", a, b))
            W.unit_bytes = 16.0 * n
            if group:
                W.close = group.close
        W.total = W.unit_bytes * world
        W.desc = f"BabelStream {wl} fp64, 2^25 elements per array on each GPU (weak scaling)"
    elif wl in ("scan_i32", "scan_u64"):
        n = (1 << 30) if wl == "scan_i32" else (1 << 28)
        dt = torch.int32 if wl == "scan_i32" else torch.int64
        b0, e0 = adist.shard_range(n, rank, world)
        x = torch.empty(e0 - b0, dtype=dt, device=dev)
        if wl == "scan_i32":
            algo.random_u32(x, SEED, start=b0, shift=28)
        else:
            algo.random_u64(x, SEED, start=b0)
        y = torch.empty_like(x)
        group = adist.PeerGroup() if dist_on else None
        incl = wl != "scan_i32"
        W.fn = (lambda: group.scan(incl, y, x)) if group else (lambda: algo._scan(incl, y, x))
        if group:
            W.close = group.close
        W.unit_bytes = 2.0 * x.element_size() * (e0 - b0)
        W.total = 2.0 * x.element_size() * n
        W.dtype = "int32" if wl == "scan_i32" else "uint64"
        W.desc = (f"{'exclusive' if wl == 'scan_i32' else 'inclusive'} scan of 2^{30 if wl == 'scan_i32' else 28} "
                  f"{'int32 in [0,16)' if wl == 'scan_i32' else 'uint64'} split across ranks (one fused launch for "
                  "the shard total and the carry over lower ranks via peer slots, then the carried single-pass scan)")
    elif wl == "nbody":
        nb = 262144
        m, px, py, pz = (torch.empty(nb, dtype=torch.float32, device=dev) for _ in range(4))
        algo.random_f32(m, SEED + 1, 0.5, 1.0)
        for k, t in enumerate((px, py, pz)):
            algo.random_f32(t, SEED + 2 + k, 0.0, 1.0)
        b0, e0 = adist.shard_range(nb, rank, world)
        v = [torch.zeros(e0 - b0, dtype=torch.float32, device=dev) for _ in range(3)]
        sim = adist.NBody(m, px, py, pz, *v, b0)
        W.fn = lambda: sim.step(1e-3, 1e-3)
        W.unit_bytes = 20.0 * (e0 - b0) * nb
        W.total = 20.0 * nb * nb + 6.0 * nb
        W.unit, W.dtype = "GFLOP/s", "f32"
        W.desc = "all-pairs nBody, 262144 fp32 bodies split across ranks, positions all-gathered every step"
    else:
        side = 32768
        hb, he = adist.shard_range(side, rank, world)
        u = torch.empty((he - hb + 2, side + 2), dtype=torch.float64, device=dev)
        dx = 1.0 / (side + 1)
        algo.heat_init(u, dx, dx, row_offset=hb, global_rows=side)
        w = u.clone()
        slab = adist.HeatSlab(u, w, 0.2, 0.2, collective=collective)
        W.fn = slab.step
        W.close = slab.close
        W.unit_bytes = 16.0 * (he - hb) * side
        W.total = 16.0 * side * side
        W.dtype = "f64"
        W.desc = ("heat 5-point stencil, 32768^2 fp64 in row slabs, one halo row exchanged with each neighbour per "
                  "step " + ("(one kernel per step: boundary rows stored into the neighbours' mailboxes over NVLink)"
                             if collective == "fused" else "(NCCL send/recv overlapped with the interior update)"))
    return W


def time_workload(torch, dist_on, W, steps, warmup, peak, peak_kind):
    """Times W.fn: K steps back to back (value, and the per-step duration of the roofline) and K steps with an event
    pair each (reported as the isolated step time: the pairs keep consecutive steps from overlapping), max over ranks;
    returns the whole-job value, ms per step and the roofline entry."""
    s = torch.cuda.current_stream()
    launches = [0]

    def step(ev):
        if ev:
            ev[0].record(s)
        W.fn()
        if ev:
            ev[1].record(s)
            launches[0] += 1

    ms, _ = time_steps(torch, dist_on, step, steps, warmup, kernel_events=False)
    _, kern = time_steps(torch, dist_on, step, steps, warmup)
    ms = max_over_ranks(torch, dist_on, ms)
    kern = max_over_ranks(torch, dist_on, kern)
    value = W.total / (ms * 1e-3) / 1e9
    per_gpu = W.unit_bytes / (ms * 1e-3) / 1e9
    if W.unit == "GFLOP/s":
        fp32_peak = FP32_PEAK / 1e9
        roof = {"bound": "fp32 pipe", "achieved": round(per_gpu, 1), "peak": round(fp32_peak, 1), "unit": "GFLOP/s",
                "frac": round(per_gpu / fp32_peak, 4), "peak_kind": "nominal (148 SMs x 128 lanes x 2 x 1.965 GHz)"}
    else:
        roof = {"bound": "hbm", "achieved": round(per_gpu, 1), "peak": peak, "unit": "GB/s",
                "frac": round(per_gpu / peak, 4), "peak_kind": peak_kind}
    roof["step_ms_per_rank"] = round(ms, 5)
    roof["isolated_step_ms_per_rank"] = round(kern, 5)
    return value, ms, roof, launches[0]


def run_workload(args):
    """The other configurations of the metric on N ranks (one JSON line from rank 0, same keys as the headline)."""
    import torch
    from alpaka3_b200 import algo, dist as adist
    world, rank, local = adist.init()
    dist_on = world > 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    algo.set_early_start(True)
    peak, peak_kind = peaks()
    W = setup_workload(torch, algo, adist, args.workload, world, rank, dev, args.collective)
    sampler = ClockSampler(pci_bus_id(torch, local))
    sampler.start()
    value, ms, roof, launches = time_workload(torch, dist_on, W, args.steps, args.warmup, peak, peak_kind)
    sampler.stop()
    W.close()
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": W.unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": W.scaling,
                "vs_baseline": None, "dtype": W.dtype, "data": "synthetic (seeded Philox4x32-10)",
                "config": {"workload": W.desc, "name": args.workload}, "roofline": roof, "gpu_launches": launches,
                "clocks": sampler.summary()}
        print(json.dumps(line), flush=True)
    if dist_on:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def bench_parts_multi(torch, algo, adist, world, rank, dev, args, peak, peak_kind):
    """N > 1: the metric's other configurations sharded over the same ranks (max-over-ranks device time)."""
    parts = {}
    dist_on = world > 1
    for wl in ("triad", "dot", "scan_i32", "scan_u64", "nbody", "heat"):
        W = setup_workload(torch, algo, adist, wl, world, rank, dev, args.collective)
        steps = 10 if wl == "nbody" else max(args.steps, 20)
        value, ms, roof, _ = time_workload(torch, dist_on, W, steps, max(args.warmup, 3), peak, peak_kind)
        W.close()
        parts[wl] = {W.unit: round(value, 1), "ms_per_step": round(ms, 5), "scaling": W.scaling,
                     "per_gpu_frac": roof["frac"], "per_gpu_achieved": roof["achieved"], "workload": W.desc}
        del W
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    return parts


def parity_checks(torch, algo, adist, world, rank, dev):
    """Small-size parity of every sharded path on these ranks, outside the timed region, against independent torch
    references computed on each rank for the whole (small) problem: the fused reduce + all-reduce (fp64 sum, rel
    1e-5), the peer-carried exclusive int32 scan with wrap-around and the inclusive uint64 scan (torch cumsum,
    bit-exact), the nBody step with the all-gather (fp64 all-pairs, rel 1e-4 normwise) and the heat step with the
    fused halo exchange (the same operation order in torch, bit-exact). Returns {check: true/false over all ranks}."""
    res = {}
    group = adist.PeerGroup() if world > 1 else None
    try:
        # transformReduce sum of squares, fp32 shards, fused peer all-reduce
        n = (1 << 24) + 5
        full = torch.empty(n, dtype=torch.float32, device=dev)
        algo.random_f32(full, SEED, -1.0, 1.0)
        b, e = adist.shard_range(n, rank, world)
        x = full[b:e].clone()
        out = torch.empty(1, dtype=torch.float32, device=dev)
        if group:
            group.transform_reduce(0.0, "plus", "square", x, out=out)
        else:
            algo.transform_reduce(0.0, out, "plus", "square", x)
        exact = float((full.double() ** 2).sum().item())
        res["reduce_sumsq_rel_le_1e-5"] = abs(float(out.item()) - exact) / exact <= 1e-5
        # exclusive int32 scan, values that make the carry wrap
        xs_full = torch.empty(n, dtype=torch.int32, device=dev)
        algo.random_u32(xs_full, SEED, shift=1)
        xs = xs_full[b:e].clone()
        ys = torch.empty_like(xs)
        if group:
            group.scan(False, ys, xs)
        else:
            algo.exclusive_scan(ys, xs)
        want = (torch.cumsum(xs_full.long(), 0) - xs_full.long()).to(torch.int32)[b:e]
        res["scan_i32_exclusive_bit_exact"] = bool(torch.equal(ys, want))
        # inclusive uint64 scan (int64 storage, wrapping adds)
        n64 = (1 << 22) + 3
        xu_full = torch.empty(n64, dtype=torch.int64, device=dev)
        algo.random_u64(xu_full, SEED)
        b6, e6 = adist.shard_range(n64, rank, world)
        xu = xu_full[b6:e6].clone()
        yu = torch.empty_like(xu)
        if group:
            group.scan(True, yu, xu)
        else:
            algo.inclusive_scan(yu, xu)
        res["scan_u64_inclusive_bit_exact"] = bool(torch.equal(yu, torch.cumsum(xu_full, 0)[b6:e6]))
        del full, x, xs_full, xs, ys, want, xu_full, xu, yu
    finally:
        if group:
            torch.cuda.synchronize()
            group.close()

    # nBody: 4096 bodies split across ranks, 3 kick + drift steps with the all-gather, against fp64 all-pairs
    nb, steps, dt, eps = 4096, 3, 1e-3, 1e-3
    m = torch.empty(nb, dtype=torch.float32, device=dev)
    algo.random_f32(m, SEED + 1, 0.5, 1.0)
    pos = [torch.empty(nb, dtype=torch.float32, device=dev) for _ in range(3)]
    for k, t in enumerate(pos):
        algo.random_f32(t, SEED + 2 + k, 0.0, 1.0)
    P = torch.stack([t.double() for t in pos], 1)
    V = torch.zeros_like(P)
    M = m.double()
    for _ in range(steps):
        d = P[None, :, :] - P[:, None, :]
        r2 = (d * d).sum(-1) + eps
        a = ((M[None, :] / torch.sqrt(r2 ** 3))[:, :, None] * d).sum(1)
        V = V + a * dt
        P = P + V * dt
    bb, eb = adist.shard_range(nb, rank, world)
    v = [torch.zeros(eb - bb, dtype=torch.float32, device=dev) for _ in range(3)]
    sim = adist.NBody(m, *pos, *v, bb)
    for _ in range(steps):
        sim.step(dt, eps)
    torch.cuda.synchronize()
    got = torch.stack([t.double() for t in pos], 1)
    res["nbody_positions_rel_le_1e-4"] = float((got - P).abs().max() / P.abs().max()) <= 1e-4

    # heat: 1000 x 1000 interior, 7 steps, row slabs with the fused halo exchange, bit-exact
    nh, hsteps, r = 1000, 7, 0.2
    dx = 1.0 / (nh + 1)
    u = torch.zeros((nh + 2, nh + 2), dtype=torch.float64, device=dev)
    algo.heat_init(u, dx, dx)
    ref = u.clone()
    for _ in range(hsteps):
        c = ref[1:-1, 1:-1]
        nxt = ref.clone()
        nxt[1:-1, 1:-1] = (c * (1.0 - 2.0 * r - 2.0 * r) + ref[1:-1, :-2] * r + ref[1:-1, 2:] * r
                           + ref[:-2, 1:-1] * r + ref[2:, 1:-1] * r)
        ref = nxt
    hb, he = adist.shard_range(nh, rank, world)
    cur = u[hb:he + 2].clone()
    slab = adist.HeatSlab(cur, cur.clone(), r, r)
    for _ in range(hsteps):
        slab.step()
    slab.close()
    torch.cuda.synchronize()
    res["heat_fused_halo_bit_exact"] = bool(torch.equal(slab.cur[1:he - hb + 1], ref[hb + 1:he + 1]))

    if world > 1:
        import torch.distributed as dist
        allres = [None] * world
        dist.all_gather_object(allres, res)
        res = {k: all(r[k] for r in allres) for k in res}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-parts", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the small-size parity checks of the sharded paths")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--workload", default="sumsq",
                    choices=["sumsq", "triad", "dot", "scan_i32", "scan_u64", "nbody", "heat"],
                    help="sumsq is the headline; the others time the remaining configurations on N ranks")
    ap.add_argument("--collective", default="fused", choices=["fused", "nccl"],
                    help="N > 1: combine the per-rank partials inside the reduction kernel over mapped peer memory "
                         "(fused) or with an NCCL all-reduce after it")
    ap.add_argument("--profile-case", default=None,
                    choices=["sumsq", "triad", "copy", "dot", "scan_i32", "scan_u64", "nbody", "heat"],
                    help="run only this kernel (for ncu captures of a small case); prints a short line")
    ap.add_argument("--log2n", type=int, default=None, help="problem size (log2 elements) for --profile-case")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.profile_case:
        run_profile_case(args)
    elif args.workload != "sumsq":
        run_workload(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
