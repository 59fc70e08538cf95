"""Benchmark: batched top-p sampling of B x 32000 fp32 logits on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload topp|fused]

One step = one pass of the logits -> token path over one batch: the top-p
workload (per GPU B=4096 rows x V=32000, Gumbel + Zipf-bonus logits,
T=0.7, topp 0.9/0.95 by row, per-row xorshift seeds 42 + global row).  With N
GPUs (torchrun, one process per GPU) the global batch is N x 4096 rows of the
one seeded workload and rank r samples global rows [4096 r, 4096 (r + 1))
(weak scaling; rows are independent, no collective on the data path).  After
the timed region the ids are gathered on every rank with the library's NCCL
all-gather (sampler_nccl_allgather_ids) and rank 0 checks rows of every rank
against the CPU oracle (the line's "parity" object).  The line's "fused"
object measures the fused classifier + sampling variant at the same N: the
global batch of 8192 hidden states sharded over the ranks.

`value` is device-timed (CUDA events, inputs resident in HBM, 524 MB per
step > the 126 MB L2, so no flush is needed), max over ranks.  `e2e` is the
same metric through the host-buffer C-ABI entry point (sampler_batched_host)
with the H2D copy of the logits from pinned memory and the D2H copy of the
ids inside the timed region.  `--impl reference` times the reference's own
CPU sampler (llama2.c sample() over rows, OpenMP over the host cores).

`--workload fused` measures the fused variant instead: the classifier
projection of B = 8192 bf16 hidden states (dim 4096, sharded over the GPUs)
against a bf16 wcls [32000, 4096] on the tensor cores, then top-p sampling
(T = 0.8, topp 0.9) of the resulting rows; its roofline is the GEMM kernel
against the measured bf16 tensor peak.

`--workload decode` measures one decode step at batch 1 (latency): the
classifier projection of one hidden state plus sampling, ours
(`classifier_sample_fused`, bf16 wcls, id read back to the host) against the
reference's step (fp32 cuBLAS GEMV of wcls as `llama2_cublas.cu:5825-5826`,
the 128 KB logits copied to the host, its own sample() on the host).
"""
import argparse
import ctypes
import hashlib
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS_PER_GPU = 4096
VOCAB = 32000
TEMP = 0.7
METRIC = "sampled tokens/sec & HBM GB/s, B×32000 fp32 logits, top-p 0.9, at 1/2/4/8 B200"
WORKLOAD = "top-p batch: B=4096 per GPU x V=32000 fp32, Gumbel+Zipf(1.1) logits, T=0.7, topp 0.9/0.95 by row"


def load_json(path, default=None):
    try:
        with open(path) as f:
            return json.load(f)
    except Exception:
        return default


def kernel_source_digest(files):
    """Digest of the kernel sources a profile was captured from (the files
    under llama2.cu_b200/csrc named), so a capture of older code is not
    reported as the current kernel's traffic."""
    h = hashlib.sha256()
    for f in files:
        with open(os.path.join(ROOT, "llama2.cu_b200", "csrc", f), "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()[:16]


STREAM_SOURCES = ["row_stream.cu", "row_stream_impl.cuh", "exact_math.cuh", "device_common.cuh",
                  "sampler_kernels.cuh"]
GEMM_SOURCES = ["classifier_gemm.cu", "device_common.cuh", "sampler_kernels.cuh"]


def profiled_traffic(name, sources):
    """DRAM bytes per launch (read + write) recorded by an ncu summary under
    profiles/ (its `traffic_bytes_per_launch:` line), provided its
    `source_digest:` line matches the current kernel sources; else None."""
    import re
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            text = f.read()
    except OSError:
        return None
    m = re.search(r"^traffic_bytes_per_launch:\s*(\d+)", text, re.M)
    d = re.search(r"^source_digest:\s*([0-9a-f]+)", text, re.M)
    if not m or not d or d.group(1) != kernel_source_digest(sources):
        return None
    return int(m.group(1))


def host_threads():
    """Every host thread this process may use (torchrun sets
    OMP_NUM_THREADS=1, which must not throttle the CPU baseline)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def make_rows(rank, rows=ROWS_PER_GPU):
    """Global rows [rank * rows, (rank + 1) * rows) of the seeded top-p
    workload (each row has its own generator, so a rank draws only its own)."""
    from __graft_entry__ import load_package
    w = load_package().workloads.topp(rows=rows, first=rank * rows)
    return w["logits"], w["topp_rows"]


def bind_to_gpu_numa_node(local):
    """Restricts this process to the host CPUs NVML lists as local to its GPU
    (read-only NVML query; no GPU setting changes), so the pinned host buffers
    of the end-to-end leg are first touched on the GPU's own memory node.
    Returns the previous CPU set to restore, or None."""
    try:
        import pynvml
        import torch
        props = torch.cuda.get_device_properties(local)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            words = pynvml.nvmlDeviceGetCpuAffinity(h, 16)
        finally:
            pynvml.nvmlShutdown()
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1}
        before = os.sched_getaffinity(0)
        cpus &= before
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return before
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during timing."""

    def __init__(self, gpu_index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = []
        with open(self.f.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def host_cpu():
    """The host's CPU model and logical CPU count (as nproc reports them)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return dict(cpu_model=model, nproc=os.cpu_count())


def cpu_baseline(x, topp_rows, rows, use_ref=True, min_seconds=10.0):
    """The reference's own sampler on all host threads: passes over the first
    `rows` rows of the workload, repeated until at least `min_seconds` of CPU
    work (a bounded sample of the same workload)."""
    import oracle
    if use_ref and oracle.ref_available():
        lib, kind = oracle.ref_sampler(), "reference"
    else:
        lib, kind = oracle.oracle(), "port"
    threads = host_threads()
    from __graft_entry__ import load_package
    seeds = load_package().workloads.row_seeds(rows)
    t0 = time.perf_counter()
    passes = 0
    while True:
        lib.sample_batch(x[:rows], TEMP, 0.9, seeds, topp_rows=topp_rows[:rows], nthreads=threads)
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    return dict(value=passes * rows / dt, unit="tokens/s", cores=threads, kind=kind,
                sample=f"{passes} passes over {rows} rows of the top-p workload (llama2.c sample() per row, "
                       f"OpenMP over rows), {dt:.1f} s", **host_cpu())


def run_reference(args):
    """--impl reference: the reference's CPU sampler on the same workload."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    rows = args.ref_rows
    x, tr = make_rows(0, rows=rows)
    import oracle
    if not oracle.ref_available():
        oracle.build(with_ref=True)
    kind = "reference" if oracle.ref_available() else "port"
    lib = oracle.ref_sampler() if kind == "reference" else oracle.oracle()
    threads = host_threads()
    from __graft_entry__ import load_package
    seeds = load_package().workloads.row_seeds(rows)
    for _ in range(args.warmup):
        lib.sample_batch(x, TEMP, 0.9, seeds, topp_rows=tr, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        lib.sample_batch(x, TEMP, 0.9, seeds, topp_rows=tr, nthreads=threads)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    value = rows / dt
    line = dict(metric=METRIC, value=value, unit="tokens/s", n_gpus=world, steps=args.steps, warmup=args.warmup,
                ms_per_step=dt * 1e3, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="f32",
                data="synthetic (seeded numpy PCG64)", impl="reference",
                config=dict(workload=WORKLOAD, rows_per_step=rows, vocab=VOCAB, parallelism="host threads"),
                cpu_baseline=dict(value=value, unit="tokens/s", cores=threads, kind=kind,
                                  sample=f"{rows} rows per step, llama2.c sample() per row, OpenMP over rows",
                                  **host_cpu()),
                e2e=dict(value=value, unit="tokens/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)
    return 0


def fused_step_setup(pkg, world, rank, dev):
    """Inputs of the fused workload for this rank: rows [row0, row0 + B) of
    the 8192 hidden states, the whole wcls."""
    import torch
    f = pkg.workloads.fused()
    Bg, D = f["hidden"].shape
    V = f["wcls"].shape[0]
    row0 = rank * Bg // world
    B = (rank + 1) * Bg // world - row0
    h_host = torch.from_numpy(f["hidden"][row0:row0 + B].view(np.int16)).view(torch.bfloat16)
    w = torch.from_numpy(f["wcls"].view(np.int16)).view(torch.bfloat16).to(dev)
    return f, Bg, D, V, row0, B, h_host, w


def measure_fused(pkg, args, world, rank, dev, with_clocks=False):
    """Fused classifier + top-p sampling, global batch 8192 sharded by rows.
    Returns (per-rank dict of times, constants) for the caller to reduce."""
    import torch
    f, Bg, D, V, row0, B, h_host, w = fused_step_setup(pkg, world, rank, dev)
    h = h_host.to(dev)
    states = torch.empty(B, dtype=torch.int64, device=dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    logits = torch.empty(B, V, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    T, TOPP = f["temperature"], f["topp"]

    def step():
        pkg.seed_states(states, f["seed"], row0)
        pkg.classifier_sample_fused(h, w, T, TOPP, states, out_ids=ids, stream=stream)
        return pkg.last_launch_count() + 1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) if with_clocks else None
    if clocks:
        time.sleep(0.25)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    ev0.record(stream)
    for _ in range(args.steps):
        launches += step()
    ev1.record(stream)
    torch.cuda.synchronize()
    # the GEMM kernel alone, per launch
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, b in kev:
        a.record(stream)
        pkg.classifier_logits(h, w, logits_out=logits, stream=stream)
        b.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks else None
    ms = ev0.elapsed_time(ev1) / args.steps
    gemm_ms = float(np.mean([a.elapsed_time(b) for a, b in kev]))
    # end to end: hidden states from pinned host memory, ids back to the host
    pin = h_host.pin_memory()
    ids_host = torch.empty(B, dtype=torch.int32).pin_memory()
    e2e_steps = max(1, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        h.copy_(pin, non_blocking=True)
        step()
        ids_host.copy_(ids, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    # parity sample: this rank's first rows through the fused call with its
    # logits returned, the ids checked on the CPU against the oracle
    nchk = min(B, 8)
    lg = torch.empty(nchk, V, dtype=torch.float32, device=dev)
    st = torch.empty(nchk, dtype=torch.int64, device=dev)
    pkg.seed_states(st, f["seed"], row0)
    chk_ids = pkg.classifier_sample_fused(h[:nchk].contiguous(), w, T, TOPP, st, logits_out=lg)
    torch.cuda.synchronize()
    mism = oracle_mismatches(lg.cpu().numpy(), chk_ids.cpu().numpy(), T, TOPP, np.full(nchk, TOPP, np.float32),
                             pkg.workloads.row_seeds(nchk, seed=f["seed"], offset=row0))
    times = dict(ms=ms, gemm_ms=gemm_ms, e2e_ms=e2e_ms, launches=launches, checked=nchk, mismatches=mism[0],
                 unexplained=mism[1])
    return times, dict(Bg=Bg, D=D, V=V, B=B, T=T, TOPP=TOPP, clocks=clk)


def fused_line_parts(times, const, world, peaks):
    """The fused variant's numbers from the max over ranks of `times`."""
    Bg, D, V, B = const["Bg"], const["D"], const["V"], const["B"]
    peak_burst = peaks.get("bf16_tflops") or 1590.0
    peak_sus = peaks.get("bf16_tflops_sustained") or 1400.0
    note = "of measured" if peaks.get("bf16_tflops") else "of fallback"
    flops = 2.0 * B * D * V
    achieved = flops / (times["gemm_ms"] * 1e-3) / 1e12
    return dict(
        value=Bg / (times["ms"] * 1e-3), ms_per_step=times["ms"], unit="tokens/s",
        workload=f"fused: H bf16 [{Bg},{D}] x wcls bf16 [{V},{D}] -> fp32 logits, T={const['T']}, "
                 f"topp {const['TOPP']}; rows sharded over {world} GPU(s), wcls replicated",
        gemm=dict(kernel="classifier_gemm_pair_kernel", ms=times["gemm_ms"], tflops=achieved,
                  frac_of_burst=achieved / peak_burst, frac_of_sustained=achieved / peak_sus,
                  peak_burst=peak_burst, peak_sustained=peak_sus, peak_source=note),
        e2e=dict(value=Bg / (times["e2e_ms"] * 1e-3), unit="tokens/s", ms_per_step=times["e2e_ms"],
                 h2d_bytes_per_step=Bg * D * 2, d2h_bytes_per_step=Bg * 4),
        parity=dict(rows_checked=int(times["checked"]), mismatches=int(times["mismatches"]),
                    ok=int(times["unexplained"]) == 0),
        gpu_launches=int(times["launches"]))


def run_fused(args):
    """--workload fused: the fused classifier + sampling as the headline line."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    pkg = load_package()
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    times, const = measure_fused(pkg, args, world, rank, dev, with_clocks=True)
    times = reduce_max(times, world, dev)
    if rank == 0:
        peaks = load_json(os.path.join(ROOT, "MEASURED_PEAKS.json"), {})
        fp = fused_line_parts(times, const, world, peaks)
        g = fp["gemm"]
        line = dict(metric="fused classifier (bf16 tcgen05 GEMM) + top-p sampling, sampled tokens/sec",
                    value=fp["value"], unit="tokens/s", n_gpus=world, steps=args.steps, warmup=args.warmup,
                    ms_per_step=fp["ms_per_step"], higher_is_better=True, scaling="strong", vs_baseline=None,
                    dtype="bf16", data="synthetic (seeded numpy PCG64: H ~ N(0,1), wcls ~ N(0, 0.02^2), bf16)",
                    config=dict(workload=fp["workload"], global_batch=const["Bg"], rows_per_gpu=const["B"],
                                parallelism=f"rows sharded over {world} GPU(s), wcls replicated, no collective",
                                l2="wcls 262 MB and logits > 126 MB L2; no flush"),
                    roofline=dict(bound="tensor", achieved=g["tflops"], peak=g["peak_burst"], unit="TFLOP/s",
                                  frac=g["frac_of_burst"],
                                  traffic=profiled_traffic("classifier_gemm_8192x4096x32000.md", GEMM_SOURCES),
                                  kernel=g["kernel"], kernel_ms=g["ms"], peak_source=g["peak_source"] + " (burst)"),
                    cpu_baseline=None, e2e=fp["e2e"], parity=fp["parity"], gpu_launches=fp["gpu_launches"],
                    clocks=const["clocks"])
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def reduce_max(times, world, dev):
    """Max over ranks of every number in `times` (counts summed where they
    are counts of checked rows and mismatches)."""
    if world == 1:
        return times
    import torch
    import torch.distributed as dist
    keys = sorted(times)
    summed = {"checked", "mismatches", "unexplained"}
    mx = torch.tensor([float(times[k]) if k not in summed else 0.0 for k in keys], dtype=torch.float64, device=dev)
    sm = torch.tensor([float(times[k]) if k in summed else 0.0 for k in keys], dtype=torch.float64, device=dev)
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return {k: (float(sm[i]) if k in summed else float(mx[i])) for i, k in enumerate(keys)}


def oracle_mismatches(logits, ids, temperature, topp, topp_rows, seeds):
    """(number of ids that differ from the CPU oracle's, number of those NOT
    explained by a coin within 1e-6 of a cdf boundary of the oracle's walk)."""
    import oracle
    orc = oracle.oracle()
    ref_ids, _, ref_p = orc.sample_batch(logits, temperature, topp, seeds, topp_rows=topp_rows, probs_out=True)
    bad = np.nonzero(np.asarray(ids) != ref_ids)[0]
    unexplained = 0
    for r in bad:
        coin, _ = orc.coin(int(seeds[r]))
        if orc.boundary_distance(ref_p[r], float(topp_rows[r]), coin) > 1e-6:
            unexplained += 1
    return len(bad), unexplained


def gather_ids_nccl(pkg, ids, world, rank, dev):
    """All ranks' ids on every rank through the library's own NCCL all-gather
    (sampler_nccl_get_unique_id / _comm_init / _allgather_ids).  Every rank
    takes the same collective steps whatever happens.  Returns (ids_all
    numpy array or None, status string)."""
    import torch
    import torch.distributed as dist
    L = pkg.lib()
    B = ids.numel()
    uid = torch.zeros(128, dtype=torch.uint8)
    # every rank loads NCCL through the library first (a rank that could not
    # would leave the others waiting in the communicator's set-up)
    rc = L.sampler_nccl_get_unique_id(ctypes.c_void_p(uid.data_ptr()))
    uid_dev = uid.to(dev)
    dist.broadcast(uid_dev, 0)
    uid.copy_(uid_dev.cpu())
    ok = torch.tensor([1 if rc == 0 else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok) == 0:
        return None, "ncclGetUniqueId failed: " + L.sampler_last_error().decode()
    comm = ctypes.c_void_p()
    rc = L.sampler_nccl_comm_init(ctypes.byref(comm), world, ctypes.c_void_p(uid.data_ptr()), rank)
    ok = torch.tensor([1 if rc == 0 else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if int(ok) == 0:
        if rc == 0:
            L.sampler_nccl_comm_destroy(comm)
        return None, "ncclCommInitRank failed: " + L.sampler_last_error().decode()
    full = torch.full((world * B,), -1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    rc = L.sampler_nccl_allgather_ids(comm, ctypes.c_void_p(ids.data_ptr()), B, ctypes.c_void_p(full.data_ptr()),
                                      ctypes.c_void_p(stream.cuda_stream))
    torch.cuda.synchronize()
    L.sampler_nccl_comm_destroy(comm)
    if rc != 0:
        return None, "ncclAllGather failed: " + L.sampler_last_error().decode()
    return full.cpu().numpy(), "sampler_nccl_allgather_ids"


def run_decode(args):
    """Batch-1 decode step latency, greedy and top-p, ours vs the reference's path."""
    import torch
    import oracle
    from __graft_entry__ import load_package
    pkg = load_package()
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    f = pkg.workloads.fused(rows=1)
    D, V = f["hidden"].shape[1], f["wcls"].shape[0]
    h = torch.from_numpy(f["hidden"].view(np.int16)).view(torch.bfloat16).to(dev)
    w = torch.from_numpy(f["wcls"].view(np.int16)).view(torch.bfloat16).to(dev)
    w32 = w.float()
    h32 = h.float()[0]
    if not oracle.ref_available():
        oracle.build(with_ref=True)
    ref = oracle.ref_sampler() if oracle.ref_available() else oracle.oracle()
    kind = "reference" if oracle.ref_available() else "port"
    st = torch.empty(1, dtype=torch.int64, device=dev)
    ids = torch.empty(1, dtype=torch.int32, device=dev)
    ids_host = torch.empty(1, dtype=torch.int32).pin_memory()
    logits_host = torch.empty(V, dtype=torch.float32).pin_memory()
    out = {}
    for temp in (0.0, f["temperature"]):
        def ours():
            pkg.seed_states(st, f["seed"])
            pkg.classifier_sample_fused(h, w, temp, f["topp"], st, out_ids=ids)
            ids_host.copy_(ids)
            return int(ids_host[0])

        def reference():
            lg = torch.mv(w32, h32)
            logits_host.copy_(lg)
            ids_r = ref.sample_batch(logits_host.numpy()[None, :], temp, f["topp"],
                                     np.array([f["seed"]], np.uint64), nthreads=1)[0]
            return int(ids_r[0])

        # the same step captured once in a CUDA graph and replayed (the
        # library's buffers exist after the eager warm-up above)
        for _ in range(3):
            ours()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            pkg.seed_states(st, f["seed"])
            pkg.classifier_sample_fused(h, w, temp, f["topp"], st, out_ids=ids)

        def ours_graph():
            graph.replay()
            ids_host.copy_(ids)
            return int(ids_host[0])

        res = {}
        for name, fn in (("ours", ours), ("ours_graph", ours_graph), ("reference_path", reference)):
            for _ in range(max(args.warmup, 3)):
                fn()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                fn()
            res[name] = (time.perf_counter() - t0) / args.steps * 1e6
        assert ours_graph() == ours()  # the replay samples what the eager call does
        out["greedy" if temp == 0.0 else "topp"] = dict(ours_us=res["ours"], ours_graph_us=res["ours_graph"],
                                                        reference_path_us=res["reference_path"])
        del graph
    # the classifier alone (classifier_gemv_kernel at one row), device-timed on
    # its stream; W (262 MB) is larger than the 126 MB L2, so no flush
    stream = torch.cuda.current_stream()
    lg = torch.empty(1, V, device=dev)
    for _ in range(5):
        pkg.classifier_logits(h, w, logits_out=lg, stream=stream)
    n_cls = 50
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n_cls):
        pkg.classifier_logits(h, w, logits_out=lg, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    cls_us = e0.elapsed_time(e1) / n_cls * 1e3
    peaks = load_json(os.path.join(ROOT, "MEASURED_PEAKS.json"), {})
    peak, peak_note = peaks.get("hbm_gbs"), "of measured"
    if not peak:
        peak, peak_note = 6650.0, "of fallback"
    alg_bytes = V * D * 2 + D * 2 + V * 4  # wcls + hidden row + fp32 logits
    achieved = alg_bytes / (cls_us * 1e-6) / 1e9
    roof = dict(bound="hbm", kernel="classifier_gemv_kernel", achieved=achieved, peak=peak, unit="GB/s",
                frac=achieved / peak, traffic=profiled_traffic("classifier_gemv_kernel_decode_1x4096x32000.md", GEMM_SOURCES),
                note=f"{peak_note} HBM copy bandwidth; {cls_us:.1f} us per call")
    line = dict(metric="decode step latency at batch 1 (classifier + sampling), us", value=out["topp"]["ours_us"],
                unit="us", n_gpus=1, steps=args.steps, warmup=args.warmup, higher_is_better=False,
                vs_baseline=None, dtype="bf16", data="synthetic (seeded numpy PCG64)",
                config=dict(workload=f"decode: hidden bf16 [1,{D}] x wcls [{V},{D}], T={f['temperature']}, "
                                     f"topp {f['topp']}; greedy T=0"),
                latency=out, reference_kind=kind, roofline=roof,
                reference_path="torch.mv fp32 wcls (cuBLAS GEMV) + 128 KB D2H + reference sample() on one host thread")
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package
    pkg = load_package()
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    # host work and pinned buffers on the GPU's own memory node
    cpus_before = bind_to_gpu_numa_node(local)

    data_rank = rank if args.rows_of_rank is None else args.rows_of_rank
    x_host, topp_host = make_rows(data_rank)
    B = x_host.shape[0]
    row0 = data_rank * B
    seeds = pkg.workloads.row_seeds(B, offset=row0)
    x = torch.from_numpy(x_host).to(dev)
    topp_rows = torch.from_numpy(topp_host).to(dev)
    states = torch.empty(B, dtype=torch.int64, device=dev)
    ids = torch.empty(B, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    def step():
        pkg.seed_states(states, 42, row0)
        pkg.sample_batched(x, TEMP, 0.9, states, topp_rows=topp_rows, out_ids=ids, stream=stream)
        return pkg.last_launch_count() + 1

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    time.sleep(0.25)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    ev0.record(stream)
    for _ in range(args.steps):
        launches += step()
    ev1.record(stream)
    torch.cuda.synchronize()
    # per-launch duration of the row kernel alone (events around each launch)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    pkg.seed_states(states, 42, row0)
    for a, b in kev:
        a.record(stream)
        pkg.sample_batched(x, TEMP, 0.9, states, topp_rows=topp_rows, out_ids=ids, stream=stream)
        b.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / args.steps
    kernel_ms = float(np.mean([a.elapsed_time(b) for a, b in kev]))
    t = torch.tensor([ms, kernel_ms], dtype=torch.float64, device=dev)
    rank_ms = [ms]
    if world > 1:
        every = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(every, t)
        rank_ms = [float(v[0]) for v in every]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, kernel_ms = float(t[0]), float(t[1])

    # parity: the step's ids (from the seeded states) gathered on every rank
    # by the library's NCCL all-gather; rank 0 checks rows of every rank
    pkg.seed_states(states, 42, row0)
    step()
    torch.cuda.synchronize()
    if world > 1:
        ids_all, how = gather_ids_nccl(pkg, ids, world, rank, dev)
    else:
        ids_all, how = ids.cpu().numpy(), "local"
    parity = None
    if rank == 0:
        parity = dict(gathered_by=how, ranks=world, rows_checked=0, mismatches=0, ok=False)
        if ids_all is not None:
            per = max(1, args.parity_rows // world)
            checked = mism = unexplained = 0
            for r in range(world):
                dr = r if args.rows_of_rank is None else args.rows_of_rank
                local_rows = np.linspace(0, B - 1, per).astype(np.int64)
                xs = np.stack([pkg.workloads.topp(rows=1, first=dr * B + int(i))["logits"][0] for i in local_rows])
                tps = np.where((dr * B + local_rows) % 2 == 0, 0.9, 0.95).astype(np.float32)
                sd = pkg.workloads.row_seeds(B, offset=dr * B)[local_rows]
                got = ids_all[r * B + local_rows]
                m, u = oracle_mismatches(xs, got, TEMP, 0.9, tps, sd)
                checked += len(local_rows)
                mism += m
                unexplained += u
            parity.update(rows_checked=checked, mismatches=mism, ok=unexplained == 0,
                          rule="ids equal the CPU oracle's, or the coin lies within 1e-6 of a cdf boundary")

    # end to end through the host-buffer C-ABI call: pinned logits in,
    # ids and states out, copies inside the timed region
    pin = torch.from_numpy(x_host).pin_memory()
    xh = pin.numpy()
    st_host = np.empty(B, dtype=np.uint64)
    e2e_steps = max(1, min(args.steps, 10))
    for _ in range(2):
        st_host[:] = seeds
        pkg.sample_batched_host(xh, TEMP, 0.9, st_host, topp_rows_np=topp_host)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        st_host[:] = seeds
        pkg.sample_batched_host(xh, TEMP, 0.9, st_host, topp_rows_np=topp_host)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms)
    del pin, xh, x
    torch.cuda.empty_cache()

    # the fused classifier + sampling variant at the same number of GPUs
    fused = None
    if not args.no_fused:
        ftimes, fconst = measure_fused(pkg, args, world, rank, dev)
        ftimes = reduce_max(ftimes, world, dev)
        if rank == 0:
            fused = fused_line_parts(ftimes, fconst, world, load_json(os.path.join(ROOT, "MEASURED_PEAKS.json"), {}))

    if cpus_before is not None:
        os.sched_setaffinity(0, cpus_before)  # the CPU baseline uses every host thread
    if rank == 0:
        peaks = load_json(os.path.join(ROOT, "MEASURED_PEAKS.json"), {})
        peak = peaks.get("hbm_gbs")
        peak_note = "of measured"
        if not peak:
            peak, peak_note = 6650.0, "of fallback"
        alg_bytes = B * VOCAB * 4 + B * (8 + 8 + 4 + 4)  # logits + state r/w + topp + ids
        achieved = alg_bytes / (kernel_ms * 1e-3) / 1e9
        traffic = profiled_traffic("row_stream_kernel_topp_4096x32000.md", STREAM_SOURCES)
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_baseline(x_host, topp_host, args.cpu_rows)
        value = world * B / (ms * 1e-3)
        workload = WORKLOAD if args.rows_of_rank is None else WORKLOAD + f" (rows of rank {args.rows_of_rank})"
        line = dict(metric=METRIC, value=value, unit="tokens/s", n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling="weak", vs_baseline=None,
                    dtype="f32", data="synthetic (seeded numpy PCG64: Gumbel + Zipf(1.1) ranked bonus)",
                    config=dict(workload=workload, global_batch=world * B, rows_per_gpu=B, vocab=VOCAB,
                                temperature=TEMP, parallelism=f"rows sharded over {world} GPU(s), no collective",
                                l2="inputs 524 MB per GPU > 126 MB L2; no flush"),
                    hbm_gbs=world * alg_bytes / (ms * 1e-3) / 1e9, ms_per_step_by_rank=rank_ms,
                    roofline=dict(bound="hbm", achieved=achieved, peak=peak, unit="GB/s", frac=achieved / peak,
                                  traffic=traffic, kernel="row_stream_kernel", kernel_ms=kernel_ms,
                                  peak_source=peak_note),
                    cpu_baseline=cpu,
                    e2e=dict(value=world * B / (e2e_ms * 1e-3), unit="tokens/s",
                             h2d_bytes_per_step=B * VOCAB * 4 + B * 12, d2h_bytes_per_step=B * 12,
                             ms_per_step=e2e_ms, host_memory="pinned, on the GPU's NUMA node" if cpus_before
                             else "pinned"),
                    gpu_launches=launches, clocks=clk, parity=parity, fused=fused)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=4096)
    ap.add_argument("--ref-rows", type=int, default=4096)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="topp", choices=["topp", "fused", "decode"])
    ap.add_argument("--no-fused", action="store_true", help="skip the fused variant's sub-object")
    ap.add_argument("--parity-rows", type=int, default=64, help="rows checked against the oracle (all ranks)")
    ap.add_argument("--rows-of-rank", type=int, default=None,
                    help="sample the global rows of rank K instead of this rank's (diagnosis on one GPU)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "decode":
        return run_decode(args)
    return run_fused(args) if args.workload == "fused" else run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
