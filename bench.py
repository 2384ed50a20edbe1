#!/usr/bin/env python3
"""bench.py — CSR SpMV with compressed column indices on B200: GFLOP/s (2·nnz/t) and effective HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload stencil27]
                    [--layout lp] [--tpr 8] [--no-sweep] [--no-chained]

A step is one product y = A x over the whole matrix (at N GPUs: every rank its nnz-balanced row shard,
x replicated, no exchange — the products are independent). The default workload is the 3D 27-point
stencil on 160^3 (n = 4,096,000, nnz = 109,215,352, diagonal 26, neighbours -1) in lexicographic order,
then RCM-permuted; FP64; x uniform [-1, 1] from seed 2; the headline layout is CSR-lp at T = 8 (CSR-r16 is
not admissible there: after RCM a row spans up to 151,688 columns). The working set (1.2-1.4 GB) is ten
times the 126 MB L2, so no flush is needed between products.

Prints ONE JSON line on rank 0. `value` is device-timed whole-job GFLOP/s over exactly K back-to-back
products (CUDA events on the launching stream, barrier and synchronize on both sides, max over ranks);
`protocol` adds the same product timed with the reference's protocol (3 warm-ups, 20 samples of at least
10 ms, median). `e2e` is the same metric through the public API from pinned host memory: x copied in and y
copied out every step (at N GPUs each rank copies its 1/N slice of x and the slices are all-gathered over
NCCL). `roofline` relates the kernel's algorithmic bytes (the reference byte model, memory_of) per launch
to the measured HBM peak. `parity` is the headline y compared bit for bit with the CPU oracle's
reference-order CSR-i32 product at the same T (each rank its rows). `chained` is the block-FEM matrix
(n = 32M, 2.05 G nonzeros, FP32) row-sharded over the N GPUs, K chained products y -> x whose all-gather
runs inside the product over NVLink peer memory. At N = 1, `per_layout` sweeps every layout and T on the
stencil, the random band and the power-law matrix, `comparators` times cuSPARSE and the reference's own
kernels rebuilt for sm_100a on the same arrays, and `cpu_baseline` is the reference-order CSR-i32 product on
the host cores. `--impl reference` times that CPU implementation alone on the same workload and metric.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "spmv-index-compression_b200"))

import numpy as np  # noqa: E402

WORKLOADS = {
    "stencil27": "3D 27-point stencil 160^3, RCM-permuted, FP64, x U[-1,1] seed 2",
    "laplacian": "2D 5-point Laplacian 256^2, FP64, x U[-1,1] seed 0",
    "band": "random band n=1M, half-bandwidth 2000, Poisson(32)+diagonal, FP32, seed 1",
    "powerlaw": "power law n=8M, Zipf(1.8) row lengths in [1,100000] rescaled to mean 12, FP16, seed 3",
    "fem": "block FEM n=32M, 8x8 blocks, diagonal + 7 block-columns at offsets U[-50000,50000], FP32, seed 4",
}
DTYPE_OF = {"stencil27": "fp64", "laplacian": "fp64", "band": "fp32", "powerlaw": "fp16", "fem": "fp32"}
SEED_OF = {"stencil27": 2, "laplacian": 0, "band": 1, "powerlaw": 3, "fem": 4}
FEM_ROWS = 32_000_000
METRIC = "SpMV GFLOP/s & HBM GB/s (vs ~8 TB/s) per layout/T at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
SWEEP_TPR = {"stencil27": (8, 32), "band": (2, 4, 8, 16, 32), "powerlaw": (32,)}
SWEEP_LAYOUTS = {"stencil27": ("i32", "i16", "r16", "lp"), "band": ("i32", "i16", "r16", "lp"),
                 "powerlaw": ("i32", "i16", "r16", "lp")}


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--workload", choices=("stencil27", "laplacian", "band", "powerlaw", "fem"), default="stencil27",
                        help="the headline's matrix (fem: the block-FEM matrix of --fem-rows rows)")
    parser.add_argument("--layout", default="lp")
    parser.add_argument("--tpr", type=int, default=8)
    parser.add_argument("--physical-tpr", type=int, default=0)
    parser.add_argument("--tile-nnz", type=int, default=0)
    parser.add_argument("--fem-rows", type=int, default=FEM_ROWS,
                        help="chained: n of the block-FEM matrix (a multiple of 8; smaller n for quick runs)")
    parser.add_argument("--chain-layouts", default="i32,lp", help="chained: layouts, comma-separated")
    parser.add_argument("--chain-tpr", type=int, default=8)
    parser.add_argument("--chain-exchange", choices=("halo", "push"), default="halo",
                        help="chained: each product pulls only the entries of x its rows read from the other ranks "
                             "(halo), or stores its rows into every rank's next x (push)")
    parser.add_argument("--no-sweep", action="store_true",
                        help="skip the per-layout/T table and comparators (one GPU) or the sharded power-law leg (N GPUs)")
    parser.add_argument("--no-chained", action="store_true", help="skip the chained block-FEM products")
    parser.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline budget")
    return parser.parse_args()


# ---------------------------------------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------------------------------------
def build_matrix(spmv, workload):
    if workload == "stencil27":
        matrix = spmv.synth_stencil27(160)
        matrix = spmv.apply_symmetric_permutation(matrix, spmv.reverse_cuthill_mckee(matrix))
        matrix.name = "stencil27_160_rcm"
        return matrix
    if workload == "laplacian":
        return spmv.synth_laplacian2d(256)
    if workload == "band":
        return spmv.synth_random_band(1_000_000, 2000, 32.0, 1)
    if workload == "fem":
        return spmv.synth_block_fem(FEM_ROWS, 8, 8, 50_000, 4, 0, FEM_ROWS)
    return spmv.synth_power_law(8_000_000, 1.8, 100_000, 12.0, 3)


def fem_bounds(world):
    """Row shards of the block-FEM matrix: every row has 64 nonzeros, so equal block-aligned row ranges are
    nnz-balanced."""
    per_rank = (FEM_ROWS // 8 + world - 1) // world * 8
    return np.array([min(FEM_ROWS, rank * per_rank) for rank in range(world + 1)], dtype=np.int32)


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        peaks = json.load(open(path))
        return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs: copy read+write)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(workload, layout, tpr):
    """DRAM bytes read+written per launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.txt")
    if not os.path.exists(path):
        return None
    for line in open(path):
        fields = line.split()
        if len(fields) >= 4 and not line.startswith("#") and fields[:3] == [workload, layout, str(tpr)]:
            return float(fields[3])
    return None


def host_cores():
    """The host threads this process may run on (its affinity mask)."""
    return len(os.sched_getaffinity(0))


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of one GPU every 50 ms while active."""

    QUERY = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.process = None
        self.lines = []

    def start(self):
        try:
            self.process = subprocess.Popen(["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.QUERY}",
                                             "--format=csv,noheader,nounits", "-lms", "50"],
                                            stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            time.sleep(0.3)
        except OSError:
            self.process = None

    def _read(self):
        for line in self.process.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.process is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.process.terminate()
        try:
            self.process.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.process.kill()
        self.reader.join(timeout=2)
        sm, sm_max, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            fields = [field.strip() for field in line.split(",")]
            if len(fields) < 8:
                continue
            try:
                sm.append(float(fields[0]))
                sm_max.append(float(fields[1]))
                power.append(float(fields[2]))
            except ValueError:
                continue
            for name, flag in zip(names, fields[4:8]):
                if flag.lower() in ("active", "1", "yes"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(sm_max) if sm_max else None,
                "power_w_max": max(power) if power else None, "reasons": sorted(reasons), "samples": len(sm)}


def sampler_for(torch, local_rank):
    gpu_id = str(torch.cuda.get_device_properties(local_rank).uuid)
    return ClockSampler(gpu_id if gpu_id.startswith("GPU-") else f"GPU-{gpu_id}")


# ---------------------------------------------------------------------------------------------------------
# the oracle's legs: the CPU baseline, the reference arm, and the checker of the products (never timed,
# never the product: the oracle restates the reference's CSR-i32 kernel order on the host)
# ---------------------------------------------------------------------------------------------------------
def oracle_module(threads):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    oracle.set_threads(max(1, threads))   # a launcher's OMP_NUM_THREADS=1 would hold it to one core
    return oracle


def cpu_product_rate(matrix, dtype_code, tpr, seconds_budget, steps=None, warmup=0):
    """Times the CPU oracle's CSR-i32 product on every host thread of this process. With steps, times
    exactly that many samples after warmup, each a row block sized so the whole run fits the budget;
    otherwise as many full products as fit in the budget. Returns (GFLOP/s, description, cores)."""
    import spmvb200 as spmv
    cores = host_cores()
    oracle = oracle_module(cores)
    row_ptr, col_ind, values = matrix.arrays()
    x = spmv.fill_uniform(dtype_code, matrix.cols, 7)
    typed = oracle.convert_values(values, dtype_code)
    start = time.perf_counter()
    oracle.spmv(dtype_code, oracle.I32, tpr, row_ptr, typed, x, columns=col_ind, threads=cores)
    full = time.perf_counter() - start
    nnz = col_ind.size
    if steps is None:
        count = max(1, int(seconds_budget / max(full, 1e-6)))
        start = time.perf_counter()
        for _ in range(count):
            oracle.spmv(dtype_code, oracle.I32, tpr, row_ptr, typed, x, columns=col_ind, threads=cores)
        elapsed = time.perf_counter() - start
        return 2.0 * nnz * count / elapsed / 1e9, f"{count} full products of the workload", cores
    fraction = min(1.0, seconds_budget / max((steps + warmup) * full, 1e-9))
    rows = max(1, int(matrix.rows * fraction))
    sample_ptr = row_ptr[:rows + 1]
    sample_nnz = int(sample_ptr[-1])
    for _ in range(warmup):
        oracle.spmv(dtype_code, oracle.I32, tpr, sample_ptr, typed, x, columns=col_ind, threads=cores)
    start = time.perf_counter()
    for _ in range(steps):
        oracle.spmv(dtype_code, oracle.I32, tpr, sample_ptr, typed, x, columns=col_ind, threads=cores)
    elapsed = time.perf_counter() - start
    return (2.0 * sample_nnz * steps / elapsed / 1e9,
            f"rows [0, {rows}) of the workload ({sample_nnz} nonzeros, {100 * fraction:.2f}%) per step", cores)


def oracle_mismatches(row_ptr, col_ind, values, x, y, dtype_code, tpr, threads):
    """Rows of y that differ in any bit from the oracle's reference-order CSR-i32 product at T, and the
    largest absolute difference."""
    oracle = oracle_module(threads)
    want = oracle.spmv_csr(row_ptr, col_ind, values, x, dtype_code, oracle.I32, tpr, threads=threads)
    got = np.ascontiguousarray(y)
    differ = got.view(np.uint8).reshape(got.size, -1) != want.view(np.uint8).reshape(want.size, -1)
    rows = int(np.count_nonzero(differ.any(axis=1)))
    delta = np.abs(got.astype(np.float64) - want.astype(np.float64))
    delta = delta[np.isfinite(delta)]   # rows of inf or NaN are counted as mismatched by their bits alone
    return rows, float(delta.max()) if delta.size else 0.0


def run_reference(args, rank, world):
    import spmvb200 as spmv
    if rank != 0:
        return
    matrix = build_matrix(spmv, args.workload)
    dtype_code = spmv.DTYPE_BY_NAME[DTYPE_OF[args.workload]]
    budget = 120.0
    rate, sample, cores = cpu_product_rate(matrix, dtype_code, args.tpr, budget, steps=args.steps, warmup=args.warmup)
    line = {
        "metric": METRIC, "value": round(rate, 3), "unit": "GFLOP/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": DTYPE_OF[args.workload], "data": "synthetic",
        "config": {"workload": WORKLOADS[args.workload].replace("n=32M", f"n={FEM_ROWS}"), "layout": "i32",
                   "tpr": args.tpr, "rows": matrix.rows,
                   "nnz": matrix.nnz, "parallelism": f"host threads (OpenMP over rows), {cores} cores"},
        "cpu_baseline": {"value": round(rate, 3), "unit": "GFLOP/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(rate, 3), "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU SpMV; this is its CSR-i32 kernel order restated in C (oracle/spmv_oracle.c)",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------
# timing
# ---------------------------------------------------------------------------------------------------------
def event_ms(torch, stream, body, repeats):
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(repeats):
        body()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end)


def protocol_median_ms(torch, stream, body, samples=20, warmup=3, min_sample_ms=10.0):
    """The reference's protocol (bench_csr_width.cu:631-663): warm-ups, then samples of a batch of back-to-back
    products lasting at least min_sample_ms; median time of one product."""
    for _ in range(warmup):
        body()
    torch.cuda.synchronize()
    batch = 1
    while True:
        elapsed = event_ms(torch, stream, body, batch)
        if elapsed >= 0.25 * min_sample_ms or batch >= 1 << 20:
            break
        batch *= 4
    batch = int(min(1 << 20, max(1, np.ceil(batch * min_sample_ms / max(elapsed, 1e-3)))))
    times = [event_ms(torch, stream, body, batch) / batch for _ in range(samples)]
    return statistics.median(times), batch


class Ranks:
    """The job's process group (None on one GPU): barriers and reductions over the ranks."""

    def __init__(self, torch, dist, local_rank):
        self.torch, self.dist, self.local_rank = torch, dist, local_rank

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier(device_ids=[self.local_rank])
        self.torch.cuda.synchronize()

    def max(self, values):
        if self.dist is None:
            return list(values)
        tensor = self.torch.tensor(list(values), dtype=self.torch.float64, device=f"cuda:{self.local_rank}")
        self.dist.all_reduce(tensor, op=self.dist.ReduceOp.MAX)
        return tensor.tolist()

    def sum(self, values):
        if self.dist is None:
            return list(values)
        tensor = self.torch.tensor(list(values), dtype=self.torch.float64, device=f"cuda:{self.local_rank}")
        self.dist.all_reduce(tensor, op=self.dist.ReduceOp.SUM)
        return tensor.tolist()

    def gather_objects(self, item, world):
        if self.dist is None:
            return [item]
        out = [None] * world
        self.dist.all_gather_object(out, item)
        return out


# ---------------------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import spmvb200 as spmv
    dist = None
    if world > 1:
        import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    ranks = Ranks(torch, dist, local_rank)
    dtype_name = DTYPE_OF[args.workload]
    dtype_code = spmv.DTYPE_BY_NAME[dtype_name]
    torch_dtype = {"fp64": torch.float64, "fp32": torch.float32, "fp16": torch.float16}[dtype_name]
    layout = spmv.LAYOUT_BY_NAME[args.layout]
    value_bytes = spmv.VALUE_BYTES[dtype_code]
    threads = max(1, host_cores() // world)

    matrix = build_matrix(spmv, args.workload)
    total_nnz, rows, cols = matrix.nnz, matrix.rows, matrix.cols
    bounds = spmv.shard_rows(matrix, world)
    first, last = int(bounds[rank]), int(bounds[rank + 1])
    shard = matrix if world == 1 else matrix.slice_rows(first, last)
    facts = spmv.facts_of(shard)
    if not spmv.configuration_admissible(shard, facts, spmv.Configuration.of(layout, dtype_code, args.tpr)):
        raise SystemExit(f"layout {args.layout} at T={args.tpr} is not admissible for {args.workload}")
    op = spmv.Operator(shard, layout, dtype_code, args.tpr, physical_tpr=args.physical_tpr, tile_nnz=args.tile_nnz,
                       device=local_rank)
    info = op.info()
    algorithmic_bytes = info.memory.total
    x_host = spmv.fill_uniform(dtype_code, cols, SEED_OF[args.workload])
    x = torch.from_numpy(x_host).to(device)
    y = torch.empty(shard.rows, dtype=torch_dtype, device=device)
    launch = lambda: op.run(x.data_ptr(), y.data_ptr(), stream.cuda_stream)  # noqa: E731

    # warm-up, then exactly K timed products bracketed by barrier + synchronize
    for _ in range(args.warmup):
        launch()
    ranks.barrier()
    sampler = sampler_for(torch, local_rank)
    sampler.start()
    ranks.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        launch()
    end.record(stream)
    ranks.barrier()
    elapsed_ms = start.elapsed_time(end)
    op.check()
    (elapsed_ms,) = ranks.max([elapsed_ms])
    ms_per_step = elapsed_ms / args.steps
    value = 2.0 * total_nnz * args.steps / (elapsed_ms * 1e-3) / 1e9
    # the kernel is the only launch of a step: its average duration is the device time per step
    achieved_gbs = algorithmic_bytes / (ms_per_step * 1e-3) / 1e9

    # the same product under the reference's protocol (3 warm-ups, 20 samples of at least 10 ms); the clock
    # samples cover it too, since K products can take less than one sampling interval
    protocol_ms, protocol_batch = protocol_median_ms(torch, stream, launch)
    clocks = sampler.stop()
    clocks["window"] = "the timed products and the reference-protocol samples of the same product that follow them"
    (protocol_ms,) = ranks.max([protocol_ms])

    # parity: this rank's rows of y against the oracle's reference-order CSR-i32 product at the same T
    launch()
    torch.cuda.synchronize()
    y_host = y.cpu().numpy()
    s_ptr, s_col, s_val = shard.arrays()
    mismatched, max_abs = oracle_mismatches(s_ptr, s_col, s_val, x_host, y_host, dtype_code, args.tpr, threads)
    mismatched_total, = ranks.sum([mismatched])
    (max_abs,) = ranks.max([max_abs])
    parity = {"checked": True, "against": f"oracle reference-order CSR-i32 product at T={args.tpr} (oracle/spmv_oracle.c)",
              "rows": rows, "mismatched_rows": int(mismatched_total), "max_abs_diff": max_abs,
              "bit_identical": mismatched_total == 0}

    # end to end through the public API from pinned host buffers: every step copies its x in (at N GPUs each
    # rank its 1/N slice, all-gathered over NCCL) and its y out, overlapped with the neighbouring products
    x_pinned = torch.from_numpy(x_host).pin_memory()
    y_pinned = torch.empty(shard.rows, dtype=torch_dtype).pin_memory()
    e2e_steps = max(1, min(args.steps, 200))
    pitch = lambda count: (count * value_bytes + 15) // 16 * 16  # noqa: E731
    y_pair = torch.empty(2 * pitch(shard.rows), dtype=torch.uint8, device=device)
    comm = None
    if world == 1:
        x_pair = torch.empty(2 * pitch(cols), dtype=torch.uint8, device=device)
        batch = lambda steps: op.run_host_batch(x_pinned.data_ptr(), 0, y_pinned.data_ptr(), 0, steps,  # noqa: E731
                                                x_pair.data_ptr(), y_pair.data_ptr(), stream.cuda_stream)
    else:
        box = ranks.gather_objects(spmv.comm_unique_id() if rank == 0 else None, world)
        comm = spmv.Comm(world, rank, box[0], device=local_rank)
        slice_count = (cols + world - 1) // world
        x_pair = torch.empty(2 * pitch(slice_count * world), dtype=torch.uint8, device=device)
        batch = lambda steps: spmv.shard_run_host_batch(op, comm, x_pinned.data_ptr(), 0, y_pinned.data_ptr(), 0,  # noqa: E731
                                                        steps, x_pair.data_ptr(), y_pair.data_ptr(), stream.cuda_stream)
    batch(3)
    ranks.barrier()
    # the given stream waits for the last copy out, so its events bracket the whole batch
    e2e_ms = event_ms(torch, stream, lambda: batch(e2e_steps), 1)
    ranks.barrier()
    (e2e_ms,) = ranks.max([e2e_ms])
    e2e_value = 2.0 * total_nnz * e2e_steps / (e2e_ms * 1e-3) / 1e9
    if comm is not None:
        comm.check(stream.cuda_stream, 60000)
        comm.close()
    e2e_y_ok = bool(np.array_equal(y_pinned.numpy().view(np.uint8), y_host.view(np.uint8)))

    extras = {}
    chained = None
    if not args.no_chained:
        del x, y
        op.close()
        chained = chained_leg(args, torch, spmv, ranks, rank, world, local_rank, stream, threads)
    if world > 1 and not args.no_sweep:
        extras["sharded_powerlaw"] = sharded_leg(args, torch, spmv, ranks, rank, world, local_rank, stream, threads)
    if world == 1 and not args.no_sweep:
        extras = sweep(args, torch, spmv, matrix, dtype_code, torch_dtype, stream)
        rate, sample, cores = cpu_product_rate(matrix, dtype_code, args.tpr, args.cpu_seconds)
        extras["cpu_baseline"] = {"value": round(rate, 3), "unit": "GFLOP/s", "cores": cores, "kind": "port",
                                  "sample": sample + " (reference-order CSR-i32, oracle/spmv_oracle.c)"}
    if rank != 0:
        return
    peak, peak_source = measured_peak()
    # the committed ncu capture is of the whole matrix on one GPU; a shard's traffic was not captured
    traffic = profiled_traffic(args.workload, args.layout, args.tpr) if world == 1 else None
    # x gathers: one per nonzero; against the measured rate of random single-element gathers from an
    # array the size of x (the ceiling for scattered columns, where each element costs a 32-byte sector)
    gather_ceiling = spmv.gather_rate(cols, value_bytes, 10)
    gather_rate = total_nnz / (ms_per_step * 1e-3)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": dtype_name, "data": "synthetic",
        "config": {"workload": WORKLOADS[args.workload].replace("n=32M", f"n={FEM_ROWS}"), "layout": args.layout,
                   "tpr": args.tpr,
                   "physical_tpr": info.physical_tpr, "tile_nnz": info.tile_nnz, "rows": rows, "cols": cols,
                   "nnz": total_nnz, "parallelism": f"row shards x{world} (nnz-balanced, x replicated)",
                   "l2": f"no flush: working set {algorithmic_bytes / 1e9:.2f} GB per rank > 126 MB L2",
                   "schedule": "classes" if info.schedule == spmv.SCHEDULE_CLASSES else "tiles",
                   "tiles": info.tiles, "listed_rows": info.listed_rows, "long_rows": info.long_rows},
        "protocol": {"value": f"{args.steps} back-to-back products between CUDA events after {args.warmup} warm-ups",
                     "reference_protocol_ms": round(protocol_ms, 6), "reference_protocol_batch": protocol_batch,
                     "reference_protocol_gflops": round(2.0 * total_nnz / (protocol_ms * 1e-3) / 1e9, 3),
                     "reference_protocol": "3 warm-ups, 20 samples of back-to-back products lasting >= 10 ms, "
                                           "median (bench_csr_width.cu:631-663)"},
        "parity": parity,
        "effective_gbs": round(achieved_gbs * world, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "traffic": traffic, "peak_source": peak_source,
                     "kernel": "k_spmv_classes" if info.schedule == spmv.SCHEDULE_CLASSES else "k_spmv_tiles",
                     "algorithmic_bytes_per_launch": algorithmic_bytes,
                     "traffic_note": None if world == 1 else "per-shard DRAM traffic not captured"},
        "x_gathers": {"per_step": total_nnz, "achieved_per_s": round(gather_rate, 1),
                      "random_gather_ceiling_per_s": round(gather_ceiling, 1),
                      "frac": round(gather_rate / gather_ceiling, 4),
                      "note": "ceiling measured by spmv_gather_rate on an array of cols elements; above 1 means the "
                              "gathers reuse L1/L2 lines"},
        "clocks": clocks,
        "e2e": {"value": round(e2e_value, 3), "unit": "GFLOP/s", "h2d_bytes_per_step": cols * value_bytes,
                "d2h_bytes_per_step": rows * value_bytes, "steps": e2e_steps, "y_matches_device_run": e2e_y_ok,
                "path": "spmv_operator_run_host_batch" if world == 1 else
                        "spmv_shard_run_host_batch: each rank copies its 1/N slice of x, NCCL all-gather, product, "
                        "its rows of y out"},
        "gpu_launches": args.steps,
    }
    if chained is not None:
        line["chained"] = chained
    line.update(extras)
    print(json.dumps(line), flush=True)


def chained_leg(args, torch, spmv, ranks, rank, world, local_rank, stream, threads):
    """Config 5: the block-FEM matrix row-sharded over the ranks (each rank builds only its rows), K chained
    products y -> x over NVLink peer memory (spmv_chain_run_peer), each followed by a barrier of the GPUs.
    The exchange is the halo (each product pulls only the entries of the next x its rows read from the
    other ranks) or the push (each product stores its rows into every rank's next x). The product kernels
    alone are timed too, and two chained products are checked against the oracle on a block of each rank's
    rows whose columns reach into the previous rank's rows."""
    dtype = spmv.F32
    tpr = args.chain_tpr
    bounds = fem_bounds(world)
    first, last = int(bounds[rank]), int(bounds[rank + 1])
    started = time.time()
    shard = spmv.synth_block_fem(FEM_ROWS, 8, 8, 50_000, 4, first, last)
    facts = spmv.facts_of(shard)
    x_host = spmv.fill_uniform(dtype, FEM_ROWS, SEED_OF["fem"])
    group = spmv.PeerGroup(world, rank, x_host.nbytes, device=local_rank)
    if world > 1:
        group.open(ranks.gather_objects(group.export(), world))
    halo_entries = group.set_halo(shard, bounds) if args.chain_exchange == "halo" else None
    peak, _ = measured_peak()
    total_nnz = 64 * FEM_ROWS
    # the parity block: the first rows of this rank's shard; their columns reach into the previous rank's rows,
    # so their second chained product reads entries of the first that came through the exchange
    sample_rows = min(4096, last - first)
    sample = spmv.synth_block_fem(FEM_ROWS, 8, 8, 50_000, 4, first, first + sample_rows)
    s_ptr, s_col, s_val = sample.arrays()
    reach = (int(s_col.min()), int(s_col.max()) + 1)   # the entries of the first product the block reads
    around = spmv.synth_block_fem(FEM_ROWS, 8, 8, 50_000, 4, reach[0], reach[1])
    a_ptr, a_col, a_val = around.arrays()
    x_first = x_host.copy()
    x_first[reach[0]:reach[1]] = oracle_product(a_ptr, a_col, a_val, x_host, dtype, tpr, threads)
    x_second_block = oracle_product(s_ptr, s_col, s_val, x_first, dtype, tpr, threads)
    out = {"workload": WORKLOADS["fem"].replace("n=32M", f"n={FEM_ROWS}"), "rows": FEM_ROWS, "nnz": total_nnz,
           "tpr": tpr, "steps": args.steps, "warmup": args.warmup, "n_gpus": world, "exchange": args.chain_exchange,
           "parallelism": f"row shards x{world} (block-aligned, equal nonzeros); " + (
               f"each product pulls the {halo_entries} entries of the next x its rows read from the other ranks' memory"
               if args.chain_exchange == "halo" else
               "each product stores its rows into every rank's next x") + " over NVLink, after a barrier of the GPUs",
           "layouts": {}}
    if halo_entries is not None:
        out["halo_entries_per_rank"] = halo_entries
    y_alone = torch.empty(last - first, dtype=torch.float32, device=f"cuda:{local_rank}")
    for name in [item for item in args.chain_layouts.split(",") if item]:
        layout = spmv.LAYOUT_BY_NAME[name]
        if not spmv.configuration_admissible(shard, facts, spmv.Configuration.of(layout, dtype, tpr)):
            out["layouts"][name] = {"status": "not admissible"}
            continue
        op = spmv.Operator(shard, layout, dtype, tpr, device=local_rank)
        info = op.info()
        # two chained products from x0, a block of this rank's rows checked bit for bit against the oracle
        # (checked this early because the matrix is diagonally dominant: x grows by about 64 each product
        # and overflows FP32 within the timed products)
        group.write_x(x_host.ctypes.data, x_host.nbytes)
        ranks.barrier()
        spmv.chain_run_peer(op, group, bounds, 2, stream.cuda_stream, timeout_ms=60000)
        group.check()
        x_after = np.empty_like(x_host)
        group.read_x(x_after.ctypes.data, x_after.nbytes)
        got = x_after[first:first + sample_rows]
        mismatched = int(np.count_nonzero(got.view(np.uint32) != x_second_block.view(np.uint32)))
        delta = np.abs(got.astype(np.float64) - x_second_block.astype(np.float64))
        delta = delta[np.isfinite(delta)]
        max_abs = float(delta.max()) if delta.size else 0.0
        ranks.barrier()
        spmv.chain_run_peer(op, group, bounds, args.warmup, stream.cuda_stream, timeout_ms=60000)
        group.check()
        ranks.barrier()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        spmv.chain_run_peer(op, group, bounds, args.steps, stream.cuda_stream, timeout_ms=60000)
        end.record(stream)
        end.synchronize()
        group.check()
        chain_ms = start.elapsed_time(end)
        ranks.barrier()
        # the product kernels alone on this rank's rows, x held still (no exchange, no barrier)
        x_now = group.x(0)
        kernel_ms = event_ms(torch, stream, lambda: op.run(x_now, y_alone.data_ptr(), stream.cuda_stream),
                             args.steps) / args.steps
        op.check()
        chain_ms, kernel_ms, max_abs = ranks.max([chain_ms, kernel_ms, max_abs])
        (mismatched,) = ranks.sum([mismatched])
        ms_per_step = chain_ms / args.steps
        bytes_per_rank = info.memory.total
        out["layouts"][name] = {
            "status": "ok", "ms_per_step": round(ms_per_step, 6),
            "gflops": round(2.0 * total_nnz / (ms_per_step * 1e-3) / 1e9, 3),
            "kernel_ms": round(kernel_ms, 6), "exposed_exchange_ms": round(ms_per_step - kernel_ms, 6),
            "kernel_gbs_per_rank": round(bytes_per_rank / (kernel_ms * 1e-3) / 1e9, 1),
            "kernel_frac_per_rank": round(bytes_per_rank / (kernel_ms * 1e-3) / 1e9 / peak, 4),
            "physical_tpr": info.physical_tpr, "tile_nnz": info.tile_nnz,
            "gpu_launches_per_step": 3 if args.chain_exchange == "halo" and world > 1 else 2,
            "parity": {"checked": True, "rows_per_rank": sample_rows, "mismatched_rows": int(mismatched),
                       "max_abs_diff": max_abs, "bit_identical": mismatched == 0,
                       "against": f"oracle reference-order CSR-i32 products at T={tpr}: the second chained product "
                                  "from x0 on the first rows of each rank's shard, whose columns reach into the "
                                  "previous rank's rows"}}
        op.close()
    ranks.barrier()
    group.close()
    out["setup_s"] = round(time.time() - started, 1)
    return out


def sharded_leg(args, torch, spmv, ranks, rank, world, local_rank, stream, threads):
    """Config 4 at N GPUs: the power-law matrix (n = 8M, FP16) in nnz-balanced row shards, x replicated, CSR-i32
    and CSR-lp at T = 32 (rows by length); the product of every rank timed with the reference's protocol, max
    over ranks; each rank's rows checked bit for bit against the oracle."""
    matrix = build_matrix(spmv, "powerlaw")
    dtype = spmv.DTYPE_BY_NAME["fp16"]
    bounds = spmv.shard_rows(matrix, world)
    first, last = int(bounds[rank]), int(bounds[rank + 1])
    shard = matrix.slice_rows(first, last)
    x_host = spmv.fill_uniform(dtype, matrix.cols, SEED_OF["powerlaw"])
    x = torch.from_numpy(x_host).to(f"cuda:{local_rank}")
    y = torch.empty(shard.rows, dtype=torch.float16, device=f"cuda:{local_rank}")
    s_ptr, s_col, s_val = shard.arrays()
    out = {"workload": WORKLOADS["powerlaw"], "rows": matrix.rows, "nnz": matrix.nnz, "tpr": 32, "n_gpus": world,
           "parallelism": f"row shards x{world} (nnz-balanced, x replicated)", "layouts": {}}
    facts = spmv.facts_of(shard)
    for name in ("i32", "lp"):
        layout = spmv.LAYOUT_BY_NAME[name]
        if not spmv.configuration_admissible(shard, facts, spmv.Configuration.of(layout, dtype, 32)):
            out["layouts"][name] = {"status": "not admissible"}
            continue
        with spmv.Operator(shard, layout, dtype, 32, device=local_rank) as op:
            body = lambda: op.run(x.data_ptr(), y.data_ptr(), stream.cuda_stream)  # noqa: E731
            ranks.barrier()
            ms, batch = protocol_median_ms(torch, stream, body)
            body()
            torch.cuda.synchronize()
            op.check()
        mismatched, max_abs = oracle_mismatches(s_ptr, s_col, s_val, x_host, y.cpu().numpy(), dtype, 32, threads)
        ms, max_abs = ranks.max([ms, max_abs])
        (mismatched,) = ranks.sum([mismatched])
        out["layouts"][name] = {"status": "ok", "t_ms": round(ms, 6), "gflops": round(2.0 * matrix.nnz / (ms * 1e-3) / 1e9, 2),
                                "parity": {"checked": True, "rows": matrix.rows, "mismatched_rows": int(mismatched),
                                           "max_abs_diff": max_abs, "bit_identical": mismatched == 0}}
    return out


def oracle_product(row_ptr, col_ind, values, x, dtype_code, tpr, threads):
    """The oracle's reference-order CSR-i32 product at T (the checker of the chained products)."""
    oracle = oracle_module(threads)
    return oracle.spmv_csr(row_ptr, col_ind, values, x, dtype_code, oracle.I32, tpr, threads=threads)


def sweep(args, torch, spmv, stencil, dtype_code, torch_dtype, stream):
    """Every layout and T on the stencil, the random band and the power-law matrix with the reference's
    timing protocol, each layout's y compared bit for bit with CSR-i32's at the same T; cuSPARSE on each
    matrix and the reference's own kernels rebuilt for sm_100a on the stencil's arrays."""
    peak, _ = measured_peak()
    rows_out = []
    comparators = {}
    for workload in ("stencil27", "band", "powerlaw"):
        matrix = stencil if workload == "stencil27" else build_matrix(spmv, workload)
        dtype = spmv.DTYPE_BY_NAME[DTYPE_OF[workload]]
        tdtype = {"fp64": torch.float64, "fp32": torch.float32, "fp16": torch.float16}[DTYPE_OF[workload]]
        bits_type = {"fp64": torch.int64, "fp32": torch.int32, "fp16": torch.int16}[DTYPE_OF[workload]]
        facts = spmv.facts_of(matrix)
        x = torch.from_numpy(spmv.fill_uniform(dtype, matrix.cols, SEED_OF[workload])).cuda()
        y = torch.empty(matrix.rows, dtype=tdtype, device="cuda")
        for tpr in SWEEP_TPR[workload]:
            i32_ms, i32_bits = None, None
            for name in SWEEP_LAYOUTS[workload]:
                layout = spmv.LAYOUT_BY_NAME[name]
                configuration = spmv.Configuration.of(layout, dtype, tpr)
                memory = spmv.memory_of(matrix, facts, configuration)
                entry = {"matrix": workload, "layout": name, "tpr": tpr, "bytes": memory.total}
                if not spmv.configuration_admissible(matrix, facts, configuration):
                    entry["status"] = "not admissible"
                    rows_out.append(entry)
                    continue
                with spmv.Operator(matrix, layout, dtype, tpr) as op:
                    body = lambda: op.run(x.data_ptr(), y.data_ptr(), stream.cuda_stream)  # noqa: E731
                    ms, batch = protocol_median_ms(torch, stream, body)
                    body()
                    torch.cuda.synchronize()
                    op.check()
                    info = op.info()
                    if workload == "stencil27" and name in ("i32", "lp"):
                        comparators.setdefault("reference_sm100a", []).append(
                            reference_kernels(torch, spmv, op, matrix, dtype, layout, tpr, x, y, ms))
                    if workload == "band" and name == "r16":
                        comparators.setdefault("r16_controls", []).extend(
                            r16_controls(torch, spmv, op, matrix, dtype, tpr, x, ms, i32_bits, bits_type))
                bits = y.view(bits_type).clone()
                if name == "i32":
                    i32_ms, i32_bits = ms, bits
                gbs = memory.total / (ms * 1e-3) / 1e9
                entry.update(status="ok", physical_tpr=info.physical_tpr, tile_nnz=info.tile_nnz,
                             schedule="classes" if info.schedule == spmv.SCHEDULE_CLASSES else "tiles",
                             t_ms=round(ms, 6), batch=batch, gflops=round(2.0 * matrix.nnz / (ms * 1e-3) / 1e9, 2),
                             gbs=round(gbs, 1), frac=round(gbs / peak, 4),
                             speedup_vs_i32=round(i32_ms / ms, 4) if i32_ms else None,
                             bits_equal_i32=bool(torch.equal(bits, i32_bits)) if i32_bits is not None else None)
                rows_out.append(entry)
        comparators.setdefault("cusparse", {})[workload] = cusparse_comparator(torch, spmv, matrix, facts, dtype, tdtype,
                                                                                x, stream)
        del x, y
        if workload != "stencil27":
            del matrix
    return {"per_layout": rows_out, "comparators": comparators}


def cusparse_comparator(torch, spmv, matrix, facts, dtype, tdtype, x, stream):
    try:
        row_ptr, col_ind, values = matrix.arrays()
        import warnings
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            compute = torch.float32 if tdtype == torch.float16 else tdtype
            a = torch.sparse_csr_tensor(torch.from_numpy(row_ptr), torch.from_numpy(col_ind),
                                        torch.from_numpy(values).to(tdtype).to(compute), size=(matrix.rows, matrix.cols),
                                        device=x.device)
            xc = x.to(compute).unsqueeze(1)
            ms, batch = protocol_median_ms(torch, stream, lambda: torch.sparse.mm(a, xc))
            i32 = spmv.memory_of(matrix, facts, spmv.Configuration.of(spmv.I32, dtype, 8)).total
            out = {"via": "torch.sparse.mm (cusparseSpMV, int32 CSR)", "t_ms": round(ms, 6),
                   "gflops": round(2.0 * matrix.nnz / (ms * 1e-3) / 1e9, 2), "gbs": round(i32 / (ms * 1e-3) / 1e9, 1),
                   "compute": str(compute).replace("torch.", "")}
            del a
            return out
    except Exception as failure:  # the comparator is optional
        return {"error": str(failure)[:200]}


def r16_controls(torch, spmv, op, matrix, dtype, tpr, x, library_ms, i32_bits, bits_type):
    """The reference's control builds of CSR-r16 (bench_csr_width.cu:34-42: lane-major offsets, the same two to
    a 32-bit load, 32-bit offsets, the loop unrolled 16 times) launched on the r16 operator's arrays, each timed
    with the reference's protocol and its y compared bit for bit with CSR-i32's at the same T."""
    out = []
    arrays = op.arrays()
    lane = torch.from_numpy(spmv.encode_relative_lane(matrix, tpr).view(np.int16)).cuda()
    wide = torch.from_numpy(spmv.encode_relative(matrix, 4).view(np.int32)).cuda()
    facts = spmv.facts_of(matrix)
    base = spmv.memory_of(matrix, facts, spmv.Configuration.of(spmv.R16, dtype, tpr)).total
    for name, control in spmv.R16_CONTROLS.items():
        offsets = {"lane": lane, "pair": lane, "wide": wide}.get(name)
        y = torch.empty(matrix.rows, dtype=x.dtype, device="cuda")
        device = spmv.DeviceMatrix(rows=matrix.rows, cols=matrix.cols, nnz=matrix.nnz, row_ptr=arrays.row_ptr,
                                   columns=offsets.data_ptr() if offsets is not None else arrays.columns,
                                   row_base=arrays.row_base, values=arrays.values, x=x.data_ptr(), y=y.data_ptr())
        body = lambda: spmv.launch_r16_control(control, dtype, tpr, device, torch.cuda.current_stream().cuda_stream)  # noqa: E731
        ms, batch = protocol_median_ms(torch, torch.cuda.current_stream(), body)
        body()
        torch.cuda.synchronize()
        total = base + (2 * matrix.nnz if name == "wide" else 0)
        out.append({"control": name, "tpr": tpr, "t_ms": round(ms, 6), "batch": batch,
                    "gflops": round(2.0 * matrix.nnz / (ms * 1e-3) / 1e9, 2), "bytes": total,
                    "library_r16_t_ms": round(library_ms, 6), "library_speedup": round(ms / library_ms, 4),
                    "bits_equal_i32": bool(torch.equal(y.view(bits_type), i32_bits)) if i32_bits is not None else None})
        del y
    del lane, wide
    return out


def reference_kernels(torch, spmv, op, matrix, dtype, layout, tpr, x, y, library_ms):
    """The reference's launch<T> (bench_csr_width.cu:607-629) rebuilt for sm_100a from its own sources
    (oracle/_ref, built where the reference tree was present), timed with the same protocol on the
    operator's own device arrays, outside the product path; its y compared with the library's."""
    name = spmv.LAYOUT_NAMES[layout]
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        if not oracle.Reference.available():
            return {"layout": name, "tpr": tpr, "unavailable": "oracle/_ref/libspmvref.so is not built"}
        reference = oracle.Reference()
        arrays = op.arrays()
        mine = y.clone()
        theirs = torch.zeros_like(y)
        call = lambda: reference.launch_async(dtype, layout, tpr, matrix.rows, matrix.cols, matrix.nnz,  # noqa: E731
                                              arrays.row_ptr, arrays.columns, arrays.row_base, arrays.row_word,
                                              arrays.row_width, arrays.words, arrays.values, x.data_ptr(),
                                              theirs.data_ptr())
        ms, batch = protocol_median_ms(torch, torch.cuda.default_stream(), call)
        torch.cuda.synchronize()
        peak, _ = measured_peak()
        memory = op.info().memory.total
        return {"layout": name, "tpr": tpr, "t_ms": round(ms, 6), "batch": batch,
                "gflops": round(2.0 * matrix.nnz / (ms * 1e-3) / 1e9, 2),
                "frac": round(memory / (ms * 1e-3) / 1e9 / peak, 4),
                "bits_equal_library": bool(torch.equal(mine.view(torch.int64) if mine.dtype == torch.float64 else mine,
                                                       theirs.view(torch.int64) if theirs.dtype == torch.float64 else theirs)),
                "library_t_ms": round(library_ms, 6), "library_speedup": round(ms / library_ms, 4)}
    except Exception as failure:  # the comparator is optional
        return {"layout": name, "tpr": tpr, "error": str(failure)[:200]}


def main():
    global FEM_ROWS
    args = parse_args()
    if args.fem_rows <= 0 or args.fem_rows % 8:
        raise SystemExit("--fem-rows must be a positive multiple of 8")
    FEM_ROWS = args.fem_rows
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        cpus = host_cores()
        os.environ.setdefault("SPMV_HOST_THREADS", str(max(1, cpus // world)))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
        try:
            run_ours(args, rank, world, local_rank)
        finally:
            dist.destroy_process_group()
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
