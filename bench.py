#!/usr/bin/env python3
"""bench.py — CSR SpMV with compressed column indices on B200: GFLOP/s (2·nnz/t) and effective HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload stencil27]
                    [--layout lp] [--tpr 8] [--no-sweep]

A step is one product y = A x over the whole matrix (at N GPUs: every rank its nnz-balanced row shard,
x replicated, no exchange — the products are independent). The default workload is the 3D 27-point
stencil on 160^3 (n = 4,096,000, nnz = 109,215,352, diagonal 26, neighbours -1) in lexicographic order,
then RCM-permuted; FP64; x uniform [-1, 1] from seed 2; the headline layout is CSR-lp at T = 8 (CSR-r16 is
not admissible there: after RCM a row spans up to 151,688 columns). The working set (1.2-1.4 GB) is ten
times the 126 MB L2, so no flush is needed between products.

Prints ONE JSON line on rank 0. `value` is device-timed whole-job GFLOP/s (CUDA events, barrier and
synchronize on both sides, max over ranks); `e2e` is the same metric through the public API from pinned
host memory (x copied in and y copied out every step); `roofline` relates the kernel's algorithmic bytes
(the reference byte model, memory_of) per launch to the measured HBM peak; `cpu_baseline` is the
reference-order CSR-i32 product on the host cores (the CPU oracle, a restatement of the reference kernel).
`--impl reference` times that CPU implementation alone on the same workload and metric.
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
    "fem": "block FEM n=32M, 8x8 blocks, diagonal + 7 block-columns at offsets U[-50000,50000], FP32, seed 4; "
           "chained products y -> x with an NCCL all-gather of y",
}
DTYPE_OF = {"stencil27": "fp64", "laplacian": "fp64", "band": "fp32", "powerlaw": "fp16", "fem": "fp32"}
SEED_OF = {"stencil27": 2, "laplacian": 0, "band": 1, "powerlaw": 3, "fem": 4}
FEM_ROWS = 32_000_000
METRIC = "SpMV GFLOP/s & HBM GB/s (vs ~8 TB/s) per layout/T at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default="stencil27")
    parser.add_argument("--layout", default="lp")
    parser.add_argument("--tpr", type=int, default=8)
    parser.add_argument("--physical-tpr", type=int, default=0)
    parser.add_argument("--tile-nnz", type=int, default=0)
    parser.add_argument("--fem-rows", type=int, default=FEM_ROWS,
                        help="fem: n of the block-FEM matrix (a multiple of 8; smaller n for profiling captures)")
    parser.add_argument("--blocks-per-rank", type=int, default=0,
                        help="fem: interleaved row blocks per rank whose all-gathers overlap the next block's "
                             "product (0: 4 on more than one GPU, else 1; 1: one shard and spmv_chain_run)")
    parser.add_argument("--no-sweep", action="store_true", help="skip the per-layout/T table and comparators")
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


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of one GPU every 100 ms while active."""

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
                                             "--format=csv,noheader,nounits", "-lms", "100"],
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


# ---------------------------------------------------------------------------------------------------------
# the reference arm: the reference-order CPU product (the oracle)
# ---------------------------------------------------------------------------------------------------------
def cpu_product_rate(matrix, dtype_code, tpr, seconds_budget, steps=None, warmup=0):
    """Times the CPU oracle's CSR-i32 product on all host threads. With steps, times exactly that many
    samples after warmup, each a row block sized so the whole run fits the budget; otherwise as many full
    products as fit in the budget. Returns (GFLOP/s, description, cores)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import spmvb200 as spmv
    row_ptr, col_ind, values = matrix.arrays()
    x = spmv.fill_uniform(dtype_code, matrix.cols, 7)
    typed = oracle.convert_values(values, dtype_code)
    cores = oracle.max_threads()
    start = time.perf_counter()
    oracle.spmv(dtype_code, oracle.I32, tpr, row_ptr, typed, x, columns=col_ind)
    full = time.perf_counter() - start
    nnz = col_ind.size
    if steps is None:
        count = max(1, int(seconds_budget / max(full, 1e-6)))
        start = time.perf_counter()
        for _ in range(count):
            oracle.spmv(dtype_code, oracle.I32, tpr, row_ptr, typed, x, columns=col_ind)
        elapsed = time.perf_counter() - start
        return 2.0 * nnz * count / elapsed / 1e9, f"{count} full products of the workload", cores
    fraction = min(1.0, seconds_budget / max((steps + warmup) * full, 1e-9))
    rows = max(1, int(matrix.rows * fraction))
    sample_ptr = row_ptr[:rows + 1]
    sample_nnz = int(sample_ptr[-1])
    for _ in range(warmup):
        oracle.spmv(dtype_code, oracle.I32, tpr, sample_ptr, typed, x, columns=col_ind)
    start = time.perf_counter()
    for _ in range(steps):
        oracle.spmv(dtype_code, oracle.I32, tpr, sample_ptr, typed, x, columns=col_ind)
    elapsed = time.perf_counter() - start
    return (2.0 * sample_nnz * steps / elapsed / 1e9,
            f"rows [0, {rows}) of the workload ({sample_nnz} nonzeros, {100 * fraction:.2f}%) per step", cores)


def run_reference(args, rank, world):
    import spmvb200 as spmv
    if rank != 0:
        return
    if args.workload == "fem":   # a row range of the 2.05 G-nonzero matrix stands in (host memory)
        matrix = spmv.synth_block_fem(FEM_ROWS, 8, 8, 50_000, 4, 0, min(FEM_ROWS, 2_000_000))
    else:
        matrix = build_matrix(spmv, args.workload)
    dtype_code = spmv.DTYPE_BY_NAME[DTYPE_OF[args.workload]]
    budget = 120.0
    rate, sample, cores = cpu_product_rate(matrix, dtype_code, args.tpr, budget, steps=args.steps, warmup=args.warmup)
    line = {
        "metric": METRIC, "value": round(rate, 3), "unit": "GFLOP/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": DTYPE_OF[args.workload], "data": "synthetic",
        "config": {"workload": WORKLOADS[args.workload], "layout": "i32", "tpr": args.tpr, "rows": matrix.rows,
                   "nnz": matrix.nnz, "parallelism": "host threads (OpenMP over rows)"},
        "cpu_baseline": {"value": round(rate, 3), "unit": "GFLOP/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(rate, 3), "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU SpMV; this is its CSR-i32 kernel order restated in C (oracle/spmv_oracle.c)",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------------------
# our arm
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


def run_ours(args, rank, world, local_rank):
    if args.workload == "fem":
        run_fem(args, rank, world, local_rank)
        return
    import torch
    import spmvb200 as spmv
    dist = None
    if world > 1:
        import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    dtype_name = DTYPE_OF[args.workload]
    dtype_code = spmv.DTYPE_BY_NAME[dtype_name]
    torch_dtype = {"fp64": torch.float64, "fp32": torch.float32, "fp16": torch.float16}[dtype_name]
    layout = spmv.LAYOUT_BY_NAME[args.layout]

    matrix = build_matrix(spmv, args.workload)
    total_nnz, rows, cols = matrix.nnz, matrix.rows, matrix.cols
    bounds = spmv.shard_rows(matrix, world)
    shard = matrix if world == 1 else matrix.slice_rows(int(bounds[rank]), int(bounds[rank + 1]))
    facts = spmv.facts_of(shard)
    admissible = spmv.configuration_admissible(shard, facts, spmv.Configuration.of(layout, dtype_code, args.tpr))
    if not admissible:
        raise SystemExit(f"layout {args.layout} at T={args.tpr} is not admissible for {args.workload}")
    op = spmv.Operator(shard, layout, dtype_code, args.tpr, physical_tpr=args.physical_tpr, tile_nnz=args.tile_nnz,
                       device=local_rank)
    info = op.info()
    algorithmic_bytes = info.memory.total
    x_host = spmv.fill_uniform(dtype_code, cols, SEED_OF[args.workload])
    x = torch.from_numpy(x_host).to(device)
    y = torch.empty(shard.rows, dtype=torch_dtype, device=device)
    launch = lambda: op.run(x.data_ptr(), y.data_ptr(), stream.cuda_stream)  # noqa: E731

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    # warm-up, then exactly K timed products bracketed by barrier + synchronize
    for _ in range(args.warmup):
        launch()
    barrier()
    gpu_id = torch.cuda.get_device_properties(local_rank).uuid
    sampler = ClockSampler(f"GPU-{gpu_id}" if not str(gpu_id).startswith("GPU-") else str(gpu_id))
    sampler.start()
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        launch()
    end.record(stream)
    barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(end)
    op.check()
    if dist is not None:
        timing = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
        dist.all_reduce(timing, op=dist.ReduceOp.MAX)
        elapsed_ms = timing.item()
    ms_per_step = elapsed_ms / args.steps
    value = 2.0 * total_nnz * args.steps / (elapsed_ms * 1e-3) / 1e9
    # the kernel is the only launch of a step: its average duration is the device time per step
    achieved_gbs = algorithmic_bytes / (ms_per_step * 1e-3) / 1e9

    # end to end through the public API from pinned host buffers: copy x in, multiply, copy y out, wait
    value_bytes = spmv.VALUE_BYTES[dtype_code]
    x_pinned = torch.from_numpy(x_host).pin_memory()
    y_pinned = torch.empty(shard.rows, dtype=torch_dtype).pin_memory()
    # a stream of e2e_steps products through spmv_operator_run_host_batch: every step copies its x in from
    # pinned host memory and its y out, overlapped with the products of the neighbouring steps
    e2e_steps = max(1, min(args.steps, 200))
    pitch = lambda count: (count * value_bytes + 15) // 16 * 16  # noqa: E731
    x_pair = torch.empty(2 * pitch(cols), dtype=torch.uint8, device=device)
    y_pair = torch.empty(2 * pitch(shard.rows), dtype=torch.uint8, device=device)
    batch = lambda steps: op.run_host_batch(x_pinned.data_ptr(), 0, y_pinned.data_ptr(), 0, steps,  # noqa: E731
                                            x_pair.data_ptr(), y_pair.data_ptr(), stream.cuda_stream)
    batch(3)
    barrier()
    # the given stream waits for the last copy out, so its events bracket the whole batch
    e2e_ms = event_ms(torch, stream, lambda: batch(e2e_steps), 1)
    barrier()
    if dist is not None:
        timing = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
        dist.all_reduce(timing, op=dist.ReduceOp.MAX)
        e2e_ms = timing.item()
    e2e_value = 2.0 * total_nnz * e2e_steps / (e2e_ms * 1e-3) / 1e9

    extras = {}
    if world == 1 and not args.no_sweep:
        extras = sweep(args, torch, spmv, matrix, dtype_code, torch_dtype, x, stream)
        rate, sample, cores = cpu_product_rate(matrix, dtype_code, args.tpr, args.cpu_seconds)
        extras["cpu_baseline"] = {"value": round(rate, 3), "unit": "GFLOP/s", "cores": cores, "kind": "port",
                                  "sample": sample + " (reference-order CSR-i32, oracle/spmv_oracle.c)"}
    if rank != 0:
        return
    peak, peak_source = measured_peak()
    traffic = profiled_traffic(args.workload, args.layout, args.tpr)
    # x gathers: one per nonzero; against the measured rate of random single-element gathers from an
    # array the size of x (the ceiling for scattered columns, where each element costs a 32-byte sector)
    gather_ceiling = spmv.gather_rate(cols, value_bytes, 10)
    gather_rate = total_nnz / (ms_per_step * 1e-3)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": dtype_name, "data": "synthetic",
        "config": {"workload": WORKLOADS[args.workload], "layout": args.layout, "tpr": args.tpr,
                   "physical_tpr": info.physical_tpr, "tile_nnz": info.tile_nnz, "rows": rows, "cols": cols,
                   "nnz": total_nnz, "parallelism": f"row shards x{world} (nnz-balanced, x replicated)",
                   "l2": f"no flush: working set {algorithmic_bytes * world / 1e9:.2f} GB > 126 MB L2",
                   "schedule": "classes" if info.schedule == spmv.SCHEDULE_CLASSES else "tiles",
                   "tiles": info.tiles, "listed_rows": info.listed_rows, "long_rows": info.long_rows},
        "effective_gbs": round(achieved_gbs * world, 1),
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "traffic": traffic, "peak_source": peak_source,
                     "kernel": "k_spmv_classes" if info.schedule == spmv.SCHEDULE_CLASSES else "k_spmv_tiles",
                     "algorithmic_bytes_per_launch": algorithmic_bytes},
        "x_gathers": {"per_step": total_nnz, "achieved_per_s": round(gather_rate, 1),
                      "random_gather_ceiling_per_s": round(gather_ceiling, 1),
                      "frac": round(gather_rate / gather_ceiling, 4),
                      "note": "ceiling measured by spmv_gather_rate on an array of cols elements; above 1 means the "
                              "gathers reuse L1/L2 lines"},
        "clocks": clocks,
        "e2e": {"value": round(e2e_value, 3), "unit": "GFLOP/s", "h2d_bytes_per_step": cols * value_bytes * world,
                "d2h_bytes_per_step": rows * value_bytes, "steps": e2e_steps},
        "gpu_launches": args.steps,
    }
    line.update(extras)
    print(json.dumps(line), flush=True)


def run_fem(args, rank, world, local_rank):
    """The block-FEM matrix row-sharded over the ranks (each rank builds only its rows), a step is one
    chained product. On one shard per rank (spmv_chain_run): every rank's shard product into its slice of
    the next x, then the slices all-gathered over NCCL. On interleaved row blocks (spmv_chain_run_blocks,
    the default on more than one GPU): rank r holds blocks c * world + r of 32M / (world * C) rows, and each
    round of blocks is all-gathered while the next block computes. The kernel alone is also timed for the
    roofline."""
    import torch
    import spmvb200 as spmv
    dist = None
    if world > 1:
        import torch.distributed as dist
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(device)
    dtype_code = spmv.DTYPE_BY_NAME["fp32"]
    layout = spmv.LAYOUT_BY_NAME[args.layout]
    blocks_per_rank = args.blocks_per_rank or (4 if world > 1 else 1)
    total_nnz = 64 * FEM_ROWS
    if blocks_per_rank == 1:
        bounds = fem_bounds(world)
        ranges = [(int(bounds[rank]), int(bounds[rank + 1]))]
    else:
        block_rows = FEM_ROWS // (world * blocks_per_rank)
        if block_rows * world * blocks_per_rank != FEM_ROWS or block_rows % 8:
            raise SystemExit(f"{FEM_ROWS} rows do not divide into {world * blocks_per_rank} blocks of whole 8x8 blocks")
        ranges = [((c * world + rank) * block_rows, (c * world + rank + 1) * block_rows) for c in range(blocks_per_rank)]
    ops = []
    for first, last in ranges:
        shard = spmv.synth_block_fem(FEM_ROWS, 8, 8, 50_000, 4, first, last)
        facts = spmv.facts_of(shard)
        if not spmv.configuration_admissible(shard, facts, spmv.Configuration.of(layout, dtype_code, args.tpr)):
            raise SystemExit(f"layout {args.layout} at T={args.tpr} is not admissible for fem")
        ops.append(spmv.Operator(shard, layout, dtype_code, args.tpr, physical_tpr=args.physical_tpr,
                                 tile_nnz=args.tile_nnz, device=local_rank))
        del shard
    info = ops[0].info()
    algorithmic_bytes = sum(op.info().memory.total for op in ops)
    box = [spmv.comm_unique_id() if rank == 0 else None]
    if dist is not None:
        dist.broadcast_object_list(box, src=0)
    comm = spmv.Comm(world, rank, box[0], device=local_rank)
    x_host = spmv.fill_uniform(dtype_code, FEM_ROWS, SEED_OF["fem"])
    x_current = torch.from_numpy(x_host).to(device)
    x_next = torch.zeros_like(x_current)
    y_alone = torch.empty(max(last - first for first, last in ranges), dtype=torch.float32, device=device)

    def barrier():
        if dist is not None:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize()

    if blocks_per_rank == 1:
        chain = lambda count: spmv.chain_run(ops[0], comm, bounds, x_current.data_ptr(), x_next.data_ptr(),  # noqa: E731
                                             count, stream.cuda_stream)
    else:
        chain = lambda count: spmv.chain_run_blocks(ops, block_rows, comm, x_current.data_ptr(),  # noqa: E731
                                                    x_next.data_ptr(), count, stream.cuda_stream)
    chain(args.warmup)
    comm.check(stream.cuda_stream, 120000)
    barrier()
    gpu_id = torch.cuda.get_device_properties(local_rank).uuid
    sampler = ClockSampler(f"GPU-{gpu_id}" if not str(gpu_id).startswith("GPU-") else str(gpu_id))
    sampler.start()
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    chain(args.steps)
    end.record(stream)
    comm.check(stream.cuda_stream, 120000)
    barrier()
    clocks = sampler.stop()
    elapsed_ms = start.elapsed_time(end)

    # the product kernels alone on this rank's rows (x held still), for the roofline
    def products_alone():
        for op in ops:
            op.run(x_current.data_ptr(), y_alone.data_ptr(), stream.cuda_stream)
    kernel_steps = max(3, min(args.steps, 50))
    kernel_ms = event_ms(torch, stream, products_alone, kernel_steps)
    for op in ops:
        op.check()
    # end to end: x in from pinned host memory, one chained product, this rank's new rows of x out
    x_pinned = torch.from_numpy(x_host).pin_memory()
    own_rows = sum(last - first for first, last in ranges)
    y_pinned = torch.empty(own_rows, dtype=torch.float32).pin_memory()
    e2e_steps = max(1, min(args.steps, 10))

    def e2e_step():
        x_current.copy_(x_pinned, non_blocking=True)
        chain(1)
        offset = 0
        for first, last in ranges:
            y_pinned[offset:offset + last - first].copy_(x_next[first:last], non_blocking=True)
            offset += last - first
    barrier()
    e2e_ms = event_ms(torch, stream, e2e_step, e2e_steps)
    comm.check(stream.cuda_stream, 120000)
    barrier()
    times = torch.tensor([elapsed_ms, kernel_ms, e2e_ms], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed_ms, kernel_ms, e2e_ms = times.tolist()
    comm.close()
    if rank != 0:
        return
    ms_per_step = elapsed_ms / args.steps
    kernel_ms_per_launch = kernel_ms / kernel_steps
    achieved_gbs = algorithmic_bytes / (kernel_ms_per_launch * 1e-3) / 1e9
    peak, peak_source = measured_peak()
    if blocks_per_rank == 1:
        parallelism = (f"row shards x{world} (block-aligned, nnz-balanced), NCCL all-gather of y between chained "
                       "products")
    else:
        parallelism = (f"interleaved row blocks x{world * blocks_per_rank} ({blocks_per_rank} per rank, "
                       f"{block_rows} rows each), each round's NCCL all-gather beside the next block's product")
    line = {
        "metric": METRIC, "value": round(2.0 * total_nnz * args.steps / (elapsed_ms * 1e-3) / 1e9, 3), "unit": "GFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": WORKLOADS["fem"].replace("n=32M", f"n={FEM_ROWS}") if FEM_ROWS != 32_000_000
                   else WORKLOADS["fem"], "layout": args.layout, "tpr": args.tpr, "rows": FEM_ROWS,
                   "nnz": total_nnz, "parallelism": parallelism,
                   "l2": f"no flush: {algorithmic_bytes / 1e9:.2f} GB per rank > 126 MB L2",
                   "physical_tpr": info.physical_tpr, "tile_nnz": info.tile_nnz,
                   "tiles": sum(op.info().tiles for op in ops)},
        "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved_gbs / peak, 4), "traffic": None, "peak_source": peak_source,
                     "kernel": "k_spmv_tiles", "algorithmic_bytes_per_launch": algorithmic_bytes // len(ops),
                     "kernel_ms": round(kernel_ms_per_launch / len(ops), 6)},
        "clocks": clocks,
        "e2e": {"value": round(2.0 * total_nnz * e2e_steps / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GFLOP/s",
                "h2d_bytes_per_step": FEM_ROWS * 4 * world, "d2h_bytes_per_step": FEM_ROWS * 4, "steps": e2e_steps},
        "gpu_launches": args.steps * len(ops),
    }
    for op in ops:
        op.close()
    print(json.dumps(line), flush=True)


def sweep(args, torch, spmv, matrix, dtype_code, torch_dtype, x, stream):
    """Every layout at T = 8 and 32 with the reference's timing protocol, and cuSPARSE on the same matrix."""
    peak, _ = measured_peak()
    facts = spmv.facts_of(matrix)
    rows = []
    i32_ms = {}
    y = torch.empty(matrix.rows, dtype=torch_dtype, device=x.device)
    for tpr in (8, 32):
        for name in ("i32", "i16", "r16", "lp"):
            layout = spmv.LAYOUT_BY_NAME[name]
            configuration = spmv.Configuration.of(layout, dtype_code, tpr)
            memory = spmv.memory_of(matrix, facts, configuration)
            entry = {"layout": name, "tpr": tpr, "bytes": memory.total}
            if not spmv.configuration_admissible(matrix, facts, configuration):
                entry["status"] = "not admissible"
                rows.append(entry)
                continue
            with spmv.Operator(matrix, layout, dtype_code, tpr) as op:
                ms, batch = protocol_median_ms(torch, stream, lambda: op.run(x.data_ptr(), y.data_ptr(), stream.cuda_stream))
                entry.update(status="ok", physical_tpr=op.info().physical_tpr, tile_nnz=op.info().tile_nnz,
                             schedule="classes" if op.info().schedule == spmv.SCHEDULE_CLASSES else "tiles",
                             t_ms=round(ms, 6), batch=batch,
                             gflops=round(2.0 * matrix.nnz / (ms * 1e-3) / 1e9, 2),
                             gbs=round(memory.total / (ms * 1e-3) / 1e9, 1),
                             frac=round(memory.total / (ms * 1e-3) / 1e9 / peak, 4))
            if name == "i32":
                i32_ms[tpr] = ms
            entry["speedup_vs_i32"] = round(i32_ms[tpr] / entry["t_ms"], 4) if tpr in i32_ms else None
            rows.append(entry)
    comparators = {}
    try:
        row_ptr, col_ind, values = matrix.arrays()
        import warnings
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            compute = torch.float32 if torch_dtype == torch.float16 else torch_dtype
            a = torch.sparse_csr_tensor(torch.from_numpy(row_ptr), torch.from_numpy(col_ind),
                                        torch.from_numpy(values).to(torch_dtype).to(compute), size=(matrix.rows, matrix.cols),
                                        device=x.device)
            xc = x.to(compute).unsqueeze(1)
            ms, batch = protocol_median_ms(torch, stream, lambda: torch.sparse.mm(a, xc))
            i32 = spmv.memory_of(matrix, facts, spmv.Configuration.of(spmv.I32, dtype_code, 8)).total
            comparators["cusparse"] = {"via": "torch.sparse.mm (cusparseSpMV, int32 CSR)", "t_ms": round(ms, 6),
                                       "gflops": round(2.0 * matrix.nnz / (ms * 1e-3) / 1e9, 2),
                                       "gbs": round(i32 / (ms * 1e-3) / 1e9, 1)}
            del a
    except Exception as failure:  # the comparator is optional
        comparators["cusparse"] = {"error": str(failure)[:200]}
    return {"per_layout": rows, "comparators": comparators}


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
        cpus = len(os.sched_getaffinity(0))
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
