"""The multi-GPU host logic on CPU ranks (gloo, world size 2): nnz-balanced row shards, each rank's shard
product (the oracle stands in for the GPU), the all-gather of unequal shards into the next x, chained
products, the interleaved row blocks whose rounds are all-gathered one by one, and a rank that leaves
before a collective being detected by the other rank's timeout."""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def free_port():
    with socket.socket() as probe:
        probe.bind(("127.0.0.1", 0))
        return probe.getsockname()[1]


def setup(rank, world, port, seconds=60):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "spmv-index-compression_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=seconds))


def gather_shards(y_shard, bounds):
    """All-gather of unequal shards: pad to the largest, gather, keep each rank's rows."""
    world = len(bounds) - 1
    counts = np.diff(bounds)
    padded = torch.zeros(int(counts.max()), dtype=torch.float64)
    padded[:y_shard.size] = torch.from_numpy(y_shard)
    pieces = [torch.zeros_like(padded) for _ in range(world)]
    dist.all_gather(pieces, padded)
    return np.concatenate([pieces[r][:counts[r]].numpy() for r in range(world)])


def chained_worker(rank, world, port):
    setup(rank, world, port)
    import oracle
    import spmvb200 as spmv
    matrix = spmv.synth_random_band(4000, 300, 10.0, 1)
    bounds = spmv.shard_rows(matrix, world)
    row_ptr, col_ind, values = matrix.arrays()
    counts = np.diff(row_ptr[bounds])
    assert abs(int(counts[0]) - int(counts[1])) <= 2 * int(np.diff(row_ptr).max())
    shard = matrix.slice_rows(int(bounds[rank]), int(bounds[rank + 1]))
    s_ptr, s_col, s_val = shard.arrays()
    x = spmv.fill_uniform(spmv.F64, matrix.cols, 5)
    expected = x.copy()
    for _ in range(3):
        expected = oracle.spmv_csr(row_ptr, col_ind, values, expected, spmv.F64, spmv.LP, 8)
        y_shard = oracle.spmv_csr(s_ptr, s_col, s_val, x, spmv.F64, spmv.LP, 8)
        x = gather_shards(y_shard, bounds)
    assert np.array_equal(x.view(np.uint64), expected.view(np.uint64))
    dist.destroy_process_group()


def interleaved_worker(rank, world, port):
    """spmv_chain_run_blocks' exchange: rank r holds blocks c * world + r; after each of its blocks, the
    round of blocks c * world .. c * world + world - 1 is all-gathered into its place in the next x."""
    setup(rank, world, port)
    import oracle
    import spmvb200 as spmv
    blocks_per_rank, block_rows = 3, 500
    n = world * blocks_per_rank * block_rows
    matrix = spmv.synth_random_band(n, 200, 9.0, 2)
    row_ptr, col_ind, values = matrix.arrays()
    mine = spmv.interleaved_block_rows(row_ptr, col_ind, values, world, blocks_per_rank, rank)
    x = spmv.fill_uniform(spmv.F64, n, 6)
    expected = x.copy()
    for _ in range(3):
        expected = oracle.spmv_csr(row_ptr, col_ind, values, expected, spmv.F64, spmv.LP, 8)
        x_next = np.zeros_like(x)
        for c, (b_ptr, b_col, b_val) in enumerate(mine):
            y_block = oracle.spmv_csr(b_ptr, b_col, b_val, x, spmv.F64, spmv.LP, 8)
            pieces = [torch.zeros(block_rows, dtype=torch.float64) for _ in range(world)]
            dist.all_gather(pieces, torch.from_numpy(y_block))
            first = c * world * block_rows
            x_next[first:first + world * block_rows] = np.concatenate([piece.numpy() for piece in pieces])
        x = x_next
    assert np.array_equal(x.view(np.uint64), expected.view(np.uint64))
    dist.destroy_process_group()


def leaving_worker(rank, world, port):
    setup(rank, world, port, seconds=5)
    if rank == 1:
        os._exit(0)   # leaves between steps, before the collective, with nothing in flight
    try:
        dist.all_reduce(torch.ones(1))
        raise AssertionError("the collective completed without the other rank")
    except RuntimeError:
        pass          # the timeout (or the closed connection) is reported, not a hang


def test_sharded_chained_products_match_the_whole_matrix():
    mp.spawn(chained_worker, args=(2, free_port()), nprocs=2, join=True)


def test_interleaved_row_blocks_match_the_whole_matrix():
    mp.spawn(interleaved_worker, args=(2, free_port()), nprocs=2, join=True)


def test_a_rank_that_leaves_is_detected_by_timeout():
    mp.spawn(leaving_worker, args=(2, free_port()), nprocs=2, join=True)
