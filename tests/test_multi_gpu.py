"""Chained products over NCCL on two GPUs (spmv_chain_run): each rank's CSR-lp shard product into its
slice of the next x, the slices all-gathered (grouped broadcasts for nnz-balanced shards of unequal rows,
one all-gather for equal ones), three times; and over interleaved row blocks whose all-gathers run beside
the next block's product (spmv_chain_run_blocks); and over peer memory, each product storing its rows into
both GPUs' next x (spmv_chain_run_peer); the results bit-identical to the oracle's chain on the whole
matrix; and in halo mode, each product pulling only the entries of x the rank's rows read from the other
GPU."""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as probe:
        probe.bind(("127.0.0.1", 0))
        return probe.getsockname()[1]


def worker(rank, world, port):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "spmv-index-compression_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import oracle
    import spmvb200 as spmv
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    box = [spmv.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    comm = spmv.Comm(world, rank, box[0], device=rank)
    matrix = spmv.synth_random_band(20000, 500, 12.0, 3)
    row_ptr, col_ind, values = matrix.arrays()
    x0 = spmv.fill_uniform(spmv.F64, matrix.cols, 9)
    expected = x0.copy()
    for _ in range(3):
        expected = oracle.spmv_csr(row_ptr, col_ind, values, expected, spmv.F64, spmv.LP, 8)
    # nnz-balanced shards (unequal: grouped broadcasts) and equal row halves (one all-gather)
    for bounds in (spmv.shard_rows(matrix, world), np.array([0, 10000, 20000], dtype=np.int32)):
        shard = matrix.slice_rows(int(bounds[rank]), int(bounds[rank + 1]))
        with spmv.Operator(shard, spmv.LP, spmv.F64, 8, device=rank) as op:
            x_current = torch.from_numpy(x0).cuda()
            x_next = torch.zeros_like(x_current)
            stream = torch.cuda.current_stream().cuda_stream
            spmv.chain_run(op, comm, bounds, x_current.data_ptr(), x_next.data_ptr(), 3, stream)
            comm.check(stream, 30000)
            result = x_next.cpu().numpy()    # an odd count of products ends in x_next
        assert np.array_equal(result.view(np.uint64), expected.view(np.uint64)), bounds.tolist()
    # interleaved row blocks (spmv_chain_run_blocks): 2 ranks x 4 blocks of 2500 rows; rank r holds blocks
    # r, r + 2, r + 4, r + 6; an odd and an even count of products
    blocks_per_rank, block_rows = 4, 2500
    ops = [spmv.Operator(matrix.slice_rows((c * world + rank) * block_rows, (c * world + rank + 1) * block_rows),
                         spmv.LP, spmv.F64, 8, device=rank) for c in range(blocks_per_rank)]
    fourth = oracle.spmv_csr(row_ptr, col_ind, values, expected, spmv.F64, spmv.LP, 8)
    for products, want in ((3, expected), (4, fourth)):
        x_current = torch.from_numpy(x0).cuda()
        x_next = torch.zeros_like(x_current)
        stream = torch.cuda.current_stream().cuda_stream
        spmv.chain_run_blocks(ops, block_rows, comm, x_current.data_ptr(), x_next.data_ptr(), products, stream)
        comm.check(stream, 30000)
        result = (x_next if products % 2 else x_current).cpu().numpy()
        assert np.array_equal(result.view(np.uint64), want.view(np.uint64)), products
    for op in ops:
        op.close()
    # chained products over peer memory (spmv_chain_run_peer): each product stores its rows into both
    # ranks' next x, then a barrier of the two GPUs; nnz-balanced and equal shards, 3 products then 1 more
    group = spmv.PeerGroup(world, rank, x0.nbytes, device=rank)
    handles = [None] * world
    dist.all_gather_object(handles, group.export())
    group.open(handles)
    stream = torch.cuda.current_stream().cuda_stream
    for bounds in (spmv.shard_rows(matrix, world), np.array([0, 10000, 20000], dtype=np.int32)):
        shard = matrix.slice_rows(int(bounds[rank]), int(bounds[rank + 1]))
        with spmv.Operator(shard, spmv.LP, spmv.F64, 8, device=rank) as op:
            group.write_x(x0.ctypes.data, x0.nbytes)
            dist.barrier()
            for products, want in ((3, expected), (1, fourth)):
                spmv.chain_run_peer(op, group, bounds, products, stream, timeout_ms=20000)
                group.check()
                result = np.empty_like(x0)
                group.read_x(result.ctypes.data, result.nbytes)
                assert np.array_equal(result.view(np.uint64), want.view(np.uint64)), (bounds.tolist(), products)
        dist.barrier()
    # halo mode: each product pulls only the entries of x the rank's rows read from the other rank; each
    # rank's own rows of the chain are the oracle's, and the halo is a small part of x
    for bounds in (spmv.shard_rows(matrix, world), np.array([0, 10000, 20000], dtype=np.int32)):
        first, last = int(bounds[rank]), int(bounds[rank + 1])
        shard = matrix.slice_rows(first, last)
        halo = group.set_halo(shard, bounds)
        assert 0 < halo < matrix.cols // 4, halo
        with spmv.Operator(shard, spmv.LP, spmv.F64, 8, device=rank) as op:
            group.write_x(x0.ctypes.data, x0.nbytes)
            dist.barrier()
            for products, want in ((3, expected), (1, fourth)):
                spmv.chain_run_peer(op, group, bounds, products, stream, timeout_ms=20000)
                group.check()
                result = np.empty_like(x0)
                group.read_x(result.ctypes.data, result.nbytes)
                assert np.array_equal(result[first:last].view(np.uint64), want[first:last].view(np.uint64)), \
                    ("halo", bounds.tolist(), products)
        dist.barrier()
    group.close()
    comm.close()
    dist.destroy_process_group()


def test_chained_products_over_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(worker, args=(2, free_port()), nprocs=2, join=True)
