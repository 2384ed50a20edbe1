"""Chained products over peer memory on one GPU (spmv_chain_run_peer with a group of one rank: the fused
product, the barrier and the buffer turns without peers) against the oracle's chain, bit for bit; and a
barrier whose other rank never comes, which must end in SPMV_ERR_TIMEOUT from spmv_peer_group_check after
its bounded wait, leaving the GPU usable. The two-GPU run is in test_multi_gpu.py."""
import numpy as np
import pytest

import oracle
import spmvb200 as spmv

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TORCH = {spmv.F64: torch.float64, spmv.F32: torch.float32, spmv.F16: torch.float16}


def oracle_chain(matrix, x0, dtype, layout, tpr, products):
    row_ptr, col_ind, values = matrix.arrays()
    x = x0.copy()
    for _ in range(products):
        x = oracle.spmv_csr(row_ptr, col_ind, values, x, dtype, layout, tpr)
    return x


@pytest.mark.parametrize("dtype,layout,tpr", [(spmv.F64, spmv.LP, 8), (spmv.F32, spmv.I32, 16),
                                              (spmv.F16, spmv.LP, 32)])
def test_one_rank_chain_matches_oracle(dtype, layout, tpr):
    matrix = spmv.synth_random_band(30000, 400, 10.0, 6)
    x0 = spmv.fill_uniform(dtype, matrix.cols, 4)
    group = spmv.PeerGroup(1, 0, x0.nbytes, device=0)
    bounds = np.array([0, matrix.rows], dtype=np.int32)
    stream = torch.cuda.current_stream().cuda_stream
    done = 0
    if layout == spmv.I32:   # halo mode on one rank: nothing to pull
        assert group.set_halo(matrix, bounds) == 0
    with spmv.Operator(matrix, layout, dtype, tpr, device=0) as op:
        group.write_x(x0.ctypes.data, x0.nbytes)
        for products in (1, 2, 3):   # each call continues the chain from the group's current x
            spmv.chain_run_peer(op, group, bounds, products, stream)
            group.check()
            done += products
            result = np.empty_like(x0)
            group.read_x(result.ctypes.data, result.nbytes)
            want = oracle_chain(matrix, x0, dtype, layout, tpr, done)
            assert np.array_equal(result.view(np.uint8), want.view(np.uint8)), done
    group.close()


def test_barrier_without_the_other_rank_times_out():
    """Rank 0 of a group of two whose rank 1 never opens: the barrier's wait runs out (a flag nothing
    sets), the status word says so, and the device stays usable."""
    group = spmv.PeerGroup(2, 0, 1024, device=0)
    group.barrier(timeout_ms=200, stream=torch.cuda.current_stream().cuda_stream)
    with pytest.raises(spmv.SpmvError) as failure:
        group.check()
    assert failure.value.status == spmv.ERR_TIMEOUT
    with pytest.raises(spmv.SpmvError):   # a timed-out group refuses further barriers
        group.barrier(timeout_ms=200)
    group.close()
    # the context is intact: an ordinary product still runs and matches the oracle
    matrix = spmv.synth_random_band(5000, 100, 8.0, 2)
    x = spmv.fill_uniform(spmv.F64, matrix.cols, 1)
    with spmv.Operator(matrix, spmv.I32, spmv.F64, 8) as op:
        x_device = torch.from_numpy(x).cuda()
        y_device = torch.empty(matrix.rows, dtype=torch.float64, device="cuda")
        op.run(x_device.data_ptr(), y_device.data_ptr())
        torch.cuda.synchronize()
        op.check()
    row_ptr, col_ind, values = matrix.arrays()
    want = oracle.spmv_csr(row_ptr, col_ind, values, x, spmv.F64, spmv.I32, 8)
    assert np.array_equal(y_device.cpu().numpy().view(np.uint64), want.view(np.uint64))
