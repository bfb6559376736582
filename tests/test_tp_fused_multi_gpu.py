"""The tensor-parallel layers with the peer-memory exchange, on 2 GPUs (skipped with fewer;
W4A16_TEST_WORLD=N runs it on N GPUs, N <= 8).

One child process per GPU, NCCL for set-up (handles, barriers) and for the
reference path.  For the column-parallel (N split, gather) and row-parallel (K split, fp32
reduction) layers at decode and prefill batch sizes:
* the fused path (GEMM into the exchange buffer + the library's exchange kernel) matches
  the CPU oracle within the tests' tolerance, with the one-round exchange (receive area)
  and the two-round one (none), which give the same bits;
* it gives bitwise identical y on every rank (every rank holds the same rank-order sums);
* it matches the NCCL path (all_gather_into_tensor / all_reduce) within tolerance -- the
  reduction order of NCCL's all-reduce is its own, so not bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

# ranks (GPUs) of the test; 2 by default, up to W4A16_TP_MAX_RANKS = 8 with W4A16_TEST_WORLD
WORLD = int(os.environ.get("W4A16_TEST_WORLD", "2"))
CASES = [(1, 1024, 2048), (16, 2048, 4096), (200, 512, 1024)]   # M, N, K


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _rank_main(rank, port, out):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [here, root, os.path.join(root, "w4a16-gemm_b200")]
    import torch.distributed as dist
    from helpers import make_workload
    from w4a16_opt import tp
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    res = {}
    sb, yb = max(M * N * 4 for M, N, _ in CASES), max(M * N * 2 for M, N, _ in CASES)
    ex = tp.PeerExchange(src_bytes=sb, y_bytes=yb)                    # one round at these sizes
    ex2 = tp.PeerExchange(src_bytes=sb, y_bytes=yb, push_bytes=0)     # always two rounds
    try:
        for M, N, K in CASES:
            x, q, s, Wp = make_workload(M, N, K, 128, seed=M + N + K)
            col = tp.ColumnParallelW4A16(Wp, s, N, K, exchange=ex)
            row = tp.RowParallelW4A16(Wp, s, N, K, exchange=ex)
            y_col_f = col.fused(x).clone()
            y_row_f = row.fused(row.x_slice(x)).clone()
            col.exchange = row.exchange = ex2
            y_col_2 = col.fused(x).clone()
            y_row_2 = row.fused(row.x_slice(x)).clone()
            y_col_n = col(x)
            y_row_n = row(row.x_slice(x))
            torch.cuda.synchronize()
            res[(M, N, K)] = tuple(t.float().cpu().numpy() for t in (y_col_f, y_row_f, y_col_n, y_row_n,
                                                                     y_col_2, y_row_2))
    finally:
        ex.close()
        ex2.close()
        dist.destroy_process_group()
    out[rank] = res


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason=f"needs {WORLD} GPUs")
def test_fused_exchange_two_gpus():
    from helpers import assert_close, make_workload, ref_gemm
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, port, out)) for r in range(WORLD)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank did not finish"
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(out)
    for M, N, K in CASES:
        x, q, s, _ = make_workload(M, N, K, 128, seed=M + N + K, device="cpu")
        ref = ref_gemm(x, q, s, 128)
        for rank in range(WORLD):
            y_col_f, y_row_f, y_col_n, y_row_n, y_col_2, y_row_2 = res[rank][(M, N, K)]
            assert_close(y_col_f, ref)
            assert_close(y_row_f, ref)
            assert np.array_equal(y_col_f, y_col_2) and np.array_equal(y_row_f, y_row_2)   # both protocols
            assert np.array_equal(y_col_f, y_col_n)           # the gather moves the same fp16 values
            assert_close(y_row_f, y_row_n.astype(np.float32))
        for rank in range(1, WORLD):
            for k in range(2):
                assert np.array_equal(res[0][(M, N, K)][k], res[rank][(M, N, K)][k])

