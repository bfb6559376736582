"""Tensor-parallel host logic (w4a16_opt.tp) on CPU: shard layout, and world-size-2 gloo runs.

The GEMM is injected (the oracle on the shard the rank owns), so these tests check what the
TP layer itself does -- which words and scales each rank owns, the collectives, the output
assembly -- without a GPU.  The CUDA GEMM on those shards is covered by the GPU tests.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w4a16_oracle as oracle


def _problem(M, N, K, G, seed=3):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=gen).half()
    q = torch.randint(0, 16, (N, K), generator=gen, dtype=torch.uint8)
    s = (torch.rand(K // G, N, generator=gen) * 0.018 + 0.002).half()
    Wp = torch.from_numpy(oracle.pack_int4(q.numpy()).view(np.int32))
    return x, q, s, Wp


def _oracle_gemm_out(Wp, x, scales, y, workspace=None):
    """Stand-in for w4a16_gemm_out on CPU: y = x @ dequant(Wp, scales)^T (fp32 math)."""
    ref = oracle.ref_gemm_from_packed(x.numpy(), Wp.numpy(), scales.numpy())
    y.copy_(torch.from_numpy(ref).to(y.dtype))
    return y


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_columns_is_a_column_slice(world):
    from w4a16_opt import tp
    N, K, G = 512, 1024, 128
    _, q, s, Wp = _problem(1, N, K, G)
    full = oracle.dequant_from_packed(Wp.numpy(), s.numpy(), N, K)
    n_loc = N // world
    for r in range(world):
        Wp_r, s_r = tp.shard_columns(Wp, s, N, K, r, world)
        assert Wp_r.numel() == n_loc * K // 8 and s_r.shape == (K // G, n_loc)
        part = oracle.dequant_from_packed(Wp_r.numpy(), s_r.numpy(), n_loc, K)
        assert np.array_equal(part.view(np.uint16), full[r * n_loc:(r + 1) * n_loc].view(np.uint16))


@pytest.mark.parametrize("world,G", [(2, 128), (4, 64), (8, 64)])
def test_shard_rows_is_a_k_slice(world, G):
    from w4a16_opt import tp
    N, K = 256, 4096
    _, q, s, Wp = _problem(1, N, K, G)
    full = oracle.dequant_from_packed(Wp.numpy(), s.numpy(), N, K)
    k_loc = K // world
    for r in range(world):
        Wp_r, s_r = tp.shard_rows(Wp, s, N, K, r, world)
        assert Wp_r.numel() == N * k_loc // 8 and s_r.shape == (k_loc // G, N)
        part = oracle.dequant_from_packed(Wp_r.numpy(), s_r.numpy(), N, k_loc)
        assert np.array_equal(part.view(np.uint16), full[:, r * k_loc:(r + 1) * k_loc].view(np.uint16))


def test_shard_rejects_uneven_splits():
    from w4a16_opt import tp
    _, q, s, Wp = _problem(1, 48, 192, 64)
    with pytest.raises(ValueError):
        tp.shard_columns(Wp, s, 48, 192, 0, 2)        # 3 n16 blocks over 2 ranks
    with pytest.raises(ValueError):
        tp.shard_rows(Wp, s, 48, 192, 0, 2)           # 3 chunks of 64 over 2 ranks


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _rank_main(rank, world, port, M, N, K, G, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from w4a16_opt import tp
        x, q, s, Wp = _problem(M, N, K, G)
        col = tp.ColumnParallelW4A16(Wp, s, N, K, gemm_out=_oracle_gemm_out)
        y_col = col(x)
        row = tp.RowParallelW4A16(Wp, s, N, K, gemm_out=_oracle_gemm_out)
        y_row = row(row.x_slice(x))
        # caller-provided outputs: written in place (M = 1 included), twice in a row (the
        # gather's staging buffer is reused), and the same values as the returned tensors
        y_col_out = torch.full((M, N), float("nan"), dtype=torch.float16)
        y_row_out = torch.full((M, N), float("nan"), dtype=torch.float16)
        for _ in range(2):
            assert col.gather(col.local(x), out=y_col_out) is y_col_out
            part = row.partial(row.x_slice(x))
            assert row.reduce(part, out=y_row_out) is y_row_out
        assert torch.equal(y_col_out, y_col) and torch.equal(y_row_out, y_row)
        assert len(col._gather_bufs) == (0 if M == 1 else 1)
        results[rank] = (y_col.float().numpy(), y_row.float().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [1, 3, 16])
def test_tp_world2_gloo(M):
    """Column split + all-gather and row split + fp32 all-reduce reproduce the full GEMM."""
    world, N, K, G = 2, 512, 2048, 128
    with mp.get_context("spawn").Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_rank_main, args=(world, _free_port(), M, N, K, G, results), nprocs=world, join=True)
        out = dict(results)
    x, q, s, Wp = _problem(M, N, K, G)
    ref = oracle.ref_gemm(x.numpy(), q.numpy(), s.numpy(), G)
    denom = float(np.abs(ref).max())
    for rank in range(world):
        y_col, y_row = out[rank]
        assert y_col.shape == (M, N) and y_row.shape == (M, N)
        # column split: each rank's columns are the full GEMM's columns (fp16 rounding only)
        assert float(np.abs(y_col - ref).max()) <= 2e-3 * denom
        # row split: two fp32 partial sums, one fp16 rounding
        assert float(np.abs(y_row - ref).max()) <= 2e-3 * denom
    assert np.array_equal(out[0][0], out[1][0]) and np.array_equal(out[0][1], out[1][1])


def _failing_rank_main(rank, world, port, layer, mode, timeout_s, results):
    """Rank 1 fails between steps (raises, or stalls and never joins); rank 0 runs the layer."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # rendezvous with a generous timeout (process start-up varies), then run the layers on a
    # group whose collectives time out quickly
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dist.barrier()
    group = dist.new_group(ranks=list(range(world)), timeout=datetime.timedelta(seconds=timeout_s))
    from w4a16_opt import tp
    M, N, K, G = 2, 256, 512, 128
    x, q, s, Wp = _problem(M, N, K, G)
    cls = tp.ColumnParallelW4A16 if layer == "col" else tp.RowParallelW4A16
    mod = cls(Wp, s, N, K, group=group, gemm_out=_oracle_gemm_out)
    if rank != 0:
        if mode == "raise":
            raise RuntimeError("injected failure on rank 1")
        time.sleep(timeout_s + 2)             # alive, but never enters the collective
        os._exit(0)
    t0 = time.monotonic()
    try:
        mod(x) if layer == "col" else mod(mod.x_slice(x))
        results[rank] = ("completed", time.monotonic() - t0)
    except Exception as exc:                  # the collective must end with an error, not hang
        results[rank] = (type(exc).__name__, time.monotonic() - t0)
    os._exit(0)                               # no teardown collective with a failed peer


@pytest.mark.parametrize("layer", ["col", "row"])
@pytest.mark.parametrize("mode", ["raise", "stall"])
def test_tp_peer_failure_is_an_error_not_a_hang(layer, mode):
    """A rank that dies or stalls between steps makes the surviving rank's next collective
    (all-gather or all-reduce) raise within the process-group timeout."""
    timeout_s = 3
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_failing_rank_main, args=(r, 2, port, layer, mode, timeout_s, results))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        assert not alive, "a rank did not finish"
        out = dict(results)
    assert 0 in out, "rank 0 reported nothing"
    outcome, secs = out[0]
    assert outcome != "completed", "the collective completed without its peer"
    assert secs < timeout_s + 30, f"error took {secs:.1f} s"
    assert procs[1].exitcode == (1 if mode == "raise" else 0)
    print(f"{layer}/{mode}: rank 0 raised {outcome} after {secs:.1f} s")
