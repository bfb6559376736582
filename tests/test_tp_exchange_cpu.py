"""The tensor-parallel exchange (csrc/tp_exchange.cuh) checked on the CPU.

* A thread-per-(rank, CTA) emulation of the exchange kernels' protocols -- the two-round
  pull (ready flags, per-CTA done flags) and the one-round push (contributions stored into
  parity slots of every peer's receive area, one per-CTA done flag), the rank's call count
  (epoch) that the last CTA of a call to finish advances, grids of two sizes (the kernel
  launches more CTAs for large contributions), waits that accept a flag at or past the
  expected epoch -- over shared arrays that stand in for the ranks' buffers; calls of both
  protocols and both grid sizes interleave as the C ABI chooses them by size.  Random delays move the
  threads of different ranks and calls past one another; every call must still produce the
  rank-order sum (reduce) or the column gather, on every rank.  A rank that stops joining
  (a stalled peer, injected on the host) must make the others' bounded waits end in an
  error, not a hang.
* The C ABI's checks of a group and an exchange's regions, which run before any CUDA call.
"""
import ctypes
import random
import threading
import time

import numpy as np
import pytest

# the kernel launches kTpCtasSmall (one-round calls, small two-round calls) or kTpCtasLarge
# CTAs (two-round calls of large contributions); smaller counts keep the emulation fast
CTAS_SMALL, CTAS_LARGE = 2, 4


class PeerTimeout(Exception):
    pass


class Exchange:
    """Every rank's buffer: ready[src], done[src][cta], epoch and count, the source and y regions."""

    def __init__(self, world, M, N, gather, limit_s=2.0):
        self.world, self.M, self.N, self.gather, self.limit = world, M, N, gather, limit_s
        self.ready = np.zeros((world, world), np.int64)          # [buffer][src]
        self.done = np.zeros((world, world, CTAS_LARGE), np.int64)   # [buffer][src][cta]
        self.epoch = np.zeros(world, np.int64)                   # [rank]: calls completed
        self.count = np.zeros(world, np.int64)                   # [rank]: CTAs of the current call done
        self.y = np.full((world, M, N), np.nan)
        # receive area: [buffer][parity][src] one contribution each (stale values start as NaN)
        shape = (M, N // world) if gather else (M, N)
        self.recv = np.full((world, 2, world) + shape, np.nan, np.float16 if gather else np.float32)
        self.lock = threading.Lock()

    def wait_at_least(self, get, e):
        t0 = time.monotonic()
        while True:
            with self.lock:
                if get() >= e:
                    return
            if time.monotonic() - t0 > self.limit:
                raise PeerTimeout()
            time.sleep(0.0005 * random.random())

    def start(self, rank):
        """A CTA reads the rank's call count once, when it starts."""
        with self.lock:
            return self.epoch[rank] + 1

    def count_out(self, rank, e, grid):
        """tp_count_out: the last CTA of the call to finish advances the rank's epoch."""
        with self.lock:
            self.count[rank] += 1
            if self.count[rank] == grid:
                self.count[rank] = 0
                self.epoch[rank] = e

    def push_cta(self, rank, cta, src_regions, grid=CTAS_SMALL):
        """One CTA of tp_push_kernel on `rank`: send this CTA's units of the contribution to
        slot (e & 1, rank) of every peer, one flag per peer, wait for CTA cta of every peer,
        build y from the own source region and the received slots."""
        W, M, N = self.world, self.M, self.N
        e = self.start(rank)
        par = e & 1
        own = src_regions[rank]
        flat = own.reshape(-1)
        units = flat.size // (8 if self.gather else 4)                 # 16-byte units
        per = 8 if self.gather else 4
        lo, hi = units * cta // grid * per, units * (cta + 1) // grid * per
        for t in range(W):                                             # A: stores into every peer
            if t != rank:
                self.recv[t, par, rank].reshape(-1)[lo:hi] = flat[lo:hi]
                time.sleep(0.0002 * random.random())
        with self.lock:                                                # B: flags, then wait
            for t in range(W):
                if t != rank:
                    self.done[t, rank, cta] = max(self.done[t, rank, cta], e)
        try:
            for src in range(W):
                if src != rank:
                    self.wait_at_least(lambda src=src: self.done[rank, src, cta], e)
        except PeerTimeout:
            self.count_out(rank, e, grid)
            raise
        # C: y from the same units
        if self.gather:
            nl = N // W
            for src in range(W):
                part = (own if src == rank else self.recv[rank, par, src]).reshape(-1)[lo:hi]
                for i, v in zip(range(lo, hi), part):
                    m, c = divmod(i, nl)
                    self.y[rank, m, src * nl + c] = np.float16(v)
        else:
            acc = np.zeros(hi - lo, np.float32)
            for src in range(W):                                       # rank order
                acc = acc + (own if src == rank else self.recv[rank, par, src]).reshape(-1)[lo:hi]
            self.y[rank].reshape(-1)[lo:hi] = np.float16(acc)
        self.count_out(rank, e, grid)

    def cta(self, rank, cta, src_regions, grid=CTAS_SMALL):
        """One CTA of the exchange kernel on `rank` (phases A, B, C); src_regions[r] is rank
        r's source region for this call."""
        W, M, N = self.world, self.M, self.N
        e = self.start(rank)
        with self.lock:                                           # A: ready into every buffer
            for t in range(W):
                self.ready[t, rank] = max(self.ready[t, rank], e)
        try:
            for src in range(W):
                self.wait_at_least(lambda src=src: self.ready[rank, src], e)
        except PeerTimeout:
            self.count_out(rank, e, grid)
            raise
        nl = N // W                                               # B: this CTA's share of the rank's columns
        units = M * (nl // 8)
        for u in range(units * cta // grid, units * (cta + 1) // grid):
            m, c8 = u // (nl // 8), (u % (nl // 8)) * 8
            cols = slice(rank * nl + c8, rank * nl + c8 + 8)
            if self.gather:
                vals = src_regions[rank][m, c8:c8 + 8]
            else:
                vals = np.zeros(8, np.float32)
                for src in range(W):                              # rank order
                    vals = vals + src_regions[src][m, cols]
            time.sleep(0.0002 * random.random())
            for t in range(W):
                self.y[t, m, cols] = np.float16(vals)
        with self.lock:                                           # C: done into every buffer
            for t in range(W):
                self.done[t, rank, cta] = max(self.done[t, rank, cta], e)
        try:
            for src in range(W):
                self.wait_at_least(lambda src=src: self.done[rank, src, cta], e)
        finally:
            self.count_out(rank, e, grid)


def run_calls(ex, inputs, stall_rank=None, stall_call=None, push=(), large=()):
    """Every rank issues the calls in order, with no host synchronisation between ranks (a
    fast rank runs ahead); each call's CTAs run as threads.  After each call a rank reads its
    own y: no peer may write the next call's results into it before this rank announced
    that call.  Calls in `push` take the one-round form (always the small grid), calls in
    `large` the large grid.  Returns results[rank][call], or raises the first error."""
    results = [[] for _ in range(ex.world)]
    errors = []

    def rank_main(rank):
        for i, src in enumerate(inputs):
            if rank == stall_rank and i == stall_call:
                return                                            # stops joining: never starts call i
            grid = CTAS_LARGE if i in large and i not in push else CTAS_SMALL
            threads = [threading.Thread(target=_cta, args=(rank, c, src, i in push, grid)) for c in range(grid)]
            for t in threads:
                t.start()
            for t in threads:
                t.join()
            if errors:
                return
            results[rank].append(ex.y[rank].copy())

    def _cta(rank, c, src, one_round, grid):
        try:
            (ex.push_cta if one_round else ex.cta)(rank, c, src, grid)
        except Exception as exc:                                  # noqa: BLE001
            errors.append(exc)

    ranks = [threading.Thread(target=rank_main, args=(r,)) for r in range(ex.world)]
    for t in ranks:
        t.start()
    for t in ranks:
        t.join(timeout=60)
    assert not any(t.is_alive() for t in ranks), "a rank hung"
    if errors:
        raise errors[0]
    return results


@pytest.mark.parametrize("mix", ["pull", "push", "mixed", "grids"])
@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("gather", [False, True])
def test_exchange_protocol_results(world, gather, mix):
    rng = np.random.default_rng(world)
    M, N = 3, 16 * world
    calls = 10
    push = {"pull": (), "push": tuple(range(calls)), "mixed": (1, 2, 4, 7, 8), "grids": ()}[mix]
    large = {"pull": (), "push": (), "mixed": (0, 3, 9), "grids": (1, 2, 5, 6, 9)}[mix]
    inputs = []
    for _ in range(calls):
        if gather:
            inputs.append([rng.standard_normal((M, N // world)).astype(np.float16) for _ in range(world)])
        else:
            inputs.append([rng.standard_normal((M, N)).astype(np.float32) for _ in range(world)])
    ex = Exchange(world, M, N, gather)
    results = run_calls(ex, inputs, push=push, large=large)
    assert all(len(r) == len(inputs) for r in results)
    for i, src in enumerate(inputs):
        if gather:
            want = np.concatenate(src, axis=1).astype(np.float16)
        else:
            acc = np.zeros((M, N), np.float32)
            for p in src:                                          # rank order
                acc = acc + p
            want = acc.astype(np.float16)
        for r in range(world):
            assert np.array_equal(results[r][i].astype(np.float16), want), f"rank {r}, call {i}"
    assert (ex.epoch == len(inputs)).all() and (ex.count == 0).all()


@pytest.mark.parametrize("push", [(), (0, 1, 2)])
def test_stalled_peer_is_an_error_not_a_hang(push):
    world, M, N = 3, 2, 48
    rng = np.random.default_rng(0)
    inputs = [[rng.standard_normal((M, N)).astype(np.float32) for _ in range(world)] for _ in range(3)]
    ex = Exchange(world, M, N, gather=False, limit_s=0.5)
    t0 = time.monotonic()
    with pytest.raises(PeerTimeout):
        run_calls(ex, inputs, stall_rank=2, stall_call=1, push=push)
    assert time.monotonic() - t0 < 30


# ------------------------------------------------------------------ the C ABI's host-side checks

def _group(lib_capi, world=2, rank=0, ptrs=(256, 512), nbytes=1 << 20):
    return lib_capi.TpGroup(rank, world, (ctypes.c_void_p * lib_capi.TP_MAX_RANKS)(*ptrs), nbytes)


@pytest.mark.parametrize("kw,msg", [
    (dict(world=0), "world"),
    (dict(world=9), "world"),
    (dict(rank=2), "rank"),
    (dict(ptrs=(256, 0)), "mapped"),
    (dict(ptrs=(256, 300)), "256-byte aligned"),
])
def test_exchange_rejects_bad_groups(kw, msg):
    from w4a16_opt import capi
    lib = capi.load()
    g = _group(capi, **kw)
    st = lib.w4a16_tp_allreduce(ctypes.byref(g), capi.TP_CTRL_BYTES, 1 << 19, 2, 64, None)
    assert st in (18, 1, 9) and msg in capi.last_error(lib)


@pytest.mark.parametrize("args,msg", [
    ((96, 1 << 19, 2, 64), "past the flags"),                        # source inside the flags
    ((8192, 8200, 2, 64), "multiples of 16"),
    ((8192, 8192 + 256, 2, 64), "overlap"),
    ((8192, 1 << 19, 2, 56), "multiple of 8 * world"),
    ((8192, (1 << 20) - 64, 2, 64), "inside the buffers"),            # y runs past the end
])
def test_exchange_rejects_bad_regions(args, msg):
    from w4a16_opt import capi
    lib = capi.load()
    g = _group(capi)
    st = lib.w4a16_tp_allreduce(ctypes.byref(g), *args, None)
    assert st != 0 and msg in capi.last_error(lib)


@pytest.mark.parametrize("recv,msg", [
    ((8192 + 16, 4096), "256-byte boundary"),
    ((4096, 4096), "past the flags"),
    (((1 << 20) - 2048, 4096), "inside the buffers"),
    ((1 << 19, 4096), "must not overlap"),
])
def test_exchange_rejects_bad_receive_areas(recv, msg):
    from w4a16_opt import capi
    lib = capi.load()
    g = _group(capi)
    g.recv_off, g.recv_bytes = recv
    st = lib.w4a16_tp_allreduce(ctypes.byref(g), 8192, 1 << 19, 2, 64, None)
    assert st != 0 and msg in capi.last_error(lib)


def test_peer_alloc_rejects_buffers_smaller_than_the_flags():
    from w4a16_opt import capi
    lib = capi.load()
    p, h = ctypes.c_void_p(), capi.IpcHandle()
    assert lib.w4a16_peer_alloc(1024, ctypes.byref(p), ctypes.byref(h)) == 18
    assert "W4A16_TP_CTRL_BYTES" in capi.last_error(lib)
