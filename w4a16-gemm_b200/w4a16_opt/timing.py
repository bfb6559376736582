"""Device timing of a captured step: one CUDA graph, replayed between CUDA events.

Used by ``bench.py`` (whole-step throughput) and ``gemm_benchmark`` (per-call latency in
the reference benchmark's schema).  A step is captured once -- after one eager run on a side
stream, so lazily initialised state (tensor maps, workspaces, shared-memory opt-ins) exists
before capture -- and then replayed: ``warm`` untimed replays, then timed ones, with the
events recorded on the stream the replays run on.
"""
import torch


class GraphStep:
    """``fn`` captured as one CUDA graph on the current device."""

    def __init__(self, fn):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            fn()

    def warm(self, n: int) -> None:
        for _ in range(n):
            self.graph.replay()
        torch.cuda.synchronize()

    def total_ms(self, n: int) -> float:
        """Device milliseconds of ``n`` back-to-back replays."""
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(n):
            self.graph.replay()
        t1.record()
        t1.synchronize()
        return t0.elapsed_time(t1)

    def each_ms(self, n: int) -> list:
        """Device milliseconds of each of ``n`` replays, timed one at a time."""
        out = []
        for _ in range(n):
            out.append(self.total_ms(1))
        return out

    def close(self) -> None:
        self.graph = None
