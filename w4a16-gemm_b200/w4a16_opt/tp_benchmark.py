"""Exchange-only timing of the tensor-parallel layers' collectives, one process per GPU.

    torchrun --nproc-per-node N -m w4a16_opt.tp_benchmark [--M 1,16] [--reduce-N 8192] [--gather-N 28672]

For each M it times, per call, the row-parallel reduction of an fp32 partial [M, reduce-N]
and the column-parallel gather of fp16 columns into [M, gather-N] (the Llama-3-70B down and
gate/up outputs by default), three ways on the same buffers:

* ``one_round``: the library's exchange kernel with a receive area (``PeerExchange``
  default): one flag round per call for contributions up to ``TP_PUSH_MAX_BYTES``;
* ``two_round``: the same kernel without a receive area (ready flag, then peer loads);
* ``nccl``: ``all_reduce`` of the partial + a cast to fp16, and ``all_gather_into_tensor``.

Each is captured as a CUDA graph of 20 calls, replayed 50 times between CUDA events; the
microseconds per call are the maximum over ranks.  Rank 0 prints one JSON line per case.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

from . import tp
from .timing import GraphStep

CALLS, REPS = 20, 50


def _time_us(fn) -> float:
    def step():
        for _ in range(CALLS):
            fn()
    dist.barrier()
    g = GraphStep(step)
    g.warm(5)
    dist.barrier()
    torch.cuda.synchronize()
    ms = g.total_ms(REPS)
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    g.close()
    return round(float(t.item()) * 1e3 / (REPS * CALLS), 2)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--M", default="1,16")
    ap.add_argument("--reduce-N", type=int, default=8192)
    ap.add_argument("--gather-N", type=int, default=28672)
    args = ap.parse_args(argv)
    rank = int(os.environ.get("RANK", 0))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    world = dist.get_world_size()
    ms = [int(v) for v in args.M.split(",")]
    src_bytes = max(max(ms) * args.reduce_N * 4, max(ms) * args.gather_N // world * 2)
    y_bytes = max(ms) * max(args.reduce_N, args.gather_N) * 2
    one = tp.PeerExchange(src_bytes, y_bytes)
    two = tp.PeerExchange(src_bytes, y_bytes, push_bytes=0)
    try:
        for M in ms:
            for kind, N in (("reduce", args.reduce_N), ("gather", args.gather_N)):
                row = {"kind": kind, "M": M, "N": N, "world": world}
                for name, ex in (("one_round", one), ("two_round", two)):
                    if kind == "reduce":
                        ex.src((M, N), torch.float32).copy_(torch.randn(M, N, device="cuda"))
                        row[name + "_us"] = _time_us(lambda ex=ex: ex.allreduce(M, N))
                    else:
                        ex.src((M, N // world), torch.float16).copy_(torch.randn(M, N // world, device="cuda").half())
                        row[name + "_us"] = _time_us(lambda ex=ex: ex.allgather(M, N))
                if kind == "reduce":
                    part = torch.randn(M, N, device="cuda")
                    y = torch.empty(M, N, dtype=torch.float16, device="cuda")

                    def nccl():
                        dist.all_reduce(part)
                        y.copy_(part)
                else:
                    loc = torch.randn(M, N // world, device="cuda").half()
                    buf = torch.empty(world * M, N // world, dtype=torch.float16, device="cuda")

                    def nccl():
                        dist.all_gather_into_tensor(buf, loc)
                row["nccl_us"] = _time_us(nccl)
                if rank == 0:
                    print(json.dumps(row), flush=True)
    finally:
        one.close()
        two.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
