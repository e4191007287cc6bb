"""Times the reference's own GPU kernels on the B200 (a baseline, not the product).

TEST / BASELINE INFRASTRUCTURE ONLY. Loads ``oracle/_ref/relm_mp_ref_cuda.so``
(maichmueller/relmo's ``src/_ops/mp/mp_ops.cpp`` + ``mp_cuda_kernels.cu``,
compiled for sm_100a by ``oracle/build_ref.py --cuda``) and times its six
hot ops through ``torch.ops.relm_mp`` on a seeded workload (cfg2: 2^20 rows,
2^24 messages, D=64, fp32, Zipf(1.3) destinations), each op alone with CUDA
events on the current stream (1 untimed call, then ``--reps`` timed calls).
Prints one JSON object: per op ms, GB/s of the same algorithmic bytes the bench
counts, and messages/s.

It must run in a process of its own: the reference library registers the
``relm_mp`` namespace that the B200 library registers too. ``bench.py --impl
reference`` runs it as a subprocess.

The reference kernels are SIMT grid-stride loops over (edge, column) with float
atomics (cu:412-649); on valid indices they neither fault nor wait on one
another (the atomic max is a CAS loop that exits once the stored value is not
smaller than its own).
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(ROOT))

from relmo_b200 import workloads  # noqa: E402  (pure Python, loads no library)

LIB = HERE / "_ref" / "relm_mp_ref_cuda.so"
OPS = ("fanout_fwd", "fanout_bwd", "fanin_sum_fwd", "fanin_sum_bwd", "fanin_lse_fwd", "fanin_lse_bwd")


def run_op(ops, wl, op: str, lse):
    if op == "fanout_fwd":
        return ops.fanout_scatter(wl.x, wl.src, wl.flat_dst, wl.out_rows)
    if op == "fanout_bwd":
        return ops.fanout_scatter_backward(wl.grad_slots, wl.src, wl.flat_dst, wl.x.size(0))
    if op == "fanin_sum_fwd":
        return ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 0)
    if op == "fanin_lse_fwd":
        return ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
    if op == "fanin_sum_bwd":
        return ops.fanin_reduce_sum_backward(wl.grad_nodes, wl.flat_src, wl.dst, wl.msgs.size(0))
    if op == "fanin_lse_bwd":
        return ops.fanin_reduce_logsumexp_backward(wl.grad_nodes, wl.msgs, wl.flat_src, wl.dst, lse, wl.msgs.size(0))
    raise ValueError(op)


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--workload", default="cfg2-unsorted", choices=["cfg2-unsorted", "cfg2-sorted"])
    parser.add_argument("--reps", type=int, default=3)
    args = parser.parse_args()
    if not LIB.is_file():
        print(json.dumps({"unavailable": f"{LIB.name} not built (python oracle/build_ref.py --cuda)"}))
        return 0
    torch.ops.load_library(str(LIB))
    ops = torch.ops.relm_mp
    dev = torch.device("cuda", 0)
    wl = workloads.cfg2(seed=0, device=dev, sorted_dst=args.workload == "cfg2-sorted")
    nbytes = {op: workloads.algorithmic_bytes(op, wl) for op in OPS}
    lse = ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
    stream = torch.cuda.current_stream()
    per_op = {}
    for op in OPS:
        run_op(ops, wl, op, lse)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.reps):
            run_op(ops, wl, op, lse)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / args.reps
        per_op[op] = {"ms": round(ms, 4), "gbs": round(nbytes[op] / ms / 1e6, 1),
                      "msgs_per_s": round(wl.num_edges / ms * 1e3, 1)}
    print(json.dumps({
        "kind": "reference GPU kernels (mp_cuda_kernels.cu, sm_100a build of the reference sources)",
        "workload": args.workload, "dtype": "f32", "reps": args.reps, "build_info": ops.build_info(),
        "per_op": per_op,
    }))
    return 0


if __name__ == "__main__":
    sys.exit(main())
