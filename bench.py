"""Benchmark of the relm_mp fan-out / fan-in path on B200.

One step = one pass of the hot path over one batch of the workload: the index
plans of the batch are built (the plan cache is cleared first) and the six ops
run through ``torch.ops.relm_mp`` (the reference's op API): fanout_scatter,
fanout_scatter_backward, fanin_reduce sum and logsumexp, fanin_reduce_sum_backward
and fanin_reduce_logsumexp_backward.

Default workload (N=1): cfg2, the reference's large op benchmark - N=2^20
nodes, E=2^24 messages, D=64, fp32, truncated Zipf(1.3) destinations in
generation order ("unsorted"), uniform sources, values ~N(0,1); synthetic data
from a fixed seed. Inputs are far larger than L2 (4.3 GB message matrix).

metric: GB/s of compulsory HBM traffic (each referenced input row read once,
every int64 index read once, each output row written once; plan/sort traffic
not counted), summed over the six ops and all ranks, divided by the max over
ranks of the step time (which does include the plan builds).

--gpus N (torchrun, one rank per GPU): every rank processes its own batch
(seed + rank); no collective on the data path (weak scaling). Timing uses CUDA
events between barriers; the max over ranks is taken with an NCCL all-reduce.

RelationalGNN train steps (``rgnn_train`` in the line; ``--workload cfg3|cfg4``
prints them as the headline instead): cfg3 = CentralizedRelationalGNN, emb 32,
10 layers, smoothed logsumexp, 256 states; cfg4 = decentralized RelationalGNN,
emb 128, 30 layers, sum, bf16 autocast, global batch 4096 states split evenly
over the ranks (strong scaling) and into micro-batches with gradient
accumulation, DDP gradient all-reduce over NCCL. One step = forward, loss,
backward and AdamW over the whole global batch; states/s = global states per
step / max-over-ranks step time.

LGAN step (``lgan_step`` in the line; ``--workload lgan`` prints it as the
headline): one lgan_pool_reduce and its backward (mean mode; sum alongside) on a
synthetic LGAN batch - 2^17 entities, 2^20 relation instances of arity 1..3
(~2^21 slots), 4 RR edges per instance, D=64 fp32; GB/s of compulsory traffic
(workloads.lgan_algorithmic_bytes) per step, plans built inside the step, and
per-op times with cached plans (the per-layer cost inside a model).

Also in the default line: every op's time, GB/s, fraction of the measured copy
peak and messages/s with its plans cached (``per_op``); at N=1 the same table
for cfg2 with bf16 storage (``per_op_bf16``) and for destination-sorted cfg2
(``per_op_sorted``); and, at every N, cfg5 (2^22 rows, 2^26 messages, D=32,
64 hubs x 100k) split over the ranks by work-balanced destination ranges with
no collective (``cfg5_partitioned``: step time = max over ranks, the per-rank
step times and edge counts).

--impl reference: the reference's own CPU relm_mp library
(``oracle/_ref/relm_mp_ref.so``, built from the reference sources) on the
host cores, on a bounded edge sample of the same workload; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from relmo_b200 import workloads  # noqa: E402

METRIC = "fanin/fanout GB/s vs HBM peak"
LGAN_METRIC = "lgan pool+graph step GB/s vs HBM peak"
MODEL_METRIC = "RGNN train states/s"
UNIT = "GB/s"
OPS = ("fanout_fwd", "fanout_bwd", "fanin_sum_fwd", "fanin_sum_bwd", "fanin_lse_fwd", "fanin_lse_bwd")
FANIN_OPS = ("fanin_sum_fwd", "fanin_sum_bwd", "fanin_lse_fwd", "fanin_lse_bwd")


def ops_of(workload: str) -> tuple[str, ...]:
    """cfg5 is the fan-in stress test (sum and logsumexp, forward and backward)."""

    return FANIN_OPS if workload == "cfg5" else OPS
REF_LIB = ROOT / "oracle" / "_ref" / "relm_mp_ref.so"


# ---- helpers ---------------------------------------------------------------------------


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            d = json.loads(p.read_text())
            return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def ncu_traffic() -> dict:
    """Per-launch DRAM bytes of each op's main kernel from a committed ncu summary, if any."""

    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.is_file():
        try:
            return json.loads(p.read_text())
        except Exception:
            return {}
    return {}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"relm_mp_clocks_{os.getpid()}_{gpu_index}.csv"

    def start(self) -> None:
        try:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"],
                stdout=self.fh, stderr=subprocess.DEVNULL,
            )
        except Exception:
            self.proc = None

    def settle(self, step, max_seconds: float = 3.0, samples: int = 2) -> None:
        """Run untimed steps until the sampler has recorded a few samples, so the
        samples taken around the (possibly short) timed region are under load."""

        if self.proc is None:
            return
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < max_seconds:
            step()
            torch.cuda.synchronize()
            self.fh.flush()
            try:
                if len(self.path.read_text().splitlines()) >= samples:
                    return
            except OSError:
                return

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        try:
            self.path.unlink()
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def make_workload(name: str, seed: int, device, dtype: torch.dtype, nodes=None, edges=None,
                  emb=None) -> workloads.FanWorkload:
    size = {}
    if nodes is not None:
        size["n"] = int(nodes)
    if edges is not None:
        size["edges"] = int(edges)
    if emb is not None:
        size["emb"] = int(emb)
    if name == "cfg2-unsorted":
        return workloads.cfg2(seed=seed, device=device, sorted_dst=False, dtype=dtype, **size)
    if name == "cfg2-sorted":
        return workloads.cfg2(seed=seed, device=device, sorted_dst=True, dtype=dtype, **size)
    if name == "cfg5":
        return workloads.cfg5(seed=seed, device=device, **size).to(device, dtype)
    if name == "cfg1":
        return workloads.cfg1(seed=seed, device=device).to(device, dtype)
    raise ValueError(name)


def op_bytes(wl: workloads.FanWorkload, op_list=OPS) -> dict[str, int]:
    s = wl.x.element_size()
    return {op: workloads.algorithmic_bytes(op, wl, s) for op in op_list}


def run_ops(ops, wl: workloads.FanWorkload, op_list=OPS) -> dict[str, torch.Tensor]:
    """The ops of one step, as the autograd wrappers call them (the logsumexp
    backward takes the forward's output)."""

    out, lse = {}, None
    for op in op_list:
        if op == "fanin_lse_bwd" and lse is None:
            lse = ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
        out[op] = run_one_op(ops, wl, op, lse)
        if op == "fanin_lse_fwd":
            lse = out[op]
    return out


def shard_workload(wl: workloads.FanWorkload, rank: int, world: int) -> workloads.FanWorkload:
    """The rank's part of a fan-in workload under the destination-range partition
    (its edges, the message rows they read, its output rows)."""

    from relmo_b200 import partition

    ranges = partition.balanced_destination_ranges(wl.dst, wl.dim_size, world)
    sh = partition.shard_by_destination(wl.flat_src, wl.dst, wl.dim_size, rank, world, ranges)
    none = torch.empty(0, dtype=torch.int64, device=wl.dst.device)
    return workloads.FanWorkload(
        wl.name, wl.x[:0], none, none, 0, wl.msgs.index_select(0, sh.rel_rows), sh.flat_src, sh.dst, sh.dim_size,
        wl.grad_slots[:0], wl.grad_nodes[sh.row_lo : sh.row_hi].contiguous(),
    )


def time_per_op(ops, wl: workloads.FanWorkload, op_list, reps: int, nbytes: dict) -> dict:
    """Each op on its own with its plans cached: CUDA-event time per call on the
    current stream (2 untimed calls first), GB/s of its algorithmic bytes, the
    fraction of the measured copy peak, and messages per second."""

    peak = measured_peaks()["hbm_gbs"]
    stream = torch.cuda.current_stream()
    lse = ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
    out = {}
    for op in op_list:
        for _ in range(2):
            run_one_op(ops, wl, op, lse)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(reps):
            run_one_op(ops, wl, op, lse)
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / reps
        gbs = nbytes[op] / ms / 1e6
        out[op] = {"ms": round(ms, 4), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                   "msgs_per_s": round(wl.num_edges / ms * 1e3, 1), "bytes": nbytes[op]}
    return out


def extra_per_op(ops, mp, name: str, dtype: torch.dtype, seed: int, device, reps: int) -> dict:
    """Per-op table of another cfg2 variant (bf16 storage, or destination-sorted)."""

    wl = make_workload(name, seed=seed, device=device, dtype=dtype)
    nbytes = op_bytes(wl, OPS)
    mp.clear_plan_cache()
    table = time_per_op(ops, wl, OPS, reps, nbytes)
    mp.clear_plan_cache()
    del wl
    torch.cuda.empty_cache()
    return {"workload": name, "dtype": "f32" if dtype == torch.float32 else "bf16", "per_op": table}


def cfg5_partitioned(ops, mp, device, rank: int, world: int, barrier, max_over_ranks, sum_over_ranks,
                     steps: int, warmup: int) -> dict:
    """cfg5 (2^22 rows, 2^26 messages, D=32, 64 hubs x 100k) split over the ranks
    by work-balanced destination ranges (relmo_b200.partition): each rank runs
    the four fan-in ops on its own edges, message rows and output rows, with no
    collective; one step = plan cache cleared + the four ops. Strong scaling:
    the whole job is the same at every N."""

    wl = make_workload("cfg5", seed=0, device=device, dtype=torch.float32)
    if world > 1:
        wl = shard_workload(wl, rank, world)
    wl.x = wl.x[:1].clone()  # fan-out inputs unused by the fan-in ops
    wl.grad_slots = wl.grad_slots[:1].clone()
    torch.cuda.empty_cache()
    step_bytes = sum(op_bytes(wl, FANIN_OPS).values())

    def step():
        mp.clear_plan_cache()
        run_ops(ops, wl, FANIN_OPS)

    for _ in range(max(warmup, 3)):
        step()
    barrier()
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    barrier()
    mine = ev0.elapsed_time(ev1) / steps
    elapsed_ms = max_over_ranks(mine)
    job_bytes = sum_over_ranks(step_bytes)
    per_rank = [[float(mine), float(wl.dst.numel()), float(wl.dim_size)]]  # fan-in edges of this rank
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor(per_rank[0], device=device, dtype=torch.float64)
        allv = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(allv, t)
        per_rank = [v.tolist() for v in allv]
    mp.clear_plan_cache()
    del wl
    torch.cuda.empty_cache()
    return {
        "workload": "cfg5", "ops": list(FANIN_OPS), "ranks": world, "steps": steps,
        "step": "plan builds (cache cleared) + 4 fan-in ops",
        "ms_per_step": round(elapsed_ms, 4), "value": round(job_bytes / elapsed_ms / 1e6, 1), "unit": UNIT,
        "scaling": "strong", "parallelism": f"work-balanced destination-range partition x{world}, no collective",
        "per_rank": [{"ms": round(v[0], 4), "edges": int(v[1]), "rows": int(v[2])} for v in per_rank],
    }


def run_one_op(ops, wl, op: str, lse=None):
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


# ---- CPU baselines -------------------------------------------------------------------------


def cpu_sample(workload: str, edges: int, seed: int = 0) -> workloads.FanWorkload:
    """A bounded sample of the workload: the same node count, dimension and index
    distributions, `edges` messages (generated on the CPU)."""

    if workload.startswith("cfg2"):
        return workloads.cfg2(seed=seed, device="cpu", sorted_dst=workload.endswith("sorted") and "un" not in workload,
                              edges=edges)
    if workload == "cfg5":
        frac = edges / (1 << 26)
        return workloads.cfg5(seed=seed, device="cpu", edges=edges, per_hub=max(1, int(100_000 * frac)))
    return workloads.cfg1(seed=seed)


def time_oracle_port(wl: workloads.FanWorkload, repeats: int = 1, op_list=OPS) -> tuple[float, int]:
    """Seconds per step of the C oracle (single thread) on `wl`; returns (s, bytes)."""

    from oracle import oracle

    x, msgs = wl.x.float().numpy(), wl.msgs.float().numpy()
    gs, gn = wl.grad_slots.float().numpy(), wl.grad_nodes.float().numpy()
    src, fdst, fsrc, dst = wl.src.numpy(), wl.flat_dst.numpy(), wl.flat_src.numpy(), wl.dst.numpy()
    best = math.inf
    for _ in range(repeats):
        t0 = time.perf_counter()
        if "fanout_fwd" in op_list:
            oracle.fanout_scatter(x, src, fdst, wl.out_rows)
            oracle.fanout_scatter_backward(gs, src, fdst, x.shape[0])
        oracle.fanin_reduce(msgs, fsrc, dst, wl.dim_size, 0)
        oracle.fanin_reduce_sum_backward(gn, fsrc, dst, msgs.shape[0])
        lse = oracle.fanin_reduce(msgs, fsrc, dst, wl.dim_size, 1)
        oracle.fanin_reduce_logsumexp_backward(gn, msgs, fsrc, dst, lse, msgs.shape[0])
        best = min(best, time.perf_counter() - t0)
    return best, sum(op_bytes(wl, op_list).values())


MODEL_CPU_STATES = {"cfg3": 32, "cfg4": 8}


def model_cpu_baseline(name: str, steps: int = 2, warmup: int = 1, states: int | None = None) -> dict:
    """Train steps of the RGNN workload on the host cores with relmo's torch
    formulas for the fan ops (the path relmo takes without its kernels; the
    reference model itself needs torch_geometric, not installed here), fp32,
    on a bounded sample of states. Returns states/s and the sample."""

    from relmo_b200 import model_train

    cfg = model_train.CONFIGS[name]
    n = int(states or MODEL_CPU_STATES[name])
    torch.manual_seed(0)
    model = model_train.build_model(cfg.kind, cfg.embedding_size, cfg.num_layers, cfg.aggregation, cfg.arities,
                                    use_kernels=False)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    batch = cfg.batch(seed=0, device="cpu", states=n)
    for _ in range(warmup):
        model_train.train_step(model, opt, [batch])
    t0 = time.perf_counter()
    for _ in range(steps):
        model_train.train_step(model, opt, [batch])
    dt = (time.perf_counter() - t0) / steps
    return {"value": round(n / dt, 3), "unit": "states/s", "cores": torch.get_num_threads(), "kind": "port",
            "states": n,
            "sample": f"{name} model, {n} states per step (of {cfg.global_states}), fp32, relmo's torch formulas "
                      f"for the fan ops (PyG-free restatement), {steps} steps after {warmup} warm-up"}


def reference_arm(args) -> None:
    """--impl reference: the reference's CPU ops on the host cores."""

    rank = env_int("RANK", 0)
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if args.workload in ("cfg3", "cfg4"):
        base = model_cpu_baseline(args.workload, steps=max(args.steps, 1), warmup=args.warmup)
        line = {
            "impl": "reference", "metric": MODEL_METRIC, "value": base["value"], "unit": "states/s",
            "n_gpus": args.gpus, "steps": max(args.steps, 1), "warmup": args.warmup,
            "ms_per_step": round(base["states"] / base["value"] * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload}, "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "states/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return
    if args.workload == "lgan":
        print(json.dumps(lgan_reference_line(args, threads)), flush=True)
        return
    edges = args.cpu_edges
    wl = cpu_sample(args.workload, edges)
    kind = "port"
    if REF_LIB.is_file():
        torch.ops.load_library(str(REF_LIB))
        ops = torch.ops.relm_mp
        kind = "reference"
    op_list = ops_of(args.workload)
    nbytes = sum(op_bytes(wl, op_list).values())
    times = []
    for i in range(args.warmup + args.steps):
        if kind == "reference":
            t0 = time.perf_counter()
            run_ops(ops, wl, op_list)
            dt = time.perf_counter() - t0
        else:
            dt, _ = time_oracle_port(wl, op_list=op_list)
        if i >= args.warmup:
            times.append(dt)
    step = sum(times) / len(times)
    value = nbytes / step / 1e9
    sample = (f"{args.workload} with E={edges} messages (of {1 << 24 if args.workload.startswith('cfg2') else 'n/a'}),"
              f" same N, D and index distributions; {len(op_list)} ops per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "edges_sample": edges, "nodes": int(wl.dim_size), "emb": wl.emb},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads if kind == "reference" else 1,
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.workload.startswith("cfg2") and args.reference_gpu:
        line["reference_gpu"] = reference_gpu_ops(args.workload)
    print(json.dumps(line), flush=True)


def reference_gpu_ops(workload: str) -> dict:
    """The reference's own SIMT kernels (mp_cuda_kernels.cu built for sm_100a by
    oracle/build_ref.py --cuda) timed per op on the full cfg2 workload on this
    box's GPU, in a process of their own (oracle/ref_gpu_ops.py): the same-box
    GPU baseline beside the CPU one. Not part of this arm's value."""

    if not torch.cuda.is_available():
        return {"unavailable": "no GPU in this process"}
    try:
        proc = subprocess.run([sys.executable, str(ROOT / "oracle" / "ref_gpu_ops.py"), "--workload", workload],
                              capture_output=True, text=True, timeout=900)
    except subprocess.TimeoutExpired:
        return {"unavailable": "reference GPU ops did not finish in 900 s"}
    for line in reversed(proc.stdout.splitlines()):
        if line.startswith("{"):
            return json.loads(line)
    return {"unavailable": f"reference GPU ops exited {proc.returncode}: {proc.stderr.strip()[-300:]}"}


# ---- B200 arm -------------------------------------------------------------------------------


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--workload", default="cfg2-unsorted",
                        choices=["cfg2-unsorted", "cfg2-sorted", "cfg5", "cfg1", "cfg3", "cfg4", "lgan"])
    parser.add_argument("--dtype", default="float32", choices=["float32", "bfloat16"])
    parser.add_argument("--cpu-edges", type=int, default=1 << 22, help="edge sample of the reference arm")
    parser.add_argument("--port-edges", type=int, default=1 << 20, help="edge sample of the cpu_baseline leg")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--e2e-steps", type=int, default=2)
    parser.add_argument("--ops-only", action="store_true", help="per-op kernel timing only (profiling runs)")
    parser.add_argument("--ops", default=None, help="ops timed by --ops-only (comma list; default: the workload's)")
    parser.add_argument("--reps", type=int, default=5, help="timed repetitions per op in the per-op timing")
    parser.add_argument("--nodes", type=int, default=None, help="override the workload's node count (profiling)")
    parser.add_argument("--edges", type=int, default=None, help="override the workload's edge count (profiling)")
    parser.add_argument("--emb", type=int, default=None,
                        help="override the workload's embedding width (profiling: plan builds at full index size)")
    parser.add_argument("--models", default="cfg3,cfg4",
                        help="RGNN train-step workloads added to the cfg2 line ('' for none)")
    parser.add_argument("--model-steps", type=int, default=2, help="timed train steps per model workload")
    parser.add_argument("--model-warmup", type=int, default=3)
    parser.add_argument("--model-states", type=int, default=None, help="override the global batch (states)")
    parser.add_argument("--micro-states", type=int, default=None, help="states per micro-batch (cfg4 default 512)")
    parser.add_argument("--lgan", type=int, default=1, help="add the LGAN step to the cfg2 line (0: no)")
    parser.add_argument("--extra-tables", type=int, default=1,
                        help="cfg2 line at N=1: add per-op tables of cfg2 bf16 and cfg2 sorted (0: no)")
    parser.add_argument("--reference-gpu", type=int, default=1,
                        help="--impl reference on cfg2: also time the reference's own GPU kernels (0: no)")
    parser.add_argument("--cfg5-part", type=int, default=1,
                        help="cfg2 line: add the cfg5 destination-range partition at every N (0: no)")
    parser.add_argument("--lgan-relations", type=int, default=1 << 20, help="LGAN relation instances")
    parser.add_argument("--lgan-entities", type=int, default=1 << 17, help="LGAN entities")
    parser.add_argument("--lgan-steps", type=int, default=5, help="timed LGAN steps in the cfg2 line")
    args = parser.parse_args()

    if args.impl == "reference":
        reference_arm(args)
        return 0

    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))
    else:
        torch.cuda.set_device(0)
    device = torch.device("cuda", torch.cuda.current_device())

    from relmo_b200 import capi
    from relmo_b200.ops import mp, mp_runtime

    assert mp.available(), "relm_mp library not loadable"
    if args.workload in ("cfg3", "cfg4"):
        return model_main(args, device, rank, world, local_rank)
    if args.workload == "lgan":
        return lgan_main(args, device, rank, world, local_rank)
    ops = torch.ops.relm_mp
    dtype = torch.float32 if args.dtype == "float32" else torch.bfloat16
    op_list = ops_of(args.workload)
    partitioned = args.workload == "cfg5" and world > 1
    # weak scaling: an independent batch per rank; cfg5: one global workload split by destination range
    wl = make_workload(args.workload, seed=0 if partitioned else rank, device=device, dtype=dtype,
                       nodes=args.nodes, edges=args.edges, emb=args.emb)
    global_nodes, global_edges = int(wl.dim_size), wl.num_edges
    if partitioned:
        wl = shard_workload(wl, rank, world)
        torch.cuda.empty_cache()
    nbytes = op_bytes(wl, op_list)
    step_bytes = sum(nbytes.values())
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(v: float) -> float:
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def step():
        mp.clear_plan_cache()
        return run_ops(ops, wl, op_list)

    # ---- per-op kernel timing (plans cached): roofline of each op -------------------------
    stream = torch.cuda.current_stream()
    timed_ops = op_list if not (args.ops_only and args.ops) else tuple(o for o in args.ops.split(",") if o)
    per_op = time_per_op(ops, wl, timed_ops, args.reps, nbytes)
    if args.ops_only:
        if rank == 0:
            print(json.dumps({"per_op": per_op}), flush=True)
        return 0

    # ---- the timed region ----------------------------------------------------------------
    for _ in range(max(args.warmup, 3)):
        step()
    sampler = ClockSampler(device.index if world == 1 else local_rank)
    sampler.start()
    sampler.settle(step)
    if world > 1:  # every rank ran a rank-local number of settle steps; line them up
        barrier()
    launches0 = capi.lib().relm_mp_kernel_launches()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    barrier()
    clocks = sampler.stop()
    launches = capi.lib().relm_mp_kernel_launches() - launches0
    elapsed = max_over_ranks(ev0.elapsed_time(ev1) / 1e3)
    ms_per_step = elapsed / args.steps * 1e3
    job_bytes = sum_over_ranks(step_bytes)
    value = job_bytes * args.steps / elapsed / 1e9

    # ---- plan build cost (separately) -----------------------------------------------------------
    lse = ops.fanin_reduce(wl.msgs, wl.flat_src, wl.dst, wl.dim_size, 1)
    mp.clear_plan_cache()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for op in op_list:  # the first call of each op builds its plan
        run_one_op(ops, wl, op, lse)
    t1.record(stream)
    torch.cuda.synchronize()
    first_calls_ms = t0.elapsed_time(t1)
    ops_ms = sum(v["ms"] for v in per_op.values())

    # ---- end to end through the public API with host buffers ------------------------------------
    e2e = None
    if not args.no_e2e:
        e2e = end_to_end(ops, mp, wl, args, device, world, max_over_ranks, barrier, op_list, sum_over_ranks)

    peaks = measured_peaks()
    dominant = max(per_op, key=lambda k: per_op[k]["ms"])
    achieved = per_op[dominant]["gbs"]
    # ncu traffic figures are per workload and storage type (fp32 under the bare workload name)
    traffic_key = args.workload if dtype == torch.float32 else f"{args.workload}:{args.dtype}"
    traffic = ncu_traffic().get(traffic_key, {}).get(dominant)
    roofline = {
        "bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
        "algorithmic_bytes": nbytes[dominant], "peak_source": peaks["source"],
    }
    rgnn = {}
    for name in [m for m in args.models.split(",") if m]:
        if name == "cfg3" and world > 1:
            continue  # single-GPU configuration
        rgnn[name] = model_bench(name, args, device, rank, world, max_over_ranks, barrier,
                                 steps=args.model_steps, warmup=args.model_warmup)
    lgan = None
    if args.lgan:
        lgan = lgan_bench(args, device, rank, world, max_over_ranks, sum_over_ranks, barrier,
                          steps=args.lgan_steps, warmup=3)
    extra = {}
    if world == 1 and args.workload == "cfg2-unsorted" and args.extra_tables:
        extra["per_op_bf16"] = extra_per_op(ops, mp, "cfg2-unsorted", torch.bfloat16, 0, device, args.reps)
        extra["per_op_sorted"] = extra_per_op(ops, mp, "cfg2-sorted", torch.float32, 0, device, args.reps)
    if args.workload.startswith("cfg2") and args.cfg5_part:
        extra["cfg5_partitioned"] = cfg5_partitioned(ops, mp, device, rank, world, barrier, max_over_ranks,
                                                     sum_over_ranks, steps=args.steps, warmup=3)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = cpu_sample(args.workload, args.port_edges)
        secs, sbytes = time_oracle_port(sample, op_list=op_list)
        cpu = {"value": round(sbytes / secs / 1e9, 4), "unit": UNIT, "cores": 1, "kind": "port",
               "sample": f"{args.workload} with E={args.port_edges} messages, same N, D and distributions; "
                         f"the {len(op_list)} ops once, C oracle, 1 thread"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "strong" if partitioned else "weak", "vs_baseline": None,
            "dtype": "f32" if dtype == torch.float32 else "bf16", "data": "synthetic",
            "config": {
                "workload": args.workload, "nodes": global_nodes, "edges": global_edges, "emb": wl.emb,
                "dst": "zipf(1.3)" if args.workload.startswith("cfg2") else args.workload,
                "per_rank_batches": 1, "l2": "inputs larger than L2 (no flush needed)",
                "step": f"plan builds (cache cleared) + {len(op_list)} ops",
                "parallelism": (f"work-balanced destination-range partition x{world}, no collective" if partitioned
                                else f"independent batches x{world}"),
            },
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(launches),
            "clocks": clocks,
            "per_op": per_op,
            "rgnn_train": rgnn or None,
            "lgan_step": lgan,
            "plan_and_first_call_ms": round(first_calls_ms, 3),
            "ops_only_ms": round(ops_ms, 3),
            "ops_only_gbs": round(step_bytes / ops_ms / 1e6, 1),
            "libs": mp_runtime.loaded_library_paths(),
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def model_bench(name, args, device, rank, world, max_over_ranks, barrier, *, steps: int, warmup: int,
                e2e: bool = False) -> dict:
    """Train steps of one RGNN workload over all ranks (see the module docstring).
    With ``e2e`` the batch lives in pinned host memory and every step copies its
    index tensors to the device and reads the loss back."""

    from relmo_b200 import capi, model_train

    cfg = model_train.CONFIGS[name]
    states = int(args.model_states or cfg.global_states)
    lo, hi = model_train.shard_states(states, rank, world)
    host_batch = cfg.batch(seed=0, device="cpu", states=states).state_slice(lo, hi)
    per_rank = hi - lo
    micro = int(args.micro_states or (min(per_rank, 512) if name == "cfg4" else per_rank))
    host_micro = model_train.micro_batches(host_batch, micro)
    dev_micro = [b.to(device) for b in host_micro]
    model = model_train.model_for(cfg, seed=0, device=device)
    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP

        model = DDP(model, device_ids=[device.index], gradient_as_bucket_view=True)
    opt = model_train.make_optimizer(model)
    pinned = [model_train.RelationalBatch(b.num_objects, b.num_states,
                                          {p: a.pin_memory() for p, a in b.relations.items()},
                                          b.object_state.pin_memory()) for b in host_micro]
    loss_host = torch.empty((), dtype=torch.float32, pin_memory=True)
    h2d = sum(a.numel() * a.element_size() for b in pinned for a in [*b.relations.values(), b.object_state])

    def step(from_host: bool):
        batches = [b.to(device, non_blocking=True) for b in pinned] if from_host else dev_micro
        loss = model_train.train_step(model, opt, batches, autocast=cfg.autocast)
        if from_host:
            loss_host.copy_(loss, non_blocking=True)
        return loss

    for _ in range(max(warmup, 3)):
        step(False)
    stream = torch.cuda.current_stream()
    result = {}
    for mode in ("device", "e2e") if e2e else ("device",):
        launches0 = capi.lib().relm_mp_kernel_launches()
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(steps):
            loss = step(mode == "e2e")
        ev1.record(stream)
        barrier()
        elapsed = max_over_ranks(ev0.elapsed_time(ev1) / 1e3)
        result[mode] = {"states_per_s": round(states * steps / elapsed, 2),
                        "ms_per_step": round(elapsed / steps * 1e3, 2),
                        "relm_mp_launches_per_step": (capi.lib().relm_mp_kernel_launches() - launches0) // steps}
    loss_value = float(loss)
    finite = math.isfinite(loss_value)
    out = {
        "workload": name, "model": cfg.kind, "emb": cfg.embedding_size, "layers": cfg.num_layers,
        "aggregation": cfg.aggregation, "dtype": "bf16 autocast, fp32 accumulation" if cfg.autocast else "f32",
        "global_states": states, "per_rank_states": per_rank, "micro_states": micro,
        "micro_batches": len(dev_micro), "steps": steps, "warmup": max(warmup, 3),
        "parallelism": f"ddp{world}" if world > 1 else "single", "scaling": "strong",
        "states_per_s": result["device"]["states_per_s"], "ms_per_step": result["device"]["ms_per_step"],
        "relm_mp_launches_per_step": result["device"]["relm_mp_launches_per_step"],
        "loss": round(loss_value, 6) if finite else None, "loss_finite": finite, "optimizer": "AdamW (fused)",
    }
    if e2e:
        out["e2e"] = {"value": result["e2e"]["states_per_s"], "unit": "states/s", "h2d_bytes_per_step": h2d,
                      "d2h_bytes_per_step": 4, "ms_per_step": result["e2e"]["ms_per_step"]}
    return out


def model_main(args, device, rank, world, local_rank) -> int:
    """--workload cfg3|cfg4: the RGNN train step as the headline line."""

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from relmo_b200 import capi
    from relmo_b200.ops import mp_runtime

    sampler = ClockSampler(local_rank)
    launches0 = capi.lib().relm_mp_kernel_launches()
    sampler.start()
    r = model_bench(args.workload, args, device, rank, world, max_over_ranks, barrier, steps=args.steps,
                    warmup=args.warmup, e2e=not args.no_e2e)
    clocks = sampler.stop()
    launches = capi.lib().relm_mp_kernel_launches() - launches0
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = model_cpu_baseline(args.workload)
    if rank == 0:
        line = {
            "metric": MODEL_METRIC, "value": r["states_per_s"], "unit": "states/s", "n_gpus": world,
            "steps": args.steps, "warmup": r["warmup"], "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if "bf16" in r["dtype"] else "f32",
            "data": "synthetic",
            "config": {k: r[k] for k in ("workload", "model", "emb", "layers", "aggregation", "global_states",
                                         "per_rank_states", "micro_states", "micro_batches", "parallelism")}
            | {"l2": "activations far larger than L2 (no flush needed)"},
            "roofline": None, "cpu_baseline": cpu, "e2e": r.get("e2e"),
            "gpu_launches": int(r["relm_mp_launches_per_step"] * args.steps),
            "relm_mp_launches_all_phases": int(launches), "clocks": clocks, "loss": r["loss"],
            "loss_finite": r["loss_finite"],
            "libs": mp_runtime.loaded_library_paths(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


# ---- LGAN step (lgan_pool_reduce + backward) ---------------------------------------------


def lgan_workload(args, seed: int, device, relations=None, entities=None) -> workloads.LganWorkload:
    return workloads.lgan(seed=seed, device=device, relations=int(relations or args.lgan_relations),
                          entities=int(entities or args.lgan_entities))


def lgan_ops(ops, wl: workloads.LganWorkload, mode: int):
    outs = ops.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, mode)
    grad = ops.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities, *wl.graph(),
                                         wl.relation_count, mode)
    return outs, grad


def lgan_bench(args, device, rank, world, max_over_ranks, sum_over_ranks, barrier, *, steps: int, warmup: int,
               e2e: bool = False) -> dict:
    """LGAN forward + backward per rank on its own batch (seed = rank): the full
    step with plan builds (mean and sum modes), and forward / backward alone
    with cached plans."""

    from relmo_b200.ops import mp

    ops = torch.ops.relm_mp
    wl = lgan_workload(args, rank, device)
    nbytes = workloads.lgan_algorithmic_bytes(wl)
    step_bytes = nbytes["lgan_fwd"] + nbytes["lgan_bwd"]
    stream = torch.cuda.current_stream()
    out = {
        "workload": "lgan", "entities": wl.entity_dim_size, "relations": wl.relation_count, "slots": wl.num_slots,
        "rr_edges": int(wl.rr_src.numel()), "tn_edges": int(wl.tn_rel.numel()), "nn_edges": int(wl.nn_rel.numel()),
        "emb": wl.emb, "dtype": "f32", "bytes_per_step": step_bytes,
    }
    for mode, tag in ((2, "mean"), (0, "sum")):
        # cached plans: forward and backward alone
        for _ in range(max(warmup, 3)):
            lgan_ops(ops, wl, mode)
        per_op = {}
        for name in ("lgan_fwd", "lgan_bwd"):
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            ev0.record(stream)
            for _ in range(args.reps):
                if name == "lgan_fwd":
                    ops.lgan_pool_reduce(wl.slots, wl.slot_to_rel, wl.arities, *wl.graph(), wl.entity_dim_size, mode)
                else:
                    ops.lgan_pool_reduce_backward(wl.grad_x, wl.grad_tn, wl.grad_nn, wl.slot_to_rel, wl.arities,
                                                  *wl.graph(), wl.relation_count, mode)
            ev1.record(stream)
            torch.cuda.synchronize()
            ms = ev0.elapsed_time(ev1) / args.reps
            per_op[name] = {"ms": round(ms, 4), "gbs": round(nbytes[name] / ms / 1e6, 1)}

        def step():
            mp.clear_plan_cache()
            return lgan_ops(ops, wl, mode)

        for _ in range(max(warmup, 3)):
            step()
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(steps):
            step()
        ev1.record(stream)
        barrier()
        elapsed = max_over_ranks(ev0.elapsed_time(ev1) / 1e3)
        job_bytes = sum_over_ranks(step_bytes)
        ops_ms = per_op["lgan_fwd"]["ms"] + per_op["lgan_bwd"]["ms"]
        out[tag] = {
            "value": round(job_bytes * steps / elapsed / 1e9, 2), "unit": UNIT,
            "ms_per_step": round(elapsed / steps * 1e3, 4), "steps": steps,
            "ops_only_ms": round(ops_ms, 4), "ops_only_gbs": round(step_bytes / ops_ms / 1e6, 1), "per_op": per_op,
        }
    if e2e:
        out["e2e"] = lgan_end_to_end(ops, wl, args, device, max_over_ranks, sum_over_ranks, barrier, step_bytes)
    return out


def lgan_end_to_end(ops, wl, args, device, max_over_ranks, sum_over_ranks, barrier, step_bytes) -> dict:
    """Mean-mode forward + backward through torch.ops.relm_mp with every input
    copied in from pinned host memory and every output copied back inside the
    timed region (the index copies change the indices' versions, so every step
    also rebuilds its plans, as a new batch would)."""

    names = ("slots", "slot_to_rel", "arities", "rr_src", "rr_dst", "tn_rel", "tn_ent", "nn_rel", "nn_ent",
             "grad_x", "grad_tn", "grad_nn")
    host = {n: getattr(wl, n).cpu().pin_memory() for n in names}
    dev = {n: torch.empty_like(getattr(wl, n)) for n in names}
    dwl = workloads.LganWorkload("lgan", *(dev[n] for n in names[:9]), wl.entity_dim_size,
                                 *(dev[n] for n in names[9:]))
    compute = torch.cuda.current_stream()
    outs_host = []

    def one():
        for n in names:
            dev[n].copy_(host[n], non_blocking=True)
        outs, grad = lgan_ops(ops, dwl, 2)
        res = list(outs) + [grad]
        if not outs_host:
            outs_host.extend(torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in res)
        for h, t in zip(outs_host, res):
            h.copy_(t, non_blocking=True)

    one()
    torch.cuda.synchronize()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in outs_host)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(compute)
    for _ in range(args.e2e_steps):
        one()
    ev1.record(compute)
    barrier()
    elapsed = max_over_ranks(ev0.elapsed_time(ev1) / 1e3)
    return {
        "value": round(sum_over_ranks(step_bytes) * args.e2e_steps / elapsed / 1e9, 3), "unit": UNIT,
        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
        "ms_per_step": round(elapsed / args.e2e_steps * 1e3, 2), "steps": args.e2e_steps,
        "copies": "pinned host buffers, copies and ops in order on the current stream",
    }


def lgan_cpu_port(relations: int = 1 << 18, entities: int = 1 << 15) -> dict:
    """The C oracle (one thread) on a bounded LGAN sample: forward + backward, mean."""

    from oracle import oracle

    wl = workloads.lgan(seed=0, device="cpu", relations=relations, entities=entities)
    nb = workloads.lgan_algorithmic_bytes(wl)
    graph = [t for t in wl.graph()]
    t0 = time.perf_counter()
    oracle.lgan_pool_reduce(wl.slots.numpy(), wl.slot_to_rel, wl.arities, *graph, wl.entity_dim_size, 2)
    oracle.lgan_pool_reduce_backward(wl.grad_x.numpy(), wl.grad_tn.numpy(), wl.grad_nn.numpy(), wl.slot_to_rel,
                                     wl.arities, *graph, wl.relation_count, 2)
    secs = time.perf_counter() - t0
    return {"value": round((nb["lgan_fwd"] + nb["lgan_bwd"]) / secs / 1e9, 4), "unit": UNIT, "cores": 1,
            "kind": "port", "sample": f"lgan with {relations} relation instances, {entities} entities (same arity, "
                                      f"RR density and D), mean forward + backward once, C oracle, 1 thread"}


def lgan_reference_line(args, threads: int) -> dict:
    """--impl reference --workload lgan: the reference's CPU library (ATen
    formulas) on a bounded sample, all host threads."""

    relations, entities = 1 << 19, 1 << 16
    wl = workloads.lgan(seed=0, device="cpu", relations=relations, entities=entities)
    nb = workloads.lgan_algorithmic_bytes(wl)
    step_bytes = nb["lgan_fwd"] + nb["lgan_bwd"]
    if REF_LIB.is_file():
        torch.ops.load_library(str(REF_LIB))
        ops, kind, cores = torch.ops.relm_mp, "reference", threads
        run = lambda: lgan_ops(ops, wl, 2)  # noqa: E731
    else:
        from oracle import oracle

        kind, cores = "port", 1

        def run():
            graph = list(wl.graph())
            oracle.lgan_pool_reduce(wl.slots.numpy(), wl.slot_to_rel, wl.arities, *graph, wl.entity_dim_size, 2)
            oracle.lgan_pool_reduce_backward(wl.grad_x.numpy(), wl.grad_tn.numpy(), wl.grad_nn.numpy(),
                                             wl.slot_to_rel, wl.arities, *graph, wl.relation_count, 2)
    times = []
    for i in range(args.warmup + max(args.steps, 1)):
        t0 = time.perf_counter()
        run()
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    step = sum(times) / len(times)
    value = step_bytes / step / 1e9
    sample = f"lgan with {relations} relation instances, {entities} entities, mean forward + backward per step"
    return {
        "impl": "reference", "metric": LGAN_METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
        "steps": max(args.steps, 1), "warmup": args.warmup, "ms_per_step": round(step * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "lgan", "relations_sample": relations, "entities_sample": entities, "emb": wl.emb},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def lgan_main(args, device, rank, world, local_rank) -> int:
    """--workload lgan: the LGAN step (mean) as the headline line."""

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()

    def reduce(v: float, op) -> float:
        if world == 1:
            return v
        import torch.distributed as dist

        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=op)
        return float(t.item())

    import torch.distributed as dist

    from relmo_b200 import capi
    from relmo_b200.ops import mp_runtime

    max_over_ranks = lambda v: reduce(v, dist.ReduceOp.MAX)  # noqa: E731
    sum_over_ranks = lambda v: reduce(v, dist.ReduceOp.SUM)  # noqa: E731
    sampler = ClockSampler(local_rank)
    sampler.start()
    launches0 = capi.lib().relm_mp_kernel_launches()
    r = lgan_bench(args, device, rank, world, max_over_ranks, sum_over_ranks, barrier, steps=args.steps,
                   warmup=args.warmup, e2e=not args.no_e2e)
    launches = capi.lib().relm_mp_kernel_launches() - launches0
    clocks = sampler.stop()
    peaks = measured_peaks()
    mean = r["mean"]
    achieved = mean["ops_only_gbs"]
    cpu = lgan_cpu_port() if rank == 0 and world == 1 and not args.no_cpu_baseline else None
    if rank == 0:
        line = {
            "metric": LGAN_METRIC, "value": mean["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": mean["ms_per_step"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {k: r[k] for k in ("workload", "entities", "relations", "slots", "rr_edges", "tn_edges",
                                         "nn_edges", "emb")}
            | {"mode": "mean", "step": "plan builds (cache cleared) + lgan_pool_reduce + backward",
               "l2": "inputs larger than L2 (no flush needed)", "parallelism": f"independent batches x{world}"},
            "roofline": {
                "bound": "hbm", "kernel": "lgan_pool_reduce + backward, plans cached", "achieved": achieved,
                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                "traffic": ncu_traffic().get("lgan", {}).get("lgan_step"), "algorithmic_bytes": r["bytes_per_step"],
                "peak_source": peaks["source"],
            },
            "cpu_baseline": cpu, "e2e": r.get("e2e"), "gpu_launches": int(launches), "clocks": clocks,
            "lgan_step": r, "libs": mp_runtime.loaded_library_paths(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


OP_INPUTS = {
    "fanout_fwd": ("x", "src", "flat_dst"),
    "fanout_bwd": ("grad_slots", "src", "flat_dst"),
    "fanin_sum_fwd": ("msgs", "flat_src", "dst"),
    "fanin_sum_bwd": ("grad_nodes", "flat_src", "dst"),
    "fanin_lse_fwd": ("msgs", "flat_src", "dst"),
    "fanin_lse_bwd": ("grad_nodes", "msgs", "flat_src", "dst"),
}


E2E_ORDER = ("fanin_sum_bwd", "fanout_fwd", "fanin_sum_fwd", "fanin_lse_fwd", "fanin_lse_bwd", "fanout_bwd")


def end_to_end(ops, mp, wl, args, device, world, max_over_ranks, barrier, op_list=OPS, sum_over_ranks=None) -> dict:
    """Same step through torch.ops.relm_mp with the inputs copied in from pinned
    host memory and every op output copied back, all inside the timed region.

    The copies run on their own streams, ordered by first use: an op starts as
    soon as its own inputs are on the device (the host-to-device copy of the next
    op's inputs overlaps it) and its output goes back to the host while the next
    op runs. One step's copies wait for the previous step's ops (same buffers).
    The same ops as the timed step, in E2E_ORDER."""

    # Ops whose outputs are large and inputs small go first, so the long
    # device-to-host copies start early and overlap the long host-to-device ones.
    op_list = [op for op in E2E_ORDER if op in op_list]
    names_in = []
    for op in op_list:
        for n in OP_INPUTS[op]:
            if n not in names_in:
                names_in.append(n)
    host = {n: getattr(wl, n).cpu().pin_memory() for n in names_in}
    dev = {n: torch.empty_like(getattr(wl, n)) for n in names_in}
    for n in ("x", "src", "flat_dst", "msgs", "flat_src", "dst", "grad_slots", "grad_nodes"):
        dev.setdefault(n, getattr(wl, n))
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    dwl = workloads.FanWorkload(
        wl.name, dev["x"], dev["src"], dev["flat_dst"], wl.out_rows, dev["msgs"], dev["flat_src"], dev["dst"],
        wl.dim_size, dev["grad_slots"], dev["grad_nodes"],
    )
    outs_host = {}
    compute = torch.cuda.current_stream()
    h2d_stream = torch.cuda.Stream(device=device)
    d2h_stream = torch.cuda.Stream(device=device)

    def one():
        step_start = torch.cuda.Event()
        step_start.record(compute)
        h2d_stream.wait_event(step_start)  # previous step's ops are done with the buffers
        ready = {}
        with torch.cuda.stream(h2d_stream):
            for n in names_in:
                dev[n].copy_(host[n], non_blocking=True)
                ready[n] = torch.cuda.Event()
                ready[n].record(h2d_stream)
        lse = None
        done = []
        for op in op_list:
            for n in OP_INPUTS[op]:
                compute.wait_event(ready[n])
            if op == "fanin_lse_bwd" and lse is None:
                lse = ops.fanin_reduce(dwl.msgs, dwl.flat_src, dwl.dst, dwl.dim_size, 1)
            out = run_one_op(ops, dwl, op, lse)
            if op == "fanin_lse_fwd":
                lse = out
            ev = torch.cuda.Event()
            ev.record(compute)
            d2h_stream.wait_event(ev)
            if op not in outs_host:
                outs_host[op] = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
            with torch.cuda.stream(d2h_stream):
                out.record_stream(d2h_stream)
                outs_host[op].copy_(out, non_blocking=True)
            done.append(out)
        fin = torch.cuda.Event()
        fin.record(d2h_stream)
        compute.wait_event(fin)
        return done

    one()
    torch.cuda.synchronize()
    d2h = sum(t.numel() * t.element_size() for t in outs_host.values())
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(compute)
    for _ in range(args.e2e_steps):
        one()
    ev1.record(compute)
    barrier()
    elapsed = max_over_ranks(ev0.elapsed_time(ev1) / 1e3)
    step_bytes = sum(op_bytes(wl, op_list).values())
    job_bytes = sum_over_ranks(step_bytes) if sum_over_ranks is not None else step_bytes * world
    return {
        "value": round(job_bytes * args.e2e_steps / elapsed / 1e9, 3), "unit": UNIT,
        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
        "ms_per_step": round(elapsed / args.e2e_steps * 1e3, 2), "steps": args.e2e_steps,
        "copies": "pinned host buffers, H2D / compute / D2H on three streams, ordered by first use",
        "op_order": list(op_list),
    }

if __name__ == "__main__":
    sys.exit(main())
