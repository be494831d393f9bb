"""Training-step throughput of the B200 engine (samples/s, fwd+bwd+Adam).

Default workload: the transformer encoder fine-tune (token + positional
embedding 8192x256 / 128x256, four pre-norm layers of d_model 256, 4 heads, FFN
1024 GELU, mean-pool, Gemm 256->2; global batch 256 sequences x 128 tokens
sharded across ranks; cross-entropy; Adam 1e-4), the largest of the five
configurations on one GPU.  ``--workload`` selects another one
(mlp_policy, mlp_classifier, ppo, cnn).
One step = zero_grad, forward, fused softmax-cross-entropy, backward (with the
NCCL gradient all-reduce inside backward when N > 1) and one Adam step,
captured once with ``tynx_b200.compile`` and replayed as a CUDA graph.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--math tf32|3xtf32|fp32] [--impl ours|reference]

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events
on the engine's stream with an L2 flush (a 512 MiB write, larger than the
126 MB L2) between steps outside the events; the per-rank total is the sum of
the K step times; barrier + synchronize on both sides; the job time is the max
over ranks.  ``e2e`` repeats the measurement through the public API with the
step's inputs copied from pinned host memory and the loss read back each step
(host clock, max over ranks).  ``--impl reference`` times the CPU oracle (the
numpy restatement of the reference's Flex training step) with every host
thread, each step on a bounded sample of the global batch; it imports only the
host-side workload and ONNX modules, never the CUDA library.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

if "--impl" in sys.argv and "reference" in sys.argv:
    # The CPU arm uses every host thread for BLAS, whatever the launcher set
    # (torchrun exports OMP_NUM_THREADS=1 to every rank).
    for _var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_var] = str(os.cpu_count() or 1)

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def _dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


class Clocks:
    """Sample SM clocks and throttle reasons with nvidia-smi during a region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        query = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={query}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in Path(self.path).read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(int(r[1]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def _np_dtype(name: str):
    return {"float32": np.float32, "int64": np.int64, "bool": np.bool_}[name]


def _flush_l2(tx, buf):
    # writing 512 MiB evicts the 126 MB L2
    from tynx_b200 import _native as N

    ctx = buf.ctx
    ctx.check(N.lib.tx_memset(ctx.handle, buf.ptr, 0, buf.nbytes))


def _cpu_step_fn(wl):
    """The oracle's training step on the workload (for the CPU baseline)."""
    from oracle import flex_oracle as fo
    from tynx_b200.onnx import ir

    model = fo.OracleModel(ir.load_training_graph(wl.onnx))
    opt = fo.Adam(model.named_parameters(), lr=wl.lr)
    key = "ids" if wl.name == "transformer" else ("obs" if wl.loss == "ppo" else "x")

    def step(batch):
        opt.zero_grad()
        if wl.loss == "ppo":
            out = model(batch["obs"])
            n = batch["obs"].shape[0]
            loss = fo.ppo_loss(out["logits"], out["value"], batch["actions"],
                               np.zeros(n, np.float32), batch["advantages"], batch["returns"])
        else:
            loss = fo.cross_entropy(model(batch[key]), batch["y"])
        loss.backward()
        opt.step()
        return loss.item()

    return step


def _head(batch: dict, rows: int) -> dict:
    """The first `rows` samples of a batch (every per-sample array sliced)."""
    return {k: (v[:rows] if isinstance(v, np.ndarray) and v.ndim >= 1 else v) for k, v in batch.items()}


def _sample_rows(wl, step, per_step_s: float) -> tuple[int, float]:
    """Rows of the global batch one CPU step may take so that it lasts about
    per_step_s: one cold step on 1/16 of the batch, then a timed one, scaled."""
    rows = max(1, wl.batch // 16)
    step(_head(wl.make_batch(0), rows))  # cold
    t0 = time.perf_counter()
    step(_head(wl.make_batch(1), rows))
    per_row = (time.perf_counter() - t0) / rows
    fit = int(per_step_s / max(per_row, 1e-9))
    # a power-of-two fraction of the batch, at least 1/16 of it
    sample = wl.batch
    while sample > rows and sample > fit:
        sample //= 2
    return sample, per_row


def bench_config(wl, world: int) -> dict:
    """The workload description both arms print (identical dicts)."""
    return {"workload": wl.name, "global_batch": wl.batch, "per_gpu_batch": wl.batch // world,
            "parallelism": f"dp{world}", "l2": "flushed between steps (512 MiB write)",
            "flop_per_step": wl.flop_per_step}


def cpu_baseline(wl, budget_s: float = 15.0) -> dict:
    """Time the oracle's step on the host cores: a bounded sample of the
    workload (whole steps on a slice of the global batch), all host threads."""
    step = _cpu_step_fn(wl)
    sample, _ = _sample_rows(wl, step, budget_s / 8)
    times = []
    start = time.perf_counter()
    i = 2
    while time.perf_counter() - start < budget_s and i < 50:
        b = _head(wl.make_batch(i), sample)
        t0 = time.perf_counter()
        step(b)
        times.append(time.perf_counter() - t0)
        i += 1
    med = float(np.median(times))
    cores = os.cpu_count() or 1
    return {"value": sample / med, "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": f"{len(times)} {wl.name} training steps of the numpy oracle on {sample} of the "
                      f"{wl.batch} samples of a global batch (multithreaded BLAS, {cores} host "
                      f"threads), median step {med * 1e3:.1f} ms"}


def run_reference(args) -> None:
    """The reference arm: the oracle's training step (the CPU restatement of the
    reference's Flex step), every host thread, on a bounded sample per step.
    Under torchrun only rank 0 runs; the other ranks exit without work."""
    world, rank, _ = _dist_env()
    if rank != 0:
        return
    from tynx_b200 import workloads  # host-side module: the CUDA library stays unmapped

    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(os.cpu_count() or 1)
    except Exception:  # pragma: no cover - the environment variables already ask for it
        pass
    wl = make_workload(workloads, args)
    step = _cpu_step_fn(wl)
    # the whole run (warm-up + timed) stays near two minutes of host time
    sample, _ = _sample_rows(wl, step, 120.0 / (args.steps + args.warmup))
    for i in range(args.warmup):
        step(_head(wl.make_batch(i), sample))
    times = []
    for i in range(args.steps):
        b = _head(wl.make_batch(args.warmup + i), sample)
        t0 = time.perf_counter()
        step(b)
        times.append(time.perf_counter() - t0)
    total = float(sum(times))
    value = sample * args.steps / total
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": "train samples/s (fwd+bwd+Adam)", "value": value,
        "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy; the reference names no dataset)",
        "config": bench_config(wl, world),
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": cores, "kind": "port",
                         "sample": f"each step: the numpy restatement of the Flex training step on "
                                   f"{sample} of the {wl.batch} samples of the global batch "
                                   f"({cores} host threads)"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def make_workload(workloads, args):
    """The workload at its configured size, or at --global-batch."""
    if not args.global_batch:
        return workloads.WORKLOADS[args.workload]()
    key = "minibatch" if args.workload == "ppo" else "batch"
    return workloads.WORKLOADS[args.workload](**{key: args.global_batch})


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=50)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--workload", default="transformer")
    parser.add_argument("--math", default="tf32", choices=["tf32", "3xtf32", "fp32", "tf32trunc"])
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-budget", type=float, default=15.0)
    parser.add_argument("--bucket-mb", type=float, default=2.0,
                        help="gradient all-reduce bucket size when N > 1")
    parser.add_argument("--global-batch", type=int, default=0,
                        help="override the workload's global batch (PPO: the minibatch); with --gpus 1 "
                             "at the N-GPU per-rank batch it times the same per-GPU work without the exchange")
    args = parser.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    world, rank, local = _dist_env()
    os.environ.setdefault("TYNX_CUDA_MATH", args.math)
    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    import tynx_b200 as tx
    from tynx_b200 import _core, workloads
    from tynx_b200 import _native as N
    from tynx_b200.distributed import init_data_parallel, shard

    tx.set_math_mode(args.math)
    wl = make_workload(workloads, args)
    per_rank = wl.batch // world
    rows = shard(wl.batch, world, rank)
    ctx = _core.context()
    model = tx.load(wl.onnx, trainable="auto")
    opt = tx.optim.Adam(model.named_parameters(), lr=wl.lr)
    if world > 1:
        init_data_parallel(world, rank)
        model.enable_data_parallel(bucket_mb=args.bucket_mb)

    if wl.loss == "ppo":
        # the captured PPO minibatch update: clipped surrogate + 0.5 value MSE
        # - 0.01 entropy; behaviour log-probs come from the initial policy
        with tx.no_grad():
            obs_all = wl.notes["rollout_obs"]
            logits = model(tx.Tensor(obs_all))["logits"]
        from tynx_b200.distributions import Categorical

        dtypes = ("float32", "int64", "float32", "float32", "float32")
        # log-probs of every rollout action under the initial policy
        all_actions = np.empty(obs_all.shape[0], np.int64)
        for j in range(obs_all.shape[0] // wl.batch):
            b = wl.make_batch(j)
            all_actions[b["index"]] = b["actions"]
        with tx.no_grad():
            old_all = Categorical(logits=logits).log_prob(tx.Tensor(all_actions, dtype="int64")).numpy()

        def host_inputs(i):
            b = wl.make_batch(i)
            return (b["obs"], b["actions"], old_all[b["index"]], b["advantages"], b["returns"])

        @tx.compile(fullgraph=True)
        def train_step(obs, actions, old_logp, adv, ret):
            opt.zero_grad()
            out = model(obs)
            # the clipped surrogate + 0.5 value MSE - 0.01 entropy, as one fused
            # kernel pair (the same objective the reference composes from
            # Categorical, minimum, clamp and mse_loss)
            loss = tx.nn.functional.ppo_loss(out["logits"], out["value"], actions, old_logp, adv, ret)
            loss.backward()
            opt.step()
            return loss
    else:
        key = "ids" if args.workload == "transformer" else "x"
        dtypes = ("int64" if key == "ids" else "float32", "int64")

        def host_inputs(i):
            b = wl.make_batch(i)
            return (b[key], b["y"])

        @tx.compile(fullgraph=True)
        def train_step(x, y):
            opt.zero_grad()
            loss = tx.nn.functional.cross_entropy(model(x), y)
            loss.backward()
            opt.step()
            return loss

    # device-resident batches (one per step) for the kernel-time measurement
    n_batches = args.warmup + args.steps
    host = [host_inputs(i) for i in range(n_batches)]
    dev = [tuple(tx.Tensor(a[rows], dtype=dt) for a, dt in zip(h, dtypes)) for h in host]
    flush = tx.zeros(128 << 20)  # 512 MiB

    stream = ctypes_stream(ctx)
    ext = torch.cuda.ExternalStream(stream, device=torch.device("cuda", ctx.index))

    def barrier():
        tx.synchronize()
        if world > 1:
            dist.barrier()

    # warm-up (first call captures, later calls replay)
    for i in range(args.warmup):
        train_step(*dev[i])
    entry = train_step.entry_for(*dev[0])
    launches_per_step = entry.kernel_count if entry is not None else None
    barrier()

    # ---- device-timed steps --------------------------------------------------------
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with Clocks(ctx.index) as clocks:
        barrier()
        for i in range(args.steps):
            # stage this step's batch into the graph's input buffers, then evict L2
            for dst, src in zip(entry.static_inputs, dev[args.warmup + i]):
                ctx.check(N.lib.tx_d2d(ctx.handle, dst.ptr, src.ptr, src.nbytes))
            _flush_l2(tx, flush)
            starts[i].record(ext)
            ctx.check(N.lib.tx_exec_launch(entry.exec), "graph replay")
            ends[i].record(ext)
            entry.apply_post_state()
        barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = float(sum(step_ms))
    if world > 1:
        t = torch.tensor([total_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = wl.batch * args.steps / (total_ms / 1e3)

    # ---- roofline of the dominant kernel (the largest forward GEMM) -----------------
    roofline = gemm_roofline(tx, ctx, ext, wl, per_rank, args.math)

    # ---- end to end through the public API with host buffers -------------------------
    # A Prefetcher uploads the next two batches on its copy stream while step i
    # runs; every step still includes its own upload and the read-back of its loss.
    pinned = [tuple(tx.pinned(np.ascontiguousarray(a[rows], dtype=np.dtype(_np_dtype(dt))))
                    for a, dt in zip(h, dtypes)) for h in host[args.warmup:]]
    prefetch = tx.Prefetcher(*pinned[0], depth=3)
    barrier()
    t0 = time.perf_counter()
    losses = []
    for i in range(min(2, args.steps)):
        prefetch.put(*pinned[i])
    for i in range(args.steps):
        inputs = prefetch.get()
        loss = train_step(*inputs)
        if i + 2 < args.steps:
            prefetch.put(*pinned[i + 2])
        losses.append(loss.item())
    barrier()
    e2e_s = time.perf_counter() - t0
    prefetch.close()
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    h2d = sum(a.nbytes for a in pinned[0])
    e2e = {"value": wl.batch * args.steps / e2e_s, "unit": "samples/s",
           "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": 4}

    if rank == 0:
        line = {
            "metric": "train samples/s (fwd+bwd+Adam)",
            "value": value,
            "unit": "samples/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "tf32" if args.math == "tf32" else args.math,
            "data": "synthetic (seeded numpy; the reference names no dataset)",
            "config": bench_config(wl, world),
            "math": args.math,
            "achieved_tflops": wl.flop_per_step / (ms_per_step / 1e3) / 1e12,
            "roofline": roofline,
            "e2e": e2e,
            "gpu_launches": (launches_per_step * args.steps) if launches_per_step else None,
            "clocks": clocks.summary(),
            "final_loss": losses[-1],
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = cpu_baseline(wl, args.cpu_budget)
        elif world == 1:
            line["cpu_baseline"] = None
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def ctypes_stream(ctx) -> int:
    import ctypes as C

    from tynx_b200 import _native as N

    out = C.c_void_p()
    ctx.check(N.lib.tx_stream(ctx.handle, C.byref(out)))
    return out.value


def gemm_roofline(tx, ctx, ext, wl, per_rank: int, math: str) -> dict:
    """Time the step's largest forward GEMM alone (CUDA events on the engine stream),
    with the operand layout and epilogue it has in the step."""
    import torch

    from tynx_b200 import _core

    peaks, source = _peaks()
    # largest GEMM of the MLP classifier / policy: hidden x hidden forward
    tb, act, with_bias, with_preact = True, "relu", True, False
    if wl.name in ("mlp_classifier", "mlp_policy"):
        hidden = 1024 if wl.name == "mlp_classifier" else 256
        M, N_, K = per_rank, hidden, hidden
    elif wl.name == "transformer":
        # the first FFN MatMul: weight stored K x N, GELU, pre-activation kept
        M, N_, K = per_rank * 128, 1024, 256
        tb, act, with_bias, with_preact = False, "gelu", False, True
    elif wl.name == "ppo":
        M, N_, K = per_rank, 512, 512
    else:
        M, N_, K = per_rank * 256, 64, 288
    from tynx_b200 import _native as N

    rng = np.random.default_rng(0)
    A = tx.Tensor(rng.standard_normal((M, K)).astype(np.float32))
    B = tx.Tensor(rng.standard_normal((N_, K) if tb else (K, N_)).astype(np.float32))
    Cm = tx.zeros(M, N_)
    bias = tx.zeros(N_)
    pre = tx.zeros(M, N_) if with_preact else None
    flags = 0
    if math == "tf32":
        # as in the step: the activation arrives TF32-rounded from the previous
        # epilogue, the weight from the TF32 shadow, and the output is stored
        # rounded for the next contraction
        for t in (A, B):
            ctx.check(N.lib.tx_round_tf32(ctx.handle, t.ptr, t.ptr, t.nbytes // 4))
        flags = N.TX_GEMM_A_TF32 | N.TX_GEMM_B_TF32 | N.TX_GEMM_ROUND_OUT

    def launch():
        _core.gemm(ctx, M, N_, K, A.ptr, K, False, B.ptr, K if tb else N_, tb, Cm.ptr, N_,
                   bias=bias.ptr if with_bias else None, act=act, flags=flags,
                   preact=pre.ptr if pre is not None else None)

    for _ in range(5):
        launch()
    tx.synchronize()
    # one event pair per launch: the device time of the kernel, not the host's
    # enqueue rate; L2 is flushed before each launch (inputs > L2 is not given)
    reps = 20
    flush = tx.zeros(128 << 20)
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(reps)]
    for s, e in pairs:
        _flush_l2(tx, flush)
        # a device-side spin after the flush keeps the GPU busy while the host
        # enqueues the launch, so the event pair brackets device work only
        with torch.cuda.stream(ext):
            torch.cuda._sleep(400000)
        s.record(ext)
        launch()
        e.record(ext)
    pairs[-1][1].synchronize()
    ms = sum(s.elapsed_time(e) for s, e in pairs) / reps
    flops = 2.0 * M * N_ * K
    achieved = flops / (ms / 1e3) / 1e12
    # dense TF32 peak: the measured dense bf16 rate halved (B200: tf32 dense = 1/2 bf16 dense)
    if math == "fp32":
        peak = 80.0
        note = "fp32 SIMT nominal (no tensor cores)"
    else:
        peak = peaks["bf16_tflops"] / 2.0
        note = f"dense TF32 = 1/2 of {source} bf16 burst ({peaks['bf16_tflops']} TF/s)"
    # DRAM bytes per launch of this kernel from an ncu capture of the same
    # command (dram__bytes_read.sum + dram__bytes_write.sum), where one exists
    traffic = None
    tpath = ROOT / "profiles" / "roofline_traffic.json"
    if tpath.exists() and math == "tf32":
        entry = json.loads(tpath.read_text()).get(wl.name)
        if entry and per_rank == wl.batch == entry.get("batch"):
            traffic = entry["traffic_bytes"]
    epi = ("+bias" if with_bias else "") + f"+{act}" + ("+preact" if with_preact else "")
    # algorithmic HBM bytes: A and B read once, C (and the pre-activation) written once
    nbytes = 4.0 * (M * K + K * N_ + M * N_ * (2 if with_preact else 1) + (N_ if with_bias else 0))
    out = {"kernel": f"gemm {M}x{N_}x{K} {epi} ({math})", "flops": flops, "algorithmic_bytes": nbytes,
           "traffic": traffic, "traffic_unit": "bytes/launch", "duration_us": ms * 1e3}
    if nbytes / (peaks["hbm_gbs"] * 1e9) > flops / (peak * 1e12):
        # the stores outweigh the math: bound by HBM
        gbs = nbytes / (ms / 1e3) / 1e9
        out.update({"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": gbs / peaks["hbm_gbs"], "peak_source": f"{source} HBM copy bandwidth",
                    "tflops": achieved})
    else:
        out.update({"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                    "frac": achieved / peak, "peak_source": note})
    return out


if __name__ == "__main__":
    main()
