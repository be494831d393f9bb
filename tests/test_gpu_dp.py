"""Data-parallel training on two GPUs (skipped with fewer than two).

Two ranks, one process per GPU, each training the MLP classifier on its half
of the global batch with the NCCL gradient average inside backward.  In the
exact fp32 mode the averaged gradients must equal a full-batch run on the same
GPU up to summation order (relative L2 1e-5), and after Adam every rank must
hold bit-identical parameters.  The communicator id travels through the
TCPStore path; NVLS is off (no multicast objects).
"""

import hashlib
import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def _gpus() -> int:
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank_main(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0",
                      NCCL_DEBUG="WARN")
    sys.path.insert(0, str(ROOT))
    try:
        import tynx_b200 as tx
        from tynx_b200 import workloads
        from tynx_b200.distributed import init_data_parallel, shard

        tx.set_math_mode("fp32")
        wl = workloads.mlp_classifier(batch=512)
        model = tx.load(wl.onnx, trainable="auto")
        ref = tx.load(wl.onnx, trainable="auto")
        init_data_parallel(world, rank, timeout_ms=60000)
        model.enable_data_parallel(bucket_mb=1)
        opt = tx.optim.Adam(model.named_parameters(), lr=wl.lr)
        ref_opt = tx.optim.Adam(ref.named_parameters(), lr=wl.lr)
        rows = shard(wl.batch, world, rank)
        worst = 0.0
        for step in range(3):
            batch = wl.make_batch(step)
            opt.zero_grad()
            ref_opt.zero_grad()
            loss = tx.nn.functional.cross_entropy(model(tx.Tensor(batch["x"][rows])),
                                                  tx.Tensor(batch["y"][rows]))
            loss.backward()
            ref_loss = tx.nn.functional.cross_entropy(ref(tx.Tensor(batch["x"])), tx.Tensor(batch["y"]))
            ref_loss.backward()
            got = dict(model.named_parameters())
            for name, p in ref.named_parameters():
                g, r = got[name].grad.numpy(), p.grad.numpy()
                err = float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30))
                worst = max(worst, err)
            opt.step()
            ref_opt.step()
        digest = hashlib.sha256()
        for name, p in model.named_parameters():
            digest.update(p.numpy().tobytes())
        tx.synchronize()
        queue.put((rank, True, (worst, digest.hexdigest())))
    except BaseException as exc:  # report, never hang the parent
        queue.put((rank, False, f"{type(exc).__name__}: {exc}"))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_two_gpu_data_parallel_matches_full_batch():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 240
    while len(results) < 2 and time.time() < deadline:
        try:
            rank, ok, value = queue.get(timeout=1.0)
            results[rank] = (ok, value)
        except Exception:
            if all(not p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    assert len(results) == 2, f"ranks that reported: {sorted(results)}"
    for rank, (ok, value) in results.items():
        assert ok, f"rank {rank}: {value}"
    (w0, h0), (w1, h1) = results[0][1], results[1][1]
    assert max(w0, w1) < 1e-5, (w0, w1)
    assert h0 == h1
