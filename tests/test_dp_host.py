"""Host-side logic of the data-parallel step, run as two ``gloo`` ranks on CPU.

The CUDA path averages gradients with ``ncclAvg`` inside backward; what that
relies on, and what is tested here without a GPU:

* the communicator id made by rank 0 reaches every rank unchanged, through an
  initialised process group or the ``TCPStore`` fallback;
* a rank that never joins ends the other ranks' wait with an error (bounded);
* ``shard`` splits a global batch into equal, disjoint, covering shards;
* averaging per-shard mean-loss gradients over the ranks gives the
  global-batch gradient (the oracle on each shard, ``all_reduce`` over gloo),
  and Adam on the averaged gradients leaves every rank with the same
  parameters -- the replicated-optimizer invariant.
"""

from __future__ import annotations

import os
import socket
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from tynx_b200.distributed import exchange_unique_id, shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(fn, world: int, *args) -> list:
    """Run ``fn(rank, world, port, *args)`` on ``world`` spawned ranks; return results."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_wrap, args=(fn, r, world, port, queue) + args) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 120
    while len(results) < world and time.time() < deadline:
        try:
            rank, ok, value = queue.get(timeout=1.0)
        except Exception:
            if all(not p.is_alive() for p in procs) and queue.empty():
                break
            continue
        results[rank] = (ok, value)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
            p.join()
    assert len(results) == world, f"ranks that reported: {sorted(results)}"
    for rank, (ok, value) in sorted(results.items()):
        assert ok, f"rank {rank}: {value}"
    return [results[r][1] for r in range(world)]


def _wrap(fn, rank, world, port, queue, *args):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    try:
        queue.put((rank, True, fn(rank, world, port, *args)))
    except BaseException as exc:  # report, never hang the parent
        queue.put((rank, False, f"{type(exc).__name__}: {exc}"))


def _fake_id() -> bytes:
    return bytes(range(128))


# -- communicator id exchange -----------------------------------------------------------

def _id_via_group(rank, world, port):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        return exchange_unique_id(rank, world, make_id=_fake_id)
    finally:
        dist.destroy_process_group()


def _id_via_store(rank, world, port):
    return exchange_unique_id(rank, world, make_id=_fake_id, timeout_s=30)


def test_unique_id_reaches_every_rank_over_gloo():
    assert _spawn(_id_via_group, 2) == [_fake_id()] * 2


def test_unique_id_reaches_every_rank_over_store():
    assert _spawn(_id_via_store, 2) == [_fake_id()] * 2


def _id_rank0_absent(rank, world, port):
    # only rank 1 runs: it hosts nothing and waits for rank 0's store
    t0 = time.time()
    try:
        exchange_unique_id(1, 2, make_id=_fake_id, timeout_s=2)
    except Exception as exc:  # the bounded wait ends with an error
        return ("error", time.time() - t0, type(exc).__name__)
    return ("returned", time.time() - t0, "")


def test_missing_rank_ends_the_wait_with_an_error():
    [(what, waited, _)] = _spawn(_id_rank0_absent, 1)
    assert what == "error"
    assert waited < 60


def test_unique_id_length_checked():
    with pytest.raises(ValueError):
        exchange_unique_id(0, 1, make_id=lambda: b"short")


# -- shards -------------------------------------------------------------------------------

@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_are_equal_disjoint_and_cover(world):
    n = 4096
    covered = np.zeros(n, np.int64)
    for r in range(world):
        s = shard(n, world, r)
        assert s.stop - s.start == n // world
        covered[s] += 1
    assert (covered == 1).all()


def test_shard_rejects_ragged_batch():
    with pytest.raises(ValueError):
        shard(4097, 2, 0)


# -- averaged shard gradients == global gradient ---------------------------------------

def _dp_step(rank, world, port, name, kw):
    import torch
    import torch.distributed as dist

    from oracle import flex_oracle as fo
    from tynx_b200 import workloads
    from tynx_b200.onnx import ir

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        wl = workloads.WORKLOADS[name](**kw)
        graph = ir.load_training_graph(wl.onnx)
        model = fo.OracleModel(graph)
        opt = fo.Adam(model.named_parameters(), lr=wl.lr)
        key = "ids" if "ids" in wl.make_batch(0) else "x"
        out = []
        for step in range(2):
            batch = wl.make_batch(step)
            rows = shard(wl.batch, world, rank)
            opt.zero_grad()
            loss = fo.cross_entropy(model(batch[key][rows]), batch["y"][rows])
            loss.backward()
            for _, p in model.named_parameters():
                g = torch.from_numpy(np.ascontiguousarray(p.grad, np.float64))
                dist.all_reduce(g)  # sum, then / world: the ncclAvg of the CUDA path
                p.grad = (g.numpy() / world).astype(np.float32)
            grads = {n: p.grad.copy() for n, p in model.named_parameters()}
            opt.step()
            out.append((grads, {n: p.data.copy() for n, p in model.named_parameters()}))
        return out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,kw", [("mlp_policy", {}), ("mlp_classifier", {"batch": 512})])
def test_averaged_shard_gradients_equal_global_gradients(name, kw):
    from oracle import flex_oracle as fo
    from tynx_b200 import workloads
    from tynx_b200.onnx import ir

    ranks = _spawn(_dp_step, 2, name, kw)
    wl = workloads.WORKLOADS[name](**kw)
    model = fo.OracleModel(ir.load_training_graph(wl.onnx))
    opt = fo.Adam(model.named_parameters(), lr=wl.lr)
    for step in range(2):
        batch = wl.make_batch(step)
        opt.zero_grad()
        fo.cross_entropy(model(batch["x"]), batch["y"]).backward()
        glob = {n: p.grad.copy() for n, p in model.named_parameters()}
        opt.step()
        for n, g in glob.items():
            # only the summation order differs between the shard mean and the global mean
            for r in range(2):
                got = ranks[r][step][0][n]
                err = np.linalg.norm(got - g) / max(np.linalg.norm(g), 1e-30)
                assert err < 1e-5, (step, n, r, err)
            # replicated optimizer: the ranks hold bit-identical parameters
            np.testing.assert_array_equal(ranks[0][step][1][n], ranks[1][step][1][n])
