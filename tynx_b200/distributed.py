"""Data-parallel training across the GPUs of one node (one process per GPU).

The reference is single-device; this is the exchange step of the data-parallel
step: every rank holds replicated parameters and a shard of the batch, and
parameter gradients are averaged inside backward by NCCL over NVLink in
buckets on a side stream (``tx_graph_set_dp`` / ``tx_dp_init``).

Rendezvous uses ``torch.distributed`` when a process group is initialised (the
NCCL unique id is broadcast from rank 0), else a ``TCPStore`` from the usual
``MASTER_ADDR`` / ``MASTER_PORT`` environment.
"""

from __future__ import annotations

import ctypes as C
import os
from datetime import timedelta
from typing import Callable, Optional

from ._core import Device, context
from ._native import lib


def _nccl_unique_id() -> bytes:
    buf = (C.c_uint8 * 128)()
    code = lib.tx_dp_unique_id(buf)
    if code:
        raise RuntimeError("ncclGetUniqueId failed")
    return bytes(buf)


def exchange_unique_id(rank: int, world: int, make_id: Callable[[], bytes] = _nccl_unique_id,
                       timeout_s: float = 120.0) -> bytes:
    """Rank 0 makes the communicator id; every rank returns the same 128 bytes.

    Uses the initialised ``torch.distributed`` group when there is one (any
    backend), else a ``TCPStore`` at ``MASTER_ADDR:MASTER_PORT+1``.  A rank that
    never joins ends the others' wait with an error after ``timeout_s``.
    """
    ident = make_id() if rank == 0 else None
    if ident is not None and len(ident) != 128:
        raise ValueError("a communicator id is 128 bytes")
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        obj = [ident]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]
    from torch.distributed import TCPStore

    host = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ.get("MASTER_PORT", "29500")) + 1
    store = TCPStore(host, port, world, rank == 0, timeout=timedelta(seconds=timeout_s))
    if rank == 0:
        store.set("tynx_nccl_id", ident)
    ident = store.get("tynx_nccl_id")
    store.set(f"tynx_nccl_id_ack_{rank}", b"1")
    if rank == 0:
        # rank 0 hosts the store: keep it up until every rank has read the id
        store.wait([f"tynx_nccl_id_ack_{r}" for r in range(world)])
    return ident


def init_data_parallel(world: Optional[int] = None, rank: Optional[int] = None,
                       device: Optional[Device] = None, timeout_ms: int = 120000) -> None:
    """Create this rank's NCCL communicator on its GPU (bounded wait)."""
    world = int(os.environ.get("WORLD_SIZE", "1")) if world is None else world
    rank = int(os.environ.get("RANK", "0")) if rank is None else rank
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    ctx = context(device)
    ident = exchange_unique_id(rank, world, timeout_s=timeout_ms / 1e3)
    buf = (C.c_uint8 * 128).from_buffer_copy(ident)
    ctx.check(lib.tx_dp_init(ctx.handle, world, rank, buf, timeout_ms), "data-parallel init")


def shutdown_data_parallel(device: Optional[Device] = None) -> None:
    ctx = context(device)
    ctx.check(lib.tx_dp_destroy(ctx.handle))


def shard(n: int, world: int, rank: int) -> slice:
    """Contiguous batch shard of rank ``rank`` (equal sizes; ``n`` must divide)."""
    if n % world:
        raise ValueError(f"global batch {n} does not divide across {world} ranks")
    per = n // world
    return slice(rank * per, (rank + 1) * per)
