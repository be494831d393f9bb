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
from typing import Optional

from ._core import Device, context
from ._native import lib


def _unique_id_bytes(rank: int, world: int) -> bytes:
    buf = (C.c_uint8 * 128)()
    if rank == 0:
        code = lib.tx_dp_unique_id(buf)
        if code:
            raise RuntimeError("ncclGetUniqueId failed")
    try:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            obj = [bytes(buf) if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            return obj[0]
    except ImportError:  # pragma: no cover
        pass
    from torch.distributed import TCPStore

    host = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ.get("MASTER_PORT", "29500")) + 1
    store = TCPStore(host, port, world, rank == 0)
    if rank == 0:
        store.set("tynx_nccl_id", bytes(buf))
    return store.get("tynx_nccl_id")


def init_data_parallel(world: Optional[int] = None, rank: Optional[int] = None,
                       device: Optional[Device] = None, timeout_ms: int = 120000) -> None:
    """Create this rank's NCCL communicator on its GPU (bounded wait)."""
    world = int(os.environ.get("WORLD_SIZE", "1")) if world is None else world
    rank = int(os.environ.get("RANK", "0")) if rank is None else rank
    ctx = context(device)
    ident = _unique_id_bytes(rank, world)
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
