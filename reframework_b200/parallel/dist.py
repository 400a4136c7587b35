"""Process-group context and collectives — same API as reframework/parallel/dist.py.

``init`` / ``run`` / ``current`` / ``all_reduce_sum`` / ``all_gather`` /
``all_to_all`` / ``send`` / ``recv`` / ``barrier`` / ``destroy`` keep the
reference's names, arguments and errors (dist.py:49-227): the layout is
row-major ``pp x ep`` (``pp_rank = rank // ep_size``, ``ep_rank = rank %
ep_size``); ``current()`` raises RuntimeError when no group is live; ``run``
raises RuntimeError when a child exits non-zero.  The backend is NCCL on GPUs
(one process per GPU over NVLink/NVSwitch) and gloo for CPU tests.

Added for expert parallelism: ``all_to_all_v`` (variable split sizes), a
``timeout`` on ``init`` so ranks waiting on a dead peer end with an error, and
``bind_to_device_cpus`` (host threads and first-touch pinned buffers on the
CPUs next to this rank's GPU, so eight ranks' host copies do not cross the
socket link).
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

__all__ = ["ParallelContext", "init", "run", "is_initialized", "current", "get_rank", "get_world_size",
           "all_reduce_sum", "all_gather", "all_to_all", "all_to_all_v", "send", "recv", "barrier",
           "destroy", "device_local_cpus", "bind_to_device_cpus"]


@dataclass(frozen=True)
class ParallelContext:
    backend: str
    rank: int
    world_size: int
    group: Optional[dist.ProcessGroup] = None
    pp_size: int = 1
    ep_size: int = 1
    pp_rank: int = 0
    ep_rank: int = 0


_current: Optional[ParallelContext] = None


def is_initialized() -> bool:
    return _current is not None and dist.is_initialized()


def current() -> ParallelContext:
    if _current is None:
        raise RuntimeError("No process group is initialised — call parallel.init()/run() first "
                           "(or run single-process without PP/EP).")
    return _current


def get_rank() -> int:
    return current().rank


def get_world_size() -> int:
    return current().world_size


def init(*, backend: str = "gloo", init_method: Optional[str] = None, rank: Optional[int] = None,
         world_size: Optional[int] = None, pp_size: int = 1, ep_size: int = 1,
         group: Optional[dist.ProcessGroup] = None, timeout_s: float = 300.0,
         device_id: Optional[torch.device] = None) -> ParallelContext:
    """Initialise (or re-initialise) the process group and the parallel context."""
    global _current
    if dist.is_initialized():
        destroy()
    kw = {}
    if device_id is not None and backend == "nccl":
        kw["device_id"] = device_id
    dist.init_process_group(backend=backend, init_method=init_method, rank=rank, world_size=world_size,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)
    rank = dist.get_rank()
    world = dist.get_world_size()
    if pp_size > 1 or ep_size > 1:
        if pp_size * ep_size != world:
            raise ValueError(f"pp_size({pp_size}) * ep_size({ep_size}) must equal world_size({world})")
        pp_rank = rank // ep_size if ep_size > 1 else 0
        ep_rank = rank % ep_size if ep_size > 1 else 0
    else:
        pp_rank = ep_rank = 0
    _current = ParallelContext(backend=backend, rank=rank, world_size=world, group=group or dist.group.WORLD,
                               pp_size=pp_size, ep_size=ep_size, pp_rank=pp_rank, ep_rank=ep_rank)
    return _current


def run(target, *, world_size: int, backend: str = "gloo", init_method: Optional[str] = None,
        pp_size: int = 1, ep_size: int = 1, args: tuple = (), start_method: str = "fork",
        timeout_s: float = 120.0) -> List[int]:
    """Spawn ``world_size`` local processes, each calling ``target(rank, ctx, *args)``
    inside an initialised group (dist.py:135-176).  Raises RuntimeError on any
    non-zero exit code."""
    import torch.multiprocessing as mp

    ctx_mp = mp.get_context(start_method)
    procs = [ctx_mp.Process(target=_worker, args=(r, target, world_size, backend, init_method, pp_size,
                                                  ep_size, args, timeout_s)) for r in range(world_size)]
    for p in procs:
        p.start()
    for p in procs:
        p.join()
    codes = [p.exitcode for p in procs]
    if any(c != 0 for c in codes):
        raise RuntimeError(f"parallel run failed with exit codes {codes}")
    return codes


def _worker(rank, target, world_size, backend, init_method, pp_size, ep_size, args, timeout_s):
    os.environ["RANK"] = str(rank)
    os.environ["WORLD_SIZE"] = str(world_size)
    ctx = init(backend=backend, init_method=init_method, rank=rank, world_size=world_size,
               pp_size=pp_size, ep_size=ep_size, timeout_s=timeout_s)
    try:
        target(rank, ctx, *args)
    finally:
        destroy()


def _group():
    return current().group if _current is not None else None


def all_reduce_sum(t: torch.Tensor) -> torch.Tensor:
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=_group())
    return t


def all_gather(t: torch.Tensor) -> List[torch.Tensor]:
    out = [torch.empty_like(t) for _ in range(get_world_size())]
    dist.all_gather(out, t, group=_group())
    return out


def all_to_all(t: torch.Tensor, scatter_dim: int = 0) -> torch.Tensor:
    """Equal-chunk all-to-all along ``scatter_dim`` (dist.py:194-206)."""
    world = get_world_size()
    chunks = t.chunk(world, dim=scatter_dim)
    flat = torch.cat([c.contiguous().view(-1) for c in chunks])
    out = torch.empty_like(flat)
    # all_to_all_single (gloo implements it, unlike the list form) on equal chunks
    dist.all_to_all_single(out, flat, group=_group())
    received = [piece.view(chunks[0].shape) for piece in out.view(world, -1).unbind(0)]
    return torch.stack(received, dim=scatter_dim).reshape_as(t)


def all_to_all_v(out: torch.Tensor, inp: torch.Tensor, out_splits: Sequence[int],
                 in_splits: Sequence[int], group=None) -> torch.Tensor:
    """Variable-size all-to-all along dim 0 (rows); ``out`` must hold sum(out_splits) rows."""
    dist.all_to_all_single(out, inp, output_split_sizes=list(out_splits),
                           input_split_sizes=list(in_splits), group=group or _group())
    return out


def send(t: torch.Tensor, dst: int) -> None:
    dist.send(t.contiguous(), dst=dst)


def recv(shape, dtype: torch.dtype, src: int) -> torch.Tensor:
    out = torch.empty(tuple(shape), dtype=dtype)
    dist.recv(out, src=src)
    return out


def barrier() -> None:
    dist.barrier()


def destroy() -> None:
    global _current
    if dist.is_initialized():
        dist.destroy_process_group()
    _current = None


# ------------------------------------------------------------- host placement
def _parse_cpulist(text: str) -> List[int]:
    """``"0-3,8,10-11"`` -> [0, 1, 2, 3, 8, 10, 11]."""
    cpus: List[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.extend(range(int(a), int(b) + 1))
        else:
            cpus.append(int(part))
    return cpus


def device_local_cpus(domain: int, bus: int, device: int, sysfs: str = "/sys") -> Optional[List[int]]:
    """CPUs on the same NUMA node as the PCI device ``domain:bus:device.0``
    (its ``local_cpulist`` in sysfs), or None when sysfs does not say."""
    path = os.path.join(sysfs, "bus", "pci", "devices", f"{domain:04x}:{bus:02x}:{device:02x}.0", "local_cpulist")
    try:
        with open(path) as f:
            cpus = _parse_cpulist(f.read())
    except (OSError, ValueError):
        return None
    return cpus or None


def bind_to_device_cpus(device: torch.device, sysfs: str = "/sys") -> Optional[List[int]]:
    """Restrict this process to the CPUs next to ``device`` (intersected with
    the CPUs it may use) and return them; None (nothing changed) when the
    topology is unknown or the intersection is empty.  Call it before pinned
    host buffers are allocated: their pages are placed on first touch."""
    props = torch.cuda.get_device_properties(device)
    cpus = device_local_cpus(props.pci_domain_id, props.pci_bus_id, props.pci_device_id, sysfs)
    if not cpus or not hasattr(os, "sched_setaffinity"):
        return None
    allowed = os.sched_getaffinity(0)
    mine = sorted(set(cpus) & allowed)
    if not mine or set(mine) == allowed:
        return mine or None
    os.sched_setaffinity(0, mine)
    return mine
