"""One process per GPU: contiguous sample shards of a batched use_model.

roseNNa evaluates one independent sample per use_model call
(fLibrary/modelCreator.fpp:42), so a batch shards across ranks with no
exchange on the data path: rank r evaluates the contiguous samples
[a_r, b_r) on its own GPU with the weights replicated, and the first n % world
ranks take one extra sample (the rule the library applies between the devices
of one process, rosenna_use_model_f32).  Collectives appear only around the
data path: gathering the shards' outputs for a caller that wants the whole
batch on every rank, and the max over ranks of a timing.

Arrays are in the batched reference layout viewed as (rows, n) matrices (row r
holds per-sample element r of every sample), so a shard is a column range.
Ranks and devices come from the torchrun environment (RANK, LOCAL_RANK,
WORLD_SIZE); torch.distributed carries the collectives (nccl between GPUs,
gloo on the host).
"""
from __future__ import annotations

import os
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np


def env() -> Tuple[int, int, int]:
    """(rank, local_rank, world_size) of this process; (0, 0, 1) outside torchrun."""
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def shard_bounds(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Samples [a, b) of a batch of n that rank `rank` of `world` evaluates."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} rank={rank} world={world}")
    base, rem = divmod(n, world)
    a = rank * base + min(rank, rem)
    return a, a + base + (1 if rank < rem else 0)


def shard_rows(inputs_rows: Sequence[np.ndarray], rank: int, world: int) -> Tuple[int, int, List[np.ndarray]]:
    """This rank's samples of every input, as contiguous arrays: columns of a
    (rows, n) input, or axis 1 of a (post, n, pre) input (one whose batch is
    not its first dimension, in the reference layout)."""
    n = int(inputs_rows[0].shape[1])
    for x in inputs_rows:
        if x.ndim not in (2, 3) or x.shape[1] != n:
            raise ValueError("inputs must be (rows, n) or (post, n, pre) arrays over the same n samples")
    a, b = shard_bounds(n, rank, world)
    return a, b, [np.ascontiguousarray(x[:, a:b], dtype=np.float32) for x in inputs_rows]


def use_model_shard(inputs_rows: Sequence[np.ndarray], rank: int, world: int,
                    run: Optional[Callable[[List[np.ndarray], int], List[np.ndarray]]] = None):
    """Evaluates this rank's shard of a batch given whole on every rank.

    run(shard_inputs, n_shard) -> (rows, n_shard) outputs; the default is the
    engine's use_model on the current GPU (rosenna_b200.api.use_model_rows).
    Returns (a, b, outputs of samples [a, b))."""
    a, b, ins = shard_rows(inputs_rows, rank, world)
    if run is None:
        from . import api

        run = lambda xs, m: api.use_model_rows(xs, m)  # noqa: E731
    return a, b, run(ins, b - a)


def _collective_device(group=None):
    import torch
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def gather_shards(local_outputs: Sequence[np.ndarray], n: int, group=None) -> List[np.ndarray]:
    """All ranks' shards joined into the (rows, n) outputs of the whole batch, on
    every rank.  Shards differ by at most one sample, so each is padded to the
    largest for one all_gather per output."""
    import torch
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    dev = _collective_device(group)
    bounds = [shard_bounds(n, r, world) for r in range(world)]
    width = max(b - a for a, b in bounds)
    a0, b0 = bounds[rank]
    full = []
    for y in local_outputs:
        if y.shape[1] != b0 - a0:
            raise ValueError(f"rank {rank} holds {y.shape[1]} samples, its shard is {b0 - a0}")
        buf = torch.zeros((y.shape[0], width), dtype=torch.float32, device=dev)
        buf[:, : b0 - a0] = torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32))
        parts = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf, group=group)
        full.append(np.concatenate([p[:, : b - a].cpu().numpy() for p, (a, b) in zip(parts, bounds)], axis=1))
    return full


def max_over_ranks(x: float, group=None) -> float:
    """The largest x over the ranks (the job's time is its slowest rank's)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=_collective_device(group))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def values_over_ranks(x: float, group=None) -> List[float]:
    """Every rank's x, in rank order (a per-rank record beside the max)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return [float(x)]
    dev = _collective_device(group)
    parts = [torch.zeros(1, dtype=torch.float64, device=dev) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, torch.tensor([float(x)], dtype=torch.float64, device=dev), group=group)
    return [float(p.item()) for p in parts]


def _parse_cpulist(text: str) -> List[int]:
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


def bind_host_to_device(device: int) -> Optional[dict]:
    """Restricts this process to the host CPUs of the NUMA node its GPU hangs
    off (sysfs local_cpulist of the GPU's PCI device), so that pinned host
    buffers allocated afterwards live on that node and host<->device copies do
    not cross the inter-socket link.  Returns {"node", "cpus"} or None when the
    topology cannot be read (the affinity is then left as it is)."""
    try:
        import torch

        pr = torch.cuda.get_device_properties(device)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        base = os.path.join("/sys/bus/pci/devices", bus)
        with open(os.path.join(base, "local_cpulist")) as f:
            cpus = _parse_cpulist(f.read())
        node = -1
        try:
            with open(os.path.join(base, "numa_node")) as f:
                node = int(f.read().strip())
        except (OSError, ValueError):
            pass
        allowed = set(os.sched_getaffinity(0))
        cpus = [c for c in cpus if c in allowed]
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return {"node": node, "cpus": len(cpus)}
    except Exception:
        return None
