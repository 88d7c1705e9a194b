"""Data-parallel replicas: one process per GPU, each holding a full copy of the action head.

Independent robot observations are partitioned across ranks on the host; every rank runs its
shard through its own B200ExpandedActionHeadChain with no device-to-device traffic.  The only
cross-rank operations are host-side (gathering the actions back to the serving process, and
liveness checks through the rendezvous store), never on the GPU step path.  The reference
serves one GPU per server process and batches only inside one process
(rldx/model/core/rldx.py:1072-1082); this module adds the multi-GPU split.
"""

from __future__ import annotations

import datetime
import time
from typing import Callable, Dict, Sequence

import torch


def shard_bounds(n_items: int, world: int, rank: int) -> tuple:
    """Contiguous, balanced partition of n_items over world ranks: [start, end) of `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if n_items < 0:
        raise ValueError("n_items must be >= 0")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(observations: Dict[str, torch.Tensor], world: int, rank: int) -> Dict[str, torch.Tensor]:
    """This rank's slice (dim 0) of every observation tensor."""
    n = {v.shape[0] for v in observations.values()}
    if len(n) != 1:
        raise ValueError(f"observation tensors disagree on the batch size: {sorted(n)}")
    s, e = shard_bounds(n.pop(), world, rank)
    return {k: v[s:e] for k, v in observations.items()}


def gather_to_rank0(local: torch.Tensor, world: int, rank: int, counts: Sequence[int], group=None):
    """Host-side gather of per-rank action chunks (CPU tensors) to rank 0 over a CPU (gloo)
    group; returns the concatenation on rank 0 and None elsewhere."""
    import torch.distributed as dist

    if world == 1:
        return local
    maxn = max(counts)
    buf = torch.zeros((maxn,) + tuple(local.shape[1:]), dtype=local.dtype)
    buf[: local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)] if rank == 0 else None
    dist.gather(buf, parts, dst=0, group=group)
    if rank != 0:
        return None
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)


def serve_sharded(step: Callable[[Dict[str, torch.Tensor]], torch.Tensor],
                  observations: Dict[str, torch.Tensor], world: int, rank: int, group=None):
    """Runs `step` on this rank's shard and gathers all actions to rank 0."""
    n = next(iter(observations.values())).shape[0]
    counts = [shard_bounds(n, world, r)[1] - shard_bounds(n, world, r)[0] for r in range(world)]
    mine = shard(observations, world, rank)
    out = step(mine)
    return gather_to_rank0(out.detach().cpu(), world, rank, counts, group)


class Heartbeat:
    """Liveness through the rendezvous store: each rank bumps `hb/<rank>` between steps; a peer
    that has not bumped within `timeout_s` is reported dead before the next launch, so no rank
    ever enters a step waiting on a replica that is gone."""

    def __init__(self, store, world: int, rank: int, timeout_s: float = 5.0):
        self.store, self.world, self.rank, self.timeout_s = store, world, rank, timeout_s
        self.beat()

    def beat(self) -> None:
        self.store.set(f"hb/{self.rank}", repr(time.time()))

    def dead_peers(self) -> list:
        now, dead = time.time(), []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                self.store.wait([f"hb/{r}"], datetime.timedelta(seconds=self.timeout_s))
                last = float(self.store.get(f"hb/{r}").decode())
            except Exception:  # noqa: BLE001  (the peer never joined within the timeout)
                dead.append(r)
                continue
            if now - last > self.timeout_s:
                dead.append(r)
        return dead


class ReplicaPool:
    """One serving endpoint over several GPUs of one process: a replica of the action head per
    device, each device's contiguous share of a batch of independent observations (shard_bounds)
    copied in, run through its chain's captured graph and copied back on that device's own
    stream, so one host thread keeps every GPU busy at once and no device reads another's memory.

        pool = ReplicaPool(lambda dev: B200ExpandedActionHeadChain(gs, dev), ["cuda:0", "cuda:1"])
        actions = pool(vl_embs=..., state=..., embodiment_id=..., init_noise=..., ...)  # CPU tensor

    The keyword arguments are the chain's forward() arguments, batch-major tensors on the host
    (pinned memory lets the copies overlap) or on any device; actions come back as one CPU tensor
    in the input order.  A replica binds its shard's shapes on the first call, so later batches
    must split the same way (the chain raises on shape drift).  The reference serves one GPU per
    process and batches inside it (rldx/model/core/rldx.py:1072-1082)."""

    def __init__(self, make_chain: Callable, devices: Sequence):
        if not devices:
            raise ValueError("ReplicaPool needs at least one device")
        self.devices = [torch.device(d) for d in devices]
        self.chains = [make_chain(d) for d in self.devices]
        self.streams = []
        for d in self.devices:
            with torch.cuda.device(d):
                self.streams.append(torch.cuda.Stream(d))
        self._host_out = None

    def __len__(self) -> int:
        return len(self.chains)

    def __call__(self, **observations) -> torch.Tensor:
        batch = {k: v for k, v in observations.items() if isinstance(v, torch.Tensor)}
        n = {v.shape[0] for v in batch.values()}
        if len(n) != 1:
            raise ValueError(f"observation tensors disagree on the batch size: {sorted(n)}")
        n = n.pop()
        world = len(self.chains)
        outs, spans = [], []
        for r, (chain, dev, stream) in enumerate(zip(self.chains, self.devices, self.streams)):
            s, e = shard_bounds(n, world, r)
            spans.append((s, e))
            if e == s:
                outs.append(None)
                continue
            with torch.cuda.device(dev), torch.cuda.stream(stream):
                args = {k: (v[s:e].to(dev, non_blocking=True) if k in batch else v)
                        for k, v in observations.items()}
                outs.append(chain(**args))
        for o in outs:
            if o is not None:
                shape = (n,) + tuple(o.shape[1:])
                break
        else:
            raise ValueError("empty batch")
        if self._host_out is None or tuple(self._host_out.shape) != shape:
            self._host_out = torch.empty(shape, dtype=torch.bfloat16).pin_memory()
        for o, (s, e), dev, stream in zip(outs, spans, self.devices, self.streams):
            if o is not None:
                with torch.cuda.device(dev), torch.cuda.stream(stream):
                    self._host_out[s:e].copy_(o, non_blocking=True)
        for o, stream in zip(outs, self.streams):
            if o is not None:
                stream.synchronize()
        for chain in self.chains:
            code = chain.device_status(wait=False) if hasattr(chain, "device_status") else 0
            if code:
                from ._lib import RLDX_ERR_DEVICE, RldxError

                raise RldxError(RLDX_ERR_DEVICE, f"device error 0x{code:x} recorded by a replica")
        return self._host_out.clone()
