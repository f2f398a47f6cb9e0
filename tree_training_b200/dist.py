"""Data-parallel plumbing for tree training: one process per GPU, whole trees
per rank, parameter gradients averaged after each rank's tree step.

The reference trains one trajectory tree per process and leaves data
parallelism to the launcher: the per-tree step is ``tree_grad_hybrid``
(tree_grad_hybrid.py:434-539), which only accumulates ``.grad``.  This module
supplies the rest for the multi-GPU configurations:

* ``assign_trees`` — rank r takes trees r, r+W, r+2W, ... (independent units,
  no communication inside the attention or GDN operators);
* ``GradAverager`` — bucketed all-reduce of the gradients (sum, then / W) over
  flat per-dtype buffers in a fixed parameter order, so every rank issues the
  same collectives in the same order; optionally overlapped with the last
  backward pass (``attach`` + ``arm``: each bucket is reduced as soon as all
  of its gradients are final);
* ``RankWatch`` — host-side liveness check through the process group's store:
  before a step's collectives each rank posts a heartbeat and waits, with a
  short limit, for everyone else's, so a rank that died between steps is
  reported by name instead of as a hung collective.
"""
from __future__ import annotations

import datetime
import os
import time
from typing import Dict, Iterable, List, Optional, Sequence

import torch
import torch.distributed as dist


def assign_trees(n_trees: int, world: int, rank: int) -> List[int]:
    """Indices of the trees rank ``rank`` of ``world`` processes: round robin,
    so W in {1, 2, 4, 8} splits config 3's 8 trees evenly."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_trees < 0:
        raise ValueError("n_trees must be >= 0")
    return list(range(rank, n_trees, world))


def init_process_group(backend: str, timeout_s: float = 60.0, rank: Optional[int] = None,
                       world: Optional[int] = None) -> None:
    """``torch.distributed.init_process_group`` from the torchrun environment
    with a short timeout, so ranks blocked on a dead peer fail instead of
    waiting for the library default of 10 minutes."""
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kw = {}
    if rank is not None:
        kw["rank"] = rank
    if world is not None:
        kw["world_size"] = world
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)


class GradAverager:
    """Average ``.grad`` of ``params`` over the default process group.

    Gradients are packed into flat buffers of at most ``bucket_bytes`` (one
    dtype and device per bucket, parameters in the order given), each buffer is
    all-reduced with SUM and divided by the world size, then copied back.
    Parameters whose ``.grad`` is None on this rank contribute zeros, so every
    rank issues identical collectives even when a partition did not touch a
    parameter.

    Overlap with the backward: after ``attach()`` (post-accumulate-grad hooks
    on every parameter), ``arm()`` declares that the NEXT gradient accumulation
    of each parameter is its last of the step (``tree_grad_hybrid`` calls it
    through ``before_last_backward`` before the last partition's single
    backward traversal).  From then on a bucket is packed and its all-reduce
    issued (asynchronously, on NCCL's stream) once all of its parameters have
    their final gradient, and buckets are issued strictly from the last to the
    first, so that every rank issues the same collectives in the same order.
    ``average()`` issues whatever is left in the same order, waits, divides and
    copies back."""

    def __init__(self, params: Iterable[torch.nn.Parameter], bucket_bytes: int = 256 << 20):
        self.params = [p for p in params if p.requires_grad]
        self._hooks: list = []
        self._armed = False
        self._ready: List[set] = []
        self._next = -1
        self._pending: list = []
        self.buckets: List[List[torch.nn.Parameter]] = []
        cur: List[torch.nn.Parameter] = []
        cur_bytes = 0
        key = None
        for p in self.params:
            k = (p.dtype, p.device)
            nb = p.numel() * p.element_size()
            if cur and (k != key or cur_bytes + nb > bucket_bytes):
                self.buckets.append(cur)
                cur, cur_bytes = [], 0
            cur.append(p)
            cur_bytes += nb
            key = k
        if cur:
            self.buckets.append(cur)

    def bytes_per_step(self) -> int:
        return sum(p.numel() * p.element_size() for p in self.params)

    def _active(self, group=None) -> bool:
        return dist.is_initialized() and dist.get_world_size(group) > 1

    def attach(self) -> "GradAverager":
        """Register the hooks that let ``arm()`` overlap the all-reduce with the
        backward (no effect on a single process)."""
        if self._hooks or not self._active():
            return self
        where = {}
        for bi, bucket in enumerate(self.buckets):
            for p in bucket:
                where[id(p)] = bi
        for p in self.params:
            self._hooks.append(p.register_post_accumulate_grad_hook(
                lambda q, _bi=where[id(p)]: self._on_grad(_bi, q)))
        return self

    def detach(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []

    def arm(self) -> None:
        """The next accumulation of every parameter's gradient is its last one
        of this step (see the class docstring)."""
        if not self._hooks:
            return
        self._armed = True
        self._ready = [set() for _ in self.buckets]
        self._next = len(self.buckets) - 1
        self._pending = []

    def _on_grad(self, bi: int, p: torch.nn.Parameter) -> None:
        if not self._armed:
            return
        self._ready[bi].add(id(p))
        while self._next >= 0 and len(self._ready[self._next]) == len(self.buckets[self._next]):
            self._issue(self._next)
            self._next -= 1

    def _issue(self, bi: int, group=None) -> None:
        bucket = self.buckets[bi]
        flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1)
                          for p in bucket])
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=True)
        self._pending.append((bucket, flat, work))

    def issued_during_backward(self) -> int:
        """Buckets whose all-reduce the hooks issued before ``average()``."""
        return len(self._pending) if self._armed else 0

    def average(self, group=None) -> None:
        if not self._active(group):
            self._armed = False
            return                      # a single process: nothing to average
        world = dist.get_world_size(group)
        if not self._armed:
            self._pending, self._next = [], len(self.buckets) - 1
        while self._next >= 0:          # what the hooks did not issue, same order
            self._issue(self._next, group)
            self._next -= 1
        pending, self._pending, self._armed = self._pending, [], False
        for bucket, flat, work in pending:
            work.wait()
            flat.div_(world)
            off = 0
            for p in bucket:
                n = p.numel()
                g = flat[off:off + n].view_as(p)
                if p.grad is None:
                    p.grad = g.clone()
                else:
                    p.grad.copy_(g)
                off += n


class RankFailure(RuntimeError):
    """A peer rank did not post its heartbeat within the limit."""

    def __init__(self, step: int, missing: Sequence[int]):
        super().__init__(f"step {step}: no heartbeat from rank(s) {list(missing)}")
        self.step = step
        self.missing = list(missing)


class RankWatch:
    """Per-step heartbeats through a ``torch.distributed`` store.

    ``beat(step)`` posts this rank's key for the step and waits up to
    ``timeout_s`` for every other rank's; ranks that never post are reported in
    a ``RankFailure``.  Call it between steps, before the step's first
    collective, so that no kernel or collective is in flight when a rank
    leaves."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0,
                 prefix: str = "tt_alive"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s = timeout_s
        self.prefix = prefix

    def _key(self, step: int, r: int) -> str:
        return f"{self.prefix}/{step}/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), "1")
        deadline = time.monotonic() + self.timeout_s
        missing = [r for r in range(self.world) if r != self.rank]
        while missing:
            missing = [r for r in missing if not self.store.check([self._key(step, r)])]
            if not missing:
                break
            if time.monotonic() > deadline:
                raise RankFailure(step, missing)
            time.sleep(0.01)


def world_info() -> Dict[str, int]:
    """RANK / LOCAL_RANK / WORLD_SIZE from the torchrun environment."""
    return {"rank": int(os.environ.get("RANK", 0)),
            "local_rank": int(os.environ.get("LOCAL_RANK", 0)),
            "world": int(os.environ.get("WORLD_SIZE", 1))}
