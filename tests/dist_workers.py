"""Rank bodies for the world-size-2 tests of tree_training_b200.dist (gloo on
CPU; NCCL on two GPUs with NVLS off).

Each worker runs in a spawned process with the process group already set up by
``run_ranks``; it returns a picklable result or raises."""
from __future__ import annotations

import datetime
import os
import queue
import socket
import traceback

import torch
import torch.distributed as dist


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# bodies after which a rank may be gone: the survivors do not tear the group down
_PEER_MAY_BE_GONE = ("fail_rank1", "nccl_fail_rank1")


def _entry(rank, world, port, fn_name, args, pg_timeout, q, backend):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    try:
        kw = {}
        if backend == "nccl":
            os.environ["NCCL_NVLS_ENABLE"] = "0"      # no NVLink multicast objects
            torch.cuda.set_device(rank)
            kw["device_id"] = torch.device("cuda", rank)
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=pg_timeout), **kw)
        res = globals()[fn_name](rank, world, *args)
        q.put((rank, "ok", res))
    except BaseException as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, "err", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))
    finally:
        if dist.is_initialized() and fn_name not in _PEER_MAY_BE_GONE:
            dist.destroy_process_group()


def run_ranks(fn_name: str, world: int = 2, args=(), pg_timeout: float = 20.0,
              limit_s: float = 120.0, expect=None, backend: str = "gloo"):
    """Start ``world`` spawned ranks running ``fn_name``; return {rank: (status,
    result)} for the ranks that reported within ``limit_s`` (waiting only for
    the ranks in ``expect``, default all)."""
    expect = set(range(world)) if expect is None else set(expect)
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry,
                         args=(r, world, port, fn_name, args, pg_timeout, q, backend))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        while not expect.issubset(out):
            try:
                r, status, res = q.get(timeout=limit_s)
            except queue.Empty:
                break
            out[r] = (status, res)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join()
    return out


# ---------------------------------------------------------------------------
# rank bodies
# ---------------------------------------------------------------------------

def _toy_model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Embedding(64, 16), torch.nn.Linear(16, 64)).double()


def _tree_loss(model, roots):
    """A per-tree loss over the packed tree (ids and depth-based position ids)."""
    from tree_training_b200 import build_dfs_tree_info
    info = build_dfs_tree_info(roots)
    ids = torch.as_tensor(info.dfs_token_ids_np % 64, dtype=torch.long)
    pos = torch.as_tensor(info.dfs_pos_ids_np, dtype=torch.float64)
    logits = model(ids) * (1.0 + 1e-3 * pos[:, None])
    return torch.nn.functional.cross_entropy(logits, (ids + 1) % 64)


def _trees(n):
    from tree_training_b200.synthetic import random_branching_tree
    return [random_branching_tree(100 + i, 60 + 7 * i, 3, 12) for i in range(n)]


def dp_tree_step(rank, world, n_trees, bucket_bytes):
    """Each rank runs its assigned trees, then gradients are averaged; returns
    the averaged gradients."""
    from tree_training_b200.dist import GradAverager, assign_trees
    model = _toy_model()
    trees = _trees(n_trees)
    mine = assign_trees(n_trees, world, rank)
    for i in mine:
        (_tree_loss(model, trees[i]) * (world / n_trees)).backward()
    GradAverager(model.parameters(), bucket_bytes=bucket_bytes).average()
    return {"assigned": mine, "grads": [p.grad.clone() for p in model.parameters()]}


def dp_overlap_step(rank, world, n_trees, bucket_bytes):
    """As dp_tree_step, with the all-reduce overlapped: the averager is armed
    before each rank's last backward, so the hooks issue the buckets during it."""
    from tree_training_b200.dist import GradAverager, assign_trees
    model = _toy_model()
    avg = GradAverager(model.parameters(), bucket_bytes=bucket_bytes).attach()
    trees = _trees(n_trees)
    mine = assign_trees(n_trees, world, rank)
    for j, i in enumerate(mine):
        if j == len(mine) - 1:
            avg.arm()
        (_tree_loss(model, trees[i]) * (world / n_trees)).backward()
    issued = avg.issued_during_backward()
    avg.average()
    avg.detach()
    return {"grads": [p.grad.clone() for p in model.parameters()], "issued": issued,
            "buckets": len(avg.buckets)}


def single_process_grads(n_trees):
    model = _toy_model()
    for roots in _trees(n_trees):
        (_tree_loss(model, roots) / n_trees).backward()
    return [p.grad.clone() for p in model.parameters()]


def average_with_missing_grad(rank, world):
    """Rank 1 leaves one parameter without a gradient: it counts as zero."""
    from tree_training_b200.dist import GradAverager
    a = torch.nn.Parameter(torch.zeros(5, dtype=torch.float64))
    b = torch.nn.Parameter(torch.zeros(3, dtype=torch.float32))
    a.grad = torch.full((5,), float(rank + 1), dtype=torch.float64)
    if rank == 0:
        b.grad = torch.full((3,), 4.0)
    GradAverager([a, b], bucket_bytes=16).average()
    return a.grad.tolist(), b.grad.tolist()


def heartbeat_all_alive(rank, world):
    from tree_training_b200.dist import RankWatch
    w = RankWatch(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=10.0)
    for step in range(3):
        w.beat(step)
    return "ok"


def fail_rank1(rank, world):
    """Rank 1 leaves after step 0 (between steps, nothing in flight); rank 0
    must learn of it on the host at the next step's heartbeat, and a
    collective issued anyway must end with an error within the short process
    group timeout instead of hanging."""
    import time
    from tree_training_b200.dist import RankFailure, RankWatch
    w = RankWatch(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=3.0)
    w.beat(0)
    if rank == 1:
        os._exit(0)
    out = {}
    t0 = time.monotonic()
    try:
        w.beat(1)
        out["heartbeat"] = "no error"
    except RankFailure as e:
        out["heartbeat"] = f"RankFailure {e.missing}"
    out["heartbeat_s"] = time.monotonic() - t0
    t0 = time.monotonic()
    try:
        x = torch.ones(4)
        dist.all_reduce(x)
        out["collective"] = "no error"
    except Exception as e:  # noqa: BLE001 - the error type depends on the backend
        out["collective"] = type(e).__name__
    out["collective_s"] = time.monotonic() - t0
    return out


# ---------------------------------------------------------------------------
# NCCL rank bodies (one GPU per rank)
# ---------------------------------------------------------------------------

def _attn_model(dev):
    torch.manual_seed(0)
    m = torch.nn.ModuleDict({"emb": torch.nn.Embedding(256, 64),
                             "q": torch.nn.Linear(64, 4 * 128), "k": torch.nn.Linear(64, 128),
                             "v": torch.nn.Linear(64, 128)})
    return m.to(dev)


def _attn_tree_loss(model, roots, dev):
    """Tree attention (bf16, tcgen05 path) over one packed tree; scalar loss."""
    import tree_training_b200 as tt
    info = tt.build_dfs_tree_info(roots)
    meta = info.attn_meta()
    ids = torch.as_tensor(info.dfs_token_ids_np % 256, dtype=torch.long, device=dev)
    x = model["emb"](ids)
    n = ids.shape[0]
    q = model["q"](x).view(n, 4, 128).to(torch.bfloat16)
    k = model["k"](x).view(n, 1, 128).to(torch.bfloat16)
    v = model["v"](x).view(n, 1, 128).to(torch.bfloat16)
    out = tt.tree_attention(q, k, v, meta)
    return out.float().square().mean()


def _attn_trees():
    from tree_training_b200.synthetic import bfs_tree
    return [bfs_tree(300 + i, 2048, 32, 256, 256) for i in range(2)]


def nccl_dp_attention_step(rank, world):
    """Each rank backpropagates the tree attention of its own tree and the
    gradients are averaged over NCCL; each rank also computes both trees'
    gradients alone on its GPU.  Returns the largest relative difference."""
    from tree_training_b200.dist import GradAverager, RankWatch
    dev = torch.device("cuda", rank)
    trees = _attn_trees()
    watch = RankWatch(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=20.0)
    model = _attn_model(dev)
    watch.beat(0)
    (_attn_tree_loss(model, trees[rank], dev) / world).backward()
    GradAverager(model.parameters()).average()
    got = [p.grad.detach().clone() for p in model.parameters()]
    ref_model = _attn_model(dev)
    for roots in trees:
        # the average divides the sum over ranks by W again
        (_attn_tree_loss(ref_model, roots, dev) / (world * world)).backward()
    torch.cuda.synchronize(dev)
    diff = max(float((g - p.grad).abs().max() / (p.grad.abs().max() + 1e-30))
               for g, p in zip(got, ref_model.parameters()))
    watch.beat(1)
    return diff


def nccl_fail_rank1(rank, world):
    """After one data-parallel step, rank 1 leaves between steps (its kernels
    and collectives finished); rank 0 learns of it from the heartbeat before
    launching anything for the next step, and issues no collective."""
    import time
    from tree_training_b200.dist import GradAverager, RankFailure, RankWatch
    dev = torch.device("cuda", rank)
    watch = RankWatch(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=3.0)
    model = _attn_model(dev)
    watch.beat(0)
    _attn_tree_loss(model, _attn_trees()[rank], dev).backward()
    GradAverager(model.parameters()).average()
    torch.cuda.synchronize(dev)
    if rank == 1:
        os._exit(0)
    out = {}
    t0 = time.monotonic()
    try:
        watch.beat(1)
        out["heartbeat"] = "no error"
    except RankFailure as e:
        out["heartbeat"] = f"RankFailure {e.missing}"
    out["heartbeat_s"] = time.monotonic() - t0
    return out
