"""CPU, 2 gloo ranks: the sharded search's host logic (shard ranges, global ids, all-gather layout, merge) gives
the single-process result exactly; and a rank that never reaches the collective makes the other rank fail with
an error within the process-group timeout instead of hanging (host-side fault injection; no GPU involved).

The per-shard search and the merge here are the CPU oracle's; on GPUs bench.py runs the same host logic with the
CUDA search, NCCL and vk_merge_topk_device.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import REPO, assert_same_topk


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sharded_worker(rank, world, port, data, k, out_path):
    import sys
    sys.path.insert(0, str(REPO))
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import oracle
    from veckern_b200.shard import gather_and_merge, shard_of

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    cent, codes, q = data
    sh = shard_of(codes.shape[0], world, rank)
    P = oracle.port()
    d, i = P.adc_search(cent, codes[sh.lo:sh.hi], q, k)
    i = np.where(i >= 0, i + sh.lo, -1).astype(np.int32)  # global ids
    pairs = np.stack([d.view(np.int32), i], axis=-1).view(np.int64)[..., 0]  # [nq, k] (dist, id) pairs
    local = torch.from_numpy(np.ascontiguousarray(pairs))
    gathered = torch.empty((world,) + tuple(local.shape), dtype=torch.int64)

    def all_gather(buf, x):
        dist.all_gather(list(buf.unbind(0)), x)

    def merge(buf, layout):
        arr = buf.numpy().view(np.int32).reshape(world, q.shape[0], k, 2)
        md, mi = P.merge_topk(arr[..., 0].view(np.float32).transpose(1, 0, 2).copy(),
                              arr[..., 1].transpose(1, 0, 2).copy(), k)
        if rank == 0:
            np.savez(out_path, d=md, i=mi)

    gather_and_merge(local, gathered, q.shape[0], k, all_gather, merge)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_search_equals_single(golden, tmp_path, world):
    g = golden("gpu_fixture")
    k = 33
    out = tmp_path / "merged.npz"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, world, port, (g["centroids"], g["codes"], g["queries"]), k,
                                                        str(out))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    z = np.load(out)
    assert_same_topk(z["d"], z["i"], g[f"d_k{k}"], g[f"i_k{k}"], f"{world} shards merged")


def _stuck_worker(rank, world, port, q):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        q.put("rank 1 leaves without joining the collective")
        return  # exits between steps, with no collective in flight
    t = torch.zeros(4, dtype=torch.int64)
    try:
        dist.all_gather([torch.empty_like(t) for _ in range(world)], t)
        q.put("rank 0: all_gather returned")
    except Exception as e:  # noqa: BLE001 - any error type is the detection
        q.put(f"rank 0 detected: {type(e).__name__}")


def test_missing_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stuck_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    msgs = [q.get(timeout=5) for _ in range(2)]
    assert any(m.startswith("rank 0 detected") for m in msgs), msgs
    assert all(p.exitcode is not None for p in procs), "a rank hung"
