"""Host-side tensor-parallel logic (no GPU): the shard plan of every rank
(q3xb_tp_plan) and its exchange between gloo ranks."""
import os

import pytest

from qwen3x_b200 import modelfile
from qwen3x_b200.backend import tp_plan

DENSE = [27008, 38027, 9000, 9091]


def covered(plans, start, count, total):
    spans = sorted((p[start], p[start] + p[count]) for p in plans)
    return spans[0][0] == 0 and spans[-1][1] == total and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


@pytest.mark.parametrize("mid", DENSE)
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plans_tile_every_dimension(mid, world):
    c = modelfile.CONFIGS[mid]
    try:
        plans = [tp_plan(mid, r, world) for r in range(world)]
    except ValueError:
        assert c.KH % world or c.VH % world or c.AH % world or (c.I // world) % 32 or c.I % world
        return
    for start, count, total in [("kh0", "KH", c.KH), ("vh0", "VH", c.VH), ("ah0", "AH", c.AH),
                                ("i0", "I", c.I), ("v0", "V", c.V)]:
        assert covered(plans, start, count, total), (start, plans)
    G = c.AH // c.KVH
    for p in plans:
        # every query head of the rank reads one of the rank's KV heads
        assert p["kv0"] == p["ah0"] // G
        assert (p["ah0"] + p["AH"] - 1) // G < p["kv0"] + p["KVH"]
        # value heads follow their key heads
        assert p["vh0"] // (c.VH // c.KH) == p["kh0"]
        assert (p["I"] % 32) == 0
    if c.KVH % world == 0:
        assert covered(plans, "kv0", "KVH", c.KVH)


@pytest.mark.parametrize("mid", [36035, 35091])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_expert_parallel_plans(mid, world):
    """MoE models: the routed experts tile [0, E) over the ranks; heads,
    FFN-free dims and the vocabulary stay whole (replicated)."""
    c = modelfile.CONFIGS[mid]
    plans = [tp_plan(mid, r, world) for r in range(world)]
    assert covered(plans, "e0", "experts", c.experts)
    for p in plans:
        assert p["experts"] == c.experts // world
        assert (p["KH"], p["VH"], p["AH"], p["KVH"], p["V"]) == (c.KH, c.VH, c.AH, c.KVH, c.V)
        assert p["kh0"] == p["vh0"] == p["ah0"] == p["v0"] == 0


def test_plan_rejections():
    with pytest.raises(ValueError, match="experts"):
        tp_plan(35091, 0, 3)  # 16 experts over 3 ranks
    with pytest.raises(ValueError, match="split"):
        tp_plan(27008, 0, 3)
    with pytest.raises(ValueError, match="rank"):
        tp_plan(27008, 2, 2)
    with pytest.raises(ValueError, match="unsupported"):
        tp_plan(1234, 0, 1)


def _gloo_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from qwen3x_b200.backend import tp_plan, tp_unique_id

    dist.init_process_group("gloo", rank=rank, world_size=world)
    ids = [tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    plans = [None] * world
    dist.all_gather_object(plans, (tp_plan(27008, rank, world), ids[0]))
    dist.destroy_process_group()
    q.put((rank, plans))


def test_gloo_ranks_agree_on_plan_and_communicator_id():
    """World-2 gloo ranks on CPU: the NCCL id made by rank 0 reaches rank 1
    unchanged, and the gathered plans tile the model."""
    import multiprocessing as mp
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        plans = [pl for pl, _ in results[rank]]
        ids = {i for _, i in results[rank]}
        assert len(ids) == 1 and len(next(iter(ids))) == 128
        assert [p["rank"] for p in plans] == [0, 1]
        c = modelfile.CONFIGS[27008]
        assert covered(plans, "vh0", "VH", c.VH) and covered(plans, "i0", "I", c.I)
