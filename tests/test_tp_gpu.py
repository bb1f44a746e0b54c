"""Multi-GPU backend on 2 GPUs (one process per GPU, NCCL + peer memory):
tensor parallelism (dense test model) and expert parallelism (MoE test model)
give the same logits and greedy tokens as the single-GPU backend.  Needs 2
GPUs; on a 1-GPU box it is skipped (the host-side logic is covered by
tests/test_tp.py on CPU)."""
import os

import numpy as np
import pytest

from qwen3x_b200 import modelfile

pytestmark = pytest.mark.gpu

# decode (GEMV path) and prompt (split-precision dequant-GEMM, FP32-grade):
# partial sums of the row-parallel projections / of the ranks' experts are
# added in another order, so results agree to FP32 rounding, within the
# reference's cross-backend bar of 5e-4
TOL = {"decode": 1e-4, "prefill": 5e-4}


def _tp_rank(rank, world, port, path, out, prompt, steps):
    # one node: NCCL's bootstrap over loopback
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", NCCL_SOCKET_IFNAME="lo")
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from qwen3x_b200.backend import Model, State, tp_unique_id

    # one communicator per state: a fresh id for each (an id bootstraps one communicator)
    ids = [(tp_unique_id(), tp_unique_id()) if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    model = Model(path, rank, world)
    res = {}
    def exchange(handle):  # IPC handles of the peer all-reduce buffers, in rank order
        out = [None] * world
        dist.all_gather_object(out, handle)
        return out

    for k, mode in enumerate(("decode", "prefill")):
        # the decode-mode state all-reduces over peer memory, the other one with NCCL
        st = State(model, 256, ids[0][k], exchange=exchange if mode == "decode" else None)
        if mode == "decode":
            for t in prompt:
                st.forward([int(t)])
        else:
            st.forward(prompt)
        res[mode + "_logits"] = st.logits()
        toks = []
        for _ in range(steps):
            toks.append(st.argmax())
            st.forward([toks[-1]])
        res[mode + "_tokens"] = np.array(toks)
        res[mode + "_final"] = st.logits()
        assert st.tp_error() == 0
        dist.barrier()  # no rank unmaps a peer buffer that another still reads
        st.close()
    model.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        np.savez(out, **res)


@pytest.mark.parametrize("mid", [9091, 35091], ids=["tensor-parallel", "expert-parallel"])
def test_tp2_matches_single_gpu(cuda, tmp_path, mid):
    import multiprocessing as mp
    import socket

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs 2 GPUs (host-side logic: tests/test_tp.py)")
    path = modelfile.write_model(tmp_path / "m.bin", modelfile.CONFIGS[mid], seed=5)
    prompt = np.random.default_rng(8).integers(0, modelfile.CONFIGS[mid].V, 40).astype(np.int32)
    steps = 24
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    out = tmp_path / "tp.npz"
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, str(path), str(out), prompt, steps)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    tp = np.load(out)

    from qwen3x_b200.backend import Model, State

    model = Model(path)
    for mode in ("decode", "prefill"):
        st = State(model, 256)
        if mode == "decode":
            for t in prompt:
                st.forward([int(t)])
        else:
            st.forward(prompt)
        ref = st.logits()
        scale = max(1.0, float(np.abs(ref).max()))
        assert float(np.abs(tp[mode + "_logits"] - ref).max()) <= TOL[mode] * scale, mode
        toks = []
        for _ in range(steps):
            toks.append(st.argmax())
            st.forward([toks[-1]])
        assert toks == list(tp[mode + "_tokens"]), mode
        ref = st.logits()
        assert float(np.abs(tp[mode + "_final"] - ref).max()) <= TOL[mode] * max(1.0, float(np.abs(ref).max())), mode
        st.close()
