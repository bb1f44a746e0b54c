"""Benchmark of qwen3x's packed-weight matrix path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (the metric's "Q8_0 GEMV HBM GB/s"):
y = W x with W 12288x4096 Q8_0 (w ~ N(0, 0.02), d = max|w|/127), x ~ N(0, 1)
FP32, y FP32.  One step = one GEMV of x against each of COPIES resident copies
of W (COPIES x 53.5 MB > the 126 MB L2, so every step streams W from HBM).
Steps are replayed from a CUDA graph; the timed region is bracketed by a
barrier and a device synchronize, timed with CUDA events, max over ranks.

value       algorithmic bytes of all ranks / max device time (GB/s), W resident
e2e         the same metric through q3xk_try_mv_host (x from pinned host memory,
            y back to pinned host memory, synchronous, inside the timed region)
roofline    the GEMV kernel against the measured HBM copy bandwidth
cpu_baseline the reference's own arch/cpu.cpp mv (oracle/_ref), 1 thread as
            the reference runs on Linux, a bounded sample of the same workload
--impl reference   the reference CPU implementation with all host threads.

N > 1: rank r streams row block r of a (12288 N) x 4096 matrix (x replicated,
y sharded, no data-path collective), so scaling is "weak".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ROWS, COLS = 12288, 4096
COPIES = 6
GRAPH_STEPS = 50
FALLBACK_HBM_GBS = 6650.0


def algorithmic_bytes(mtype: int, rows: int = ROWS, cols: int = COLS) -> int:
    """Packed weight bytes + x + y: 53,542,912 B for the Q8_0 12288x4096 matvec."""
    per_row = cols // 32 * (34 if mtype == 1 else 18)
    return rows * per_row + 4 * cols + 4 * rows


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def measured_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes of the kernel from the committed ncu summary."""
    p = ROOT / "profiles" / f"{name}.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


def recorded_reference_programs():
    """The reference's own CUDA and CPU programs timed on a B200 box
    (profiles/reference_programs_b200.md, made by oracle/time_reference_cli.py):
    read from the committed summary, not run here."""
    p = ROOT / "profiles" / "reference_programs_b200.md"
    if not p.exists():
        return None
    text = p.read_text()
    try:
        block = text.split("```json", 1)[1].split("```", 1)[0]
        d = json.loads(block)
    except Exception:
        return None
    d["source"] = "recorded: profiles/reference_programs_b200.md (oracle/time_reference_cli.py, same model.bin)"
    return d


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        import torch

        try:  # nvidia-smi ignores CUDA_VISIBLE_DEVICES: address the GPU by UUID
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.index = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.index = str(device_index)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)  # first sample before the timed region starts
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()
        return False

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").strip().splitlines():
            f = [s.strip() for s in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxes.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


def dist_setup(n_gpus: int):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        os.environ.setdefault("NCCL_SOCKET_IFNAME", "lo")  # one node: bootstrap over loopback
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def make_matrix(mtype: int, device):
    """This rank's row block of the GEMV matrix: with N ranks the workload is
    one (12288 N) x 4096 matrix split by rows, block r drawn from seed
    1 + 1000 r (block 0 is BASELINE config 1's matrix), x the same on every
    rank; no step needs a collective (y stays sharded)."""
    import os

    from qwen3x_b200 import quant
    from qwen3x_b200.linear import Linear

    rank = int(os.environ.get("RANK", "0"))
    w = quant.gaussian((ROWS, COLS), 1 + 1000 * rank, 0.02)
    packed = quant.quantize(w, mtype)
    return [Linear.from_packed(packed, mtype, ROWS, COLS, device=device) for _ in range(COPIES)], packed


def time_gemv(mtype: int, steps: int, warmup: int, device, world: int, sample_clocks: bool):
    """Graph-replayed GEMV steps; returns (seconds_max_over_ranks, launches, clocks)."""
    import torch
    import torch.distributed as dist

    from qwen3x_b200 import capi, quant
    from qwen3x_b200.linear import mv

    mats, _ = make_matrix(mtype, device)
    x = torch.from_numpy(quant.gaussian(COLS, 2)).to(device)
    ys = [torch.empty(ROWS, device=device) for _ in range(COPIES)]

    def step():
        for m, y in zip(mats, ys):
            mv(m, x, y)

    for _ in range(max(warmup, 3)):
        step()
    torch.cuda.synchronize()
    # K <= GRAPH_STEPS (the usual case): one graph holds exactly the K timed
    # steps between two event-record nodes, so the events time the device
    # execution of those steps and not the host's submission of the graph
    # (~70 us for 120 kernel nodes, which would otherwise sit inside the
    # timed region).  Larger K: graphs of GRAPH_STEPS steps replayed back to
    # back between host-recorded events (the submission then overlaps them).
    inner = steps <= GRAPH_STEPS
    g_steps = steps if inner else GRAPH_STEPS
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    lib = capi.lib()
    start = torch.cuda.Event(enable_timing=True, external=inner)
    end = torch.cuda.Event(enable_timing=True, external=inner)
    with torch.cuda.stream(s):
        lib.q3xk_reset_launch_count()
        with torch.cuda.graph(graph, stream=s):
            if inner:
                start.record(s)
            for _ in range(g_steps):
                step()
            if inner:
                end.record(s)
        per_graph = lib.q3xk_launch_count()
    torch.cuda.current_stream().wait_stream(s)
    replays, rem = divmod(steps, g_steps)
    graph.replay()  # warm the graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(torch.cuda.current_device()) if sample_clocks else None
    if sampler:
        sampler.__enter__()
    lib.q3xk_reset_launch_count()
    if not inner:
        start.record()
    for _ in range(replays):
        graph.replay()
    for _ in range(rem):
        step()
    if not inner:
        end.record()
    torch.cuda.synchronize()
    eager_launches = lib.q3xk_launch_count()
    if sampler:
        sampler.__exit__(None, None, None)
    if world > 1:
        dist.barrier()
    secs = start.elapsed_time(end) / 1e3
    if world > 1:
        t = torch.tensor([secs], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
    launches = replays * per_graph + eager_launches
    del graph
    return secs, launches, (sampler.summary() if sampler else None)


def time_e2e(mtype: int, steps: int, warmup: int, device, world: int):
    """Steps through q3xk_try_mv_host: H2D x, GEMV, D2H y, synchronous."""
    import torch
    import torch.distributed as dist

    from qwen3x_b200 import quant
    from qwen3x_b200.linear import try_mv

    mats, _ = make_matrix(mtype, device)
    xh = torch.from_numpy(quant.gaussian(COLS, 2)).pin_memory()
    yh = torch.empty(ROWS, dtype=torch.float32).pin_memory()
    ws = torch.empty(COLS + ROWS, dtype=torch.float32, device=device)
    for _ in range(max(warmup, 3)):
        for m in mats:
            try_mv(m, xh, yh, ws)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        for m in mats:
            try_mv(m, xh, yh, ws)
    end.record()
    torch.cuda.synchronize()
    secs = start.elapsed_time(end) / 1e3
    if world > 1:
        dist.barrier()
        t = torch.tensor([secs], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
    return secs, {"h2d_bytes_per_step": COPIES * COLS * 4, "d2h_bytes_per_step": COPIES * ROWS * 4}


def time_gemm(mtype: int, T: int, reps: int, device, world: int, precision=None):
    """Prefill dequant-GEMM Y[T, 12288] = X[T, 4096] W^T at
    `precision` (None = q3xk_gemm's split default); returns seconds per call,
    max over ranks.  The calls are replayed from a CUDA graph (no host time in
    the measurement) and rotate over weight copies whose total exceeds the
    126 MB L2 (3 x 53.5 MB for Q8_0, 5 x 28.3 MB for Q4_0), so every call
    streams its weights from HBM as a prompt chunk does."""
    import torch
    import torch.distributed as dist

    from qwen3x_b200 import quant
    from qwen3x_b200.linear import Linear, batch_mv, gemm_workspace_bytes

    packed = quant.quantize(quant.gaussian((ROWS, COLS), 1, 0.02), mtype)
    copies = 3 if mtype == 1 else 5
    lins = [Linear.from_packed(packed, mtype, ROWS, COLS, device=device) for _ in range(copies)]
    X = torch.from_numpy(quant.gaussian((T, COLS), 3)).to(device)
    Y = torch.empty(T, ROWS, device=device)
    ws = torch.empty(gemm_workspace_bytes(T, COLS), dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device)
    per_graph = max(1, reps // copies) * copies
    with torch.cuda.stream(stream):
        for lin in lins:  # warm-up (configures the kernels before capture)
            batch_mv(lin, X, Y, workspace=ws, stream=stream, precision=precision)
        stream.synchronize()
        # events as the graph's first and last nodes: device time of the calls
        start = torch.cuda.Event(enable_timing=True, external=True)
        end = torch.cuda.Event(enable_timing=True, external=True)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            start.record(stream)
            for i in range(per_graph):
                batch_mv(lins[i % copies], X, Y, workspace=ws, stream=stream, precision=precision)
            end.record(stream)
        g.replay()
        stream.synchronize()
    if world > 1:
        dist.barrier()
    with torch.cuda.stream(stream):  # the graph replays on the current stream
        g.replay()
    end.synchronize()
    secs = start.elapsed_time(end) / 1e3 / per_graph
    del g
    if world > 1:
        t = torch.tensor([secs], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
    return secs


def cpu_reference_gbs(mtype: int, threads: int, budget_s: float, rows_cap=None):
    """The reference's arch/cpu.cpp mv (oracle/_ref) on host cores: GB/s over a
    bounded sample (whole 12288x4096 matvecs until `budget_s` elapses, or a
    row-sample of one when even one call would take longer)."""
    import numpy as np

    import oracle
    from qwen3x_b200 import quant

    ref = oracle.reference()
    kind = "reference"
    if ref is None:
        kind = "port"
    w = quant.gaussian((ROWS, COLS), 1, 0.02)
    packed = quant.quantize(w, mtype)
    x = quant.gaussian(COLS, 2)
    rows = ROWS if rows_cap is None else min(ROWS, rows_cap)
    sample = packed[:rows]
    calls, t0 = 0, time.perf_counter()
    while True:
        oracle.mv(sample, mtype, rows, COLS, x, threads=threads,
                  impl="reference" if kind == "reference" else "port")
        calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    gbs = calls * algorithmic_bytes(mtype, rows) / el / 1e9
    return gbs, kind, f"{calls} x Q{'8' if mtype == 1 else '4'}_0 matvec {rows}x{COLS} in {el:.1f} s"


def decode_bytes_per_token(c, position: int) -> int:
    """Algorithmic HBM bytes of one decode step at `position`: every matrix
    once (model.bin packed size; one embedding row), the DeltaNet memory and
    conv history read and written, the KV cache read up to `position`."""
    from qwen3x_b200 import modelfile

    entries, _ = modelfile.layout(c)
    weights = sum(b for name, kind, shape, off, b in entries
                  if kind == "matrix" and name != "embedding")
    weights += modelfile.nbytes(c, "matrix", (1, c.H))
    if c.experts:  # only top_k routed experts of each pool are read
        pools = sum(b for name, kind, shape, off, b in entries if name.endswith(("moe.gate_up", "moe.down")))
        weights -= pools - pools * c.top_k // c.experts
    attn = c.N // c.AI
    delta = c.N - attn
    state = delta * (c.VH * c.KD * c.VD + c.DQKV * (c.CK - 1)) * 4 * 2
    kv = attn * position * c.KVH * c.AD * 4 * 2
    return weights + state + kv


def model_file_dir(size: int) -> str:
    import shutil
    import tempfile

    for d in ("/dev/shm", tempfile.gettempdir()):
        if os.path.isdir(d) and shutil.disk_usage(d).free > size + (4 << 30):
            return d
    return tempfile.gettempdir()


def time_engine(cfg_id: int, prompt_len: int, decode_steps: int, device, cpu_sample: bool,
                rank: int = 0, world: int = 1):
    """The backend end to end (q3x_backend.h via qwen3x_b200.backend) on a
    seeded synthetic model.bin of config `cfg_id`: prefill `prompt_len`
    uniform-random tokens in one state_forward call, then `decode_steps`
    greedy steps (state_argmax + state_forward of that token), as the
    reference's runtime drives the backend.  Times are CUDA events on the
    state's stream (max over ranks); weights (GBs) are far larger than L2.
    world > 1: one rank per GPU (rank 0 writes the file) -- tensor parallelism
    for dense configs, expert parallelism for MoE configs."""
    import numpy as np
    import torch

    from qwen3x_b200 import modelfile
    from qwen3x_b200.backend import Model, State, tp_unique_id

    c = modelfile.CONFIGS[cfg_id]
    size = modelfile.file_size(c)
    dist = None
    if world > 1:
        import torch.distributed as dist
    tag = os.environ.get("TORCHELASTIC_RUN_ID", str(os.getpid())) if world > 1 else str(os.getpid())
    path = os.path.join(model_file_dir(size), f"q3x_bench_{cfg_id}_{tag}.bin")
    out = {"config": f"{cfg_id} ({c.name})", "prompt_tokens": prompt_len, "decode_steps": decode_steps,
           "parallelism": (f"ep{world}" if c.experts else f"tp{world}") if world > 1 else "single GPU"}
    t0 = time.time()
    try:
        if rank == 0:
            modelfile.write_model(path, c, seed=7, device=device)
        if dist:
            dist.barrier()
        out["model_write_s"] = round(time.time() - t0, 1)
        t1 = time.time()
        model = Model(path, rank, world)
        out["model_load_s"] = round(time.time() - t1, 1)
        out["model_device_gb"] = round(model.device_bytes / 1e9, 2)
        nccl_id = None
        if dist:
            ids = [tp_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(ids, src=0)
            nccl_id = ids[0]
        exchange = None
        if dist:
            def exchange(handle):  # IPC handles of the peer all-reduce buffers, in rank order
                out_h = [None] * world
                dist.all_gather_object(out_h, handle)
                return out_h
        st = State(model, prompt_len + decode_steps + 72, nccl_id, exchange=exchange)
        stream = torch.cuda.ExternalStream(st.stream)
        prompt = np.random.default_rng(11).integers(0, c.V, prompt_len).astype(np.int32)
        for _ in range(3):  # warm-up: a short prompt and a few decode steps (captures the graph)
            st.forward(prompt[:min(64, prompt_len)])
            for _ in range(4):
                st.forward([st.argmax()])
            st.reset()
        st.synchronize()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        with ClockSampler(device.index) as clk:
            torch.cuda.nvtx.range_push("prefill")  # ncu --nvtx-include "prefill/"
            e0.record(stream)
            st.forward(prompt)
            e1.record(stream)
            torch.cuda.nvtx.range_pop()
            # untimed: the prompt's logits at fixed vocabulary entries (the
            # multi-GPU legs' parity check against the single-GPU run)
            full = st.logits()
            sample_idx = np.random.default_rng(5).choice(c.V, 256, replace=False)
            out["prompt_logit_sample"] = [round(float(v), 6) for v in full[sample_idx]]
            out["prompt_logit_absmax"] = round(float(np.abs(full).max()), 6)
            e1b = torch.cuda.Event(enable_timing=True)
            e1b.record(stream)
            tokens = []
            for _ in range(decode_steps):
                tokens.append(st.argmax())
                st.forward([tokens[-1]])
            e2.record(stream)
            e2.synchronize()
            # decode without the per-step host round trip (graph replays back to back)
            e3, e4 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push("decode")  # ncu --nvtx-include "decode/" selects these launches
            e3.record(stream)
            for t in tokens[:64]:
                st.forward([t])
            e4.record(stream)
            e4.synchronize()
            torch.cuda.nvtx.range_pop()
        prefill_s = e0.elapsed_time(e1) / 1e3
        decode_s = e1b.elapsed_time(e2) / 1e3
        dev_step_s = e3.elapsed_time(e4) / 1e3 / len(tokens[:64])
        if dist:  # max over ranks
            t = torch.tensor([prefill_s, decode_s, dev_step_s], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            prefill_s, decode_s, dev_step_s = (float(v) for v in t.tolist())
        mid = prompt_len + decode_steps // 2
        bpt = decode_bytes_per_token(c, mid)
        peak, peak_kind = measured_peaks()
        out.update({
            "prefill_tok_s": round(prompt_len / prefill_s, 1),
            "prefill_ms": round(prefill_s * 1e3, 2),
            "decode_tok_s": round(decode_steps / decode_s, 2),
            "decode_ms_per_token": round(decode_s / decode_steps * 1e3, 3),
            "decode_device_ms_per_token": round(dev_step_s * 1e3, 3),
            "decode_bytes_per_token": bpt,
            "decode_roofline": {"bound": "hbm", "achieved": round(bpt / dev_step_s / 1e9, 1), "peak": peak,
                                "peak_kind": peak_kind, "unit": "GB/s",
                                "frac": round(bpt / dev_step_s / 1e9 / peak, 4)},
            "clocks": clk.summary(),
            "first_tokens": tokens[:8],
        })
        if dist:
            out["tp_error"] = st.tp_error()
            dist.barrier()
        st.close()
        model.close()
        if cpu_sample and rank == 0:
            out["cpu_baseline"] = cpu_engine_tok_s(path, c)
        if dist:
            dist.barrier()
    finally:
        if rank == 0 and os.path.exists(path):
            os.unlink(path)
    return out


def time_engine_batch(cfg_id: int, prompt_len: int, decode_steps: int, batch: int, device):
    """Batched decode through q3xb_state_forward_batch (one GPU): `batch`
    independent sequences, each prefilled with its own uniform-random
    `prompt_len`-token prompt, then `decode_steps` greedy steps in which every
    sequence takes one token per call (every matrix read once for all of
    them).  Reported next to the same decode with one sequence (state_forward),
    as tokens per second over all sequences; CUDA events on the lead state's
    stream, host argmax round trips included as in the single-sequence leg."""
    import numpy as np
    import torch

    from qwen3x_b200 import modelfile
    from qwen3x_b200.backend import Model, State, forward_batch

    c = modelfile.CONFIGS[cfg_id]
    size = modelfile.file_size(c)
    path = os.path.join(model_file_dir(size), f"q3x_bench_batch_{cfg_id}_{os.getpid()}.bin")
    out = {"config": f"{cfg_id} ({c.name})", "prompt_tokens": prompt_len, "decode_steps": decode_steps,
           "batch": batch, "parallelism": "single GPU"}
    try:
        t0 = time.time()
        modelfile.write_model(path, c, seed=7, device=device)
        out["model_write_s"] = round(time.time() - t0, 1)
        model = Model(path)
        ctx = prompt_len + decode_steps + 8
        states = [State(model, ctx) for _ in range(batch)]
        rng = np.random.default_rng(13)
        t1 = time.time()
        for s in states:
            s.forward(rng.integers(0, c.V, prompt_len).astype(np.int32))
        states[0].synchronize()
        for s in states:
            s.synchronize()
        out["prefill_all_s"] = round(time.time() - t1, 1)
        stream = torch.cuda.ExternalStream(states[0].stream)
        for s in states[1:]:
            s.checkpoint_save()
        states[0].checkpoint_save()
        # warm-up step, then restore the prompts' end state
        forward_batch(model, states, [s.argmax() for s in states])
        for s in states:
            s.checkpoint_restore()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(device.index) as clk:
            toks = [s.argmax() for s in states]
            torch.cuda.nvtx.range_push("batch")  # ncu --nvtx-include "batch/" selects these launches
            e0.record(stream)
            for _ in range(decode_steps):
                forward_batch(model, states, toks)
                toks = [s.argmax() for s in states]
            e1.record(stream)
            e1.synchronize()
            torch.cuda.nvtx.range_pop()
        batch_s = e0.elapsed_time(e1) / 1e3
        # the same decode with one sequence through state_forward
        for s in states:
            s.checkpoint_restore()
        s0 = states[0]
        stream0 = torch.cuda.ExternalStream(s0.stream)
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tok = s0.argmax()
        e2.record(stream0)
        for _ in range(decode_steps):
            s0.forward([tok])
            tok = s0.argmax()
        e3.record(stream0)
        e3.synchronize()
        single_s = e2.elapsed_time(e3) / 1e3
        out.update({
            "batch_decode_tok_s": round(batch * decode_steps / batch_s, 1),
            "batch_ms_per_step": round(batch_s / decode_steps * 1e3, 3),
            "single_decode_tok_s": round(decode_steps / single_s, 1),
            "single_ms_per_token": round(single_s / decode_steps * 1e3, 3),
            "speedup": round((batch * decode_steps / batch_s) / (decode_steps / single_s), 2),
            "clocks": clk.summary(),
        })
        for s in states:
            s.close()
        model.close()
    finally:
        if os.path.exists(path):
            os.unlink(path)
    return out


def recorded_single_gpu():
    """The single-GPU engine legs' prompt logits (at 256 fixed vocabulary
    entries) and first greedy tokens, recorded from bench.py on one B200
    (tests/golden/bench_single_gpu.json): the parity check of the tensor- and
    expert-parallel legs."""
    p = ROOT / "tests" / "golden" / "bench_single_gpu.json"
    try:
        return json.loads(p.read_text())
    except Exception:
        return {}


def sharded_parity(res: dict, ref: dict) -> dict:
    """Prompt logits of an N-GPU run against the single-GPU run (bar 5e-4 of
    max(1, max|logit|), the reference's cross-backend bar) and where the greedy
    tokens first differ (random-init logits have near-ties that FP32-grade
    rounding differences can flip, so tokens are reported, not required)."""
    a = res.get("prompt_logit_sample")
    b = ref.get("prompt_logit_sample")
    out = {"bar": 5e-4}
    if a and b and len(a) == len(b):
        scale = max(1.0, float(ref.get("prompt_logit_absmax", 1.0)))
        err = max(abs(x - y) for x, y in zip(a, b)) / scale
        out["prompt_logits_max_err"] = round(err, 8)
        out["prompt_logits_within_bar"] = err <= 5e-4
    ta, tb = res.get("first_tokens", []), ref.get("first_tokens", [])
    n = min(len(ta), len(tb))
    first = next((i for i in range(n) if ta[i] != tb[i]), None)
    out["first_tokens_equal"] = first is None
    out["first_token_divergence_step"] = first
    return out


def cpu_engine_tok_s(path, c, prompt=2, steps=2):
    """The reference CPU forward (engine.cpp via oracle/_ref; single-threaded,
    one token per forward as the reference runs) on the same model.bin: a
    bounded sample of prompt + decode tokens."""
    import numpy as np

    import oracle

    if oracle.reference() is None:
        return None
    e = oracle.RefEngine(path, c if c.id not in (800, 4000, 9000, 36035, 38027) else None, context=64)
    toks = np.random.default_rng(11).integers(0, c.V, prompt).astype(np.int32)
    t0 = time.time()
    e.forward(toks)
    for _ in range(steps):
        e.forward([e.argmax()])
    dt = time.time() - t0
    e.close()
    return {"value": round((prompt + steps) / dt, 4), "unit": "tok/s", "cores": 1, "kind": "reference",
            "sample": f"{prompt}-token prompt + {steps} greedy steps of the same model.bin (reference forward "
                      "is one token at a time, so prefill and decode rates coincide)"}


def run_reference(args):
    """--impl reference: the reference CPU path with all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    import oracle

    kind = "reference" if oracle.reference() is not None else "port"
    from qwen3x_b200 import quant

    w = quant.gaussian((ROWS, COLS), 1, 0.02)
    packed = quant.quantize_q8_0(w)
    x = quant.gaussian(COLS, 2)
    for _ in range(args.warmup):
        oracle.mv(packed, 1, ROWS, COLS, x, threads=threads, impl=kind if kind == "reference" else "port")
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _c in range(COPIES):
            oracle.mv(packed, 1, ROWS, COLS, x, threads=threads, impl=kind if kind == "reference" else "port")
    el = time.perf_counter() - t0
    value = args.steps * COPIES * algorithmic_bytes(1) / el / 1e9
    line = {
        "impl": "reference", "metric": "Q8_0 GEMV HBM GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{args.steps} steps x {COPIES} Q8_0 matvecs {ROWS}x{COLS}, "
                                   f"rows split over {threads} threads"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config():
    return {"workload": "cfg1: Q8_0 GEMV y=Wx, W 12288x4096 (w~N(0,0.02)), x~N(0,1) FP32",
            "rows": ROWS, "cols": COLS, "weight_copies": COPIES,
            "l2": f"inputs larger than L2: {COPIES} resident weight copies x 53.5 MB rotated per step",
            "step": f"{COPIES} GEMV calls (one per weight copy), CUDA-graph replay",
            "timing": "CUDA events recorded as the first and last nodes of the replayed graph "
                      "(device time of the K steps; host graph submission excluded) when K <= 50",
            "parallelism": "weak, row split: rank r streams row block r of a (12288 N) x 4096 matrix "
                           "(x replicated, y sharded, no collective per step)"}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg (profiling)")
    ap.add_argument("--no-engine", action="store_true", help="skip the end-to-end model legs")
    ap.add_argument("--engine-config", type=int, default=9000,
                    help="model ID of the end-to-end leg: 9000 (cfg3, 9B Q8_0), 36035 (cfg4, 35B-A3B "
                         "MoE Q4_0), 27008 (cfg5, 27B-shaped Q8_0)")
    ap.add_argument("--engine-prompt", type=int, default=None, help="prompt tokens (default per config)")
    ap.add_argument("--engine-decode", type=int, default=256)
    ap.add_argument("--engine-batch", type=int, default=0,
                    help="with --only engine: batched decode of this many sequences (one GPU)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="N > 1: skip the tensor-/expert-parallel engine legs")
    ap.add_argument("--only", choices=["gemv", "gemm", "engine"], default=None,
                    help="run one kernel family only (for profiling; no JSON line)")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)

    import torch

    from qwen3x_b200 import capi

    capi.lib()  # fails loudly without the kernels
    rank, world, local = dist_setup(args.gpus)
    device = torch.device("cuda", torch.cuda.current_device())
    if args.only == "gemm":
        for precision, pname in ((None, "split"), (capi.GEMM_FP16, "fp16")):
            for mtype in (1, 2):
                for T in (1, 2, 8, 16, 32, 64, 128, 512, 4096):
                    secs = time_gemm(mtype, T, 10 if T >= 512 else 50, device, world, precision)
                    if rank == 0:
                        print(f"gemm {pname} type={mtype} T={T}: {secs * 1e6:.1f} us "
                              f"{2 * T * ROWS * COLS / secs / 1e12:.1f} TFLOP/s "
                              f"{algorithmic_bytes(mtype) / secs / 1e9:.0f} GB/s(weights)", flush=True)
        return 0

    prompts = {9000: 4096, 36035: 2048, 27008: 16384}  # BASELINE configs 3, 4, 5
    if args.engine_prompt is None:
        args.engine_prompt = prompts.get(args.engine_config, 4096)
    if args.only == "engine" and args.engine_batch > 0 and world == 1:
        print(json.dumps(time_engine_batch(args.engine_config, args.engine_prompt, args.engine_decode,
                                           args.engine_batch, device)), flush=True)
        return 0
    if args.only == "engine":
        res = time_engine(args.engine_config, args.engine_prompt, args.engine_decode, device,
                          rank == 0 and world == 1 and not args.no_cpu_baseline, rank, world)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
        return 0

    secs, launches, clocks = time_gemv(1, args.steps, args.warmup, device, world, rank == 0)
    bytes_q8 = algorithmic_bytes(1)
    total = world * args.steps * COPIES * bytes_q8
    value = total / secs / 1e9
    per_launch_s = secs / (args.steps * COPIES)
    peak, peak_kind = measured_peaks()
    achieved = bytes_q8 / per_launch_s / 1e9

    q4_secs, _, _ = time_gemv(2, max(args.steps // 2, 10), args.warmup, device, world, False)
    q4_bytes = algorithmic_bytes(2)
    q4_per_launch = q4_secs / (max(args.steps // 2, 10) * COPIES)
    q4_achieved = q4_bytes / q4_per_launch / 1e9

    e2e_steps = max(args.steps // 10, 20)
    if args.no_e2e:
        e2e_secs, e2e_io = float("inf"), {}
    else:
        e2e_secs, e2e_io = time_e2e(1, e2e_steps, args.warmup, device, world)
    e2e_value = world * e2e_steps * COPIES * bytes_q8 / e2e_secs / 1e9

    gemm = {}
    if args.only is None:
        peak_tf = measured_tflops()
        for precision, suffix in ((None, ""), (capi.GEMM_FP16, "_fp16")):
            for mtype, name in ((1, "q8_0"), (2, "q4_0")):
                for T in (1, 8, 64, 512, 4096):
                    gemm_secs = time_gemm(mtype, T, 10 if T >= 512 else 50, device, world, precision)
                    tf = world * 2 * T * ROWS * COLS / gemm_secs / 1e12
                    gemm[f"{name}{suffix}_T{T}"] = {"us": round(gemm_secs * 1e6, 1), "tflops": round(tf, 1),
                                                    "frac_of_bf16_peak": round(tf / world / peak_tf[0], 4)}
        gemm["peak_tflops"] = peak_tf[0]
        gemm["peak_kind"] = peak_tf[1]

    engine = None
    if args.only is None and not args.no_engine and world == 1:
        engine = time_engine(args.engine_config, args.engine_prompt, args.engine_decode, device,
                             rank == 0 and world == 1 and not args.no_cpu_baseline)
    # N > 1: the sharded paths, each rank holding a share of one model --
    # tensor parallelism on the 27B-shaped dense model (16K prompt, 256 greedy
    # steps) and expert parallelism on the 35B-A3B MoE (2K prompt) -- with the
    # greedy tokens checked against the recorded single-GPU run
    sharded = {}
    if args.only is None and world > 1 and not args.no_sharded:
        golden = recorded_single_gpu()
        for cfg_id, key in ((27008, "engine_tp27b"), (36035, "engine_ep35b")):
            try:
                res = time_engine(cfg_id, prompts[cfg_id], 256, device, False, rank, world)
            except Exception as exc:  # report the failed leg; the line itself still prints
                sharded[key] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
                print(f"bench: sharded leg {key} failed on rank {rank}: {exc}", file=sys.stderr, flush=True)
                continue
            ref = golden.get(str(cfg_id))
            if ref is not None:
                res["parity_vs_single_gpu"] = sharded_parity(res, ref)
                res["single_gpu"] = {k: ref[k] for k in ("prefill_tok_s", "decode_tok_s") if k in ref}
            res.pop("prompt_logit_sample", None)
            sharded[key] = res

    if engine:
        engine.pop("prompt_logit_sample", None)
    ref_programs = recorded_reference_programs()
    if ref_programs and engine and args.engine_config == 9000:
        rc = ref_programs.get("reference_cuda_9000", {})
        if rc.get("prefill_tok_s") and rc.get("decode_tok_s"):
            ref_programs["engine_9b_vs_reference_cuda"] = {
                "prefill": round(engine["prefill_tok_s"] / rc["prefill_tok_s"], 2),
                "decode": round(engine["decode_tok_s"] / rc["decode_tok_s"], 2)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, kind, sample = cpu_reference_gbs(1, threads=1, budget_s=10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": 1, "kind": kind, "sample": sample}

    if rank == 0:
        line = {
            "metric": "Q8_0 GEMV HBM GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(secs / args.steps * 1e3, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": profile_traffic("gemv_q8_cfg1"),
                         "bytes_per_launch": bytes_q8,
                         "kernel": "q3xk::gemv_ring_kernel<Q8_0, 24 warps, 2 stages>"},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", **e2e_io,
                    "path": "q3xk_try_mv_host (pinned host x/y, synchronous)",
                    "note": "host-latency-bound by the synchronous try_mv contract (one H2D copy, the "
                            "GEMV, one D2H copy and a stream sync per call, ~49 us per 53.5 MB call); "
                            "the end-to-end figure of the model path is extra.engine_9b.decode_tok_s "
                            "(host argmax round trip per token) beside decode_device_ms_per_token"},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "cpu_baseline": cpu,
            "extra": {
                "q4_0_gemv": {"value": round(world * q4_bytes / q4_per_launch / 1e9, 2),
                              "unit": "GB/s", "achieved_per_gpu": round(q4_achieved, 1),
                              "frac": round(q4_achieved / peak, 4),
                              "bytes_per_launch": q4_bytes},
                "gemm_cfg2": dict(gemm, workload="cfg2: Y[T,12288] = X[T,4096] W^T, dequant-GEMM on "
                                                  "tcgen05, T sweep; q8_0_T*/q4_0_T*: split precision "
                                                  "(default: hi+lo FP16 planes of X and d*q, 3 MMAs per "
                                                  "K-step, FP32-grade); *_fp16_T*: FP16 operands, 1 MMA"),
                "engine_9b": engine,
                **sharded,
                "reference_programs": ref_programs,
            },
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
