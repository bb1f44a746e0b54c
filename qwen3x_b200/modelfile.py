"""model.bin: configurations, tensor schema and a seeded synthetic writer.

The file format is qwen3x's (model_config.h:10-39, engine.cpp:461-559,
scripts/pack_weights.py:212-289): the 8-byte magic "Q3XMODL\\0", 16 uint32
header fields, then every tensor in a fixed order, each starting on a 64-byte
boundary.  Large matrices use the model's matrix type (Q8_0/Q4_0 blocks); the
MoE router and shared-expert gate are BF16; norms BF16 (stored as w', applied
as 1 + w'); DeltaNet A_log and norm FP32; dt_bias and conv BF16.

Configurations: the reference's registered model IDs with their shapes
(model_config.h:57-101), plus IDs this build adds:
  27008  the 27B-shaped hybrid with Q8_0 matrices (benchmark config 5; the
         reference only registers a Q4_0 27B, id 38027)
  9091, 9092, 35091  small test models (dense Q8_0, dense Q4_0, MoE Q4_0)
         with the real head sizes, used for fast end-to-end parity tests.

The synthetic weights follow the benchmark configs: matrices from
w ~ N(0, 0.02) quantised with the configs' encoders, BF16 router ~ N(0, 0.02),
RMSNorm w' ~ N(0, 0.01) (effective 1 + w'), DeltaNet norm 1 + N(0, 0.01),
A_log = 0, dt_bias = 0, conv ~ N(0, 0.1).
"""
from __future__ import annotations

import dataclasses
import struct
from pathlib import Path

import numpy as np

from .quant import BF16, Q4_0, Q8_0, quantize, to_bf16_bits

MAGIC = b"Q3XMODL\0"
MAX_CONTEXT = 262144
ALIGN = 64


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    id: int
    name: str
    V: int
    H: int
    I: int
    N: int
    AI: int
    AH: int
    KVH: int
    AD: int
    RD: int
    KH: int
    VH: int
    KD: int
    VD: int
    CK: int
    experts: int
    top_k: int
    shared_I: int
    matrix_type: int
    tied: bool

    @property
    def DQKV(self):
        return 2 * self.KH * self.KD + self.VH * self.VD

    @property
    def DO(self):
        return self.VH * self.VD

    @property
    def AS(self):
        return self.AH * self.AD

    @property
    def KVW(self):
        return self.KVH * self.AD

    def header(self) -> bytes:
        fields = (self.id, self.V, self.H, self.I, self.N, self.AI, self.AH, self.KVH, self.AD,
                  self.RD, self.KH, self.VH, self.KD, self.VD, self.CK, MAX_CONTEXT)
        return MAGIC + struct.pack("<16I", *fields)

    def is_delta(self, layer: int) -> bool:
        return layer % self.AI != self.AI - 1


def _c(*a):
    return ModelConfig(*a)


CONFIGS = {c.id: c for c in [
    # id, name, V, H, I, N, AI, AH, KVH, AD, RD, KH, VH, KD, VD, CK, experts, top_k, shared_I, type, tied
    _c(800, "Qwen3.5-0.8B", 248320, 1024, 3584, 24, 4, 8, 2, 256, 64, 16, 16, 128, 128, 4, 0, 0, 0, BF16, True),
    _c(4000, "Qwen3.5-4B", 248320, 2560, 9216, 32, 4, 16, 4, 256, 64, 16, 32, 128, 128, 4, 0, 0, 0, BF16, True),
    _c(9000, "Qwen3.5-9B", 248320, 4096, 12288, 32, 4, 16, 4, 256, 64, 16, 32, 128, 128, 4, 0, 0, 0, Q8_0, False),
    _c(36035, "Qwen3.6-35B-A3B", 248320, 2048, 512, 40, 4, 16, 2, 256, 64, 16, 32, 128, 128, 4, 256, 8, 512,
       Q4_0, False),
    _c(38027, "Qwen3.8-27B", 248320, 5120, 17408, 64, 4, 24, 4, 256, 64, 16, 48, 128, 128, 4, 0, 0, 0, Q4_0,
       False),
    # added by this build
    _c(27008, "27B-shaped Q8_0", 248320, 5120, 17408, 64, 4, 24, 4, 256, 64, 16, 48, 128, 128, 4, 0, 0, 0,
       Q8_0, False),
    _c(9091, "test dense Q8_0", 4096, 512, 1024, 8, 4, 2, 1, 256, 64, 2, 4, 128, 128, 4, 0, 0, 0, Q8_0, False),
    _c(9092, "test dense Q4_0", 4096, 512, 1024, 4, 4, 2, 1, 256, 64, 2, 4, 128, 128, 4, 0, 0, 0, Q4_0, False),
    _c(35091, "test MoE Q4_0", 4096, 512, 128, 4, 4, 2, 1, 256, 64, 2, 4, 128, 128, 4, 16, 4, 128, Q4_0, False),
]}


def tensors(c: ModelConfig):
    """(name, kind, shape) in file order; kind is 'matrix' (model type), 'bf16' or 'f32'
    (engine.cpp:521-555)."""
    yield "embedding", "matrix", (c.V, c.H)
    if not c.tied:
        yield "lm_head", "matrix", (c.V, c.H)
    yield "final_norm", "bf16", (c.H,)
    for i in range(c.N):
        p = f"layers.{i}."
        yield p + "input_norm", "bf16", (c.H,)
        if c.is_delta(i):
            yield p + "delta.qkv", "matrix", (c.DQKV, c.H)
            yield p + "delta.z", "matrix", (c.DO, c.H)
            yield p + "delta.a", "matrix", (c.VH, c.H)
            yield p + "delta.b", "matrix", (c.VH, c.H)
            yield p + "delta.conv", "bf16", (c.DQKV, c.CK)
            yield p + "delta.alog", "f32", (c.VH,)
            yield p + "delta.dt", "bf16", (c.VH,)
            yield p + "delta.norm", "f32", (c.VD,)
            yield p + "delta.out", "matrix", (c.H, c.DO)
        else:
            yield p + "attn.q", "matrix", (2 * c.AS, c.H)
            yield p + "attn.k", "matrix", (c.KVW, c.H)
            yield p + "attn.v", "matrix", (c.KVW, c.H)
            yield p + "attn.qnorm", "bf16", (c.AD,)
            yield p + "attn.knorm", "bf16", (c.AD,)
            yield p + "attn.out", "matrix", (c.H, c.AS)
        yield p + "post_norm", "bf16", (c.H,)
        if c.experts:
            yield p + "moe.router", "bf16", (c.experts, c.H)
            yield p + "moe.gate_up", "matrix", (c.experts * 2 * c.I, c.H)
            yield p + "moe.down", "matrix", (c.experts * c.H, c.I)
            yield p + "moe.shared_gate", "matrix", (c.shared_I, c.H)
            yield p + "moe.shared_up", "matrix", (c.shared_I, c.H)
            yield p + "moe.shared_down", "matrix", (c.H, c.shared_I)
            yield p + "moe.shared_scale", "bf16", (1, c.H)
        else:
            yield p + "ffn.gate", "matrix", (c.I, c.H)
            yield p + "ffn.up", "matrix", (c.I, c.H)
            yield p + "ffn.down", "matrix", (c.H, c.I)


def nbytes(c: ModelConfig, kind: str, shape) -> int:
    n = int(np.prod(shape))
    if kind == "matrix":
        if c.matrix_type == Q8_0:
            return n // 32 * 34
        if c.matrix_type == Q4_0:
            return n // 32 * 18
        return n * 2
    return n * (2 if kind == "bf16" else 4)


def layout(c: ModelConfig):
    """[(name, kind, shape, offset, bytes)], total file size."""
    out, cursor = [], len(c.header())
    for name, kind, shape in tensors(c):
        cursor += (-cursor) % ALIGN
        b = nbytes(c, kind, shape)
        out.append((name, kind, shape, cursor, b))
        cursor += b
    return out, cursor


def file_size(c: ModelConfig) -> int:
    return layout(c)[1]


def _std(name: str) -> float:
    if "norm" in name:
        return 0.01
    if name.endswith("conv"):
        return 0.1
    return 0.02


def _torch_quantize(w, mtype):
    """Benchmark-config encoders on the GPU (bit-identical to quant.py's numpy
    versions: IEEE division, round half away from zero, RNE to FP16)."""
    import torch

    b = w.reshape(-1, 32)
    if mtype == Q8_0:
        scale = b.abs().amax(dim=1) / 127.0
    else:
        scale = b.abs().amax(dim=1) / 8.0
    inv = torch.where(scale != 0, 1.0 / torch.where(scale != 0, scale, torch.ones_like(scale)),
                      torch.zeros_like(scale))
    n = b * inv[:, None]
    r = torch.sign(n) * torch.floor(n.abs() + 0.5)
    h = scale.to(torch.float16).view(torch.int16).to(torch.int32) & 0xFFFF
    if mtype == Q8_0:
        q = r.clamp(-127, 127).to(torch.int8).view(torch.uint8).to(torch.int32)
        blocks = torch.empty(b.shape[0], 34, dtype=torch.uint8, device=w.device)
        blocks[:, 2:] = q.to(torch.uint8)
    else:
        q = (r + 8).clamp(0, 15).to(torch.int32)
        blocks = torch.empty(b.shape[0], 18, dtype=torch.uint8, device=w.device)
        blocks[:, 2:] = (q[:, :16] | (q[:, 16:] << 4)).to(torch.uint8)
    blocks[:, 0] = (h & 0xFF).to(torch.uint8)
    blocks[:, 1] = (h >> 8).to(torch.uint8)
    return blocks


def tensor_bytes(c: ModelConfig, name: str, kind: str, shape, seed: int, device=None) -> bytes:
    """Deterministic synthetic contents of one tensor.  With `device` (a CUDA
    device) matrices are generated and quantised on the GPU, otherwise numpy."""
    n = int(np.prod(shape))
    tseed = (seed * 1000003 + sum(name.encode()) * 7919 + len(name)) % (2**63)
    if kind == "f32":
        if name.endswith("alog"):
            return np.zeros(n, np.float32).tobytes()
        # DeltaNet norm: 1 + N(0, 0.01)
        return (1.0 + np.random.default_rng(tseed).standard_normal(n, dtype=np.float32)
                * np.float32(0.01)).astype(np.float32).tobytes()
    if kind == "bf16":
        if name.endswith("delta.dt"):
            return np.zeros(n, np.uint16).tobytes()
        v = np.random.default_rng(tseed).standard_normal(n, dtype=np.float32) * np.float32(_std(name))
        return to_bf16_bits(v).tobytes()
    if device is not None and c.matrix_type in (Q8_0, Q4_0):
        import torch

        g = torch.Generator(device=device)
        g.manual_seed(tseed)
        out = []
        rows, cols = shape
        step = max(1, (1 << 26) // cols)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            w = torch.randn((r1 - r0) * cols, generator=g, device=device, dtype=torch.float32) * 0.02
            out.append(_torch_quantize(w, c.matrix_type).cpu().numpy().tobytes())
        return b"".join(out)
    v = np.random.default_rng(tseed).standard_normal(shape, dtype=np.float32) * np.float32(0.02)
    return quantize(v, c.matrix_type).tobytes()


def write_model(path, c: ModelConfig | int, seed: int = 1, device=None) -> Path:
    """Write a synthetic model.bin for config `c` (a ModelConfig or an id)."""
    if isinstance(c, int):
        c = CONFIGS[c]
    path = Path(path)
    entries, total = layout(c)
    with open(path, "wb") as f:
        f.write(c.header())
        for name, kind, shape, off, b in entries:
            f.write(b"\0" * (off - f.tell()))
            data = tensor_bytes(c, name, kind, shape, seed, device)
            if len(data) != b:
                raise AssertionError(f"{name}: {len(data)} != {b}")
            f.write(data)
    if path.stat().st_size != total:
        raise AssertionError("model.bin size mismatch")
    return path
