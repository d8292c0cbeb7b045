"""Seeded random-init MoE layers of the benchmark architectures (checkpoint layouts).

No public dataset or checkpoint is available offline; these tensors are the whole
benchmark workload, and the parity tests draw the same tensors.
Everything comes from ``numpy.random.default_rng(seed)`` drawn in a fixed order:
router, routed experts ``0..E-1`` (gate, up, down), shared experts (gate, up, down),
then activations.  Within one matrix: AWQ ``qweight``, ``qzeros``, ``scales``; FP8
``weight``, ``scale``.  Distributions:

* router fp32 ``N(0, 0.02)``; activations bf16 ``N(0, 1)`` (fp32 draw rounded to bf16);
* AWQ nibbles and zero-points uniform in ``[0, 15]`` (uniform 32-bit words), scales
  fp16 ``|N(0, 0.02)| + 1e-3``;
* FP8 values ``N(0, 1)`` clipped to +-448 and rounded to e4m3 (nearest-even), block
  scales fp32 log-uniform in ``[1e-3, 1e-1]``;
* per-channel FP8 (``fp8_channel``, the reference's own FP8): the same codes, one fp32
  scale per output channel, log-uniform in ``[1e-3, 1e-1]``;
* signed int4 (``int4_sym_g128``, the reference's ``int4_w4a16_sym``): values uniform in
  ``[-8, 7]``, one fp32 scale per input column, ``|N(0, 0.02)| + 1e-3`` drawn per 128-k
  group (the scale is constant within each group, as the kernels require).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, replace

import numpy as np


__all__ = [
    "MoeLayerConfig",
    "CONFIGS",
    "AwqMatrix",
    "Fp8Matrix",
    "Fp8ChannelMatrix",
    "Int4SymMatrix",
    "ExpertWeights",
    "LayerWeights",
    "make_layer",
    "make_layer_device",
    "scaled_config",
    "bf16_bits_from_f32",
    "GROUP",
    "BLOCK",
]

GROUP = 128  # AWQ group size along K
BLOCK = 128  # FP8 block edge


def bf16_bits_from_f32(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round-to-nearest-even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rnd = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((u + rnd) >> np.uint32(16)).astype(np.uint16)
    return np.where(np.isnan(np.asarray(x, dtype=np.float32)), np.uint16(0x7FC0), out).astype(np.uint16)


@dataclass(frozen=True)
class MoeLayerConfig:
    name: str
    hidden: int
    inter: int
    num_experts: int
    top_k: int
    num_shared: int
    shared_inter: int
    fmt: str  # "awq_int4_g128" | "fp8_b128" | "fp8_channel" | "int4_sym_g128"
    routing: str  # "softmax_topk" | "topk_softmax" | "sigmoid_group"
    n_group: int = 1
    topk_group: int = 1
    routed_scaling: float = 1.0
    tokens: tuple = ()

    @property
    def route_kw(self) -> dict:
        if self.routing == "sigmoid_group":
            return {"n_group": self.n_group, "topk_group": self.topk_group, "routed_scaling": self.routed_scaling}
        return {}

    def expert_bytes(self) -> int:
        """Algorithmic HBM bytes of one routed expert (weights + scales + zero-points)."""
        return _matrix_bytes(self.fmt, self.hidden, self.inter) * 2 + _matrix_bytes(self.fmt, self.inter, self.hidden)

    def shared_bytes(self) -> int:
        return self.num_shared * (
            _matrix_bytes(self.fmt, self.hidden, self.shared_inter) * 2
            + _matrix_bytes(self.fmt, self.shared_inter, self.hidden)
        )


def _matrix_bytes(fmt: str, k: int, n: int) -> int:
    """Checkpoint bytes of one matrix (weights + scales + zero-points)."""
    if fmt == "awq_int4_g128":
        groups = k // GROUP
        return k * n // 2 + groups * n * 2 + groups * n // 2
    if fmt == "fp8_channel":
        return k * n + n * 4
    if fmt == "int4_sym_g128":
        return k * n // 2 + k * 4
    nb, kb = math.ceil(n / BLOCK), math.ceil(k / BLOCK)
    return k * n + nb * kb * 4


CONFIGS: dict[str, MoeLayerConfig] = {
    # DeepSeek-V2-Lite MoE layer, AWQ int4 g128
    "cfg0": MoeLayerConfig("cfg0", 2048, 1408, 64, 6, 2, 1408, "awq_int4_g128", "softmax_topk", tokens=(1, 8, 64)),
    # same layer, FP8 e4m3 128x128 blocks
    "cfg1": MoeLayerConfig("cfg1", 2048, 1408, 64, 6, 2, 1408, "fp8_b128", "softmax_topk", tokens=(1, 16, 64, 256, 2048)),
    # Qwen3-30B-A3B MoE layer (no shared expert), AWQ int4
    "cfg3": MoeLayerConfig("cfg3", 2048, 768, 128, 8, 0, 0, "awq_int4_g128", "topk_softmax", tokens=(64, 4096)),
    # DeepSeek-V3 MoE layer, FP8 blocks, grouped sigmoid routing
    "cfg4": MoeLayerConfig(
        "cfg4", 7168, 2048, 256, 8, 1, 2048, "fp8_b128", "sigmoid_group",
        n_group=8, topk_group=4, routed_scaling=2.5, tokens=(256, 4096, 16384),
    ),
}


def scaled_config(base: str | MoeLayerConfig, **over) -> MoeLayerConfig:
    """A smaller layer with the same format and routing (for oracle-sized parity tests)."""
    cfg = CONFIGS[base] if isinstance(base, str) else base
    return replace(cfg, **over)


@dataclass
class AwqMatrix:
    """AWQ int4 g128 matrix, [in, out] = [K, N]."""

    qweight: np.ndarray  # int32 [K, N/8]
    qzeros: np.ndarray  # int32 [K/128, N/8]
    scales: np.ndarray  # fp16 [K/128, N]


@dataclass
class Fp8Matrix:
    """FP8 e4m3 128x128-block matrix, [out, in] = [N, K]."""

    weight: np.ndarray  # uint8 [N, K]
    scale: np.ndarray  # fp32 [N/128, K/128]


@dataclass
class Fp8ChannelMatrix:
    """FP8 e4m3 with one fp32 scale per output channel, [out, in] = [N, K] (the reference's
    ``fp8_dequant_mat`` layout)."""

    weight: np.ndarray  # uint8 [N, K]
    scale: np.ndarray  # fp32 [N]


@dataclass
class Int4SymMatrix:
    """Signed int4 weight-only, [out, in] (the reference's ``WeightOnlyMethod`` layout)."""

    weight: np.ndarray  # uint8 [N, K/2], low nibble = even input column
    scale: np.ndarray  # fp32 [K], one per input column


@dataclass
class ExpertWeights:
    gate: object
    up: object
    down: object


@dataclass
class LayerWeights:
    cfg: MoeLayerConfig
    router: np.ndarray  # fp32 [E, H]
    experts: list
    shared: list
    rng_state: dict = field(repr=False, default_factory=dict)

    def make_x(self, tokens: int) -> np.ndarray:
        """bf16 activations (uint16 bit patterns) [tokens, H], drawn after the weights."""
        rng = np.random.default_rng()
        rng.bit_generator.state = self.rng_state
        x = rng.standard_normal((tokens, self.cfg.hidden), dtype=np.float32)
        return bf16_bits_from_f32(x)


def _encode_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 (already within +-448) -> e4m3fn codes, round-to-nearest-even."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def _gen_matrix(rng: np.random.Generator, fmt: str, k: int, n: int):
    if fmt == "awq_int4_g128":
        g = k // GROUP
        qweight = rng.integers(0, 2**32, size=(k, n // 8), dtype=np.uint32).view(np.int32)
        qzeros = rng.integers(0, 2**32, size=(g, n // 8), dtype=np.uint32).view(np.int32)
        scales = (np.abs(rng.normal(0.0, 0.02, size=(g, n))) + 1e-3).astype(np.float16)
        return AwqMatrix(qweight, qzeros, scales)
    if fmt == "fp8_b128":
        w = np.clip(rng.standard_normal((n, k), dtype=np.float32), -448.0, 448.0)
        nb, kb = math.ceil(n / BLOCK), math.ceil(k / BLOCK)
        scale = np.exp(rng.uniform(math.log(1e-3), math.log(1e-1), size=(nb, kb))).astype(np.float32)
        return Fp8Matrix(_encode_e4m3(w), scale)
    if fmt == "fp8_channel":
        w = np.clip(rng.standard_normal((n, k), dtype=np.float32), -448.0, 448.0)
        scale = np.exp(rng.uniform(math.log(1e-3), math.log(1e-1), size=n)).astype(np.float32)
        return Fp8ChannelMatrix(_encode_e4m3(w), scale)
    if fmt == "int4_sym_g128":
        packed = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
        sg = (np.abs(rng.normal(0.0, 0.02, size=k // GROUP)) + 1e-3).astype(np.float32)
        return Int4SymMatrix(packed, np.repeat(sg, GROUP))
    raise ValueError(f"unknown format {fmt!r}")


def _gen_expert(rng, fmt: str, hidden: int, inter: int) -> ExpertWeights:
    gate = _gen_matrix(rng, fmt, hidden, inter)
    up = _gen_matrix(rng, fmt, hidden, inter)
    down = _gen_matrix(rng, fmt, inter, hidden)
    return ExpertWeights(gate, up, down)


def make_layer_device(cfg: str | MoeLayerConfig, seed: int = 0, device="cuda") -> LayerWeights:
    """The same layer shapes and value distributions as ``make_layer``, drawn on the GPU from
    a seeded torch generator (seconds instead of minutes for the 11 GB DeepSeek-V3 layer).
    The values differ from ``make_layer``'s (another random stream): the benchmark uses it for
    the layers too large to generate on the host in a bounded time; the parity tests use
    ``make_layer``.  Matrices hold device tensors; ``make_x`` stays the host draw."""
    import torch

    cfg = CONFIGS[cfg] if isinstance(cfg, str) else cfg
    if cfg.hidden % GROUP or cfg.inter % GROUP:
        raise ValueError("hidden and inter must be multiples of 128")
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def mat(k: int, n: int):
        lo, hi = math.log(1e-3), math.log(1e-1)
        if cfg.fmt == "int4_sym_g128":
            packed = torch.randint(0, 256, (n, k // 2), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
            sg = (torch.randn((k // GROUP,), generator=g, device=device) * 0.02).abs_().add_(1e-3)
            return Int4SymMatrix(packed, sg.repeat_interleave(GROUP))
        if cfg.fmt == "fp8_channel":
            w = torch.randn((n, k), generator=g, device=device).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
            sc = torch.rand((n,), generator=g, device=device).mul_(hi - lo).add_(lo).exp_()
            return Fp8ChannelMatrix(w.view(torch.uint8), sc)
        if cfg.fmt == "awq_int4_g128":
            q = torch.randint(-2**31, 2**31, (k, n // 8), generator=g, device=device, dtype=torch.int64).to(torch.int32)
            z = torch.randint(-2**31, 2**31, (k // GROUP, n // 8), generator=g, device=device,
                              dtype=torch.int64).to(torch.int32)
            sc = (torch.randn((k // GROUP, n), generator=g, device=device) * 0.02).abs_().add_(1e-3).to(torch.float16)
            return AwqMatrix(q, z, sc)
        w = torch.randn((n, k), generator=g, device=device).clamp_(-448.0, 448.0).to(torch.float8_e4m3fn)
        nb, kb = math.ceil(n / BLOCK), math.ceil(k / BLOCK)
        sc = torch.rand((nb, kb), generator=g, device=device).mul_(hi - lo).add_(lo).exp_()
        return Fp8Matrix(w.view(torch.uint8), sc)

    def expert(inter: int) -> ExpertWeights:
        return ExpertWeights(mat(cfg.hidden, inter), mat(cfg.hidden, inter), mat(inter, cfg.hidden))

    router = (torch.randn((cfg.num_experts, cfg.hidden), generator=g, device=device) * 0.02).cpu().numpy()
    experts = [expert(cfg.inter) for _ in range(cfg.num_experts)]
    shared = [expert(cfg.shared_inter) for _ in range(cfg.num_shared)]
    rng = np.random.default_rng(seed)
    return LayerWeights(cfg, router, experts, shared, rng_state=rng.bit_generator.state)


def make_layer(cfg: str | MoeLayerConfig, seed: int = 0) -> LayerWeights:
    """Generate one MoE layer's weights (host, checkpoint layouts) from ``seed``."""
    cfg = CONFIGS[cfg] if isinstance(cfg, str) else cfg
    if cfg.hidden % GROUP or cfg.inter % GROUP:
        raise ValueError("hidden and inter must be multiples of 128")
    rng = np.random.default_rng(seed)
    router = rng.normal(0.0, 0.02, size=(cfg.num_experts, cfg.hidden)).astype(np.float32)
    experts = [_gen_expert(rng, cfg.fmt, cfg.hidden, cfg.inter) for _ in range(cfg.num_experts)]
    shared = [_gen_expert(rng, cfg.fmt, cfg.hidden, cfg.shared_inter) for _ in range(cfg.num_shared)]
    return LayerWeights(cfg, router, experts, shared, rng_state=rng.bit_generator.state)
