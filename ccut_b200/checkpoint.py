"""Checkpoint loader: one MoE layer's experts from safetensors shards into HBM.

The reference streams experts from disk at every step: ``ccut/experts/index.py:145-248``
parses the shard headers into a ``(layer, expert) -> segment`` index,
``ccut/experts/reader.py:86-334`` reads those segments on demand, and
``ccut/io_/safetensors_io.py:88-218`` is its shard reader.  Here the same headers are
parsed once, and every routed and shared expert of a layer is read through ``mmap`` and
packed into the layer's HBM tile layout (``MoeLayer``), where it stays for the life of
the layer.

Checkpoint formats (the ``quantization_config`` of ``config.json``, resolved by
``quant_method`` as in ``ccut/quant/registry.py:107-153``):

* AWQ GEMM (``"awq"``, 4 bits, group size 128, zero points):
  ``<proj>.qweight`` int32 ``[in, out/8]``, ``<proj>.qzeros`` int32 ``[in/128, out/8]``,
  ``<proj>.scales`` fp16 ``[in/128, out]``;
* FP8 block (``"fp8"``, e4m3, ``weight_block_size [128, 128]``):
  ``<proj>.weight`` F8_E4M3 ``[out, in]``, ``<proj>.weight_scale_inv`` fp32
  ``[out/128, in/128]``.

MoE shape keys follow ``ccut/models/spec.py:159-170`` (``num_experts`` or
``n_routed_experts``, ``num_experts_per_tok``, ``moe_intermediate_size``,
``norm_topk_prob``, ``n_shared_experts`` or ``moe_shared_expert_intermediate_size``),
plus the DeepSeek-V3 routing keys (``scoring_func``, ``n_group``, ``topk_group``,
``routed_scaling_factor``).  Missing tensors raise ``KeyError``, malformed files and
missing scales ``ValueError``, formats this path does not run ``NotImplementedError``,
as the reference's reader and quant methods do.
"""

from __future__ import annotations

import json
import mmap
import re
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

__all__ = [
    "SafetensorsShard",
    "CheckpointReader",
    "MoeCheckpointSpec",
    "NameTemplates",
    "expert_pattern",
    "quant_format",
    "moe_spec_from_config",
    "load_layer_weights",
    "load_moe_layer",
    "DecoderNames",
    "DecoderCheckpointSpec",
    "decoder_spec_from_config",
    "load_decoder_weights",
    "load_decoder",
]

# safetensors dtype -> numpy dtype of the stored bytes (BF16 and FP8 stay as raw bits)
_DTYPES = {
    "F64": np.float64, "F32": np.float32, "F16": np.float16, "BF16": np.uint16,
    "I64": np.int64, "U64": np.uint64, "I32": np.int32, "U32": np.uint32, "I16": np.int16, "U16": np.uint16,
    "I8": np.int8, "U8": np.uint8, "BOOL": np.bool_, "F8_E4M3": np.uint8, "F8_E5M2": np.uint8,
}
_MAX_HEADER = 100 * 1024 * 1024


@dataclass(frozen=True)
class TensorInfo:
    dtype: str
    shape: tuple[int, ...]
    begin: int  # byte offsets inside the data section
    end: int


class SafetensorsShard:
    """One safetensors file: an 8-byte little-endian header length, a JSON header mapping
    tensor names to ``dtype`` / ``shape`` / ``data_offsets``, then the tensor bytes.
    Tensors are read as read-only views of an ``mmap`` of the file."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        with open(self.path, "rb") as fh:
            head = fh.read(8)
            if len(head) < 8:
                raise ValueError(f"{self.path}: too short for a safetensors file")
            (n,) = struct.unpack("<Q", head)
            if n > _MAX_HEADER:
                raise ValueError(f"{self.path}: header of {n} bytes, file corrupt")
            raw = fh.read(n)
            if len(raw) < n:
                raise ValueError(f"{self.path}: truncated header")
        try:
            meta = json.loads(raw.decode("utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise ValueError(f"{self.path}: header is not JSON ({e})") from None
        self.metadata = meta.pop("__metadata__", {}) or {}
        self.data_start = 8 + n
        size = self.path.stat().st_size
        self.tensors: dict[str, TensorInfo] = {}
        for name, d in meta.items():
            if d.get("dtype") not in _DTYPES:
                raise NotImplementedError(f"{self.path}: tensor {name!r} has unsupported dtype {d.get('dtype')!r}")
            shape = tuple(int(v) for v in d["shape"])
            b, e = (int(v) for v in d["data_offsets"])
            count = int(np.prod(shape, dtype=np.int64)) if shape else 1
            if e - b != count * np.dtype(_DTYPES[d["dtype"]]).itemsize or b < 0 or self.data_start + e > size:
                raise ValueError(f"{self.path}: tensor {name!r} offsets [{b}, {e}) disagree with its shape or the file")
            self.tensors[name] = TensorInfo(d["dtype"], shape, b, e)
        self._mm: mmap.mmap | None = None

    @property
    def names(self) -> list[str]:
        return list(self.tensors)

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def info(self, name: str) -> TensorInfo:
        try:
            return self.tensors[name]
        except KeyError:
            raise KeyError(f"{self.path}: no tensor {name!r}") from None

    def array(self, name: str) -> np.ndarray:
        """Read-only view of a tensor's bytes with its shape (BF16 / FP8 as raw bits)."""
        t = self.info(name)
        if self._mm is None:
            with open(self.path, "rb") as fh:
                self._mm = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
        dt = np.dtype(_DTYPES[t.dtype])
        a = np.frombuffer(self._mm, dtype=dt, count=(t.end - t.begin) // dt.itemsize, offset=self.data_start + t.begin)
        return a.reshape(t.shape)

    def close(self) -> None:
        self._mm = None  # the views keep the mapping alive while they exist


class CheckpointReader:
    """A model directory: ``config.json`` plus one ``model.safetensors`` or the shards
    listed in ``model.safetensors.index.json`` (``weight_map``: tensor -> shard file)."""

    def __init__(self, model_dir: str | Path):
        self.dir = Path(model_dir)
        cfg = self.dir / "config.json"
        if not cfg.exists():
            raise FileNotFoundError(f"{cfg}: no config.json")
        self.config = json.loads(cfg.read_text())
        index = self.dir / "model.safetensors.index.json"
        self._shards: dict[str, SafetensorsShard] = {}
        self.weight_map: dict[str, str] = {}
        if index.exists():
            wm = json.loads(index.read_text()).get("weight_map")
            if not isinstance(wm, dict):
                raise ValueError(f"{index}: no weight_map")
            self.weight_map = {str(k): str(v) for k, v in wm.items()}
        else:
            files = sorted(self.dir.glob("*.safetensors"))
            if not files:
                raise FileNotFoundError(f"{self.dir}: no safetensors files")
            for f in files:
                for name in self._shard(f.name).names:
                    self.weight_map[name] = f.name

    def _shard(self, fname: str) -> SafetensorsShard:
        sh = self._shards.get(fname)
        if sh is None:
            sh = self._shards[fname] = SafetensorsShard(self.dir / fname)
        return sh

    @property
    def text_config(self) -> dict:
        return self.config.get("text_config", self.config)

    def has(self, name: str) -> bool:
        return name in self.weight_map

    def tensor(self, name: str) -> np.ndarray:
        if name not in self.weight_map:
            raise KeyError(f"{self.dir}: no tensor {name!r} in the checkpoint")
        return self._shard(self.weight_map[name]).array(name)

    def dtype(self, name: str) -> str:
        if name not in self.weight_map:
            raise KeyError(f"{self.dir}: no tensor {name!r} in the checkpoint")
        return self._shard(self.weight_map[name]).info(name).dtype


# ---------------------------------------------------------------- config
def _compressed_tensors_format(q: dict) -> str:
    """The format of this path that a compressed-tensors ``quantization_config`` stores (the
    scheme kinds of ``ccut/quant/compressed_tensors.py:44-71``): one config group of int4
    weights, group strategy with group size 128, no activation quantization and no
    activation reordering (``pack-quantized``, repacked into AWQ's layout at load), or of FP8
    weights with the ``block`` strategy and 128 x 128 blocks (``float-quantized``; its
    activations run in 16 bits here, whatever ``input_activations`` says)."""
    groups = q.get("config_groups") or {}
    if len(groups) != 1:
        raise NotImplementedError(f"compressed-tensors with {len(groups)} config groups (have one)")
    g = next(iter(groups.values()))
    w = g.get("weights") or {}
    kind, bits, strategy = str(w.get("type", "")).lower(), int(w.get("num_bits") or 0), str(w.get("strategy", "")).lower()
    if kind == "int" and bits == 4 and strategy == "group" and int(w.get("group_size") or 0) == 128:
        if g.get("input_activations") or w.get("actorder") not in (None, False, "none"):
            raise NotImplementedError("compressed-tensors int4 with activation quantization or activation reordering")
        stored = str(g.get("format") or q.get("format") or "pack-quantized").lower()
        if stored != "pack-quantized":
            raise NotImplementedError(f"compressed-tensors int4 stored as {stored!r} (have pack-quantized)")
        # symmetric: signed int4 with its fp32 group scales as they are; asymmetric: AWQ's
        # unsigned codes and zero points (fp16 scales)
        return "int4_sym_g128" if w.get("symmetric", True) else "awq_int4_g128"
    if kind == "float" and bits == 8 and strategy == "block" and [int(v) for v in (w.get("block_structure") or [])] \
            == [128, 128]:
        return "fp8_b128"
    if kind == "float" and bits == 8 and strategy in ("channel", "tensor"):
        # the reference's own FP8 (its checkpoints' weights are per-channel static,
        # ccut/quant/compressed_tensors.py:3-10); per-token dynamic activations run in 16 bits
        # here, as the reference computes them (dequantized weights, ccut/quant/method.py:131-139)
        return "fp8_channel"
    raise NotImplementedError(f"compressed-tensors weights type={kind!r} num_bits={bits} strategy={strategy!r} are not "
                              "supported (int4 group 128, FP8 per channel / per tensor / 128 x 128 blocks)")


def quant_format(config: dict) -> str:
    """Weight format of this path for a checkpoint's ``quantization_config``: AWQ
    (``quant_method = "awq"``), FP8 blocks (``"fp8"``), or the compressed-tensors schemes that
    store the same values (``_compressed_tensors_format``)."""
    tc = config.get("text_config", config)
    q = tc.get("quantization_config") or config.get("quantization_config")
    if not q:
        raise NotImplementedError("unquantized checkpoint: this path runs AWQ int4 g128 or FP8 e4m3 128x128 weights")
    method = str(q.get("quant_method", "")).lower()
    if method == "awq":
        bits, group = int(q.get("bits", q.get("w_bit", 4))), int(q.get("group_size", q.get("q_group_size", 128)))
        version = str(q.get("version", "gemm")).lower()
        if bits != 4 or group != 128 or not q.get("zero_point", True) or version != "gemm":
            raise NotImplementedError(f"AWQ variant bits={bits} group_size={group} version={version!r} is not supported"
                                      " (4-bit, group 128, zero points, GEMM packing)")
        return "awq_int4_g128"
    if method == "fp8":
        block = q.get("weight_block_size")
        fmt = str(q.get("fmt", "e4m3")).lower()
        if block is None or [int(v) for v in block] != [128, 128] or fmt != "e4m3":
            raise NotImplementedError(f"FP8 variant fmt={fmt!r} weight_block_size={block} is not supported"
                                      " (e4m3, 128 x 128 blocks)")
        return "fp8_b128"
    if method == "compressed-tensors":
        return _compressed_tensors_format(q)
    raise NotImplementedError(f"quant_method {method!r} is not supported (have 'awq', 'fp8', 'compressed-tensors')")


@dataclass(frozen=True)
class MoeCheckpointSpec:
    fmt: str
    hidden: int
    inter: int
    num_experts: int
    top_k: int
    routing: str  # "softmax_topk" | "topk_softmax" | "sigmoid_group"
    shared_inter: int  # 0: no shared expert
    n_group: int = 1
    topk_group: int = 1
    routed_scaling: float = 1.0


def moe_spec_from_config(config: dict) -> MoeCheckpointSpec:
    """MoE layer shape and routing of a ``config.json``."""
    tc = config.get("text_config", config)
    E = int(tc.get("num_experts") or tc.get("n_routed_experts") or 0)
    if E < 1:
        raise ValueError("config has no routed experts (num_experts / n_routed_experts)")
    I = int(tc.get("moe_intermediate_size", 0))
    if I < 1:
        raise ValueError("config has no moe_intermediate_size")
    shared = int(tc.get("moe_shared_expert_intermediate_size", 0) or tc.get("shared_expert_intermediate_size", 0))
    if not shared and int(tc.get("n_shared_experts", 0) or 0):
        shared = int(tc["n_shared_experts"]) * I
    scoring = str(tc.get("scoring_func", "softmax")).lower()
    norm = bool(tc.get("norm_topk_prob", False))
    if scoring == "sigmoid":
        if not norm:
            raise NotImplementedError("sigmoid scoring without norm_topk_prob is not supported")
        routing = "sigmoid_group"
    elif scoring == "softmax":
        routing = "topk_softmax" if norm else "softmax_topk"
        # DeepSeek-V2's group-limited greedy top-k and its routed scaling of softmax weights are
        # other routings (the softmax modes here take the top-k over all experts, weights as is)
        if str(tc.get("topk_method", "greedy")).lower() == "group_limited_greedy" and int(tc.get("n_group") or 1) > 1:
            raise NotImplementedError("group-limited greedy softmax routing (topk_method = group_limited_greedy)")
        if float(tc.get("routed_scaling_factor", 1.0) or 1.0) != 1.0:
            raise NotImplementedError("softmax routing with routed_scaling_factor != 1")
    else:
        raise NotImplementedError(f"scoring_func {scoring!r} is not supported")
    return MoeCheckpointSpec(
        fmt=quant_format(config), hidden=int(tc["hidden_size"]), inter=I, num_experts=E,
        top_k=int(tc.get("num_experts_per_tok", 1)), routing=routing, shared_inter=shared,
        n_group=int(tc.get("n_group", 1) or 1), topk_group=int(tc.get("topk_group", 1) or 1),
        routed_scaling=float(tc.get("routed_scaling_factor", 1.0) or 1.0),
    )


# ---------------------------------------------------------------- tensor names
@dataclass(frozen=True)
class NameTemplates:
    """Tensor-name templates of one model family ({layer}, {expert}, {proj} placeholders;
    {proj} is gate / up / down).  The defaults are the Hugging Face DeepSeek / Qwen MoE names."""

    expert: str = "model.layers.{layer}.mlp.experts.{expert}.{proj}_proj"
    router: str = "model.layers.{layer}.mlp.gate.weight"
    bias: str = "model.layers.{layer}.mlp.gate.e_score_correction_bias"
    shared: tuple[str, ...] = ("model.layers.{layer}.mlp.shared_experts.{proj}_proj",
                               "model.layers.{layer}.mlp.shared_expert.{proj}_proj")
    shared_gate: str = "model.layers.{layer}.mlp.shared_expert_gate.weight"


def expert_pattern(template: str) -> re.Pattern[str]:
    """Regex of an expert tensor-name template: ``{layer}`` and ``{expert}`` match digits,
    ``{proj}`` a lower-case word; the template is anchored at the start only, so that the
    ``.qweight`` / ``.weight`` / ``.weight_scale_inv`` suffix follows the match (the same
    placeholder convention as ``ccut/experts/index.py:parse_expert_pattern``)."""
    out, pos = [], 0
    for m in re.finditer(r"\{(layer|expert|proj)\}", template):
        out.append(re.escape(template[pos:m.start()]))
        out.append({"layer": r"(?P<layer>\d+)", "expert": r"(?P<expert>\d+)", "proj": r"(?P<proj>[a-z]+)"}[m.group(1)])
        pos = m.end()
    out.append(re.escape(template[pos:]))
    return re.compile("^" + "".join(out))


_SUFFIXES = {"awq_int4_g128": ("qweight", "qzeros", "scales"), "fp8_b128": ("weight", "weight_scale_inv"),
             "fp8_channel": ("weight", "weight_scale"), "int4_sym_g128": ("weight_packed", "weight_scale")}


def _read_compressed_tensors(reader: CheckpointReader, prefix: str, fmt: str) -> dict | None:
    """A compressed-tensors matrix in this path's tensors, or None when ``prefix`` has none:
    int4 ``weight_packed`` / ``weight_scale`` / ``weight_zero_point`` repacked into AWQ's
    (``quant.ct_int4_to_awq``); FP8 ``weight`` with its block scales under ``weight_scale``."""
    from ccut_b200.quant import ct_int4_to_awq, ct_int4_to_sym

    if fmt == "int4_sym_g128":
        if not reader.has(f"{prefix}.weight_packed"):
            return None
        if reader.has(f"{prefix}.weight_g_idx"):
            raise NotImplementedError(f"{prefix}: activation reordering (weight_g_idx) is not supported")
        if reader.has(f"{prefix}.weight_zero_point"):
            raise ValueError(f"{prefix}: a symmetric int4 matrix has no zero points")
        if reader.dtype(f"{prefix}.weight_packed") != "I32" or not reader.has(f"{prefix}.weight_scale"):
            raise ValueError(f"{prefix}: int4 tensors must be an I32 weight_packed with a weight_scale")
        shape = reader.tensor(f"{prefix}.weight_shape") if reader.has(f"{prefix}.weight_shape") else None
        return ct_int4_to_sym(reader.tensor(f"{prefix}.weight_packed"), _float_tensor(reader, f"{prefix}.weight_scale"),
                              shape)
    if fmt == "fp8_channel":
        if not reader.has(f"{prefix}.weight"):
            return None
        if reader.dtype(f"{prefix}.weight") != "F8_E4M3" or not reader.has(f"{prefix}.weight_scale"):
            raise ValueError(f"{prefix}: FP8 tensors must be an F8_E4M3 weight with a weight_scale")
        return {"weight": reader.tensor(f"{prefix}.weight"),
                "weight_scale": _float_tensor(reader, f"{prefix}.weight_scale").reshape(-1)}
    if fmt == "awq_int4_g128" and reader.has(f"{prefix}.weight_packed"):
        if reader.has(f"{prefix}.weight_g_idx"):
            raise NotImplementedError(f"{prefix}: activation reordering (weight_g_idx) is not supported")
        if reader.dtype(f"{prefix}.weight_packed") != "I32":
            raise ValueError(f"{prefix}: weight_packed must be I32")
        if not reader.has(f"{prefix}.weight_scale"):
            raise ValueError(f"{prefix}: missing scale tensor {prefix + '.weight_scale'!r}")
        zp = reader.tensor(f"{prefix}.weight_zero_point") if reader.has(f"{prefix}.weight_zero_point") else None
        shape = reader.tensor(f"{prefix}.weight_shape") if reader.has(f"{prefix}.weight_shape") else None
        return ct_int4_to_awq(reader.tensor(f"{prefix}.weight_packed"), _float_tensor(reader, f"{prefix}.weight_scale"),
                              zp, shape)
    if (fmt == "fp8_b128" and reader.has(f"{prefix}.weight") and reader.has(f"{prefix}.weight_scale")
            and not reader.has(f"{prefix}.weight_scale_inv")):
        if reader.dtype(f"{prefix}.weight") != "F8_E4M3":
            raise ValueError(f"{prefix}: FP8 tensors must be an F8_E4M3 weight")
        return {"weight": reader.tensor(f"{prefix}.weight"),
                "weight_scale_inv": _float_tensor(reader, f"{prefix}.weight_scale")}
    return None


def _has_matrix(reader: CheckpointReader, prefix: str, fmt: str) -> bool:
    """Whether ``prefix`` names a matrix in ``fmt`` (its own tensors or compressed-tensors')."""
    return reader.has(f"{prefix}.{_SUFFIXES[fmt][0]}") or (fmt == "awq_int4_g128"
                                                           and reader.has(f"{prefix}.weight_packed"))


def _read_matrix(reader: CheckpointReader, prefix: str, fmt: str) -> dict:
    ct = _read_compressed_tensors(reader, prefix, fmt)
    if ct is not None:
        return ct
    main = _SUFFIXES[fmt][0]
    if fmt in ("fp8_channel", "int4_sym_g128"):  # only compressed-tensors checkpoints store these
        raise KeyError(f"no tensor {prefix}.{main!s} in the checkpoint")
    if not reader.has(f"{prefix}.{main}"):
        raise KeyError(f"no tensor {prefix}.{main!s} in the checkpoint")
    out = {}
    for suf in _SUFFIXES[fmt]:
        name = f"{prefix}.{suf}"
        if not reader.has(name):
            raise ValueError(f"{prefix}: missing scale tensor {name!r}")
        out[suf] = reader.tensor(name)
    if fmt == "awq_int4_g128":
        if reader.dtype(f"{prefix}.qweight") != "I32" or reader.dtype(f"{prefix}.scales") not in ("F16",):
            raise ValueError(f"{prefix}: AWQ tensors must be I32 qweight/qzeros and F16 scales")
    else:
        if reader.dtype(f"{prefix}.weight") != "F8_E4M3" or reader.dtype(f"{prefix}.weight_scale_inv") != "F32":
            raise ValueError(f"{prefix}: FP8 tensors must be F8_E4M3 weight and F32 weight_scale_inv")
    return out


def _float_tensor(reader: CheckpointReader, name: str) -> np.ndarray:
    a, dt = reader.tensor(name), reader.dtype(name)
    if dt == "BF16":
        return (a.astype(np.uint32) << np.uint32(16)).view(np.float32)
    if dt in ("F32", "F16", "F64"):
        return a.astype(np.float32)
    raise ValueError(f"{name}: expected a float tensor, got {dt}")


def load_layer_weights(model_dir: str | Path, layer: int, names: NameTemplates | None = None):
    """Host-side view of one MoE layer of a checkpoint: ``(spec, router fp32 [E, H],
    experts [{gate, up, down}], shared [{gate, up, down}] or [], bias fp32 [E] or None)``.
    Matrices are dicts of the checkpoint's tensors (read-only mmap views)."""
    return _layer_weights(CheckpointReader(model_dir), layer, names or NameTemplates())


def _layer_weights(rd: CheckpointReader, layer: int, names: NameTemplates):
    spec = moe_spec_from_config(rd.config)
    rx = expert_pattern(names.expert)
    found: dict[int, set[str]] = {}
    for name in rd.weight_map:
        m = rx.match(name)
        if m and int(m.group("layer")) == layer:
            found.setdefault(int(m.group("expert")), set()).add(m.group("proj"))
    missing = [e for e in range(spec.num_experts) if found.get(e, set()) < {"gate", "up", "down"}]
    if missing:
        raise ValueError(f"layer {layer}: experts {missing[:8]}{'...' if len(missing) > 8 else ''} are missing "
                         f"gate/up/down tensors (template {names.expert!r})")
    extra = sorted(e for e in found if e >= spec.num_experts)
    if extra:
        raise ValueError(f"layer {layer}: expert ids {extra[:8]} beyond num_experts={spec.num_experts}")
    fmt = spec.fmt

    def matrices(template: str, **kw) -> dict:
        return {p: _read_matrix(rd, template.format(layer=layer, proj=p, **kw), fmt) for p in ("gate", "up", "down")}

    experts = [matrices(names.expert, expert=e) for e in range(spec.num_experts)]
    shared = []
    if spec.shared_inter:
        if rd.has(names.shared_gate.format(layer=layer)):
            raise NotImplementedError("a per-token shared-expert gate (shared_expert_gate) is not supported")
        for t in names.shared:
            if _has_matrix(rd, t.format(layer=layer, proj="gate"), fmt):
                shared = [matrices(t)]
                break
        else:
            raise KeyError(f"layer {layer}: config has a shared expert but no tensors match {names.shared}")
    router = _float_tensor(rd, names.router.format(layer=layer))
    if router.shape != (spec.num_experts, spec.hidden):
        raise ValueError(f"router {names.router.format(layer=layer)} has shape {router.shape}, "
                         f"expected {(spec.num_experts, spec.hidden)}")
    bname = names.bias.format(layer=layer)
    bias = _float_tensor(rd, bname) if rd.has(bname) else None
    return spec, router, experts, shared, bias


def load_moe_layer(model_dir: str | Path, layer: int, device="cuda", kernel: str = "auto",
                   names: NameTemplates | None = None):
    """``MoeLayer`` of a checkpoint's MoE layer ``layer``, experts packed into HBM."""
    from ccut_b200.layer import MoeLayer

    spec, router, experts, shared, bias = load_layer_weights(model_dir, layer, names)
    return MoeLayer(spec.fmt, spec.hidden, spec.inter, spec.num_experts, spec.top_k, spec.routing, router, experts,
                    shared=shared or None, shared_inter=spec.shared_inter or None, n_group=spec.n_group,
                    topk_group=spec.topk_group, routed_scaling=spec.routed_scaling, bias=bias, kernel=kernel,
                    device=device)


# ---------------------------------------------------------------- whole decoder
@dataclass(frozen=True)
class DecoderNames:
    """Tensor names of a decoder checkpoint (``{layer}``; ``{proj}`` is q / k / v / o for the
    attention projections, gate / up / down for a dense MLP).  The defaults are the Hugging
    Face Qwen / Llama / DeepSeek names."""

    embed: str = "model.embed_tokens.weight"
    final_norm: str = "model.norm.weight"
    lm_head: str = "lm_head.weight"
    input_norm: str = "model.layers.{layer}.input_layernorm.weight"
    post_norm: str = "model.layers.{layer}.post_attention_layernorm.weight"
    attn: str = "model.layers.{layer}.self_attn.{proj}_proj"
    q_norm: str = "model.layers.{layer}.self_attn.q_norm.weight"
    k_norm: str = "model.layers.{layer}.self_attn.k_norm.weight"
    mlp: str = "model.layers.{layer}.mlp.{proj}_proj"
    moe: NameTemplates = NameTemplates()
    # MLA layers (DeepSeek-V2 / V3): q / q_a / q_b / kv_b / o through ``attn``, and
    kv_a: str = "model.layers.{layer}.self_attn.kv_a_proj_with_mqa"
    kv_a_norm: str = "model.layers.{layer}.self_attn.kv_a_layernorm.weight"
    q_a_norm: str = "model.layers.{layer}.self_attn.q_a_layernorm.weight"


@dataclass(frozen=True)
class DecoderCheckpointSpec:
    fmt: str
    vocab: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    inter: int  # dense MLP intermediate size (0: none)
    eps: float
    rope_theta: float
    rope_scaling: dict | None
    tie_word_embeddings: bool
    softcap: float | None
    moe_layers: tuple  # per layer: True for a MoE block, False for a dense MLP
    mla: dict | None = None  # MLA sizes (``_mla_spec``) when the attention is multi-head latent attention


def _is_moe_layer(tc: dict, i: int) -> bool:
    """Whether layer ``i`` has a MoE block: the model has experts, ``i`` is not in
    ``mlp_only_layers``, ``i >= first_k_dense_replace``, ``(i + 1) % decoder_sparse_step == 0``
    and ``i % moe_layer_freq == 0`` (the Qwen-MoE and DeepSeek config keys; a model without
    them has a MoE block in every layer, as the reference's layer forward assumes,
    ``ccut/models/generic.py:440-446``)."""
    if not int(tc.get("num_experts") or tc.get("n_routed_experts") or 0):
        return False
    if i in [int(v) for v in (tc.get("mlp_only_layers") or [])]:
        return False
    if i < int(tc.get("first_k_dense_replace", 0) or 0):
        return False
    if (i + 1) % max(1, int(tc.get("decoder_sparse_step", 1) or 1)):
        return False
    return i % max(1, int(tc.get("moe_layer_freq", 1) or 1)) == 0


def _rope_scaling(tc: dict) -> dict | None:
    """``rope_scaling`` (or the newer ``rope_parameters``) with its kind under ``"type"``; None
    for plain RoPE."""
    rs = tc.get("rope_scaling") or tc.get("rope_parameters")
    if not rs:
        return None
    rs = dict(rs)
    kind = rs.get("type") or rs.get("rope_type")
    if kind in (None, "default"):
        return None
    rs["type"] = kind
    if kind == "yarn" and rs.get("factor") is None:  # the ratio of the context lengths (DeepSeek-V3 configs)
        rs["factor"] = float(tc["max_position_embeddings"]) / float(rs["original_max_position_embeddings"])
    return rs


def _mla_spec(tc: dict, rope_scaling: dict | None) -> dict:
    """The MLA sizes of a DeepSeek-V2 / V3 ``config.json`` and its softmax scale:
    ``(qk_nope_head_dim + qk_rope_head_dim) ** -0.5``, times ``yarn_mscale(factor,
    mscale_all_dim) ** 2`` under YaRN scaling with ``mscale_all_dim`` (the models' own attention
    code).  ``rope_interleave`` (default true): the checkpoint's rope features are stored as
    interleaved pairs."""
    from ccut_b200.rope_tables import yarn_mscale

    for key in ("qk_nope_head_dim", "qk_rope_head_dim", "v_head_dim"):
        if key not in tc:
            raise KeyError(f"config.json has no {key!r}")
    dn, dr, dv = int(tc["qk_nope_head_dim"]), int(tc["qk_rope_head_dim"]), int(tc["v_head_dim"])
    scale = (dn + dr) ** -0.5
    if rope_scaling and rope_scaling["type"] == "yarn" and rope_scaling.get("mscale_all_dim"):
        scale *= yarn_mscale(float(rope_scaling["factor"]), float(rope_scaling["mscale_all_dim"])) ** 2
    return {"kv_lora_rank": int(tc["kv_lora_rank"]), "q_lora_rank": int(tc.get("q_lora_rank") or 0),
            "qk_nope_head_dim": dn, "qk_rope_head_dim": dr, "v_head_dim": dv, "softmax_scale": float(scale),
            "rope_interleave": bool(tc.get("rope_interleave", True))}


def decoder_spec_from_config(config: dict) -> DecoderCheckpointSpec:
    """Decoder shape of a ``config.json`` (the keys ``ccut/models/spec.py:parse_model_spec``
    reads, plus the MLA keys of DeepSeek-V2 / V3: ``kv_lora_rank``, ``q_lora_rank``,
    ``qk_nope_head_dim``, ``qk_rope_head_dim``, ``v_head_dim``).  For MLA models ``head_dim`` is
    the rope dimension (the size of the RoPE table).  Linear-attention layers raise
    ``NotImplementedError``."""
    tc = config.get("text_config", config)
    if tc.get("linear_num_key_heads") or int(tc.get("full_attention_interval", 0) or 0) > 1:
        raise NotImplementedError("linear-attention layers are not supported by the decoder")
    for key in ("hidden_size", "num_hidden_layers", "num_attention_heads", "vocab_size"):
        if key not in tc:
            raise KeyError(f"config.json has no {key!r}")
    hidden, heads = int(tc["hidden_size"]), int(tc["num_attention_heads"])
    L = int(tc["num_hidden_layers"])
    cap = tc.get("attn_logit_softcapping")
    rs = _rope_scaling(tc)
    mla = _mla_spec(tc, rs) if tc.get("kv_lora_rank") else None
    theta = tc.get("rope_theta") or (tc.get("rope_parameters") or {}).get("rope_theta") or 10000.0
    return DecoderCheckpointSpec(
        fmt=quant_format(config), vocab=int(tc["vocab_size"]), hidden=hidden, layers=L, heads=heads,
        kv_heads=1 if mla else int(tc.get("num_key_value_heads", heads)),
        head_dim=mla["qk_rope_head_dim"] if mla else int(tc.get("head_dim") or hidden // heads),
        inter=int(tc.get("intermediate_size", 0) or 0), eps=float(tc.get("rms_norm_eps", 1e-6)),
        rope_theta=float(theta), rope_scaling=rs,
        tie_word_embeddings=bool(tc.get("tie_word_embeddings", False)), softcap=float(cap) if cap else None,
        moe_layers=tuple(_is_moe_layer(tc, i) for i in range(L)), mla=mla,
    )


def _rope_perm(width: int, offsets, d_rope: int) -> np.ndarray:
    """Output-channel order that turns interleaved rope pairs ``(2i, 2i + 1)`` into the half
    layout ``(i, i + d_rope / 2)`` that RoPE here rotates, for the ``d_rope`` channels starting
    at each of ``offsets`` (the other channels stay).  Scores are unchanged: q and k are permuted
    alike."""
    perm = np.arange(width, dtype=np.int64)
    half = np.concatenate([np.arange(0, d_rope, 2), np.arange(1, d_rope, 2)])
    for off in offsets:
        perm[off: off + d_rope] = off + half
    return perm


def _permute_rows(m, fmt: str, perm: np.ndarray):
    """A ``_dense_or_quant`` matrix with its output channels in ``perm`` order."""
    from ccut_b200.quant import permute_out_channels

    kind, a = m
    if kind == "dense":
        return "dense", np.ascontiguousarray(a[perm])
    return "quant", permute_out_channels(fmt, a, perm)


def _mla_attention(rd: CheckpointReader, spec: DecoderCheckpointSpec, names: DecoderNames, i: int) -> dict:
    """One MLA layer's attention tensors: ``q`` (or ``q_a`` / ``q_a_norm`` / ``q_b``),
    ``kv_a``, ``kv_a_norm`` (or None), ``kv_b``, ``o``; with ``rope_interleave`` the rope
    channels of q and of ``kv_a`` are reordered into the half layout."""
    m, H, nh = spec.mla, spec.hidden, spec.heads
    dn, dr, dv, R, qr = (m["qk_nope_head_dim"], m["qk_rope_head_dim"], m["v_head_dim"], m["kv_lora_rank"],
                         m["q_lora_rank"])
    attn = names.attn.format
    out = {}
    q_out = nh * (dn + dr)
    if qr:
        out["q_a"] = _dense_or_quant(rd, attn(layer=i, proj="q_a"), spec.fmt, qr, H)
        out["q_a_norm"] = _vector(rd, names.q_a_norm.format(layer=i), qr)
        q = _dense_or_quant(rd, attn(layer=i, proj="q_b"), spec.fmt, q_out, qr)
    else:
        q = _dense_or_quant(rd, attn(layer=i, proj="q"), spec.fmt, q_out, H)
    kv_a = _dense_or_quant(rd, names.kv_a.format(layer=i), spec.fmt, R + dr, H)
    if m["rope_interleave"]:
        q = _permute_rows(q, spec.fmt, _rope_perm(q_out, [h * (dn + dr) + dn for h in range(nh)], dr))
        kv_a = _permute_rows(kv_a, spec.fmt, _rope_perm(R + dr, [R], dr))
    out["q"], out["kv_a"] = q, kv_a
    name = names.kv_a_norm.format(layer=i)
    out["kv_a_norm"] = _vector(rd, name, R) if rd.has(name) else None
    out["kv_b"] = _dense_or_quant(rd, attn(layer=i, proj="kv_b"), spec.fmt, nh * (dn + dv), R)
    out["o"] = _dense_or_quant(rd, attn(layer=i, proj="o"), spec.fmt, H, nh * dv)
    return out


def _dense_or_quant(rd: CheckpointReader, prefix: str, fmt: str, out_dim: int, in_dim: int):
    """``("dense", fp32 [out, in])`` for a float ``<prefix>.weight``, else ``("quant", tensors)``
    in the checkpoint's format."""
    name = f"{prefix}.weight"
    if rd.has(name) and rd.dtype(name) in ("BF16", "F16", "F32"):
        a = _float_tensor(rd, name)
        if a.shape != (out_dim, in_dim):
            raise ValueError(f"{name} has shape {a.shape}, expected {(out_dim, in_dim)}")
        return "dense", a
    m = _read_matrix(rd, prefix, fmt)
    shape = m["qweight"].shape if "qweight" in m else m["weight"].shape
    want = (in_dim, out_dim // 8) if "qweight" in m else (out_dim, in_dim)
    if shape != want:
        raise ValueError(f"{prefix} has shape {shape}, expected {want}")
    return "quant", m


def _vector(rd: CheckpointReader, name: str, n: int) -> np.ndarray:
    if not rd.has(name):
        raise KeyError(f"no tensor {name!r} in the checkpoint")
    a = _float_tensor(rd, name).reshape(-1)
    if a.size != n:
        raise ValueError(f"{name} has {a.size} elements, expected {n}")
    return a


def load_decoder_weights(model_dir: str | Path, names: DecoderNames | None = None) -> dict:
    """Host-side view of a decoder checkpoint: ``{"spec", "embed", "lm_head", "final_norm",
    "layers"}``; each layer a dict with ``ln1``, ``ln2``, ``q`` / ``k`` / ``v`` / ``o``
    (``("dense", [out, in])`` or ``("quant", tensors)``), ``q_norm`` / ``k_norm`` (or None) and
    ``ffn``: ``("moe", load_layer_weights(...))`` or ``("dense", {gate, up, down})``.  An MLA
    layer has ``q`` (or ``q_a`` / ``q_a_norm`` / ``q_b`` in ``q``), ``kv_a``, ``kv_a_norm``,
    ``kv_b`` and ``o`` instead (``_mla_attention``).  Float tensors are fp32 copies, quantized
    ones read-only views (copies where rope channels were reordered)."""
    names = names or DecoderNames()
    rd = CheckpointReader(model_dir)
    spec = decoder_spec_from_config(rd.config)
    H, d = spec.hidden, spec.head_dim
    embed = _float_tensor(rd, names.embed)
    if embed.shape != (spec.vocab, H):
        raise ValueError(f"{names.embed} has shape {embed.shape}, expected {(spec.vocab, H)}")
    if rd.has(names.lm_head):
        lm_head = _float_tensor(rd, names.lm_head)
        if lm_head.shape != (spec.vocab, H):
            raise ValueError(f"{names.lm_head} has shape {lm_head.shape}, expected {(spec.vocab, H)}")
    elif spec.tie_word_embeddings:
        lm_head = embed
    else:
        raise KeyError(f"no tensor {names.lm_head!r} and tie_word_embeddings is false")
    dims = {"q": (spec.heads * d, H), "k": (spec.kv_heads * d, H), "v": (spec.kv_heads * d, H),
            "o": (H, spec.heads * d)}
    layers = []
    for i in range(spec.layers):
        lay = {"ln1": _vector(rd, names.input_norm.format(layer=i), H),
               "ln2": _vector(rd, names.post_norm.format(layer=i), H)}
        if spec.mla:
            lay.update(_mla_attention(rd, spec, names, i))
        else:
            for p, (o, n) in dims.items():
                lay[p] = _dense_or_quant(rd, names.attn.format(layer=i, proj=p), spec.fmt, o, n)
            for p, n in (("q_norm", spec.heads), ("k_norm", spec.kv_heads)):
                name = getattr(names, p).format(layer=i)
                w = _float_tensor(rd, name).reshape(-1) if rd.has(name) else None
                if w is not None and w.size not in (d, n * d):
                    raise ValueError(f"{name} has {w.size} elements, expected {d} or {n * d}")
                lay[p] = w
        if spec.moe_layers[i]:
            lay["ffn"] = ("moe", _layer_weights(rd, i, names.moe))
        else:
            if spec.inter < 1:
                raise ValueError(f"layer {i} has a dense MLP but config.json has no intermediate_size")
            lay["ffn"] = ("dense", {p: _read_matrix(rd, names.mlp.format(layer=i, proj=p), spec.fmt)
                                    for p in ("gate", "up", "down")})
        layers.append(lay)
    final_norm = _vector(rd, names.final_norm, H)
    return {"spec": spec, "embed": embed, "lm_head": lm_head, "final_norm": final_norm, "layers": layers}


def load_decoder(model_dir: str | Path, device="cuda", kernel: str = "auto", names: DecoderNames | None = None,
                 quantized_projections: bool = True, app_config=None):
    """``MoeDecoder`` of a whole checkpoint: every layer's MoE experts packed into HBM
    (``MoeLayer``) or its dense MLP (``DenseFfn``).  Quantized attention projections stay in
    their format (``quant.QuantLinear``, run by ``ccut_quant_linear``), or with
    ``quantized_projections=False`` are dequantized on the device (``quant.dequantize``) and
    kept as bf16 for cuBLAS.  RoPE from ``rope_theta`` / ``rope_scaling``: the reference's
    ``build_rope`` table (``rope_table``: none, linear, dynamic, its own yarn), whose attention
    factor the reference's layer does not apply, and neither does this decoder.  ``app_config``: the engine's config (``[experts]`` / ``[quant]``,
    ``ccut_b200.config``), checked against the checkpoint before anything is uploaded.

    MLA checkpoints (DeepSeek-V2 / V3) give ``MlaDecoderLayer`` layers: ``kv_a_proj_with_mqa``
    (576 outputs, not a multiple of the 128 the quantized-projection kernel tiles by) and
    ``kv_b_proj`` (whose per-head blocks the layer keeps) are dequantized on the device, the
    first padded with zero channels to a multiple of 128 for the export; RoPE from YaRN
    (``yarn_rope_table``) with its factor applied to ``q_pe`` squared (the models scale both
    ``cos`` and ``sin``, so the scores carry the factor twice)."""
    import torch

    from ccut_b200.dense import DenseFfn
    from ccut_b200.layer import MoeLayer
    from ccut_b200.model import DecoderLayer, MlaDecoderLayer, MoeDecoder, rope_table, yarn_rope_table
    from ccut_b200.quant import QuantLinear, dequantize, pad_out_channels

    if app_config is not None:  # the engine's [experts] / [quant] settings, checked before any upload
        from ccut_b200.config import resolve

        resolve(app_config, CheckpointReader(model_dir).config)
    w = load_decoder_weights(model_dir, names)
    spec = w["spec"]
    scaling_type = "none"
    if spec.mla and spec.rope_scaling and spec.rope_scaling["type"] == "yarn":
        inv_freq, f = yarn_rope_table(spec.head_dim, spec.rope_theta, spec.rope_scaling)
        attn_factor, scaling_type = f * f, "yarn"
    else:
        inv_freq, attn_factor = rope_table(spec.head_dim, spec.rope_theta, spec.rope_scaling)

    def dense(m, out_dim: int, in_dim: int, keep_quant: bool | None = None, dtype=torch.bfloat16):
        kind, a = m
        if kind == "dense":
            return torch.from_numpy(np.ascontiguousarray(a)).to(device=device, dtype=dtype)
        keep = quantized_projections if keep_quant is None else keep_quant
        if keep and out_dim % 128 == 0 and in_dim % 128 == 0:
            return QuantLinear(spec.fmt, a, in_dim, out_dim, device)
        padded = -(-out_dim // 128) * 128
        if padded != out_dim:
            a = pad_out_channels(spec.fmt, a, padded)
        main = "qweight" if "qweight" in a else _SUFFIXES[spec.fmt][0]
        t = dequantize(spec.fmt, a[main], {k: v for k, v in a.items() if k != main}, in_dim, padded, device)
        return t[:out_dim].to(dtype).contiguous()

    H, d = spec.hidden, spec.head_dim
    dims = {"q": (spec.heads * d, H), "k": (spec.kv_heads * d, H), "v": (spec.kv_heads * d, H),
            "o": (H, spec.heads * d)}
    layers = []
    ws: dict = {}  # the layers run one after another: one set of FFN workspaces for all of them
    for lay in w["layers"]:
        kind, f = lay["ffn"]
        if kind == "moe":
            ms, router, experts, shared, bias = f
            ffn = MoeLayer(ms.fmt, ms.hidden, ms.inter, ms.num_experts, ms.top_k, ms.routing, router, experts,
                           shared=shared or None, shared_inter=ms.shared_inter or None, n_group=ms.n_group,
                           topk_group=ms.topk_group, routed_scaling=ms.routed_scaling, bias=bias, kernel=kernel,
                           device=device, workspaces=ws)
        else:
            ffn = DenseFfn(spec.fmt, H, spec.inter, f["gate"], f["up"], f["down"], kernel=kernel, device=device,
                           workspaces=ws)
        if spec.mla:
            m, nh = spec.mla, spec.heads
            dn, dr, dv, R, qr = (m["qk_nope_head_dim"], m["qk_rope_head_dim"], m["v_head_dim"], m["kv_lora_rank"],
                                 m["q_lora_rank"])
            q = dense(lay["q"], nh * (dn + dr), qr or H)
            q_a = dense(lay["q_a"], qr, H) if qr else None
            kv_a = dense(lay["kv_a"], R + dr, H, keep_quant=False)
            kv_b = dense(lay["kv_b"], nh * (dn + dv), R, keep_quant=False, dtype=torch.float32)
            o = dense(lay["o"], H, nh * dv)
            layers.append(MlaDecoderLayer(lay["ln1"], q, kv_a, kv_b, o, lay["ln2"], ffn, lay["kv_a_norm"], heads=nh,
                                          qk_nope_head_dim=dn, qk_rope_head_dim=dr, v_head_dim=dv, kv_lora_rank=R,
                                          q_a=q_a, q_a_norm=lay.get("q_a_norm"), softmax_scale=m["softmax_scale"],
                                          device=device))
            continue
        q, k, v, o = (dense(lay[p], *dims[p]) for p in "qkvo")
        layers.append(DecoderLayer(lay["ln1"], q, k, v, o, lay["ln2"], ffn, lay["q_norm"], lay["k_norm"],
                                   heads=spec.heads, kv_heads=spec.kv_heads, head_dim=d, device=device))
    return MoeDecoder(w["embed"], layers, w["final_norm"], w["lm_head"], inv_freq=inv_freq,
                      attention_factor=attn_factor, scaling_type=scaling_type, eps=spec.eps, softcap=spec.softcap,
                      device=device)
