"""Writes small safetensors checkpoints of the seeded synthetic layers (test fixtures).

A checkpoint is a model directory with ``config.json`` (Hugging Face DeepSeek-style MoE
keys and a ``quantization_config``), two shards and ``model.safetensors.index.json``,
holding one MoE layer at index ``layer``: router, routed experts and the shared experts
merged into one MLP along the intermediate axis (as DeepSeek stores ``shared_experts``).
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from oracle import formats, inputs

_DT = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int32): "I32",
       np.dtype(np.uint8): "U8", np.dtype(np.uint16): "U16", np.dtype(np.int64): "I64"}


def write_safetensors(path: Path, tensors: dict[str, tuple[str | None, np.ndarray]], metadata=None) -> None:
    """tensors: name -> (safetensors dtype or None for the array's own, array)."""
    header, blobs, off = {}, [], 0
    for name, (dt, a) in tensors.items():
        a = np.ascontiguousarray(a)
        b = a.tobytes()
        header[name] = {"dtype": dt or _DT[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    raw = json.dumps(header).encode()
    raw += b" " * (-len(raw) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(raw)))
        fh.write(raw)
        for b in blobs:
            fh.write(b)


def _matrix_tensors(prefix: str, m) -> dict:
    if isinstance(m, inputs.AwqMatrix):
        return {f"{prefix}.qweight": (None, m.qweight), f"{prefix}.qzeros": (None, m.qzeros),
                f"{prefix}.scales": (None, m.scales)}
    return {f"{prefix}.weight": ("F8_E4M3", m.weight), f"{prefix}.weight_scale_inv": (None, m.scale)}


def _pack_sequential(cols: np.ndarray) -> np.ndarray:
    """uint8 nibbles [R, 8 C] -> int32 [R, C], nibble i of a word in bits 4i .. 4i + 3."""
    c = cols.reshape(cols.shape[0], -1, 8).astype(np.uint32)
    w = np.zeros(c.shape[:2], np.uint32)
    for i in range(8):
        w |= c[..., i] << np.uint32(4 * i)
    return w.view(np.int32)


def ct_quant_config(fmt: str) -> dict:
    """A compressed-tensors ``quantization_config`` for ``fmt``: int4 group 128 weights
    (``pack-quantized``, asymmetric for AWQ, symmetric for ``int4_sym_g128``), FP8 128 x 128
    block weights with dynamic activations, or per-channel FP8 weights with per-token dynamic
    activations (the reference's own checkpoints, ``ccut/quant/compressed_tensors.py:3-10``)."""
    if fmt == "int4_sym_g128":
        w = {"num_bits": 4, "type": "int", "symmetric": True, "strategy": "group", "group_size": 128,
             "actorder": None}
        return {"quant_method": "compressed-tensors", "format": "pack-quantized",
                "config_groups": {"group_0": {"targets": ["Linear"], "weights": w, "input_activations": None}},
                "ignore": ["lm_head", "re:.*mlp.gate$"]}
    if fmt == "fp8_channel":
        w = {"num_bits": 8, "type": "float", "symmetric": True, "strategy": "channel", "dynamic": False}
        a = {"num_bits": 8, "type": "float", "symmetric": True, "strategy": "token", "dynamic": True}
        return {"quant_method": "compressed-tensors", "format": "float-quantized",
                "config_groups": {"group_0": {"targets": ["Linear"], "weights": w, "input_activations": a}},
                "ignore": ["lm_head", "re:.*mlp.gate$"]}
    if fmt == "awq_int4_g128":
        w = {"num_bits": 4, "type": "int", "symmetric": False, "strategy": "group", "group_size": 128,
             "actorder": None}
        return {"quant_method": "compressed-tensors", "format": "pack-quantized",
                "config_groups": {"group_0": {"targets": ["Linear"], "weights": w, "input_activations": None}},
                "ignore": ["lm_head", "re:.*mlp.gate$"]}
    w = {"num_bits": 8, "type": "float", "symmetric": True, "strategy": "block", "block_structure": [128, 128]}
    a = {"num_bits": 8, "type": "float", "symmetric": True, "strategy": "group", "group_size": 128, "dynamic": True}
    return {"quant_method": "compressed-tensors", "format": "float-quantized",
            "config_groups": {"group_0": {"targets": ["Linear"], "weights": w, "input_activations": a}},
            "ignore": ["lm_head", "re:.*mlp.gate$"]}


def _ct_matrix_tensors(prefix: str, m) -> dict:
    """One matrix in compressed-tensors form with the same values: AWQ ``(q - z) * s`` as
    ``weight_packed`` (q along K, 8 per word), ``weight_zero_point`` (z along N),
    ``weight_scale`` fp16 [N, K / 128], ``weight_shape``; FP8 as ``weight`` + ``weight_scale``."""
    if isinstance(m, inputs.AwqMatrix):
        q = formats.awq_unpack(m.qweight)  # [K, N]
        z = formats.awq_unpack(m.qzeros)  # [K / 128, N]
        K, N = q.shape
        return {f"{prefix}.weight_packed": (None, _pack_sequential(np.ascontiguousarray(q.T))),
                f"{prefix}.weight_zero_point": (None, np.ascontiguousarray(_pack_sequential(z).T)),
                f"{prefix}.weight_scale": (None, np.ascontiguousarray(m.scales.T)),
                f"{prefix}.weight_shape": (None, np.array([N, K], np.int64))}
    if isinstance(m, inputs.Fp8ChannelMatrix):
        return {f"{prefix}.weight": ("F8_E4M3", m.weight), f"{prefix}.weight_scale": (None, m.scale.reshape(-1, 1))}
    if isinstance(m, inputs.Int4SymMatrix):  # signed v as v + 8, 8 per word along K; group scales [N, K/128]
        v8 = formats.int4_sym_unpack(m.weight).astype(np.int16) + 8  # [N, K]
        N, K = v8.shape
        return {f"{prefix}.weight_packed": (None, _pack_sequential(v8.astype(np.uint8))),
                f"{prefix}.weight_scale": (None, np.ascontiguousarray(np.repeat(m.scale[None, ::128], N, axis=0))),
                f"{prefix}.weight_shape": (None, np.array([N, K], np.int64))}
    return {f"{prefix}.weight": ("F8_E4M3", m.weight), f"{prefix}.weight_scale": (None, m.scale)}


def merged_shared(lw):
    """The layer's shared experts as one MLP (intermediate axis concatenated)."""
    if not lw.shared:
        return None
    out = {}
    for proj in ("gate", "up", "down"):
        mats = [getattr(s, proj) for s in lw.shared]
        if isinstance(mats[0], (inputs.Fp8ChannelMatrix, inputs.Int4SymMatrix)):
            if len(mats) != 1:  # per-channel / per-column scales do not survive a merge along K
                raise NotImplementedError("one shared expert for the per-channel formats")
            out[proj] = mats[0]
        elif isinstance(mats[0], inputs.AwqMatrix):  # [in, out]: gate/up cat along out, down along in
            ax = 1 if proj != "down" else 0
            out[proj] = inputs.AwqMatrix(*(np.concatenate([getattr(m, f) for m in mats], axis=ax)
                                           for f in ("qweight", "qzeros", "scales")))
        else:  # [out, in]
            ax = 0 if proj != "down" else 1
            out[proj] = inputs.Fp8Matrix(*(np.concatenate([getattr(m, f) for m in mats], axis=ax)
                                           for f in ("weight", "scale")))
    return out


def write_checkpoint(root: Path, lw, layer: int = 3, router_bf16: bool = False, quant: dict | None = None,
                     drop: tuple[str, ...] = (), extra_config: dict | None = None, ct: bool = False) -> Path:
    """One MoE layer of ``lw`` as a two-shard checkpoint; ``ct``: in compressed-tensors form."""
    c = lw.cfg
    root.mkdir(parents=True, exist_ok=True)
    mt = _ct_matrix_tensors if ct else _matrix_tensors
    if ct and quant is None:
        quant = ct_quant_config(c.fmt)
    q = quant or ({"quant_method": "awq", "bits": 4, "group_size": 128, "zero_point": True, "version": "gemm"}
                  if c.fmt == "awq_int4_g128" else
                  {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128],
                   "activation_scheme": "dynamic"})
    cfg = {"architectures": ["DeepseekV2ForCausalLM"], "hidden_size": c.hidden, "moe_intermediate_size": c.inter,
           "n_routed_experts": c.num_experts, "num_experts_per_tok": c.top_k,
           "n_shared_experts": c.num_shared * c.shared_inter // c.inter if c.num_shared else 0,
           "norm_topk_prob": c.routing == "topk_softmax", "scoring_func": "softmax",
           "quantization_config": q}
    cfg.update(extra_config or {})
    (root / "config.json").write_text(json.dumps(cfg))
    pre = f"model.layers.{layer}.mlp"
    t1, t2 = {}, {}
    r = lw.router.astype(np.float32)
    if router_bf16:
        t1[f"{pre}.gate.weight"] = ("BF16", inputs.synthetic.bf16_bits_from_f32(r))
    else:
        t1[f"{pre}.gate.weight"] = (None, r)
    t1["model.embed_tokens.weight"] = (None, np.zeros((4, c.hidden), np.float32))  # an unrelated tensor
    for e, ew in enumerate(lw.experts):
        dst = t1 if e < c.num_experts // 2 else t2
        for proj in ("gate", "up", "down"):
            dst.update(mt(f"{pre}.experts.{e}.{proj}_proj", getattr(ew, proj)))
    sh = merged_shared(lw)
    if sh:
        for proj in ("gate", "up", "down"):
            t2.update(mt(f"{pre}.shared_experts.{proj}_proj", sh[proj]))
    for name in drop:
        t1.pop(name, None)
        t2.pop(name, None)
    write_safetensors(root / "model-00001-of-00002.safetensors", t1, {"format": "pt"})
    write_safetensors(root / "model-00002-of-00002.safetensors", t2)
    wm = {n: "model-00001-of-00002.safetensors" for n in t1} | {n: "model-00002-of-00002.safetensors" for n in t2}
    (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    return root


def write_decoder_checkpoint(root: Path, tiny, fmt: str, qlayers: list, attn_mats: list | None = None,
                             dense: dict | None = None, dense_inter: int = 0, tie: bool = False,
                             drop: tuple[str, ...] = (), extra_config: dict | None = None) -> Path:
    """A Qwen-MoE style decoder checkpoint of a ``tests.model_helpers`` tiny model: BF16
    embedding, norms and ``lm_head``; attention projections BF16 from ``tiny.attn`` or the
    quantized ``attn_mats``; per layer the MoE block of ``qlayers[i]`` (F32 router, experts,
    the shared expert under ``shared_experts``), or for the layers of ``dense`` (layer ->
    ``ExpertWeights`` with intermediate size ``dense_inter``) a dense MLP listed in
    ``mlp_only_layers``."""
    root.mkdir(parents=True, exist_ok=True)
    bf = inputs.synthetic.bf16_bits_from_f32
    dense = dense or {}
    c0 = qlayers[0].cfg
    q = ({"quant_method": "awq", "bits": 4, "group_size": 128, "zero_point": True, "version": "gemm"}
         if fmt == "awq_int4_g128" else
         {"quant_method": "fp8", "fmt": "e4m3", "weight_block_size": [128, 128], "activation_scheme": "dynamic"})
    cfg = {"architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe", "hidden_size": tiny.hidden,
           "num_hidden_layers": tiny.layers, "num_attention_heads": tiny.heads,
           "num_key_value_heads": tiny.kv_heads, "head_dim": tiny.head_dim, "vocab_size": tiny.vocab,
           "rms_norm_eps": tiny.eps, "rope_theta": tiny.theta, "rope_scaling": None, "tie_word_embeddings": tie,
           "num_experts": c0.num_experts, "num_experts_per_tok": c0.top_k, "moe_intermediate_size": c0.inter,
           "norm_topk_prob": c0.routing == "topk_softmax", "n_shared_experts": c0.num_shared,
           "decoder_sparse_step": 1, "mlp_only_layers": sorted(dense), "intermediate_size": dense_inter,
           "quantization_config": q}
    cfg.update(extra_config or {})
    (root / "config.json").write_text(json.dumps(cfg))
    t = {"model.embed_tokens.weight": ("BF16", bf(tiny.embed)), "model.norm.weight": ("BF16", bf(tiny.final_norm))}
    if not tie:
        t["lm_head.weight"] = ("BF16", bf(tiny.lm_head))
    for i, w in enumerate(tiny.attn):
        pre = f"model.layers.{i}"
        t[f"{pre}.input_layernorm.weight"] = ("BF16", bf(w.ln1))
        t[f"{pre}.post_attention_layernorm.weight"] = ("BF16", bf(w.ln2))
        for p, m in zip("qkvo", (w.wq, w.wk, w.wv, w.wo)):
            if attn_mats is None:
                t[f"{pre}.self_attn.{p}_proj.weight"] = ("BF16", bf(m))
            else:
                t.update(_matrix_tensors(f"{pre}.self_attn.{p}_proj", attn_mats[i][p]))
        if w.q_norm is not None:
            t[f"{pre}.self_attn.q_norm.weight"] = ("BF16", bf(w.q_norm))
            t[f"{pre}.self_attn.k_norm.weight"] = ("BF16", bf(w.k_norm))
        if i in dense:
            for proj in ("gate", "up", "down"):
                t.update(_matrix_tensors(f"{pre}.mlp.{proj}_proj", getattr(dense[i], proj)))
            continue
        lw = qlayers[i]
        t[f"{pre}.mlp.gate.weight"] = (None, lw.router.astype(np.float32))
        for e, ew in enumerate(lw.experts):
            for proj in ("gate", "up", "down"):
                t.update(_matrix_tensors(f"{pre}.mlp.experts.{e}.{proj}_proj", getattr(ew, proj)))
        sh = merged_shared(lw.lw if hasattr(lw, "lw") else lw)
        if sh:
            for proj in ("gate", "up", "down"):
                t.update(_matrix_tensors(f"{pre}.mlp.shared_experts.{proj}_proj", sh[proj]))
    for name in drop:
        t.pop(name, None)
    write_safetensors(root / "model.safetensors", t, {"format": "pt"})
    return root
