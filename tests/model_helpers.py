"""Seeded tiny decoder models for the engine-wiring tests (test fixtures).

``make_tiny(seed, ...)`` draws from ``numpy.random.default_rng(seed)``, in this order: the
embedding; per layer the attention weights (``oracle.model.AttnWeights``, or with ``mla`` the
latent-attention weights ``oracle.model.MlaWeights``), a router and the
dense experts of a MoE block (``[in, out]`` like ``expert_ffn`` takes them) plus one shared
expert; then the final norm and ``lm_head``.  Every matrix is bf16-representable (fp32
draws rounded to bf16), the router stays fp32.  The GPU kernels take quantized experts, so
``quantized_layers`` draws a seeded AWQ or FP8 MoE layer of the same shape per decoder
layer (``ccut_b200.synthetic``) for the tests that run them.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from oracle import inputs, model
from oracle.model import AttnWeights, DecoderSpec, MlaWeights


def _bf16(a: np.ndarray) -> np.ndarray:
    return model.round_bf16(np.asarray(a, np.float32))


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    return (1.0 / theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)).astype(np.float32)


@dataclass
class TinyModel:
    vocab: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    num_experts: int
    top_k: int
    inter: int
    shared_inter: int
    norm_topk_prob: bool
    theta: float
    eps: float
    embed: np.ndarray = field(repr=False)
    lm_head: np.ndarray = field(repr=False)
    final_norm: np.ndarray = field(repr=False)
    attn: list = field(repr=False)
    router: list = field(repr=False)
    experts: list = field(repr=False)  # [layer][expert] = (wg [H, I], wu [H, I], wd [I, H])
    shared: list = field(repr=False)  # [layer] = (sg, su, sd) or None
    mla: dict | None = None  # the MLA sizes, when the layers are MLA layers

    @property
    def layers(self) -> int:
        return len(self.attn)

    @property
    def mode(self) -> str:
        return "topk_softmax" if self.norm_topk_prob else "softmax_topk"

    @property
    def rope_dim(self) -> int:
        return self.mla["d_rope"] if self.mla else self.head_dim

    def spec(self, inv_freq: np.ndarray | None = None) -> DecoderSpec:
        f = rope_inv_freq(self.rope_dim, self.theta) if inv_freq is None else np.asarray(inv_freq, np.float32)
        return DecoderSpec(self.hidden, self.heads, self.kv_heads, self.head_dim, f, eps=self.eps)

    def dense_ffns(self) -> list:
        return [model.moe_ffn(self.router[i], self.top_k, self.mode, (lambda e, i=i: self.experts[i][e]),
                              self.shared[i]) for i in range(self.layers)]


def make_tiny(seed: int = 0, vocab: int = 512, hidden: int = 256, heads: int = 4, kv_heads: int = 1,
              head_dim: int = 64, layers: int = 2, num_experts: int = 8, top_k: int = 2, inter: int = 128,
              shared_inter: int = 128, norm_topk_prob: bool = False, qk_norm: str | None = "flat",
              theta: float = 10000.0, eps: float = 1e-6, mla: dict | None = None) -> TinyModel:
    """qk_norm: None, ``"flat"`` (weights over the whole q / k projection) or ``"head"``.
    ``mla``: MLA layers instead, ``{"rank", "d_nope", "d_rope", "d_v"}`` and optionally
    ``"q_rank"`` (a q_a / q_b pair) and ``"kv_norm"`` (False: no ``kv_a_layernorm``)."""
    rng = np.random.default_rng(seed)
    H, d = hidden, head_dim

    def mat(out_dim: int, in_dim: int) -> np.ndarray:
        return _bf16(rng.standard_normal((out_dim, in_dim), dtype=np.float32) / np.float32(np.sqrt(in_dim)))

    def norm_w(n: int) -> np.ndarray:
        return _bf16(rng.uniform(0.5, 1.5, n).astype(np.float32))

    embed = _bf16(rng.standard_normal((vocab, H), dtype=np.float32))
    attn, router, experts, shared = [], [], [], []
    for _ in range(layers):
        ln1 = norm_w(H)
        if mla:
            R, dn, dr, dv = mla["rank"], mla["d_nope"], mla["d_rope"], mla["d_v"]
            qr = mla.get("q_rank")
            wq_a = mat(qr, H) if qr else None
            q_a_norm = norm_w(qr) if qr else None
            wq = mat(heads * (dn + dr), qr or H)
            wkv_a = mat(R + dr, H)
            kv_norm = norm_w(R) if mla.get("kv_norm", True) else None
            wkv_b = mat(heads * (dn + dv), R)
            wo = mat(H, heads * dv)
            ln2 = norm_w(H)
            attn.append(MlaWeights(ln1, wq, wkv_a, wkv_b, wo, ln2, heads, dn, dr, dv, kv_norm, wq_a, q_a_norm,
                                   mla.get("scale")))
        else:
            wq, wk, wv = mat(heads * d, H), mat(kv_heads * d, H), mat(kv_heads * d, H)
            wo = mat(H, heads * d)
            ln2 = norm_w(H)
            qn = kn = None
            if qk_norm == "flat":
                qn, kn = norm_w(heads * d), norm_w(kv_heads * d)
            elif qk_norm == "head":
                qn, kn = norm_w(d), norm_w(d)
            attn.append(AttnWeights(ln1, wq, wk, wv, wo, ln2, qn, kn))
        router.append((rng.standard_normal((num_experts, H), dtype=np.float32) * np.float32(0.1)).astype(np.float32))
        # [in, out]: gate / up [H, I], down [I, H]
        experts.append([(mat(inter, H).T.copy(), mat(inter, H).T.copy(), mat(H, inter).T.copy())
                        for _ in range(num_experts)])
        shared.append((mat(shared_inter, H).T.copy(), mat(shared_inter, H).T.copy(), mat(H, shared_inter).T.copy())
                      if shared_inter else None)
    final_norm = norm_w(H)
    lm_head = mat(vocab, H)
    return TinyModel(vocab, hidden, heads, kv_heads, head_dim, num_experts, top_k, inter, shared_inter,
                     norm_topk_prob, theta, eps, embed, lm_head, final_norm, attn, router, experts, shared,
                     dict(mla) if mla else None)


MLA_TINY = {"rank": 512, "d_nope": 32, "d_rope": 64, "d_v": 48}


def quantized_layers(tiny: TinyModel, fmt: str, seed: int = 1) -> list:
    """One seeded synthetic MoE layer (``oracle.inputs.OracleLayer``) per decoder layer, with
    the tiny model's shape, in ``fmt`` (``"awq_int4_g128"`` or ``"fp8_b128"``)."""
    base = "cfg0" if fmt == "awq_int4_g128" else "cfg1"
    cfg = inputs.scaled_config(base, hidden=tiny.hidden, inter=tiny.inter, num_experts=tiny.num_experts,
                               top_k=tiny.top_k, num_shared=1 if tiny.shared_inter else 0,
                               shared_inter=tiny.shared_inter, routing=tiny.mode)
    return [inputs.make_layer(cfg, seed + i) for i in range(tiny.layers)]


def quantized_ffns(tiny: TinyModel, layers: list) -> list:
    return [model.moe_ffn(ol.router, tiny.top_k, tiny.mode, ol.w_lookup, ol.shared_cat()) for ol in layers]


def quantized_attention(tiny: TinyModel, fmt: str, seed: int = 2, bf16: bool = True):
    """Seeded AWQ / FP8 attention projections of the tiny model's shape: per layer the
    checkpoint matrices ``{q, k, v, o}`` and the ``AttnWeights`` whose projections are their
    dequantized values, rounded to bf16 (what the decoder keeps when it dequantizes them at
    load) or exact (``bf16=False``: the quantized projections it runs as they are)."""
    from ccut_b200 import synthetic

    rng = np.random.default_rng(seed)
    d, H = tiny.head_dim, tiny.hidden
    shapes = {"q": (H, tiny.heads * d), "k": (H, tiny.kv_heads * d), "v": (H, tiny.kv_heads * d),
              "o": (tiny.heads * d, H)}  # (in, out)
    mats, attn = [], []
    for w in tiny.attn:
        m = {p: synthetic._gen_matrix(rng, fmt, k, n) for p, (k, n) in shapes.items()}
        deq = {p: inputs.dequant(m[p]).T.copy() for p in m}  # [out, in]
        if bf16:
            deq = {p: _bf16(v) for p, v in deq.items()}
        mats.append(m)
        attn.append(AttnWeights(w.ln1, deq["q"], deq["k"], deq["v"], deq["o"], w.ln2, w.q_norm, w.k_norm))
    return mats, attn
