"""ccut_b200 -- B200 (sm_100a) quantized MoE expert forward for CostCut-Infer.

The compute path is ``libccut_moe.so`` (hand-written CUDA, C ABI in ``include/ccut_moe.h``)
driven through ctypes; PyTorch supplies device memory, streams and ``torch.distributed``.
There is no CPU fallback: a missing library raises.

Public entry points
-------------------
``MoeLayer``                 HBM-resident MoE layer: ``forward``, ``route``, ``topk``,
                             ``permute``, ``expert_ffn``, ``gate_up``, ``down``, ``combine``,
                             ``dequant``
``ep.ExpertParallelMoeLayer`` the same layer with routed experts sharded over GPUs (NCCL)
``ep_a2a.AllToAllMoeLayer``  expert parallelism exchanging only the routed rows (all-to-all)
``blocks.moe``               drop-ins for ``ccut.blocks.moe`` / ``ccut.models.generic.moe_forward``
``experts``                  drop-in for ``ccut.experts.pipeline.ExpertPipeline`` over resident layers
``config``                   the reference's ``[experts]`` / ``[quant]`` settings read for this path
``quant``                    ``QuantizeMethodBase``-compatible AWQ-int4-g128 / FP8-block-128 methods
``checkpoint``               ``load_moe_layer``: a MoE layer of an AWQ / FP8-block safetensors
                             checkpoint into HBM; ``load_decoder``: a whole Qwen-MoE or
                             DeepSeek-V2 / V3 decoder
``dense.DenseFfn``           dense quantized SwiGLU FFN (the expert kernels with one expert)
``blocks.attn_gqa``          drop-ins for ``ccut.blocks.attn_gqa`` (GQA attention on tensor cores)
``blocks.norm``              drop-in for ``ccut.blocks.norm.rms_norm``
``blocks.rope``              drop-in for ``ccut.blocks.rope.apply_rope``
``blocks.attn_mla``          drop-ins for ``ccut.blocks.attn_mla`` (MLA latent attention)
``model``                    ``MoeDecoder``: embedding, decoder layers (``DecoderLayer``: GQA
                             attention, ``MlaDecoderLayer``: multi-head latent attention; norms,
                             RoPE, bf16 caches in HBM, MoE or dense FFN), final norm, ``lm_head``
                             -- the reference's generic layer forward on the GPU
``rope_tables``              RoPE tables: the reference's ``build_rope`` cases, YaRN
``backend.GenericBackend``   the ``generate_step`` backend the reference's ``Engine`` calls, over
                             a ``MoeDecoder`` (prefix-reusing sequence caches, on-device sampling)
``sampling``                 the reference's temperature / top-k / min-p / top-p transform in torch
"""

from ccut_b200.layer import MoeLayer, Permutation, Routing  # noqa: F401

__all__ = ["MoeLayer", "Permutation", "Routing"]
__version__ = "0.1.0"
