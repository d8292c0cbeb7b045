"""Generate ``tests/golden/vllm_formats.npz``: independent pins for the formats the
reference does not implement, from library code installed in this container (vLLM 0.22,
PyTorch 2.11).  Neither library travels to GPU boxes, so the vectors are committed::

    python tests/golden/make_golden_vllm.py

Fixtures
--------
``awq_*``    an unpacked int4 matrix q [K, N], zero points z [K/128, N] and fp16 scales s,
             with q and z packed by vLLM's ``awq_pack`` (the AutoAWQ GEMM layout:
             ``vllm/model_executor/layers/quantization/utils/quant_utils.py``); the test
             dequantizes the packed tensors and compares with ``(q - z) * s`` of the
             unpacked values.
``route_*``  DeepSeek-V3 grouped routing by vLLM's ``grouped_topk`` (the pure-torch path of
             ``vllm/model_executor/layers/fused_moe/router/grouped_topk_router.py``): sigmoid
             scores, a zero correction bias, 8 groups scored by their two best experts, 4
             groups kept, top-8, renormalised, times 2.5.
(The FP8 128 x 128 block format needs no fixture: its test decodes through PyTorch's
``float8_e4m3fn``, available wherever the tests run.)
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main() -> int:
    os.environ.setdefault("VLLM_LOGGING_LEVEL", "ERROR")
    os.environ["TORCHDYNAMO_DISABLE"] = "1"  # run grouped_topk's torch code as written, uncompiled
    import torch
    from vllm.model_executor.layers.fused_moe.router.grouped_topk_router import grouped_topk
    from vllm.model_executor.layers.quantization.utils.quant_utils import awq_pack

    rng = np.random.default_rng(77)
    out = {}
    # ---- AWQ GEMM packing
    K, N = 256, 128
    q = rng.integers(0, 16, (K, N), dtype=np.int64)
    z = rng.integers(0, 16, (K // 128, N), dtype=np.int64)
    s = (np.abs(rng.standard_normal((K // 128, N))) * 0.02 + 1e-3).astype(np.float16)
    qw = awq_pack(torch.from_numpy(q).int(), 4, K, N).numpy()
    qz = awq_pack(torch.from_numpy(z).int(), 4, K // 128, N).numpy()
    out.update(awq_q=q.astype(np.int8), awq_z=z.astype(np.int8), awq_s=s, awq_qweight=qw, awq_qzeros=qz)
    # ---- grouped sigmoid routing
    T, E = 96, 256
    logits = (rng.standard_normal((T, E)) * 2).astype(np.float32)
    lt = torch.from_numpy(logits)
    w, ids = grouped_topk(lt, lt, topk=8, renormalize=True, num_expert_group=8, topk_group=4,
                          scoring_func="sigmoid", routed_scaling_factor=2.5,
                          e_score_correction_bias=torch.zeros(E))
    out.update(route_logits=logits, route_ids=ids.numpy().astype(np.int64), route_w=w.numpy().astype(np.float32))
    np.savez_compressed(HERE / "vllm_formats.npz", **out)
    print("wrote", HERE / "vllm_formats.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
