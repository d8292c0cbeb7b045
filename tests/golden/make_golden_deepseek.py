"""Generate ``tests/golden/deepseek_tiny.npz``: logits of ``transformers``' own
``DeepseekV3ForCausalLM`` (fp32, eager attention) on the seeded tiny DeepSeek-V3-style models of
``tests/deepseek_helpers.py``, the published reference implementation of the architecture
the MLA loader reads (multi-head latent attention with YaRN and interleaved rope channels,
grouped sigmoid routing, shared experts, a dense first layer)::

    python tests/golden/make_golden_deepseek.py

The weights are loaded into the model's state dict as they are (the quantized matrices as the
oracle dequantizes them).  Stored per case: the tokens, the logits of every position of one
causal pass, the model's YaRN table (``inv_freq`` and the cos / sin factor) and its softmax
scale.  Needs ``transformers`` (5.x) and torch; runs on the CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from tests.deepseek_helpers import DS_CASES, DS_SEEDS, deepseek_tiny  # noqa: E402

TOKENS = 12


def main() -> int:
    import torch
    import transformers
    from transformers import DeepseekV3Config, DeepseekV3ForCausalLM

    out = {"transformers_version": np.array(transformers.__version__)}
    for name, kw in DS_CASES.items():
        seed = DS_SEEDS[name]
        cfg, _, hf = deepseek_tiny(seed, **kw)
        c = {k: v for k, v in cfg.items() if k not in ("architectures", "model_type", "quantization_config")}
        model = DeepseekV3ForCausalLM(DeepseekV3Config(**c, attn_implementation="eager")).float().eval()
        sd = model.state_dict()
        missing = set(sd) - set(hf)
        extra = set(hf) - set(sd)
        if missing or extra:
            raise SystemExit(f"{name}: state dict mismatch: missing {sorted(missing)} extra {sorted(extra)}")
        model.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)).float() for k, v in hf.items()})
        tokens = np.random.default_rng(3000 + seed).integers(0, cfg["vocab_size"], TOKENS).astype(np.int64)
        with torch.no_grad():
            logits = model(torch.from_numpy(tokens)[None]).logits[0].float().numpy()
        out[f"{name}_tokens"] = tokens
        out[f"{name}_logits"] = logits.astype(np.float32)
        out[f"{name}_inv_freq"] = model.model.rotary_emb.inv_freq.float().numpy()
        out[f"{name}_rope_factor"] = np.float64(model.model.rotary_emb.attention_scaling)
        out[f"{name}_softmax_scale"] = np.float64(model.model.layers[0].self_attn.scaling)
    np.savez_compressed(HERE / "deepseek_tiny.npz", **out)
    print("wrote", HERE / "deepseek_tiny.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
