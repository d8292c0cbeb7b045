"""Generate ``tests/golden/ct_int4.npz``: compressed-tensors ``pack-quantized`` int4 matrices
(W4A16, group 128) packed and dequantized by the ``compressed_tensors`` library itself::

    python tests/golden/make_golden_ct.py

Per case (symmetric without zero points, asymmetric with packed zero points): seeded signed
int4 values ``v`` [N, K] and zero points ``zp`` [N, K / 128] in [-8, 7], scales [N, K / 128]
that are fp16 values, ``weight_packed`` = ``pack_to_int32(v, 4)``, ``weight_zero_point`` =
``pack_to_int32(zp, 4, packed_dim=0)`` and the fp32 weight ``dequantize(unpack_from_int32(...),
scale, zp)`` with fp32 scales (exact products).  Needs ``compressed_tensors`` and torch.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# name, N, K, symmetric
CASES = [("sym", 64, 384, True), ("asym", 96, 256, False)]


def main() -> int:
    import compressed_tensors
    import torch
    from compressed_tensors.compressors.pack_quantized.helpers import pack_to_int32, unpack_from_int32
    from compressed_tensors.quantization.lifecycle.forward import dequantize

    out = {"compressed_tensors_version": np.array(compressed_tensors.__version__)}
    rng = np.random.default_rng(61)
    for name, N, K, sym in CASES:
        v = torch.from_numpy(rng.integers(-8, 8, (N, K)).astype(np.int8))
        scale = torch.from_numpy((np.abs(rng.normal(0, 0.02, (N, K // 128))) + 1e-3).astype(np.float16).astype(
            np.float32))
        packed = pack_to_int32(v, 4)
        zp = None
        if not sym:
            zp = torch.from_numpy(rng.integers(-8, 8, (N, K // 128)).astype(np.int8))
            out[f"{name}_weight_zero_point"] = pack_to_int32(zp, 4, packed_dim=0).numpy()
            zp = unpack_from_int32(torch.from_numpy(out[f"{name}_weight_zero_point"]), 4, (N, K // 128),
                                   packed_dim=0)
        w = dequantize(unpack_from_int32(packed, 4, (N, K)), scale, zp, dtype=torch.float32)
        out[f"{name}_weight_packed"] = packed.numpy()
        out[f"{name}_weight_scale"] = scale.numpy()
        out[f"{name}_weight_shape"] = np.array([N, K], np.int64)
        out[f"{name}_weight"] = w.numpy().astype(np.float32)
    np.savez_compressed(HERE / "ct_int4.npz", **out)
    print("wrote", HERE / "ct_int4.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
