"""Generate the golden fixtures under ``tests/golden/`` by running the reference itself.

Usage (only where the reference sources exist; they do not travel to GPU boxes)::

    python tests/golden/make_golden.py [--reference PATH_TO_REFERENCE/python]

The reference (CostCut-Infer, pure Python + numpy + numba) is imported read-only: numba's
``cache=True`` files go to a temporary ``NUMBA_CACHE_DIR`` and no bytecode is written.
Every fixture stores the inputs and the reference's outputs; the oracle restatement is
checked against them by ``tests/test_oracle_golden.py`` and the CUDA path by the GPU tests.

Fixtures
--------
``e4m3_table.npz``       ``fp8_e4m3_to_float32`` on all 256 codes          (kernels.py:52-74)
``fp8_rowscale.npz``     ``fp8_dequant_mat`` with per-row scales            (kernels.py:150-171)
``int4_linear.npz``      ``WeightOnlyMethod.apply`` signed int4 W4A16 whose weights equal
                         an AWQ-g128 matrix with zero-point 8 and per-group scales
                         constant along N                                   (weight_only.py:37-54)
``topk.npz``             ``topk_softmax`` both modes, incl. exact ties       (moe.py:46-89)
``silu_ffn.npz``         ``silu_mul_fused`` and ``expert_ffn``               (kernels.py:219-231, moe.py:122-141)
``combine_<fmt>.npz``    ``moe_combine`` with the oracle's dequantized experts as ``w_lookup``
                         for small AWQ and FP8-block layers               (moe.py:144-174)
``moe_forward_fp8.npz``  the reference ``moe_forward`` as-is (FakeWeightReader, FP8 per-row
                         scales) on FP8-block weights whose block scales are constant along N,
                         so both formats describe the same fp32 matrices (generic.py:348-400)
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import formats, inputs  # noqa: E402


def _import_reference(ref_python: Path):
    os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="ccut-numba-"))
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref_python))
    import ccut.blocks.moe as rmoe  # noqa: F401
    import ccut.models.generic as rgen  # noqa: F401
    import ccut.quant.kernels as rk  # noqa: F401
    import ccut.quant.weight_only as rwo  # noqa: F401
    from ccut.models.spec import MoeSpec  # noqa: F401
    from ccut.quant.spec import LayerQuantSpec, ScaleDesc, get_quant_key  # noqa: F401

    return rmoe, rgen, rk, rwo, MoeSpec, LayerQuantSpec, ScaleDesc, get_quant_key


def small_cfg(fmt: str, routing: str, top_k: int, shared: int) -> inputs.MoeLayerConfig:
    return inputs.MoeLayerConfig(
        f"small_{fmt}", hidden=256, inter=128, num_experts=8, top_k=top_k,
        num_shared=shared, shared_inter=128, fmt=fmt, routing=routing,
    )


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CCUT_REFERENCE"),
                    help="the reference's python/ directory (or set CCUT_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or CCUT_REFERENCE) must name the reference\'s python/ directory")
    rmoe, rgen, rk, rwo, MoeSpec, LayerQuantSpec, ScaleDesc, get_quant_key = _import_reference(Path(args.reference))
    rng = np.random.default_rng(20240601)

    # 1. e4m3 decode of every code
    codes = np.arange(256, dtype=np.uint8)
    np.savez_compressed(HERE / "e4m3_table.npz", codes=codes, values=rk.fp8_e4m3_to_float32(codes))

    # 2. per-row FP8 dequant
    w8 = rng.integers(0, 256, size=(16, 40), dtype=np.uint8)
    w8[w8 == 0x7F] = 0x7E  # keep NaN codes out of the matrix fixture (table covers them)
    w8[w8 == 0xFF] = 0xFE
    rs = np.exp(rng.uniform(np.log(1e-3), np.log(1e-1), size=16)).astype(np.float32)
    out = np.empty((16, 40), dtype=np.float32)
    rk.fp8_dequant_mat(w8, rs, out)
    np.savez_compressed(HERE / "fp8_rowscale.npz", w=w8, scale=rs, out=out)

    # 3. signed int4 W4A16 linear == AWQ (z = 8, scale constant along N) linear
    K, N, B = 256, 24, 5
    q = rng.integers(0, 16, size=(K, N), dtype=np.uint8)  # AWQ nibbles, [K, N]
    sigma = (np.abs(rng.normal(0.0, 0.02, size=K // 128)) + 1e-3).astype(np.float16)
    qweight = formats.awq_pack(q)
    qzeros = formats.awq_pack(np.full((K // 128, N), 8, dtype=np.uint8))
    scales = np.repeat(sigma[:, None], N, axis=1).astype(np.float16)
    v = (q.astype(np.int16) - 8).T  # signed [N, K]
    nib = (v & 0xF).astype(np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)  # [N, K/2], low nibble first
    col_scale = np.repeat(sigma.astype(np.float32), 128)  # per input column
    x = rng.standard_normal((B, K)).astype(np.float32)
    m = rwo.WeightOnlyMethod(
        LayerQuantSpec("t.int4", get_quant_key("int4_w4a16_sym"),
                       scales=(ScaleDesc(name="t.int4.weight_scale", dtype="F32", shape=(K,)),))
    )
    y = m.apply(packed.tobytes(), {"t.int4.weight_scale": col_scale}, x)
    deq = np.empty((N, K), dtype=np.float32)
    rk.int4_dequant_row(packed, col_scale, deq)
    np.savez_compressed(HERE / "int4_linear.npz", qweight=qweight, qzeros=qzeros, scales=scales,
                        x=x, y=y, dequant_out_in=deq)

    # 4. top-k routing, both modes; rows with exact ties and -0.0
    lg = rng.standard_normal((12, 64)).astype(np.float32)
    lg[0, :] = 0.5  # all tied
    lg[1, 10] = lg[1, 3] = lg[1, 40] = 3.0  # three-way tie at the top
    lg[2, :] = -0.0
    lg[3, 5] = lg[3, 6] = np.float32(2.0)
    ids_f, w_f, ids_t, w_t = {}, {}, {}, {}
    for k in (1, 2, 6, 8):
        wt, it = rmoe.topk_softmax(lg, k, False)
        w_f[k], ids_f[k] = wt, it
        wt, it = rmoe.topk_softmax(lg, k, True)
        w_t[k], ids_t[k] = wt, it
    np.savez_compressed(
        HERE / "topk.npz", logits=lg,
        **{f"ids_soft_k{k}": ids_f[k] for k in ids_f}, **{f"w_soft_k{k}": w_f[k] for k in w_f},
        **{f"ids_norm_k{k}": ids_t[k] for k in ids_t}, **{f"w_norm_k{k}": w_t[k] for k in w_t},
    )

    # 5. silu * up and one expert FFN
    g = (rng.standard_normal((7, 48)) * 4).astype(np.float32)
    u = rng.standard_normal((7, 48)).astype(np.float32)
    su = np.empty_like(g)
    rk.silu_mul_fused(g, u, su)
    xe = rng.standard_normal((7, 64)).astype(np.float32)
    wg = (rng.standard_normal((64, 48)) * 0.1).astype(np.float32)
    wu = (rng.standard_normal((64, 48)) * 0.1).astype(np.float32)
    wd = (rng.standard_normal((48, 64)) * 0.1).astype(np.float32)
    ye = rmoe.expert_ffn(xe, wg, wu, wd)
    np.savez_compressed(HERE / "silu_ffn.npz", gate=g, up=u, silu_mul=su, x=xe, wg=wg, wu=wu, wd=wd, y=ye)

    # 6. moe_combine on small oracle layers (seeded), routing from the reference
    for fmt, routing, k in (("awq_int4_g128", "softmax_topk", 2), ("fp8_b128", "topk_softmax", 3)):
        cfg = small_cfg(fmt, routing, k, shared=0)
        layer = inputs.make_layer(cfg, seed=7)
        rec = {}
        for T in (1, 5, 17):
            xb = layer.make_x(T)
            xf = formats.bf16_bits_to_f32(xb)
            logits = xf @ layer.router.T
            wts, ids = rmoe.topk_softmax(logits, k, routing == "topk_softmax")
            yb = rmoe.moe_combine(xf, ids, wts, w_lookup=layer.w_lookup)
            rec.update({f"x_T{T}": xb, f"ids_T{T}": ids, f"w_T{T}": wts, f"y_T{T}": yb})
        np.savez_compressed(HERE / f"combine_{fmt}.npz", seed=7, top_k=k, routing=routing, **rec)

    # 7. the reference moe_forward as-is, FP8 per-row scales == FP8 blocks constant along N
    cfg = small_cfg("fp8_b128", "softmax_topk", 2, shared=0)
    layer = inputs.make_layer(cfg, seed=11)
    for ew in layer.experts:  # make block scales depend on the K-block only
        for mat in (ew.gate, ew.up, ew.down):
            mat.scale[:] = mat.scale[0:1, :]
    table, shapes = {}, {}
    H, I = cfg.hidden, cfg.inter
    for e, ew in enumerate(layer.experts):
        for name, mat, (ind, outd) in (("gate", ew.gate, (H, I)), ("up", ew.up, (H, I)), ("down", ew.down, (I, H))):
            key = f"experts.{e}.{name}_proj_proj"  # the reference appends "_proj" twice (generic.py:372-374, :391)
            table[(0, key)] = np.ascontiguousarray(mat.weight.T).tobytes()  # [in, out] bytes
            table[(0, key + ".weight_scale")] = np.repeat(mat.scale[0], 128).astype(np.float32).tobytes()
            shapes[(0, key)] = (ind, outd, "fp8_e4m3")
    reader = rgen.FakeWeightReader(table, shapes)
    rec = {}
    for norm in (False, True):
        spec = MoeSpec(num_experts=cfg.num_experts, top_k=cfg.top_k, intermediate_size=I,
                       norm_topk_prob=norm, has_shared_expert=False, shared_intermediate=0)
        for T in (1, 5, 17):
            xb = layer.make_x(T)
            xf = formats.bf16_bits_to_f32(xb)
            yb = rgen.moe_forward(xf, layer.router, reader, 0, spec, None)
            rec[f"y_norm{int(norm)}_T{T}"] = yb
            rec[f"x_T{T}"] = xb
    np.savez_compressed(HERE / "moe_forward_fp8.npz", seed=11, top_k=cfg.top_k, **rec)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
