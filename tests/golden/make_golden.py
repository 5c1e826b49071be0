"""Generate golden vectors from the REFERENCE implementation's own functions.

Run in the build container, where the reference checkout is mounted read-only:

    python tests/golden/make_golden.py --reference /path/to/gpu-kernel-lab

It imports ``learning/10_cuda_decode/activation_int8.py`` and
``learning/09_int4/quantization.py`` from the reference (pure torch, CPU) and
stores their outputs on seeded inputs in ``reference_vectors.npz`` next to this
script.  The GPU box never runs this script; the tests only read the ``.npz``.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def sha256(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def bf16_as_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


def config0_inputs():
    """x bf16 [1,1024] ~ N(0,1), W f32 [3072,1024] ~ N(0,0.02), seed 0."""
    g = torch.Generator().manual_seed(0)
    w = torch.randn(3072, 1024, generator=g) * 0.02
    x = torch.randn(1, 1024, generator=g).bfloat16()
    return x, w


@torch.inference_mode()
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--out", type=Path, default=HERE / "reference_vectors.npz")
    args = ap.parse_args()
    torch.backends.cuda.matmul.allow_tf32 = False
    a8 = _load(args.reference / "learning/10_cuda_decode/activation_int8.py", "ref_activation_int8")
    q4 = _load(args.reference / "learning/09_int4/quantization.py", "ref_quantization")
    out: dict[str, np.ndarray] = {}

    # 1. calibrated int8 (test_cuda_decode.py:7-17 inputs) + a second shape.
    torch.manual_seed(1)
    w, x = torch.randn(13, 128), torch.randn(8, 128)
    cases = {"cal_a": (w, x, 128, (0.0, 0.5, 1.0)), "cal_a_rtn": (w, x, 128, (0.0,))}
    gen = torch.Generator().manual_seed(7)
    w2 = torch.randn(64, 256, generator=gen) * 0.05
    x2 = torch.randn(16, 256, generator=gen) * torch.linspace(0.1, 3.0, 256)
    cases["cal_b"] = (w2, x2, 128, (0.0, 0.5, 1.0))
    cases["cal_b_g64"] = (w2, x2, 64, (0.0, 0.5, 1.0))
    for name, (w, x, group, alphas) in cases.items():
        p = a8.quantize_int8(w, x, group_size=group, alphas=alphas)
        out[f"{name}_w"] = w.numpy()
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_group"] = np.array(group)
        out[f"{name}_alphas"] = np.array(alphas, np.float32)
        out[f"{name}_data"] = p.data.numpy()
        out[f"{name}_scales"] = p.scales.numpy()
        out[f"{name}_inverse"] = p.inverse.numpy()
        out[f"{name}_alpha"] = np.array(p.alpha)
        out[f"{name}_mse"] = np.array(p.calibration_mse)
        out[f"{name}_deq"] = a8.dequantize_int8(p).numpy()
    z = a8.quantize_int8(torch.zeros(13, 128), torch.randn(8, 128))
    out["cal_zero_deq"] = a8.dequantize_int8(z).numpy()

    # 2. projection oracle (test_cuda_decode.py:20-36 shapes): x[256], W[34,256].
    torch.manual_seed(42)
    x = torch.randn(256, dtype=torch.bfloat16)
    w = torch.randn(34, 256, dtype=torch.bfloat16)
    p = a8.quantize_int8(w, torch.randn(8, 256))
    restored = a8.dequantize_int8(p)
    expected = (restored @ x.float()).bfloat16()
    a, b = expected.chunk(2)
    out["proj_x"] = bf16_as_f32(x)
    out["proj_w"] = bf16_as_f32(w)
    out["proj_data"] = p.data.numpy()
    out["proj_scales"] = p.scales.numpy()
    out["proj_inverse"] = p.inverse.numpy()
    out["proj_alpha"] = np.array(p.alpha)
    out["proj_expected"] = bf16_as_f32(expected)
    out["proj_expected_swiglu"] = bf16_as_f32(F.silu(a) * b)
    out["proj_expected_bf16w"] = bf16_as_f32((w.float() @ x.float()).bfloat16())

    # 3. BASELINE config 0 through the reference quantiser with group = K,
    #    alpha 0 (per-row absmax/127, fp32 scale) and the reference oracle.
    x0, w0 = config0_inputs()
    p0 = a8.quantize_int8(w0, x0.float(), group_size=1024, alphas=(0.0,))
    out["cfg0_data_sha256"] = np.array(sha256(p0.data))
    out["cfg0_scales"] = p0.scales.numpy()
    out["cfg0_inverse_unique"] = np.unique(p0.inverse.numpy())
    y0 = (a8.dequantize_int8(p0) @ x0.float()[0]).bfloat16()
    out["cfg0_expected"] = bf16_as_f32(y0)
    out["cfg0_w_sha256"] = np.array(sha256(w0))
    out["cfg0_x"] = bf16_as_f32(x0)

    # 4. int4 packer (test_int4.py:7-31 inputs).
    for group in (32, 64, 128):
        wr = torch.arange(-7, 8, dtype=torch.float32).repeat(group)[:group].repeat(3, 1)
        pr = q4.quantize_int4(wr, group_size=group, chunk_rows=2)
        out[f"i4_rt{group}_w"] = wr.numpy()
        out[f"i4_rt{group}_data"] = pr.data.numpy()
        out[f"i4_rt{group}_scales"] = pr.scales.numpy()
        torch.manual_seed(5)
        we = torch.randn(7, 256)
        pe = q4.quantize_int4(we, group)
        out[f"i4_err{group}_w"] = we.numpy()
        out[f"i4_err{group}_data"] = pe.data.numpy()
        out[f"i4_err{group}_scales"] = pe.scales.numpy()
        out[f"i4_err{group}_deq"] = q4.dequantize_int4(pe).numpy()
    pz = q4.quantize_int4(torch.zeros(2, 128))
    out["i4_zero_data"] = pz.data.numpy()
    out["i4_zero_scales"] = pz.scales.numpy()

    # 5. int4 GEMV / head oracle (test_int4.py:37-66 expressions), CPU.
    torch.manual_seed(42)
    n, k = 17, 128
    wg = torch.randn(n, k, dtype=torch.bfloat16) / k ** .5
    xg = torch.randn(k, dtype=torch.bfloat16)
    pg = q4.quantize_int4(wg)
    out["i4_gemv_w"] = bf16_as_f32(wg)
    out["i4_gemv_x"] = bf16_as_f32(xg)
    out["i4_gemv_data"] = pg.data.numpy()
    out["i4_gemv_scales"] = pg.scales.numpy()
    out["i4_gemv_expected"] = bf16_as_f32((q4.dequantize_int4(pg) @ xg.float()).to(torch.bfloat16))
    torch.manual_seed(13)
    wh = torch.randn(65, 128, dtype=torch.bfloat16) / 128 ** .5
    xh = torch.randn(128, dtype=torch.bfloat16)
    ph = q4.quantize_int4(wh)
    logits = (q4.dequantize_int4(ph) @ xh.float()).to(torch.bfloat16).float()
    out["i4_head_data"] = ph.data.numpy()
    out["i4_head_scales"] = ph.scales.numpy()
    out["i4_head_x"] = bf16_as_f32(xh)
    out["i4_head_logits"] = logits.numpy()
    for top in (1, 4, 8):
        v, i = logits.topk(top)
        out[f"i4_head_top{top}_values"] = v.numpy()
        out[f"i4_head_top{top}_ids"] = i.numpy()

    # 6. torch SiLU on bf16 (the SwiGLU epilogue's activation boundary).
    gs = torch.linspace(-12, 12, 2001).bfloat16()
    us = torch.linspace(3, -3, 2001).bfloat16()
    out["swiglu_in"] = bf16_as_f32(torch.cat([gs, us]))
    out["swiglu_expected"] = bf16_as_f32(F.silu(gs) * us)

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out} ({args.out.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
