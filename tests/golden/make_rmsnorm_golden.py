"""Generate RMSNorm golden vectors from the REFERENCE implementation's own
eager functions (``learning/03_rmsnorm/qwen_rmsnorm.py:54-63``) on CPU.

    python tests/golden/make_rmsnorm_golden.py --reference /path/to/gpu-kernel-lab

The reference module imports triton at the top; only its torch functions are
called.  The cases follow the reference's tests
(``learning/03_rmsnorm/test_qwen_rmsnorm.py``): shapes, scales and dtypes.
Writes ``rmsnorm_vectors.npz`` next to this script; the tests only read it.
16-bit values are stored as their raw bits (uint16), f32 as float32.
"""
from __future__ import annotations

import argparse
import importlib.util
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
SHAPES = [(1, 128), (33, 128), (1, 1024), (17, 1024), (3, 127)]
SCALES = [0.0, 1e-4, 1.0, 100.0]


@torch.inference_mode()
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--out", type=Path, default=HERE / "rmsnorm_vectors.npz")
    args = ap.parse_args()
    spec = importlib.util.spec_from_file_location("ref_qwen_rmsnorm", args.reference / "learning/03_rmsnorm/qwen_rmsnorm.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    def store(t):
        if t.dtype == torch.float32:
            return t.numpy()
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    out = {}
    for dname, dt in DTYPES.items():
        for si, shape in enumerate(SHAPES):
            for ci, scale in enumerate(SCALES):
                if shape[0] * shape[1] > 8192 and scale < 1.0:
                    continue                      # the large shape at the unit and large scales only
                g = torch.Generator().manual_seed(1000 * si + 10 * ci + len(dname))
                x = (torch.randn(shape, generator=g) * scale).to(dt)
                r = torch.randn(shape, generator=g).to(dt)
                w = torch.randn(shape[-1], generator=g).to(dt)
                key = f"{dname}_{shape[0]}x{shape[1]}_s{ci}"
                out[key + "_x"] = store(x)
                out[key + "_r"] = store(r)
                out[key + "_w"] = store(w)
                out[key + "_y"] = store(ref.qwen_rmsnorm_reference(x, w))
                y2, c2 = ref.qwen_residual_rmsnorm_reference(x, r, w)
                out[key + "_ry"] = store(y2)
                out[key + "_rc"] = store(c2)
    np.savez_compressed(args.out, **out)
    print(f"wrote {len(out)} arrays to {args.out}")


if __name__ == "__main__":
    main()
