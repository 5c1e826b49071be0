"""numpy restatement of the reference's quantize / dequantize / matmul path.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the CUDA
path and the timed CPU baseline, never part of the product.

All arithmetic is float32 with round-half-to-even, the semantics of the
reference's torch CPU code.  bf16 values are carried as float32 arrays holding
exactly representable bf16 numbers (plus helpers for the raw uint16 bits).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------- bf16

def bf16_bits(a) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even (torch ``.bfloat16()``)."""
    u = np.ascontiguousarray(a, dtype=F32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def bf16_to_f32(bits) -> np.ndarray:
    """bf16 bit patterns -> float32 values (exact)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bf16, returned as float32."""
    return bf16_to_f32(bf16_bits(a))


# ------------------------------------------------------------- W8A16 (reference)

def _importance_pow(importance: np.ndarray, alpha: float) -> np.ndarray:
    # torch.pow(t, scalar) special-cases these exponents (0 -> ones, .5 -> sqrt,
    # 1 -> copy); mirror them so the channel vector matches bit for bit.
    if alpha == 0:
        return np.ones_like(importance)
    if alpha == 0.5:
        return np.sqrt(importance)
    if alpha == 1:
        return importance.copy()
    return np.power(importance, F32(alpha)).astype(F32)


def quantize_int8(weight, calibration, group_size=128, alphas=(0.0, 0.5, 1.0)):
    """Restates ``activation_int8.py:24-60`` (AWQ-inspired channel search).

    Returns ``dict(data int8 [N,K], scales f32 [N,K/g], inverse f32 [K],
    group_size, alpha, calibration_mse)``.
    """
    w_all = np.asarray(weight, dtype=F32)
    x = np.asarray(calibration, dtype=F32)
    if w_all.ndim != 2 or x.ndim != 2 or w_all.shape[1] != x.shape[1]:
        raise ValueError("expected weight[N,K], calibration[T,K]")
    n, k = w_all.shape
    if n == 0 or k == 0 or group_size <= 0 or k % group_size or x.shape[0] == 0:
        raise ValueError("nonempty tensors and group dividing K required")
    if not alphas or any(a < 0 or a > 1 for a in alphas):
        raise ValueError("nonempty alpha values in [0,1] required")
    if not np.isfinite(w_all).all() or not np.isfinite(x).all():
        raise ValueError("finite inputs required")
    importance = np.maximum(np.abs(x).mean(0, dtype=F32), F32(1e-4))   # :30
    best = None
    for alpha in alphas:                                               # :34
        channel = np.clip(_importance_pow(importance, alpha), F32(1e-2), F32(1e2))
        channel = channel / np.sqrt(channel.max() * channel.min())     # :36
        data = np.empty((n, k), np.int8)
        scales = np.empty((n, k // group_size), F32)
        error = 0.0
        for start in range(0, n, 256):                                 # :40
            w = w_all[start:start + 256]
            grouped = (w * channel).reshape(w.shape[0], -1, group_size)
            scale = np.abs(grouped).max(-1) / F32(127)
            scale = np.where(scale == 0, F32(1), scale).astype(F32)
            q = np.clip(np.rint(grouped / scale[..., None]), -127, 127).astype(np.int8)
            restored = (q.astype(F32) * scale[..., None]).reshape(w.shape) / channel
            error += float(np.square(x @ restored.T - x @ w.T).sum(dtype=F32))
            data[start:start + w.shape[0]] = q.reshape(w.shape)
            scales[start:start + w.shape[0]] = scale
        cand = dict(data=data, scales=scales, inverse=(F32(1) / channel).astype(F32),
                    group_size=group_size, alpha=float(alpha),
                    calibration_mse=error / (x.shape[0] * n))
        if best is None or cand["calibration_mse"] < best["calibration_mse"]:
            best = cand
    return best


def dequantize_int8(data, scales, inverse, group_size) -> np.ndarray:
    """Restates ``activation_int8.py:63-64``: ``q * s[n, k//g] * inverse[k]`` (f32)."""
    s = np.repeat(np.asarray(scales, F32), group_size, axis=1)
    return (np.asarray(data).astype(F32) * s) * np.asarray(inverse, F32)


# ------------------------------------------------------ W8A16 (BASELINE format)

def quantize_int8_rowwise(weight):
    """BASELINE.json config 0 format: per-output-row ``scale = absmax/127`` stored
    as bf16, ``q = round_half_even(W / scale_bf16)`` clamped to [-127, 127].

    This is ``activation_int8.py:47-52`` with group = K and channel = 1 (alpha 0),
    except that q is computed with the bf16-rounded scale so that the stored
    (q, scale) pair dequantises exactly.  A zero row gets scale 1 (``:48``).
    Returns ``(q int8 [N,K], scale f32 [N] holding bf16 values)``.
    """
    w = np.asarray(weight, dtype=F32)
    if w.ndim != 2 or w.shape[0] == 0 or w.shape[1] == 0:
        raise ValueError("weight must be a nonempty [N,K] matrix")
    scale = np.abs(w).max(1) / F32(127)
    scale = np.where(scale == 0, F32(1), scale).astype(F32)
    s = bf16_round(scale)
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def dequantize_int8_rowwise(q, scale) -> np.ndarray:
    return np.asarray(q).astype(F32) * np.asarray(scale, F32)[:, None]


# ------------------------------------------------------------- W4A16 (reference)

def quantize_int4(weight, group_size=128, chunk_rows=256):
    """Restates ``quantization.py:35-62``: symmetric absmax/7, values in [-7, 7],
    two's-complement nibbles, low nibble = even k.  Returns ``(data uint8 [N,K/2],
    scales f32 [N,K/g])``."""
    w_all = np.asarray(weight, dtype=F32)
    if w_all.ndim != 2:
        raise ValueError("weight must be floating-point [N,K]")
    n, k = w_all.shape
    if group_size not in (32, 64, 128) or n == 0 or k == 0 or k % group_size:
        raise ValueError("positive dimensions; group 32/64/128 must divide K")
    if chunk_rows <= 0:
        raise ValueError("chunk_rows must be positive")
    data = np.empty((n, k // 2), np.uint8)
    scales = np.empty((n, k // group_size), F32)
    for start in range(0, n, chunk_rows):
        block = w_all[start:start + chunk_rows]
        if not np.isfinite(block).all():
            raise ValueError("weights must be finite")
        grouped = block.reshape(block.shape[0], k // group_size, group_size)
        scale = np.abs(grouped).max(-1) / F32(7)
        scale = np.where(scale == 0, F32(1), scale).astype(F32)
        quant = np.clip(np.rint(grouped / scale[..., None]), -7, 7).astype(np.int16)
        codes = (quant.reshape(block.shape) & 15).astype(np.uint8)
        data[start:start + block.shape[0]] = codes[:, 0::2] | (codes[:, 1::2] << 4)
        scales[start:start + block.shape[0]] = scale
    return data, scales


def unpack_nibbles(data) -> np.ndarray:
    """uint8 [N,K/2] -> uint8 codes [N,K] (low nibble = even k)."""
    d = np.asarray(data, np.uint8)
    out = np.empty((d.shape[0], d.shape[1] * 2), np.uint8)
    out[:, 0::2] = d & 15
    out[:, 1::2] = d >> 4
    return out


def dequantize_int4(data, scales, group_size) -> np.ndarray:
    """Restates ``quantization.py:65-71``."""
    codes = unpack_nibbles(data).astype(np.int16)
    signed = np.where(codes >= 8, codes - 16, codes).astype(F32)
    return signed * np.repeat(np.asarray(scales, F32), group_size, axis=1)


# ------------------------------------------------------ W4A16 (BASELINE format)

def quantize_int4_asym(weight, group_size=128):
    """BASELINE.json config 3 format (no reference function; restated from the
    published asymmetric round-to-nearest scheme, e.g. AWQ's
    ``pseudo_quantize_tensor`` with ``zero_point=True``):

    per group of ``group_size`` along K:
      ``scale = bf16((max - min) / 15)``  (a zero range gets scale 1, as the
      reference does for zero groups, ``quantization.py:57``);
      ``zero = clamp(round(-min / scale), 0, 15)`` (an integer, exact in bf16);
      ``q = clamp(round(w / scale) + zero, 0, 15)``; nibbles packed as in
      ``quantization.py:60`` (low nibble = even k).
    Dequantised weight: ``(q - zero) * scale`` in float32, which is exact.
    Returns ``(data uint8 [N,K/2], scales f32 [N,K/g], zeros f32 [N,K/g])``.
    """
    w = np.asarray(weight, dtype=F32)
    n, k = w.shape
    if n == 0 or k == 0 or group_size <= 0 or k % group_size or group_size % 2:
        raise ValueError("positive dimensions; an even group must divide K")
    g = w.reshape(n, k // group_size, group_size)
    wmin = g.min(-1)
    wmax = g.max(-1)
    scale = (wmax - wmin) / F32(15)
    scale = np.where(scale == 0, F32(1), scale).astype(F32)
    s = bf16_round(scale)
    z = np.clip(np.rint(-wmin / s), 0, 15).astype(F32)
    q = np.clip(np.rint(g / s[..., None]) + z[..., None], 0, 15).astype(np.uint8)
    q = q.reshape(n, k)
    data = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    return data, s, z


def dequantize_int4_asym(data, scales, zeros, group_size) -> np.ndarray:
    q = unpack_nibbles(data).astype(F32)
    s = np.repeat(np.asarray(scales, F32), group_size, axis=1)
    z = np.repeat(np.asarray(zeros, F32), group_size, axis=1)
    return (q - z) * s


# ------------------------------------------------------------------- matmul path

def linear_f32(x, w_deq) -> np.ndarray:
    """fp32-accumulated ``x.float() @ W_deq.T`` (the reference oracle, before the
    final bf16 cast).  x: [M,K] (bf16 values as f32) or [K]."""
    x = np.asarray(x, F32)
    return (x @ np.asarray(w_deq, F32).T).astype(F32)


def linear(x, w_deq) -> np.ndarray:
    """``(dequantize(packed) @ x.float()).bfloat16()`` -- reference
    ``profiling/decode_stage2_benchmark.py:55`` -- generalised to x [M,K]."""
    return bf16_round(linear_f32(x, w_deq))


def silu_f32(g) -> np.ndarray:
    g = np.asarray(g, F32)
    return (g / (F32(1) + np.exp(-g))).astype(F32)


def swiglu(y) -> np.ndarray:
    """Model-ordered SwiGLU of ``warp_gemv.cu:46-50`` on bf16 projections
    ``y = [gate | up]`` (gate rows precede up rows): ``bf16(bf16(silu(g)) * u)``."""
    y = np.asarray(y, F32)
    half = y.shape[-1] // 2
    g, u = y[..., :half], y[..., half:]
    a = bf16_round(silu_f32(g))
    return bf16_round(a * u)


def head_logits(x, w_deq) -> np.ndarray:
    """lm_head logits as the reference int4 head produces them: fp32 dot, then
    rounded to the activation dtype (``09_int4/kernels.py:26``)."""
    return bf16_round(linear_f32(x, w_deq))


def topk_lowest_index(logits, k):
    """top-k values and ids; ties resolve to the lowest vocabulary index, the
    rule of ``09_int4/kernels.py:47`` (``tl.min`` over tied rows)."""
    logits = np.asarray(logits, F32)
    order = np.argsort(-logits, kind="stable")[:k]
    return logits[order], order.astype(np.int64)


# --------------------------------------------------------------------------- RMSNorm
def round_to(a, dtype: str) -> np.ndarray:
    """Round f32 values to ``dtype`` ('bf16', 'f16' or 'f32') and back to f32."""
    a = np.asarray(a, F32)
    if dtype == "bf16":
        return bf16_round(a)
    if dtype == "f16":
        return a.astype(np.float16).astype(F32)
    return a


def qwen_rmsnorm(x, weight, eps=1e-6, dtype="bf16") -> np.ndarray:
    """Qwen RMSNorm of each row, in the order of ``learning/03_rmsnorm/qwen_rmsnorm.py:54-58``:
    f32 mean of squares, ``x * rsqrt(mean + eps)`` rounded to the dtype, then the
    dtype product with the weight.  ``x`` and ``weight`` hold values of ``dtype``."""
    f = np.asarray(x, F32)
    mean = (f.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(F32)
    normalized = f * (F32(1) / np.sqrt(mean + F32(eps), dtype=F32))
    return round_to(np.asarray(weight, F32) * round_to(normalized, dtype), dtype)


def qwen_residual_rmsnorm(x, residual, weight, eps=1e-6, dtype="bf16"):
    """``(rmsnorm(c), c)`` with ``c = dtype(x + residual)`` (``qwen_rmsnorm.py:61-63``)."""
    c = round_to(np.asarray(x, F32) + np.asarray(residual, F32), dtype)
    return qwen_rmsnorm(c, weight, eps, dtype), c
