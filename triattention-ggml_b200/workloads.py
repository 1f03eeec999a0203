"""Seeded synthetic inputs for the TriAttention eviction step.

Everything here is host-side numpy (bit-reproducible across machines for a
given seed); bench.py builds its multi-GB caches on the device with the same
distributions.

Calibration stats (TRIA_FORMAT.md:61-90 layout), per (layer, head, pair f):
    q_mean = m * exp(i*phi),  m ~ |N(0,1)| + 0.1,  phi ~ U(-pi, pi)
    q_abs_mean = m + eps,     eps ~ N(0, 0.1)   (negative residuals are clamped
                                                 by the scorer, triattention.c:175-176)
    mrl = m / q_abs_mean
Key caches:
    fp32 keys  : N(0,1) scaled per dim by exp(U(-1,1))          (single-layer CPU case)
    f16 K/V    : N(0,1), each (layer, kv-head, dim) an outlier  (x8) with p = 1%
    q8_0 K/V   : ggml q8_0 blocks {f16 d = max|x|/127; int8 q = round(x/d)} of N(0,1)
Cache layout is llama.cpp's: per layer [cell][kv_head][row_bytes].
"""
from __future__ import annotations

import struct

import numpy as np

TRIA_MAGIC = 0x54524941
TRIA_HEADER = 64
TYPE_F16 = 1      # ggml type ids
TYPE_Q8_0 = 8
Q8_0_BLOCK = 34   # {f16 d; int8 q[32]}


def row_bytes(type_id: int, head_dim: int) -> int:
    if type_id == TYPE_F16:
        return 2 * head_dim
    if type_id == TYPE_Q8_0:
        assert head_dim % 32 == 0
        return head_dim // 32 * Q8_0_BLOCK
    raise ValueError(f"unsupported cache type {type_id}")


def synth_stats(num_layers, num_heads, head_dim, seed=0):
    """Per-head arrays (q_mean_real, q_mean_imag, q_abs_mean, mrl), each [L, H, fc] f32."""
    fc = head_dim // 2
    rng = np.random.default_rng(seed)
    m = np.abs(rng.standard_normal((num_layers, num_heads, fc))) + 0.1
    phi = rng.uniform(-np.pi, np.pi, (num_layers, num_heads, fc))
    eps = rng.normal(0.0, 0.1, (num_layers, num_heads, fc))
    qmr = (m * np.cos(phi)).astype(np.float32)
    qmi = (m * np.sin(phi)).astype(np.float32)
    qam = (m + eps).astype(np.float32)
    mrl = (m / (m + eps)).astype(np.float32)
    return qmr, qmi, qam, mrl


def write_tria(path, num_layers, num_heads, num_kv_heads, head_dim, rope_theta=1e6,
               attn_scale=1.0, scales=None, seed=0, version=2, arrays=None):
    """Write a TRIA v1/v2 stats file (TRIA_FORMAT.md:14-105)."""
    fc = head_dim // 2
    qmr, qmi, qam, mrl = arrays if arrays is not None else synth_stats(
        num_layers, num_heads, head_dim, seed)
    if scales is None:
        scales = np.ones(num_layers, np.float32)
    hdr = struct.pack("<IIIIIIIff", TRIA_MAGIC, version, num_layers, num_heads,
                      num_kv_heads, head_dim, fc, rope_theta, attn_scale)
    hdr += b"\0" * (TRIA_HEADER - len(hdr))
    with open(path, "wb") as f:
        f.write(hdr)
        if version >= 2:
            f.write(np.asarray(scales, "<f4").tobytes())
        for li in range(num_layers):
            for hi in range(num_heads):
                for a in (qmr, qmi, qam, mrl):
                    f.write(np.asarray(a[li, hi], "<f4").tobytes())
    return path


def fp32_keys(n, head_dim, seed=0, n_heads=1):
    """[n_heads, n, head_dim] f32 keys ~ N(0,1) * exp(U(-1,1)) per (head, dim)."""
    rng = np.random.default_rng(seed)
    scale = np.exp(rng.uniform(-1.0, 1.0, (n_heads, 1, head_dim)))
    return (rng.standard_normal((n_heads, n, head_dim)) * scale).astype(np.float32)


def split_halves(k):
    """Pair f = (x[f], x[f+fc]) (triattention_common.py:12-15)."""
    fc = k.shape[-1] // 2
    return np.ascontiguousarray(k[..., :fc]), np.ascontiguousarray(k[..., fc:])


def f16_values(num_layers, n, num_kv_heads, head_dim, seed=0, outlier_p=0.01, outlier_x=8.0):
    """[L, n, KV, hd] f32 values ~N(0,1), outlier dims (p per (layer, head, dim)) x8."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((num_layers, n, num_kv_heads, head_dim), dtype=np.float32)
    out = rng.random((num_layers, 1, num_kv_heads, head_dim)) < outlier_p
    return np.where(out, x * np.float32(outlier_x), x).astype(np.float32)


def f16_cache(num_layers, n, num_kv_heads, head_dim, seed=0, outlier_p=0.01):
    """f16 cache as raw bytes, [L, n, KV * 2*hd] uint8."""
    x = f16_values(num_layers, n, num_kv_heads, head_dim, seed, outlier_p).astype(np.float16)
    return x.view(np.uint8).reshape(num_layers, n, num_kv_heads * 2 * head_dim)


def quantize_q8_0(x):
    """ggml q8_0 of the last axis (multiple of 32): returns [..., nb*34] uint8."""
    shp = x.shape
    xb = x.reshape(-1, 32).astype(np.float32)
    amax = np.abs(xb).max(axis=1)
    d = amax / np.float32(127.0)
    inv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.rint(xb * inv[:, None]), -127, 127).astype(np.int8)
    blk = np.empty((xb.shape[0], Q8_0_BLOCK), np.uint8)
    blk[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    blk[:, 2:] = q.view(np.uint8)
    return blk.reshape(*shp[:-1], shp[-1] // 32 * Q8_0_BLOCK)


def q8_0_cache(num_layers, n, num_kv_heads, head_dim, seed=0):
    """q8_0 cache as raw bytes, [L, n, KV * hd/32*34] uint8 (from N(0,1) data)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((num_layers, n, num_kv_heads, head_dim), dtype=np.float32)
    return quantize_q8_0(x).reshape(num_layers, n, -1)


def half_to_float(h):
    return np.asarray(h, np.uint16).view(np.float16).astype(np.float32)


def rows_to_split(type_id, rows, head_dim):
    """Dequantise cache rows of one head ([n, row_bytes] uint8) to split fp32 halves."""
    n = rows.shape[0]
    if type_id == TYPE_F16:
        x = rows.reshape(n, -1).view(np.float16).astype(np.float32)
    elif type_id == TYPE_Q8_0:
        b = rows.reshape(n, head_dim // 32, Q8_0_BLOCK)
        d = b[:, :, :2].copy().view(np.float16).astype(np.float32)          # [n, nb, 1]
        q = b[:, :, 2:].view(np.int8).astype(np.float32)                    # [n, nb, 32]
        x = (q * d).reshape(n, head_dim).astype(np.float32)
    else:
        raise ValueError(type_id)
    return split_halves(x)


def layer_keep(n, layer_budget, ramp_pct):
    """Rows requested to be kept: n - floor(ramp% * (n - B) / 100) (n if n <= B)."""
    if n <= layer_budget:
        return n
    return n - (max(0, min(100, ramp_pct)) * (n - layer_budget)) // 100


def layer_budget(scale, base_budget):
    """tria_layer_budget (triattention.h:85-89): max(1, (int)(base * scale)) in fp32."""
    b = int(np.float32(np.float32(base_budget) * np.float32(scale)))
    return b if b > 0 else 1
