"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no checkpoint or dataset exists offline).

Generator: numpy PCG64 (``np.random.default_rng(seed)``), float32 normals.
  * linear / patch weights ~ N(0, 0.02), biases ~ N(0, 0.01)
  * LayerNorm gains 1, shifts 0
  * raw position embedding [1, 577, e] ~ N(0, 0.02)
  * images: pixels U[0,1) mapped through the reference normalisation
    x/127.5 - 1 of x = 255 p, i.e. 2p - 1 (sam3_processor.c:57-73)
"""
from __future__ import annotations

import numpy as np

HIERA_L = dict(img_size=1008, patch_size=14, embed_dim=1024, depth=32, n_heads=16,
               window_size=24, mlp_dim=4736)


def tiny_cfg(depth: int = 8, embed_dim: int = 128, img_size: int = 336, window_size: int = 12,
             mlp_dim: int = 320) -> dict:
    """A small encoder with the same structure (head_dim 64, a global block
    at index 7 when depth >= 8)."""
    return dict(img_size=img_size, patch_size=14, embed_dim=embed_dim, depth=depth,
                n_heads=embed_dim // 64, window_size=window_size, mlp_dim=mlp_dim)


def vit_weights(cfg: dict, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    e, m, ps = cfg["embed_dim"], cfg["mlp_dim"], cfg["patch_size"]

    def n(*shape, sd=0.02):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(sd))

    blocks = []
    for _ in range(cfg["depth"]):
        blocks.append(dict(
            ln1_w=np.ones(e, np.float32), ln1_b=np.zeros(e, np.float32),
            qkv_w=n(3 * e, e), qkv_b=n(3 * e, sd=0.01),
            proj_w=n(e, e), proj_b=n(e, sd=0.01),
            ln2_w=np.ones(e, np.float32), ln2_b=np.zeros(e, np.float32),
            fc1_w=n(m, e), fc1_b=n(m, sd=0.01),
            fc2_w=n(e, m), fc2_b=n(e, sd=0.01)))
    return dict(patch_w=n(e, ps, ps, 3), patch_b=n(e, sd=0.01), pos_raw=n(1, 577, e),
                ln_pre_w=np.ones(e, np.float32), ln_pre_b=np.zeros(e, np.float32),
                blocks=blocks)


def images(cfg: dict, n: int, seed: int = 100) -> np.ndarray:
    rng = np.random.default_rng(seed)
    s = cfg["img_size"]
    p = rng.random((n, 3, s, s), dtype=np.float32)
    return (p * np.float32(2.0) - np.float32(1.0)).astype(np.float32)


def round_weights(w: dict, fn) -> dict:
    """Apply fn (e.g. bf16 rounding) to every linear / patch weight matrix, the
    tensors the encoder stores in reduced precision."""
    out = dict(w)
    out["patch_w"] = fn(w["patch_w"])
    out["blocks"] = []
    for b in w["blocks"]:
        nb = dict(b)
        for k in ("qkv_w", "proj_w", "fc1_w", "fc2_w"):
            nb[k] = fn(b[k])
        out["blocks"].append(nb)
    return out
