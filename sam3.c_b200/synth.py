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


VIT_PREFIX = "detector_model.vision_encoder.backbone."


def vit_sam3_tensors(cfg: dict, w: dict, patch_bias: bool = True) -> list:
    """The encoder weights as the tensors of a .sam3 file: (name, array)
    under the reference's names (image_encoder.c:155, 346-452), with the
    fused QKV split back into q_proj / k_proj / v_proj."""
    e = cfg["embed_dim"]
    P = VIT_PREFIX
    t = [(P + "embeddings.patch_embeddings.projection.weight", w["patch_w"])]
    if patch_bias:
        t.append((P + "embeddings.patch_embeddings.projection.bias", w["patch_b"]))
    t += [(P + "embeddings.position_embedding.weight", w["pos_raw"]),
          (P + "layer_norm.weight", w["ln_pre_w"]), (P + "layer_norm.bias", w["ln_pre_b"])]
    for i, b in enumerate(w["blocks"]):
        L = f"{P}layers.{i}."
        t += [(L + "layer_norm1.weight", b["ln1_w"]), (L + "layer_norm1.bias", b["ln1_b"])]
        for j, q in enumerate(("q_proj", "k_proj", "v_proj")):
            t += [(L + f"attention.{q}.weight", b["qkv_w"][j * e:(j + 1) * e]),
                  (L + f"attention.{q}.bias", b["qkv_b"][j * e:(j + 1) * e])]
        t += [(L + "attention.o_proj.weight", b["proj_w"]), (L + "attention.o_proj.bias", b["proj_b"]),
              (L + "layer_norm2.weight", b["ln2_w"]), (L + "layer_norm2.bias", b["ln2_b"]),
              (L + "mlp.fc1.weight", b["fc1_w"]), (L + "mlp.fc1.bias", b["fc1_b"]),
              (L + "mlp.fc2.weight", b["fc2_w"]), (L + "mlp.fc2.bias", b["fc2_b"])]
    return t


# ---------------------------------------------------------------- TinyViT
TINYVIT_21M = dict(img_size=1008, n_layers=4, embed_dims=(96, 192, 384, 576), depths=(2, 2, 6, 2),
                   num_heads=(3, 6, 12, 18), window_sizes=(7, 7, 14, 7), embed_dim=1024, mlp_ratio=4)


def tiny_tinyvit_cfg(img_size=112):
    """A small TinyViT for parity runs (head_dim 32 everywhere)."""
    return dict(img_size=img_size, n_layers=4, embed_dims=(32, 64, 96, 128), depths=(1, 1, 2, 1),
                num_heads=(1, 2, 3, 4), window_sizes=(7, 7, 14, 7), embed_dim=64, mlp_ratio=4)


def tinyvit_weights(cfg, seed=0, std=0.02):
    """Random-init TinyViT weights in the reference's layouts (OHWI convs,
    [out, in] linears); BN running stats mean 0 / var 1, gamma 1, beta 0
    perturbed slightly; weights ~N(0, std)."""
    rng = np.random.default_rng(seed)
    n = lambda *s, sc=std: (rng.standard_normal(s) * sc).astype(np.float32)

    def bn(c):
        return dict(bn_w=1 + n(c, sc=0.05), bn_b=n(c, sc=0.05), bn_mean=n(c, sc=0.05),
                    bn_var=(1 + 0.1 * rng.random(c)).astype(np.float32))

    def conv(oc, ic, k, bias=False, with_bn=True):
        d = dict(w=n(oc, k, k, ic))
        if bias:
            d["b"] = n(oc)
        if with_bn:
            d.update(bn(oc))
        return d

    E = cfg["embed_dims"]
    r = cfg["mlp_ratio"]
    w = {"patch_embed_0": conv(E[0] // 2, 3, 3), "patch_embed_1": conv(E[0], E[0] // 2, 3), "layers": []}
    for l in range(cfg["n_layers"]):
        C = E[l]
        layer = {}
        if l == 0:
            mid = C * r
            layer["conv_blocks"] = []
            for _ in range(cfg["depths"][0]):
                c1, c2, c3 = conv(mid, C, 1), conv(mid, 1, 3), conv(C, mid, 1)
                mb = {}
                for i, cc in ((1, c1), (2, c2), (3, c3)):
                    mb[f"conv{i}_w"] = cc["w"]
                    for k in ("w", "b", "mean", "var"):
                        mb[f"bn{i}_{k}"] = cc[f"bn_{k}"]
                layer["conv_blocks"].append(mb)
        else:
            heads, ws = cfg["num_heads"][l], cfg["window_sizes"][l]
            layer["blocks"] = []
            for _ in range(cfg["depths"][l]):
                lc = conv(C, 1, 3)
                layer["blocks"].append({
                    "attn_norm_w": 1 + n(C), "attn_norm_b": n(C), "qkv_w": n(3 * C, C), "qkv_b": n(3 * C),
                    "proj_w": n(C, C), "proj_b": n(C), "attn_bias": n(heads, ws * ws, sc=0.5),
                    "lc_w": lc["w"], "lc_bn_w": lc["bn_w"], "lc_bn_b": lc["bn_b"],
                    "lc_bn_mean": lc["bn_mean"], "lc_bn_var": lc["bn_var"],
                    "mlp_norm_w": 1 + n(C), "mlp_norm_b": n(C), "fc1_w": n(r * C, C), "fc1_b": n(r * C),
                    "fc2_w": n(C, r * C), "fc2_b": n(C)})
        if l + 1 < cfg["n_layers"]:
            Cn = E[l + 1]
            layer["pm_conv1"] = conv(Cn, C, 1)
            layer["pm_conv2"] = conv(Cn, 1, 3)
            layer["pm_conv3"] = conv(Cn, Cn, 1)
        w["layers"].append(layer)
    emb, CL = cfg["embed_dim"], E[cfg["n_layers"] - 1]
    w["proj_conv1"] = dict(w=n(emb, 1, 1, CL))
    w["proj_bn"] = bn(emb)
    w["proj_conv2"] = dict(w=n(emb, 3, 3, emb), b=n(emb))
    return w


def tinyvit_images(cfg, n, seed=0):
    """Images normalised like the repo's preprocessing: U[0,1) -> 2p - 1."""
    rng = np.random.default_rng(seed)
    s = cfg["img_size"]
    return (rng.random((n, 3, s, s), dtype=np.float32) * 2 - 1).astype(np.float32)


# ---------------------------------------------------------------- FPN neck
SAM3_NECK = dict(d_model=256, dim=1024, grid=72, scales=(4.0, 2.0, 1.0, 0.5))


def neck_layer_dims(d_model, dim, sf):
    """(kind, c_in, c_out, k) per layer of one stage (necks.c:188-236)."""
    if sf >= 3.5:
        return [("t", dim, dim // 2, 2), ("t", dim // 2, dim // 4, 2), ("c", dim // 4, d_model, 1),
                ("c", d_model, d_model, 3)]
    if sf >= 1.5:
        return [("t", dim, dim // 2, 2), ("c", dim // 2, d_model, 1), ("c", d_model, d_model, 3)]
    return [("c", dim, d_model, 1), ("c", d_model, d_model, 3)]


def neck_weights(d_model, dim, scales, seed=0):
    """Random-init neck weights: OHWI convs ~N(0, 1/fan_in), biases ~N(0, 0.01)."""
    rng = np.random.default_rng(seed)
    w = {"w": [], "b": []}
    for sf in scales:
        ws, bs = [], []
        for kind, ci, co, k in neck_layer_dims(d_model, dim, sf):
            fan = ci * k * k
            ws.append((rng.standard_normal((co, k, k, ci)) / np.sqrt(fan)).astype(np.float32))
            bs.append((rng.standard_normal(co) * 0.01).astype(np.float32))
        w["w"].append(ws)
        w["b"].append(bs)
    return w
