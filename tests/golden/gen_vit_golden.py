"""Generate the golden fixtures of the full-size encoder parity tests.

Runs the UNMODIFIED reference sam3_vit_build on its own CPU backend
(oracle/_ref/libsam3_ref.so, built from the sam3.c sources by
oracle/Makefile) for the Hiera-L geometry at 1008 px with 8 blocks (seven
windowed, block 7 global) and with all 32 blocks (globals at 7/15/23/31,
image_encoder.c:35), seeded synthetic weights (sam3.c_b200/synth.py,
seed 11) and one seeded image (seed 12), in three weight precisions:
  f32  : the weights as generated
  bf16 : linear / patch weights rounded to bf16 (what the BF16 encoder holds)
  q8   : linear weights through sam3_q8_quantize / dequantize, patch bf16
and stores a fixed random sample of 16384 output positions per variant plus
whole-output statistics, so the fixture stays small (the full output is
21 MB).  Usage:
    python tests/golden/gen_vit_golden.py            # depth 8  (~5 min, 8 cores)
    python tests/golden/gen_vit_golden.py --depth 32 # depth 32 (~15 min, 8 cores)
writes tests/golden/vit_1008_depth<D>.npz.
"""
import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "sam3.c_b200")]

import oracle as O  # noqa: E402
import synth  # noqa: E402

W_SEED, IMG_SEED, N_SAMPLE = 11, 12, 16384


def variants(w):
    q8 = synth.round_weights(w, lambda a: O.q8_dequantize(O.q8_quantize(a), a.size).reshape(a.shape))
    q8["patch_w"] = O.round_bf16(w["patch_w"])
    return {"f32": w, "bf16": synth.round_weights(w, O.round_bf16), "q8": q8}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--depth", type=int, default=8)
    CFG = dict(synth.HIERA_L, depth=ap.parse_args().depth)
    w = synth.vit_weights(CFG, seed=W_SEED)
    img = synth.images(CFG, 1, seed=IMG_SEED)[0]
    rng = np.random.default_rng(0)
    n_out = (CFG["img_size"] // CFG["patch_size"]) ** 2 * CFG["embed_dim"]
    idx = np.sort(rng.choice(n_out, N_SAMPLE, replace=False)).astype(np.int64)
    out = {"idx": idx, "cfg": np.array([CFG[k] for k in ("img_size", "patch_size", "embed_dim", "depth",
                                                          "n_heads", "window_size", "mlp_dim")]),
           "seeds": np.array([W_SEED, IMG_SEED])}
    for name, wv in variants(w).items():
        t = time.time()
        y = O.ref_vit_encode(CFG, wv, img).ravel()
        print(f"{name}: {time.time() - t:.1f}s  max|y|={np.abs(y).max():.4f}", flush=True)
        out[f"{name}_sample"] = y[idx]
        out[f"{name}_stats"] = np.array([y.mean(), y.std(), np.abs(y).max(), float(np.abs(y).sum())])
    np.savez_compressed(os.path.join(HERE, f"vit_1008_depth{CFG['depth']}.npz"), **out)


if __name__ == "__main__":
    main()
