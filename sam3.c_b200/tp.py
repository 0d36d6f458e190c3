"""Single-image tensor parallelism of the ViT blocks (the optional split of
the north star): one image's encode spread over P GPUs, one process per GPU.

Per block, rank r of P holds
  * QKV rows of heads [r*H/P, (r+1)*H/P)  ->  Q|K|V of its heads [M, 3E/P]
    (column split: the heads' attention is local to the rank),
  * proj columns of the same heads [E, E/P] (row split of the contraction),
  * fc1 rows [r*F/P, (r+1)*F/P) and fc2 columns of the same slice,
and the two row-split linears (proj, fc2) end in an NCCL all-reduce of the
partial [M, E] sums over NVLink: rank 0 folds the bias and the residual
stream into its partial sum, so the all-reduce result is the new residual
stream.  LayerNorms are replicated.  The kernels are the library's own
(sam3cu.linear / layernorm / sdpa_packed through the C ABI); the
all-reduce is torch.distributed over NCCL, captured with the kernels in one
CUDA graph per rank.

This is a measurement prototype: the residual stream is kept in window
order (as the native encoder keeps it), RoPE and the patch embedding are
left out (identical work at any P), and `main()` times the 32 blocks of one
1008 px image at P = WORLD_SIZE against the same code at P = 1.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        sam3.c_b200/tp.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)


def head_cols(rank: int, world: int, e: int, heads: int) -> slice:
    """Columns [E] of rank's heads (head h spans h*hd .. h*hd + hd)."""
    if heads % world:
        raise ValueError(f"{heads} heads do not split over {world} ranks")
    hd = e // heads
    per = heads // world
    return slice(rank * per * hd, (rank + 1) * per * hd)


def mlp_cols(rank: int, world: int, f: int) -> slice:
    if f % world:
        raise ValueError(f"MLP width {f} does not split over {world} ranks")
    per = f // world
    return slice(rank * per, (rank + 1) * per)


def shard_block(b: dict, rank: int, world: int, e: int, heads: int) -> dict:
    """Rank's share of one block's F32 weights (synth.vit_weights layout:
    qkv_w [3E, E] with Q rows 0..E-1, K rows E..2E-1, V rows 2E..3E-1)."""
    hc = head_cols(rank, world, e, heads)
    mc = mlp_cols(rank, world, b["fc1_w"].shape[0])
    qkv_w = np.concatenate([b["qkv_w"][k * e:(k + 1) * e][hc] for k in range(3)], axis=0)
    qkv_b = np.concatenate([b["qkv_b"][k * e:(k + 1) * e][hc] for k in range(3)])
    return dict(ln1_w=b["ln1_w"], ln1_b=b["ln1_b"], ln2_w=b["ln2_w"], ln2_b=b["ln2_b"],
                qkv_w=np.ascontiguousarray(qkv_w), qkv_b=np.ascontiguousarray(qkv_b),
                proj_w=np.ascontiguousarray(b["proj_w"][:, hc]),
                proj_b=b["proj_b"] if rank == 0 else None,
                fc1_w=np.ascontiguousarray(b["fc1_w"][mc]), fc1_b=np.ascontiguousarray(b["fc1_b"][mc]),
                fc2_w=np.ascontiguousarray(b["fc2_w"][:, mc]),
                fc2_b=b["fc2_b"] if rank == 0 else None)


# ---------------------------------------------------------------- numpy model
def _ln(x, g, b):
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + 1e-5) * g + b


def _gelu(x):
    return 0.5 * x * (1.0 + np.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def _attn(qkv, groups, seq, heads, hd):
    e = heads * hd
    out = np.empty((qkv.shape[0], e), qkv.dtype)
    for g in range(groups):
        r = slice(g * seq, (g + 1) * seq)
        for h in range(heads):
            c = slice(h * hd, (h + 1) * hd)
            q, k, v = qkv[r, c], qkv[r, e:][:, c], qkv[r, 2 * e:][:, c]
            s = q @ k.T / np.sqrt(hd)
            p = np.exp(s - s.max(-1, keepdims=True))
            out[r, c] = (p / p.sum(-1, keepdims=True)) @ v
    return out


def block_partial_np(x, w, groups, seq, heads_local, hd, allreduce):
    """One block on one rank's shard in F32 numpy; `allreduce(y)` sums the
    partial [M, E] results over the ranks (identity at P = 1)."""
    xn = _ln(x, w["ln1_w"], w["ln1_b"])
    qkv = xn @ w["qkv_w"].T + w["qkv_b"]
    ao = _attn(qkv, groups, seq, heads_local, hd)
    y = ao @ w["proj_w"].T
    if w["proj_b"] is not None:
        y = y + w["proj_b"] + x
    x = allreduce(y)
    xn = _ln(x, w["ln2_w"], w["ln2_b"])
    h = _gelu(xn @ w["fc1_w"].T + w["fc1_b"])
    y = h @ w["fc2_w"].T
    if w["fc2_b"] is not None:
        y = y + w["fc2_b"] + x
    return allreduce(y)


# ---------------------------------------------------------------- device model
class TpBlocks:
    """Rank's shard of the encoder blocks on its GPU (BF16 weights, F32
    residual stream), forward through the library's kernels and NCCL."""

    def __init__(self, cfg: dict, blocks: list, rank: int, world: int, device, reduce_dtype="f32"):
        import torch
        import sam3cu
        self.cfg, self.rank, self.world, self.dev = cfg, rank, world, device
        self.sam3cu = sam3cu
        e, heads = cfg["embed_dim"], cfg["n_heads"]
        self.hd = e // heads
        self.heads_local = heads // world
        self.reduce_dtype = reduce_dtype

        def d16(a):
            return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device).bfloat16().contiguous()

        def d32(a):
            return None if a is None else torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)

        self.w = []
        for b in blocks:
            s = shard_block(b, rank, world, e, heads)
            self.w.append({k: (d16(v) if k.endswith("_w") and not k.startswith("ln") else d32(v))
                           for k, v in s.items()})

    def forward(self, x, bufs):
        """x: [M, E] F32 window-ordered residual stream, updated in place."""
        import torch
        import torch.distributed as dist
        sc = self.sam3cu
        cfg = self.cfg
        np_ = (cfg["img_size"] // cfg["patch_size"]) ** 2
        ws = cfg["window_size"]
        M = x.shape[0]
        n_img = M // np_
        for i, w in enumerate(self.w):
            glob = i % 8 == 7
            groups, seq = (n_img, np_) if glob else (M // (ws * ws), ws * ws)
            sc.layernorm(x, w["ln1_w"], w["ln1_b"], out=bufs["xn"])
            sc.linear(bufs["xn"], w["qkv_w"], bias=w["qkv_b"], out=bufs["qkv"])
            sc.sdpa_packed(bufs["qkv"], groups, seq, self.heads_local, self.hd, out=bufs["ao"])
            self._row_split(bufs["ao"], w["proj_w"], w["proj_b"], x, bufs)
            sc.layernorm(x, w["ln2_w"], w["ln2_b"], out=bufs["xn"])
            sc.linear(bufs["xn"], w["fc1_w"], bias=w["fc1_b"], act=sc.ACT_GELU_TANH, out=bufs["h"])
            self._row_split(bufs["h"], w["fc2_w"], w["fc2_b"], x, bufs)
        return x

    def _row_split(self, a, w, bias, x, bufs):
        """x <- x + bias + sum over ranks of a_r . w_r^T."""
        import torch.distributed as dist
        sc = self.sam3cu
        if self.world == 1:
            sc.linear(a, w, bias=bias, residual=x, out=x)
            return
        if self.reduce_dtype == "f32":
            # rank 0 folds bias and residual into its partial sum; the
            # all-reduce result is the new residual stream
            if self.rank == 0:
                sc.linear(a, w, bias=bias, residual=x, out=x)
            else:
                sc.linear(a, w, out=x)
            dist.all_reduce(x)
        else:  # bf16 partial sums on the wire, added to the f32 stream
            y = bufs["y16"]
            sc.linear(a, w, bias=bias, out=y)
            dist.all_reduce(y)
            x.add_(y)


def main():
    import torch
    import torch.distributed as dist
    import sam3cu
    import synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl")
    sam3cu.init(local)
    dev = torch.device("cuda", local)
    cfg = dict(synth.HIERA_L)
    w = synth.vit_weights(cfg, seed=0)
    e, f = cfg["embed_dim"], cfg["mlp_dim"]
    M = (cfg["img_size"] // cfg["patch_size"]) ** 2
    x0 = torch.from_numpy(np.random.default_rng(1).standard_normal((M, e)).astype(np.float32)).to(dev)
    results = {}
    for mode in (["f32", "bf16"] if world > 1 else ["f32"]):
        tp = TpBlocks(cfg, w["blocks"], rank, world, dev, reduce_dtype=mode)
        bufs = {"xn": torch.empty(M, e, dtype=torch.bfloat16, device=dev),
                "qkv": torch.empty(M, 3 * e // world, dtype=torch.bfloat16, device=dev),
                "ao": torch.empty(M, e // world, dtype=torch.bfloat16, device=dev),
                "h": torch.empty(M, f // world, dtype=torch.bfloat16, device=dev),
                "y16": torch.empty(M, e, dtype=torch.bfloat16, device=dev)}
        x = x0.clone()
        # eager warm-up (also the parity sample), then one CUDA graph per rank
        tp.forward(x, bufs)
        torch.cuda.synchronize()
        out_eager = x.clone()
        x.copy_(x0)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            tp.forward(x, bufs)  # warm the captured path once more
            torch.cuda.synchronize()
            x.copy_(x0)
            with torch.cuda.graph(g, stream=s):
                tp.forward(x, bufs)
        torch.cuda.synchronize()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        iters = 10
        a.record()
        for _ in range(iters):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / iters
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        # reference: the same blocks unsharded on this GPU (rank 0 only)
        ref = None
        if rank == 0:
            full = TpBlocks(cfg, w["blocks"], 0, 1, dev)
            xr = x0.clone()
            full.forward(xr, {"xn": bufs["xn"], "qkv": torch.empty(M, 3 * e, dtype=torch.bfloat16, device=dev),
                              "ao": torch.empty(M, e, dtype=torch.bfloat16, device=dev),
                              "h": torch.empty(M, f, dtype=torch.bfloat16, device=dev)})
            torch.cuda.synchronize()
            ref = float((out_eager - xr).abs().max() / xr.abs().max())
            del full
        results[mode] = {"ms_per_image_32_blocks": float(t.item()), "rel_err_vs_unsharded": ref}
        del tp, bufs, g
        torch.cuda.empty_cache()
    assert sam3cu.device_error() == 0
    if rank == 0:
        print(json.dumps({"tp": world, "workload": "32 Hiera-L blocks, 1 image 1008px (5184 tokens), BF16 "
                          "weights, F32 residual; RoPE and patch embed excluded",
                          "allreduce_bytes_per_block": {m: 2 * M * e * (4 if m == "f32" else 2) for m in results},
                          "results": results}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
