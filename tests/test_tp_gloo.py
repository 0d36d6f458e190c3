"""Host logic of the single-image tensor-parallel prototype (sam3.c_b200/tp.py)
on CPU: the head / MLP sharding of a block's weights and the row-split
all-reduce reproduce the unsharded block.  Two gloo ranks each run the F32
numpy block on their shard and sum the partial proj / fc2 results with
dist.all_reduce; the result must equal the unsharded block (P = 1) to F32
rounding."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import synth
import tp

CFG = synth.tiny_cfg(depth=1, embed_dim=128, img_size=168, window_size=6, mlp_dim=320)  # 2 heads of 64


def _case():
    w = synth.vit_weights(CFG, seed=4)["blocks"][0]
    # non-trivial LayerNorm parameters
    rng = np.random.default_rng(5)
    for k in ("ln1_w", "ln2_w"):
        w[k] = (1.0 + 0.1 * rng.standard_normal(CFG["embed_dim"])).astype(np.float32)
    for k in ("ln1_b", "ln2_b"):
        w[k] = (0.1 * rng.standard_normal(CFG["embed_dim"])).astype(np.float32)
    x = rng.standard_normal((144, CFG["embed_dim"])).astype(np.float32)  # 4 windows of 36
    return w, x


def test_shards_tile_the_weights():
    w, _ = _case()
    e, heads = CFG["embed_dim"], CFG["n_heads"]
    parts = [tp.shard_block(w, r, 2, e, heads) for r in range(2)]
    # proj / fc2 columns and fc1 rows concatenate back to the full matrices
    assert np.array_equal(np.concatenate([p["proj_w"] for p in parts], 1), w["proj_w"])
    assert np.array_equal(np.concatenate([p["fc2_w"] for p in parts], 1), w["fc2_w"])
    assert np.array_equal(np.concatenate([p["fc1_w"] for p in parts], 0), w["fc1_w"])
    # each rank's QKV rows are Q, K, V of its own heads
    assert parts[1]["qkv_w"].shape == (3 * e // 2, e)
    assert np.array_equal(parts[1]["qkv_w"][: e // 2], w["qkv_w"][e // 2:e])
    assert np.array_equal(parts[1]["qkv_w"][e // 2:e], w["qkv_w"][e + e // 2:2 * e])
    assert parts[0]["proj_b"] is not None and parts[1]["proj_b"] is None
    with pytest.raises(ValueError):
        tp.shard_block(w, 0, 3, e, heads)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w, x = _case()
    e, heads = CFG["embed_dim"], CFG["n_heads"]

    def allreduce(y):
        t = torch.from_numpy(np.ascontiguousarray(y, np.float32))
        dist.all_reduce(t)
        return t.numpy()

    shard = tp.shard_block(w, rank, world, e, heads)
    out = tp.block_partial_np(x.astype(np.float64), shard, 4, 36, heads // world, e // heads, allreduce)
    q.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_match_unsharded_block():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=120) for _ in procs), key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w, x = _case()
    e, heads = CFG["embed_dim"], CFG["n_heads"]
    full = tp.block_partial_np(x.astype(np.float64), tp.shard_block(w, 0, 1, e, heads), 4, 36, heads, e // heads,
                               lambda y: y)
    for _, out in res:
        assert np.abs(out - full).max() / np.abs(full).max() < 1e-5
