"""ctypes front end to the parity checkers.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.  The product (sam3.c_b200/, libsam3cu.so) never does.

Two libraries sit behind it, both built by oracle/Makefile:
  * ``lib/libsam3_oracle.so`` -- the C restatement in oracle/oracle.c.
  * ``_ref/libsam3_ref.so``   -- the unmodified sam3.c CPU backend compiled
    from the reference sources, plus oracle/ref_harness.c.  Present wherever
    it was built (it travels with the repository snapshot as a built file).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "lib", "libsam3_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libsam3_ref.so")

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
VP = C.c_void_p

_orc = None
_ref = None


def _p(a):
    return None if a is None else a.ctypes.data_as(VP)


def orc():
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing: run `make -C oracle`")
        _orc = C.CDLL(ORACLE_SO)
        _orc.orc_f32_to_bf16.restype = C.c_uint16
        _orc.orc_f32_to_bf16.argtypes = [C.c_float]
        _orc.orc_f32_to_fp16.restype = C.c_uint16
        _orc.orc_f32_to_fp16.argtypes = [C.c_float]
        _orc.orc_rope_table.argtypes = [C.c_int, C.c_int, C.c_int, C.c_float,
                                        C.c_float, VP, VP]
        _orc.orc_num_threads.argtypes = [C.c_int]
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"{REF_SO} missing: run `make -C oracle` "
                               "where the sam3.c sources are present")
        _ref = C.CDLL(REF_SO)
        _ref.ref_quiet()
    return _ref


def set_threads(n: int = 0) -> int:
    """Thread count for the restatement (OpenMP); 0 keeps the default."""
    return orc().orc_num_threads(n)


def ref_set_threads(n: int = 0) -> int:
    return ref().ref_set_threads(n)


# ---------------------------------------------------------------- formats
def round_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    orc().orc_round_bf16(_p(x), _p(out), C.c_int64(x.size))
    return out


def round_fp16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    orc().orc_round_fp16(_p(x), _p(out), C.c_int64(x.size))
    return out


Q8_DTYPE = np.dtype([("scale", "<f4"), ("data", "i1", (32,))])


def q8_quantize(x: np.ndarray) -> np.ndarray:
    """Q8_0 blocks (36 bytes each) over the flattened tensor."""
    x = np.ascontiguousarray(x, np.float32)
    nb = (x.size + 31) // 32
    out = np.zeros(nb, Q8_DTYPE)
    orc().orc_q8_quantize(_p(x), _p(out), C.c_int64(x.size))
    return out


def q8_dequantize(q: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    orc().orc_q8_dequantize(_p(q), _p(out), C.c_int64(n))
    return out


# ---------------------------------------------------------------- ops
def linear(x, w, b=None, res=None, act=0):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), np.float32)
    if b is not None:
        b = np.ascontiguousarray(b, np.float32)
    if res is not None:
        res = np.ascontiguousarray(res, np.float32)
    orc().orc_linear(_p(x), _p(w), _p(b), _p(res), _p(y), M, K, N, act)
    return y


def layernorm(x, g=None, b=None):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    orc().orc_layernorm(_p(x), _p(g), _p(b), _p(y), rows, cols)
    return y


def gelu(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    orc().orc_gelu(_p(x), _p(y), C.c_int64(x.size))
    return y


def rope_table(n_pos, grid_w, head_dim, scale, theta=10000.0):
    cs = np.empty((n_pos, head_dim // 2), np.float32)
    sn = np.empty_like(cs)
    orc().orc_rope_table(n_pos, grid_w, head_dim, scale, theta, _p(cs), _p(sn))
    return cs, sn


def rope(x, cs, sn):
    """x: [batch, seq, heads, hd]."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    B, S, H, D = x.shape
    orc().orc_rope(_p(x), _p(cs), _p(sn), _p(y), B, S, H, D)
    return y


def sdpa(q, k, v):
    """q/k/v: [BH, S, hd] (any leading dims flattened)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    S, D = q.shape[-2:]
    BH = q.size // (S * D)
    o = np.empty_like(q)
    orc().orc_sdpa(_p(q), _p(k), _p(v), _p(o), BH, S, D)
    return o


# ---------------------------------------------------------------- ViT
class _Blk(C.Structure):
    _fields_ = [(n, VP) for n in ("ln1_w", "ln1_b", "qkv_w", "qkv_b", "proj_w",
                                  "proj_b", "ln2_w", "ln2_b", "fc1_w", "fc1_b",
                                  "fc2_w", "fc2_b")]


class _VitW(C.Structure):
    _fields_ = [(n, VP) for n in ("patch_w", "patch_b", "pos_raw", "ln_pre_w",
                                  "ln_pre_b")] + [("blocks", _Blk * 32)]


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("img_size", "patch_size", "embed_dim",
                                       "depth", "n_heads", "window_size",
                                       "mlp_dim")]


BLOCK_KEYS = ("ln1_w", "ln1_b", "qkv_w", "qkv_b", "proj_w", "proj_b", "ln2_w",
              "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")


def _vit_struct(w):
    s = _VitW()
    keep = []
    for n in ("patch_w", "patch_b", "pos_raw", "ln_pre_w", "ln_pre_b"):
        a = np.ascontiguousarray(w[n], np.float32)
        keep.append(a)
        setattr(s, n, a.ctypes.data)
    for i, blk in enumerate(w["blocks"]):
        for n in BLOCK_KEYS:
            a = np.ascontiguousarray(blk[n], np.float32)
            keep.append(a)
            setattr(s.blocks[i], n, a.ctypes.data)
    return s, keep


def vit_forward(cfg: dict, w: dict, image: np.ndarray) -> np.ndarray:
    """Restated sam3_vit_build forward; image CHW F32 normalised."""
    gs = cfg["img_size"] // cfg["patch_size"]
    out = np.empty((gs * gs, cfg["embed_dim"]), np.float32)
    s, keep = _vit_struct(w)
    c = _Cfg(*(cfg[k] for k in ("img_size", "patch_size", "embed_dim", "depth",
                                "n_heads", "window_size", "mlp_dim")))
    image = np.ascontiguousarray(image, np.float32)
    orc().orc_vit_forward(C.byref(c), C.byref(s), _p(image), _p(out))
    del keep
    return out


# ---------------------------------------------------------------- reference
def ref_matmul(a, b, dt="f32"):
    """C = A[M,K] . B[K,N] with the reference kernel; dt f32|f16|bf16.

    For f16/bf16 pass uint16 bit patterns; returns the same dtype."""
    M, K = a.shape
    N = b.shape[1]
    code = {"f32": 0, "f16": 1, "bf16": 2}[dt]
    out = np.empty((M, N), np.float32 if code == 0 else np.uint16)
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    rc = ref().ref_matmul(code, _p(a), _p(b), _p(out), M, K, N)
    assert rc == 0, rc
    return out


def ref_matmul_q8(a, bq, K, N):
    a = np.ascontiguousarray(a, np.float32)
    M = a.shape[0]
    out = np.empty((M, N), np.float32)
    rc = ref().ref_matmul_q8(_p(a), _p(bq), _p(out), M, K, N)
    assert rc == 0, rc
    return out


def ref_q8_quantize(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros((x.size + 31) // 32, Q8_DTYPE)
    ref().ref_q8_quantize(_p(x), _p(out), x.size)
    return out


def ref_gelu(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    assert ref().ref_gelu(_p(x), _p(y), x.size) == 0
    return y


def ref_layernorm(x, g=None, b=None):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    assert ref().ref_layernorm(_p(x), _p(g), _p(b), _p(y), rows, cols) == 0
    return y


def ref_rope(x, cs, sn):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    B, S, H, D = x.shape
    assert ref().ref_rope(_p(x), _p(cs), _p(sn), _p(y), B, S, H, D) == 0
    return y


def ref_sdpa(q, k, v):
    """q/k/v [B, H, S, hd]."""
    q, k, v = (np.ascontiguousarray(t, np.float32) for t in (q, k, v))
    B, H, S, D = q.shape
    o = np.empty_like(q)
    assert ref().ref_sdpa(_p(q), _p(k), _p(v), _p(o), B, H, S, D) == 0
    return o


def ref_vit_encode_backend(cfg: dict, w: dict, image: np.ndarray, ops: int, be_size: int,
                           be_type: int = 2) -> np.ndarray:
    """The reference's own sam3_vit_build evaluated through another backend's
    vtable (ops = address of its struct sam3_backend_ops)."""
    gs = cfg["img_size"] // cfg["patch_size"]
    out = np.empty((gs * gs, cfg["embed_dim"]), np.float32)
    s, keep = _vit_struct(w)
    image = np.ascontiguousarray(image, np.float32)
    rc = ref().ref_vit_encode_backend(*(C.c_int(cfg[k]) for k in (
        "img_size", "patch_size", "embed_dim", "depth", "n_heads",
        "window_size", "mlp_dim")), C.byref(s), _p(image), _p(out), C.c_void_p(ops),
        C.c_size_t(be_size), C.c_int(be_type))
    del keep
    if rc != 0:
        raise RuntimeError(f"ref_vit_encode_backend failed rc={rc}")
    return out


DT = {"f32": 0, "f16": 1, "bf16": 2, "q8": 5}


def _bits(a, dt):
    """float32 array -> storage array of the reference dtype (bit patterns)."""
    if dt == "f32":
        return np.ascontiguousarray(a, np.float32)
    if dt == "bf16":
        return (np.ascontiguousarray(round_bf16(a)).view(np.uint32) >> 16).astype(np.uint16)
    if dt == "f16":
        return np.ascontiguousarray(a, np.float32).astype(np.float16).view(np.uint16)
    raise ValueError(dt)


def _unbits(a, dt):
    if dt == "f32":
        return a
    if dt == "bf16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.view(np.float16).astype(np.float32)


def ref_linear_graph(x, w, b, dt="f32", gelu=False, ops=None, be_size=0, be_type=2):
    """gh_linear (+GELU) graph built by the reference helpers, evaluated by
    the reference CPU backend (ops None) or another backend."""
    M, K = x.shape
    N = w.shape[0]
    xs, ws = _bits(x, dt), _bits(w, dt)
    bs = None if b is None else _bits(b, dt)
    out = np.empty((M, N), np.float32 if dt == "f32" else np.uint16)
    rc = ref().ref_linear_graph(DT[dt], _p(xs), _p(ws), _p(bs), _p(out), M, K, N,
                                1 if gelu else 0, C.c_void_p(ops), C.c_size_t(be_size),
                                C.c_int(be_type))
    if rc != 0:
        raise RuntimeError(f"ref_linear_graph failed rc={rc}")
    return _unbits(out, dt)


class _TDesc(C.Structure):
    _fields_ = [("dtype", C.c_int), ("n_dims", C.c_int), ("dims", C.c_int * 4),
                ("data", C.c_void_p)]


def ref_node_graph(op, ins, out_dtype, out_shape, params=(0, 0, 0, 0), ops=None, be_size=0,
                   be_type=2):
    """Single-node graph; ins: list of (storage array, dtype name, shape)."""
    if len(ins) > 6:
        raise ValueError("at most 6 inputs")
    descs = (_TDesc * 6)()
    keep = []
    for i, (arr, dt, shp) in enumerate(ins):
        a = np.ascontiguousarray(arr)
        keep.append(a)
        descs[i].dtype = DT[dt]
        descs[i].n_dims = len(shp)
        for j, d in enumerate(shp):
            descs[i].dims[j] = d
        descs[i].data = a.ctypes.data
    od = _TDesc()
    od.dtype = DT[out_dtype]
    od.n_dims = len(out_shape)
    for j, d in enumerate(out_shape):
        od.dims[j] = d
    out = np.empty(out_shape, np.float32 if out_dtype == "f32" else np.uint16)
    prm = (C.c_int * 4)(*params)
    rc = ref().ref_node_graph(op, len(ins), descs, C.byref(od), _p(out), prm, C.c_void_p(ops),
                              C.c_size_t(be_size), C.c_int(be_type))
    del keep
    if rc != 0:
        raise RuntimeError(f"ref_node_graph(op={op}) failed rc={rc}")
    return _unbits(out, out_dtype)


OP = dict(MATMUL=1, ADD=2, MUL=3, SOFTMAX=4, GELU=6, LAYERNORM=7, CONV2D=8, RESHAPE=9,
          TRANSPOSE=10, CAST=11, SLICE=13, ROPE=17, SDPA=21, BIAS_ADD=22, BATCHNORM=24)


def ref_vit_encode(cfg: dict, w: dict, image: np.ndarray) -> np.ndarray:
    gs = cfg["img_size"] // cfg["patch_size"]
    out = np.empty((gs * gs, cfg["embed_dim"]), np.float32)
    s, keep = _vit_struct(w)
    image = np.ascontiguousarray(image, np.float32)
    rc = ref().ref_vit_encode(*(C.c_int(cfg[k]) for k in (
        "img_size", "patch_size", "embed_dim", "depth", "n_heads",
        "window_size", "mlp_dim")), C.byref(s), _p(image), _p(out))
    del keep
    if rc != 0:
        raise RuntimeError(f"ref_vit_encode failed rc={rc}")
    return out


# ---------------------------------------------------------------- TinyViT
def tvit_n_offsets(ws: int) -> int:
    """Distinct (|dy|, |dx|) offsets of a ws x ws window."""
    return ws * ws


def tvit_expand_bias(compact: np.ndarray, ws: int) -> np.ndarray:
    """Restatement of expand_attention_bias: [heads, n_off] -> [heads, N, N]."""
    compact = np.ascontiguousarray(compact, np.float32)
    heads, n_off = compact.shape
    out = np.empty((heads, ws * ws, ws * ws), np.float32)
    n = orc().orc_tvit_expand_bias(_p(compact), heads, n_off, ws, _p(out))
    if n != n_off:
        raise ValueError(f"{n} offsets for ws={ws}, table has {n_off}")
    return out


def ref_tvit_expand_bias(compact: np.ndarray, ws: int) -> np.ndarray:
    """The reference's own expand_attention_bias (compiled from its source)."""
    compact = np.ascontiguousarray(compact, np.float32)
    heads, n_off = compact.shape
    out = np.empty((heads, ws * ws, ws * ws), np.float32)
    if ref().ref_tvit_expand_bias(_p(compact), heads, n_off, ws, _p(out)) != 0:
        raise RuntimeError("ref_tvit_expand_bias failed")
    return out


def tvit_window_attention(qkv: np.ndarray, nw: int, N: int, heads: int, hd: int,
                          bias: np.ndarray | None) -> np.ndarray:
    """Restatement of tvit_window_attention after the qkv linear."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    out = np.empty((nw * N, heads * hd), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    orc().orc_tvit_window_attention(_p(qkv), nw, N, heads, hd, _p(b), _p(out))
    return out


def ref_tvit_window_attention(qkv: np.ndarray, nw: int, N: int, heads: int, hd: int,
                              bias: np.ndarray | None) -> np.ndarray:
    """tvit_window_attention evaluated by the reference CPU kernels, one
    (window, head) slice at a time (the CPU MATMUL is 2-D only): MUL by the
    [1] scale tensor, TRANSPOSE, MATMUL, ADD bias, SOFTMAX, MATMUL.  The
    reshape / slice / permute nodes are exact copies, done here in numpy."""
    C = heads * hd
    x = np.ascontiguousarray(qkv, np.float32).reshape(nw, N, heads, 3 * hd)
    scale = np.array([1.0 / np.sqrt(np.float32(hd))], np.float32)
    out = np.empty((nw, N, heads, hd), np.float32)
    for w in range(nw):
        for h in range(heads):
            q = np.ascontiguousarray(x[w, :, h, :hd])
            k = np.ascontiguousarray(x[w, :, h, hd:2 * hd])
            v = np.ascontiguousarray(x[w, :, h, 2 * hd:])
            qs = ref_node_graph(OP["MUL"], [(q, "f32", (N, hd)), (scale, "f32", (1,))], "f32",
                                (N, hd))
            kt = ref_node_graph(OP["TRANSPOSE"], [(k, "f32", (N, hd))], "f32", (hd, N),
                                params=(1, 0, 0, 0))
            s = ref_node_graph(OP["MATMUL"], [(qs, "f32", (N, hd)), (kt, "f32", (hd, N))], "f32",
                               (N, N))
            if bias is not None:
                s = ref_node_graph(OP["ADD"], [(s, "f32", (N, N)),
                                               (np.ascontiguousarray(bias[h]), "f32", (N, N))],
                                   "f32", (N, N))
            p = ref_node_graph(OP["SOFTMAX"], [(s, "f32", (N, N))], "f32", (N, N))
            out[w, :, h] = ref_node_graph(OP["MATMUL"], [(p, "f32", (N, N)), (v, "f32", (N, hd))],
                                          "f32", (N, hd))
    return out.reshape(nw * N, C)


def dwconv3x3_bn(x: np.ndarray, w: np.ndarray, cb=None, bn=None, gelu=False) -> np.ndarray:
    """Restatement of a depthwise 3x3 tvit_conv_bn on NHWC x [B, H, W, C];
    w [C, 3, 3, 1]; bn = (gamma, beta, mean, var) or None."""
    x = np.ascontiguousarray(x, np.float32)
    B, H, W, Cc = x.shape
    y = np.empty_like(x)
    g = b = m = v = None
    if bn is not None:
        g, b, m, v = (np.ascontiguousarray(t, np.float32) for t in bn)
    wc = np.ascontiguousarray(w, np.float32)
    cbc = None if cb is None else np.ascontiguousarray(cb, np.float32)
    orc().orc_dwconv3x3_bn(_p(x), B, H, W, Cc, _p(wc), _p(cbc), _p(g), _p(b), _p(m), _p(v),
                           1 if gelu else 0, _p(y))
    return y


def ref_dwconv3x3_bn(x: np.ndarray, w: np.ndarray, cb=None, bn=None) -> np.ndarray:
    """The reference CONV2D (groups = C, stride 1, pad 1), BIAS_ADD and
    BATCHNORM kernels on the same inputs, as gh_conv2d + gh_batchnorm chain
    them (graph_helpers.c:1360-1395, image_encoder_tinyvit.c:655-674)."""
    x = np.ascontiguousarray(x, np.float32)
    B, H, W, Cc = x.shape
    ins = [(x, "f32", (B, H, W, Cc)), (np.ascontiguousarray(w, np.float32), "f32", (Cc, 3, 3, 1))]
    y = ref_node_graph(OP["CONV2D"], ins, "f32", (B, H, W, Cc), params=(1, 1, Cc, 0))
    if cb is not None:  # gh_conv2d adds the conv bias as a BIAS_ADD node (graph_helpers.c:1392)
        y = ref_node_graph(OP["BIAS_ADD"], [(y, "f32", (B, H, W, Cc)),
                                             (np.ascontiguousarray(cb, np.float32), "f32", (Cc,))],
                           "f32", (B, H, W, Cc))
    if bn is not None:
        g, b, m, v = (np.ascontiguousarray(t, np.float32) for t in bn)
        y = ref_node_graph(OP["BATCHNORM"], [(y, "f32", (B, H, W, Cc)), (g, "f32", (Cc,)),
                                              (b, "f32", (Cc,)), (m, "f32", (Cc,)),
                                              (v, "f32", (Cc,))], "f32", (B, H, W, Cc))
    return y


TVIT_BLOCK_KEYS = ("attn_norm_w", "attn_norm_b", "qkv_w", "qkv_b", "proj_w", "proj_b",
                   "attn_bias", "lc_w", "lc_b", "lc_bn_w", "lc_bn_b", "lc_bn_mean", "lc_bn_var",
                   "mlp_norm_w", "mlp_norm_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")


class _TvitBlk(C.Structure):
    _fields_ = [(n, VP) for n in TVIT_BLOCK_KEYS]


def tvit_block_forward(w: dict, x: np.ndarray, heads: int, ws: int) -> np.ndarray:
    """Restatement of tvit_block_forward on one NHWC image x [H, W, C];
    w['attn_bias'] is the expanded [heads, N, N] table."""
    x = np.array(x, np.float32, copy=True, order="C")
    H, W, Cc = x.shape
    s = _TvitBlk()
    keep = []
    for n in TVIT_BLOCK_KEYS:
        if w.get(n) is None:
            setattr(s, n, None)
            continue
        a = np.ascontiguousarray(w[n], np.float32)
        keep.append(a)
        setattr(s, n, a.ctypes.data)
    mlp = w["fc1_w"].shape[0]
    orc().orc_tvit_block_forward(C.byref(s), _p(x), H, W, Cc, heads, ws, mlp)
    del keep
    return x


TVIT_MBCONV_KEYS = tuple(f"{c}{i}_{k}" if c == "bn" else f"conv{i}_{k}"
                         for i in (1, 2, 3) for c, ks in (("conv", ("w", "b")),
                                                          ("bn", ("w", "b", "mean", "var")))
                         for k in ks)


class _TvitMb(C.Structure):
    _fields_ = [(n, VP) for n in TVIT_MBCONV_KEYS]


def tvit_mbconv_forward(w: dict, x: np.ndarray) -> np.ndarray:
    """Restatement of tvit_mbconv_forward on NHWC x [B, H, W, C]."""
    x = np.array(x, np.float32, copy=True, order="C")
    B, H, W, Cc = x.shape
    s = _TvitMb()
    keep = []
    for n in TVIT_MBCONV_KEYS:
        if w.get(n) is None:
            setattr(s, n, None)
            continue
        a = np.ascontiguousarray(w[n], np.float32)
        keep.append(a)
        setattr(s, n, a.ctypes.data)
    mid = w["conv1_w"].shape[0]
    orc().orc_tvit_mbconv_forward(C.byref(s), _p(x), B, H, W, Cc, mid)
    del keep
    return x


def tinyvit_forward(cfg_struct, weights_struct, image: np.ndarray) -> np.ndarray:
    """Restatement of sam3_tinyvit_build for one image [3, S, S]; the
    ctypes structs have the CUDA library's layouts (the test builds them
    with sam3cu.tinyvit_structs).  Returns [grid*grid, embed_dim]."""
    image = np.ascontiguousarray(image, np.float32)
    S = cfg_struct.img_size
    g = (S - 1) // 2 + 1
    g = (g - 1) // 2 + 1
    for _ in range(cfg_struct.n_layers - 1):
        g = (g - 1) // 2 + 1
    out = np.empty((g * g, cfg_struct.embed_dim), np.float32)
    got = orc().orc_tinyvit_forward(C.byref(cfg_struct), C.byref(weights_struct), _p(image), _p(out))
    assert got == g
    return out


def ref_tinyvit_encode(cfg_struct, weights_struct, image: np.ndarray, ops=None, be_size=0, be_type=2):
    """The reference's own sam3_tinyvit_build (image_encoder_tinyvit.c,
    compiled from source into oracle/_ref) evaluated by a backend: `ops`
    None is the reference CPU backend (which lacks the batched MATMUL the
    graph needs), else a struct sam3_backend_ops address such as the CUDA
    backend's.  Weight structs as for tinyvit_forward."""
    image = np.ascontiguousarray(image, np.float32)
    S = cfg_struct.img_size
    g = (S - 1) // 2 + 1
    g = (g - 1) // 2 + 1
    for _ in range(cfg_struct.n_layers - 1):
        g = (g - 1) // 2 + 1
    out = np.empty((g * g, cfg_struct.embed_dim), np.float32)
    rc = ref().ref_tinyvit_encode(C.byref(cfg_struct), C.byref(weights_struct), _p(image), _p(out),
                                  C.c_void_p(ops), C.c_size_t(be_size), C.c_int(be_type))
    if rc != 0:
        raise RuntimeError(f"ref_tinyvit_encode failed rc={rc}")
    return out


# ---------------------------------------------------------------- FPN neck
def _neck_ptrs(w: dict):
    """(w, b) -> two [4*4] pointer arrays (stage-major, layer-minor)."""
    W = (VP * 16)()
    B = (VP * 16)()
    keep = []
    for i, layers in enumerate(w["w"]):
        for j, a in enumerate(layers):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            W[i * 4 + j] = a.ctypes.data
            bb = np.ascontiguousarray(w["b"][i][j], np.float32)
            keep.append(bb)
            B[i * 4 + j] = bb.ctypes.data
    return W, B, keep


def neck_out_sizes(grid, scales):
    out = []
    for sf in scales:
        if sf >= 3.5:
            out.append(grid * 4)
        elif sf >= 1.5:
            out.append(grid * 2)
        elif sf >= 0.75:
            out.append(grid)
        else:
            out.append((grid - 2) // 2 + 1)
    return out


def neck_forward(d_model, dim, grid, scales, w: dict, feat: np.ndarray):
    """Restatement of sam3_neck_build: feat [grid*grid, dim] -> list of
    [H_i, H_i, d_model] arrays."""
    feat = np.ascontiguousarray(feat, np.float32)
    W, B, keep = _neck_ptrs(w)
    sizes = neck_out_sizes(grid, scales)
    outs = [np.empty((h, h, d_model), np.float32) for h in sizes]
    optr = (VP * 4)(*[o.ctypes.data for o in outs])
    sc = np.ascontiguousarray(scales, np.float32)
    orc().orc_neck_forward(d_model, dim, grid, len(scales), _p(sc), W, B, _p(feat), optr)
    return outs


def ref_neck(d_model, dim, grid, scales, w: dict, feat: np.ndarray, ops=None, be_size=0, be_type=2):
    """The reference's own sam3_neck_build (necks.c, compiled from source)
    evaluated by a backend (ops None: the reference CPU backend)."""
    feat = np.ascontiguousarray(feat, np.float32)
    W, B, keep = _neck_ptrs(w)
    sizes = neck_out_sizes(grid, scales)
    outs = [np.empty((h, h, d_model), np.float32) for h in sizes]
    optr = (VP * 4)(*[o.ctypes.data for o in outs])
    sc = np.ascontiguousarray(scales, np.float32)
    WB = (VP * 32)(*(list(W) + list(B)))  # struct rn_weights {w[4][4]; b[4][4];}
    rc = ref().ref_neck_run(d_model, dim, grid, len(scales), _p(sc), C.byref(WB), _p(feat), optr,
                            C.c_void_p(ops), C.c_size_t(be_size), C.c_int(be_type))
    if rc != 0:
        raise RuntimeError(f"ref_neck_run failed rc={rc}")
    return outs


# ---------------------------------------------------------------- .sam3 files
class _RwTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("n_dims", C.c_int),
                ("dims", C.c_int * 4), ("data", VP)]


def ref_write_sam3(path: str, tensors, quantize: bool = False, image_size: int = 0,
                   encoder_dim: int = 0, n_layers: int = 0) -> None:
    """Write a .sam3 file with the reference's own sam3_weight_write
    (weight.c:64-236).  tensors: (name, array[, dtype]) with float32 arrays
    (dtype F32) or uint16 bit patterns (dtype 1 F16 / 2 BF16).  quantize:
    the converter's Q8_0 rule (cli_convert.c:340-425)."""
    keep = []
    arr = (_RwTensor * len(tensors))()
    for i, item in enumerate(tensors):
        name, a = item[0], item[1]
        dt = item[2] if len(item) > 2 else 0
        a = np.ascontiguousarray(a, np.float32 if dt == 0 else np.uint16)
        nm = name.encode()
        keep += [a, nm]
        arr[i].name, arr[i].dtype, arr[i].n_dims = nm, dt, a.ndim
        for d in range(a.ndim):
            arr[i].dims[d] = a.shape[d]
        arr[i].data = a.ctypes.data
    rc = ref().ref_write_sam3(path.encode(), arr, len(tensors), int(quantize), image_size,
                              encoder_dim, n_layers)
    if rc != 0:
        raise RuntimeError(f"sam3_weight_write failed rc={rc}")


def ref_find_sam3(path: str, name: str):
    """sam3_weight_open + sam3_weight_find: dict like sam3cu.sam3_find, None
    if absent; raises with the sam3_error of a file the reference rejects."""
    dt, nd = C.c_int(0), C.c_int(0)
    dims = (C.c_int * 4)()
    off, nb = C.c_ulonglong(0), C.c_ulonglong(0)
    rc = ref().ref_find_sam3(path.encode(), name.encode(), C.byref(dt), C.byref(nd), dims,
                             C.byref(off), C.byref(nb))
    if rc == 1:
        return None
    if rc != 0:
        raise RuntimeError(f"sam3_weight_open failed rc={rc}")
    return dict(dtype=dt.value, dims=tuple(dims[i] for i in range(nd.value)), offset=off.value,
                nbytes=nb.value)


def ref_open_sam3(path: str) -> int:
    """sam3_weight_open's status (enum sam3_error) for a file."""
    return ref().ref_open_sam3(path.encode())


def ref_vit_encode_file(path: str, cfg: dict, image: np.ndarray) -> np.ndarray:
    """The reference encoder loaded from a .sam3 file the way an application
    loads it (sam3_weight_open, sam3_vit_load with the file, sam3_vit_build on
    the CPU backend)."""
    image = np.ascontiguousarray(image, np.float32)
    gs = cfg["img_size"] // cfg["patch_size"]
    out = np.empty((gs * gs, cfg["embed_dim"]), np.float32)
    rc = ref().ref_vit_encode_file(path.encode(), cfg["img_size"], cfg["patch_size"], cfg["embed_dim"],
                                   cfg["depth"], cfg["n_heads"], cfg["window_size"], cfg["mlp_dim"],
                                   _p(image), _p(out))
    if rc != 0:
        raise RuntimeError(f"ref_vit_encode_file failed rc={rc}")
    return out
