"""Generates tests/golden/*.npz by running the reference's own Python code.

JAX/Flax are not installed here, so the reference modules cannot be imported
as a whole. Instead this script reads the reference sources, extracts the
functions on the attention hot path with `ast`, and executes them unchanged
in a namespace where `jax` / `jnp` are a small numpy shim:

* src/vidax/models/ltx2_5/diffusion_vae.py: `_window_start`, `_gather_window`,
  `neighborhood_attention_3d` (lines 152-234);
* src/vidax/core/attention.py: `chunk_by_rank`, `local_attention`,
  `dot_product_attention`, `sequence_parallel_self_attention`,
  `sequence_parallel_joint_self_attention` (lines 132-146, 321-533), run on
  P threads (one per emulated device) whose `jax.lax.all_to_all` /
  `all_gather` / `axis_index` meet at a barrier;
* src/vidax/core/rope3d.py: `_axis_freqs`, `create_rope3d_freqs`,
  `apply_rope3d` (lines 33-111);
* src/vidax/core/attention.py: `RMSNorm.__call__` (lines 149-162), run as a
  plain function on a stand-in module object;
* src/vidax/core/rope3d.py: `sinusoidal_embedding_1d` (lines 15-30);
* src/vidax/models/ltx2_5/diffusion_vae.py: `_default_rope_dim_split`,
  `_rope_inv_freqs`, `_apply_abs_rope_axis`, `_apply_abs_rope` (lines
  96-150), and `NeighborhoodAttention3D.__call__` (lines 252-284) with its
  Dense layers replaced by given projections.

The shim restates the third-party jax primitives the code calls: `jnp.take`,
`jnp.moveaxis`, `jnp.einsum` (bf16 operands, f32 accumulation, result in the
operand dtype, as XLA does), `jax.nn.softmax`, `jax.lax.scan`, `jax.vmap`,
`jax.lax.all_to_all(tiled=True)`, and `jax.nn.dot_product_attention` (f32
logits, f32 softmax, weights cast to the input dtype, bf16 einsum). The
vidax code around them -- window starts, gather indices, key ordering, the
scan/vmap structure, dtype handling, dispatch, default scale and the Ulysses
split/concat axes -- is the reference's own.

Run from the repository root with the path of a vidax checkout:
    python tests/golden/make_golden.py <path-to-vidax>
The fixtures are committed; tests only read them (the reference checkout is
not needed to run the tests).
"""
from __future__ import annotations

import ast
import os
import sys
import threading
import types

import ml_dtypes
import numpy as np

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("VIDAX_REFERENCE", "")
OUT_DIR = os.path.dirname(os.path.abspath(__file__))
BF16 = ml_dtypes.bfloat16


# ----------------------------------------------------------------- jax shim
def _einsum(spec, *ops, **kw):
    dt = np.result_type(*[o.dtype for o in ops])
    res = np.einsum(spec, *[np.asarray(o, np.float32) for o in ops], optimize=True)
    return res.astype(dt)


def _softmax(x, axis=-1):
    x = np.asarray(x)
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(x.dtype)


def _scan(f, init, xs):
    n = len(xs[0]) if isinstance(xs, (tuple, list)) else len(xs)
    carry, ys = init, []
    for i in range(n):
        x_i = tuple(x[i] for x in xs) if isinstance(xs, (tuple, list)) else xs[i]
        carry, y = f(carry, x_i)
        ys.append(y)
    return carry, np.stack(ys)


def _vmap(f, in_axes=0, out_axes=0):
    def g(x):
        outs = [f(np.take(x, i, axis=in_axes)) for i in range(x.shape[in_axes])]
        return np.stack(outs, axis=out_axes)
    return g


def _dot_product_attention(q, k, v, bias=None, mask=None, scale=None, **kw):
    dt = q.dtype
    D = q.shape[-1]
    scale = D ** -0.5 if scale is None else scale
    logits = np.einsum("btnh,bsnh->bnts", np.asarray(q, np.float32), np.asarray(k, np.float32))
    logits = logits * np.float32(scale)
    if bias is not None:
        logits = logits + np.asarray(bias, np.float32)
    if mask is not None:
        logits = np.where(mask, logits, np.float32(-0.7 * np.finfo(np.float32).max))
    p = _softmax(logits.astype(np.float32), axis=-1).astype(dt)
    out = np.einsum("bnts,bsnh->btnh", np.asarray(p, np.float32), np.asarray(v, np.float32))
    return out.astype(dt)


class _Device:
    platform = "cpu"
    device_kind = "cpu"


class _Collective:
    """Thread-per-device stand-in for a mesh axis: all_to_all / axis_index."""

    def __init__(self, P):
        self.P = P
        self.barrier = threading.Barrier(P)
        self.slots = [None] * P
        self.local = threading.local()

    def axis_index(self, name):
        return self.local.rank

    def all_to_all(self, x, axis_name, split_axis, concat_axis, tiled=False):
        assert tiled
        r = self.local.rank
        self.slots[r] = np.split(np.asarray(x), self.P, axis=split_axis)
        self.barrier.wait()
        res = np.concatenate([self.slots[src][r] for src in range(self.P)], axis=concat_axis)
        self.barrier.wait()
        return res

    def all_gather(self, x, axis_name, axis, tiled=False):
        assert tiled
        r = self.local.rank
        self.slots[r] = np.asarray(x)
        self.barrier.wait()
        res = np.concatenate([self.slots[src] for src in range(self.P)], axis=axis)
        self.barrier.wait()
        return res

    def dynamic_slice_in_dim(self, x, start, size, axis=0):
        return np.take(x, np.arange(int(start), int(start) + size), axis=axis)


def make_namespace(coll=None):
    jnp = types.SimpleNamespace(
        take=lambda a, idx, axis=None: np.take(a, np.asarray(idx), axis=axis),
        moveaxis=np.moveaxis, asarray=np.asarray, einsum=_einsum,
        promote_types=np.promote_types, float32=np.float32, bfloat16=BF16,
        ndarray=np.ndarray, pad=np.pad, where=np.where, arange=np.arange,
        broadcast_to=np.broadcast_to, transpose=np.transpose, concatenate=np.concatenate)
    lax = types.SimpleNamespace(scan=_scan)
    if coll is not None:
        lax.all_to_all = coll.all_to_all
        lax.all_gather = coll.all_gather
        lax.axis_index = coll.axis_index
        lax.dynamic_slice_in_dim = coll.dynamic_slice_in_dim
    else:
        lax.dynamic_slice_in_dim = lambda x, s, n, axis=0: np.take(
            x, np.arange(int(s), int(s) + n), axis=axis)
    jax = types.SimpleNamespace(
        lax=lax, vmap=_vmap, nn=types.SimpleNamespace(
            softmax=_softmax, dot_product_attention=_dot_product_attention),
        devices=lambda: [_Device()], device_count=lambda: 1)
    from typing import Optional, Tuple
    return {"jax": jax, "jnp": jnp, "np": np, "Optional": Optional, "Tuple": Tuple,
            "Mesh": object, "P": lambda *a: a}


def load_functions(relpath, names, ns):
    path = os.path.join(REF, relpath)
    src = open(path).read()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            seg = ast.get_source_segment(src, node)
            exec(compile("\n" * (node.lineno - 1) + seg, path, "exec"), ns)
    missing = [n for n in names if n not in ns]
    if missing:
        raise RuntimeError(f"functions {missing} not found in {path}")
    return ns


# ----------------------------------------------------------------- fixtures
def seeded(shape, seed, scale=None):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal(shape, dtype=np.float32)
    if scale is not None:
        x = x * np.float32(scale)
    return x.astype(BF16)


def gen_na3d():
    ns = load_functions("src/vidax/models/ltx2_5/diffusion_vae.py",
                        ["_window_start", "_gather_window", "neighborhood_attention_3d"],
                        make_namespace())
    out = {}
    # window starts for every (length, kernel) in a grid of small sizes
    lens, kers, starts = [], [], []
    for L in range(1, 40):
        for kk in range(1, 14):
            s = np.asarray(ns["_window_start"](L, kk), np.int64)
            lens.append(L)
            kers.append(kk)
            starts.append(np.pad(s, (0, 40 - L), constant_values=-1))
    out["ws_length"] = np.array(lens, np.int32)
    out["ws_kernel"] = np.array(kers, np.int32)
    out["ws_start"] = np.array(starts, np.int32)
    cases = [((1, 3, 5, 7, 2, 16), (3, 3, 5)), ((1, 4, 6, 9, 1, 32), (3, 5, 5)),
             ((2, 2, 3, 4, 1, 8), (5, 9, 9)), ((1, 5, 4, 6, 2, 16), (3, 7, 7)),
             ((1, 3, 5, 9, 2, 128), (3, 3, 5)), ((1, 4, 7, 10, 1, 128), (5, 9, 9)),
             # head_dim 64 with LTX-2.5's decoder windows (diffusion_vae.py:547-553);
             # T = 2 < kt clamps the time window to the whole grid
             ((1, 4, 6, 10, 2, 64), (3, 5, 5)), ((1, 2, 9, 9, 1, 64), (3, 7, 7))]
    for i, (shape, kernel) in enumerate(cases):
        q = seeded(shape, 40 + i, scale=shape[-1] ** -0.5)
        k = seeded(shape, 50 + i)
        v = seeded(shape, 60 + i)
        o = ns["neighborhood_attention_3d"](q, k, v, kernel)
        assert o.dtype == BF16 and o.shape == shape
        out[f"na{i}_q"], out[f"na{i}_k"], out[f"na{i}_v"] = (x.astype(np.float32) for x in (q, k, v))
        out[f"na{i}_o"] = o.astype(np.float32)
        out[f"na{i}_kernel"] = np.array(kernel, np.int32)
    return out


def gen_attention():
    names = ["chunk_by_rank", "local_attention", "dot_product_attention",
             "sequence_parallel_self_attention"]
    out = {}
    ns = load_functions("src/vidax/core/attention.py", names, make_namespace())
    # dot_product_attention on the CPU path: default scale and explicit scale
    q, k, v = seeded((2, 37, 3, 16), 70), seeded((2, 29, 3, 16), 71), seeded((2, 29, 3, 16), 72)
    out["dpa_q"], out["dpa_k"], out["dpa_v"] = (x.astype(np.float32) for x in (q, k, v))
    out["dpa_o_default"] = ns["dot_product_attention"](q, k, v).astype(np.float32)
    out["dpa_o_scale1"] = ns["dot_product_attention"](q, k, v, scale=1.0).astype(np.float32)
    out["local_o"] = ns["local_attention"](q, k, v).astype(np.float32)
    # head_dim 128 (the sm_100a kernel's size): self- and cross-attention
    q, k, v = seeded((1, 300, 2, 128), 73), seeded((1, 300, 2, 128), 74), seeded((1, 300, 2, 128), 75)
    out["dpa128_q"], out["dpa128_k"], out["dpa128_v"] = (x.astype(np.float32) for x in (q, k, v))
    out["dpa128_o"] = ns["dot_product_attention"](q, k, v).astype(np.float32)
    kx, vx = seeded((1, 77, 2, 128), 76), seeded((1, 77, 2, 128), 77)
    out["cross128_k"], out["cross128_v"] = kx.astype(np.float32), vx.astype(np.float32)
    out["cross128_o"] = ns["local_attention"](q, kx, vx).astype(np.float32)
    # key padding through the public API: an additive 0 / -inf key bias
    # (B, 1, 1, Sk) and the boolean-mask form, ragged valid lengths
    q, k, v = seeded((2, 33, 2, 128), 78), seeded((2, 41, 2, 128), 79), seeded((2, 41, 2, 128), 80)
    lens = np.array([41, 19], np.int32)
    valid = np.arange(41)[None, :] < lens[:, None]
    bias = np.where(valid, 0.0, -np.inf).astype(np.float32)[:, None, None, :]
    out["keypad_q"], out["keypad_k"], out["keypad_v"] = (x.astype(np.float32) for x in (q, k, v))
    out["keypad_len"] = lens
    out["keypad_o_bias"] = ns["dot_product_attention"](q, k, v, bias=bias).astype(np.float32)
    out["keypad_o_mask"] = ns["dot_product_attention"](q, k, v, mask=valid[:, None, None, :]).astype(np.float32)
    # a batch item with no visible key at all (every key masked / -inf)
    lens0 = np.array([41, 0], np.int32)
    valid0 = np.arange(41)[None, :] < lens0[:, None]
    bias0 = np.where(valid0, 0.0, -np.inf).astype(np.float32)[:, None, None, :]
    out["keypad0_len"] = lens0
    with np.errstate(invalid="ignore"):
        out["keypad0_o_bias"] = ns["dot_product_attention"](q, k, v, bias=bias0).astype(np.float32)
    out["keypad0_o_mask"] = ns["dot_product_attention"](q, k, v, mask=valid0[:, None, None, :]).astype(np.float32)
    # Ulysses over P emulated devices, each holding its chunk_by_rank share
    for P, (B, S, H, D) in ((2, (1, 16, 4, 8)), (4, (2, 24, 8, 8)), (8, (1, 256, 8, 128))):
        coll = _Collective(P)
        ns_p = load_functions("src/vidax/core/attention.py", names, make_namespace(coll))
        qg, kg, vg = seeded((B, S, H, D), 80 + P), seeded((B, S, H, D), 90 + P), seeded((B, S, H, D), 100 + P)
        results = [None] * P

        def worker(r):
            coll.local.rank = r
            loc = [ns_p["chunk_by_rank"](x, 1, P, r) for x in (qg, kg, vg)]
            results[r] = ns_p["sequence_parallel_self_attention"](*loc, "sp")

        threads = [threading.Thread(target=worker, args=(r,)) for r in range(P)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        out[f"sp{P}_q"], out[f"sp{P}_k"], out[f"sp{P}_v"] = (x.astype(np.float32) for x in (qg, kg, vg))
        out[f"sp{P}_o"] = np.stack([np.asarray(r).astype(np.float32) for r in results])
    # joint [text; visual] Ulysses (CogVideoX layout): text replicated, visual chunked
    # (the head_dim-128 case is the size the sm_100a kernel takes)
    # (joint4d128 / joint2d64: the kernel's head dims at 4 and 2 ranks, distinct seeds)
    for tag, P, (B, T, S, H, D), seed0 in (
            ("joint2", 2, (1, 5, 16, 4, 8), None), ("joint4", 4, (2, 7, 24, 8, 8), None),
            ("joint2d128", 2, (1, 13, 80, 4, 128), None),
            ("joint4d128", 4, (2, 7, 96, 8, 128), 230), ("joint2d64", 2, (1, 11, 64, 4, 64), 240)):
        coll = _Collective(P)
        ns_p = load_functions("src/vidax/core/attention.py",
                              names + ["sequence_parallel_joint_self_attention"],
                              make_namespace(coll))
        if seed0 is None:
            seed0 = 110 + P + (D > 8) * 7
        qg, kg, vg = (seeded((B, T + S, H, D), seed0 + i) for i in range(3))
        results = [None] * P
        S_loc = S // P

        def worker(r):
            coll.local.rank = r
            loc = [np.concatenate([x[:, :T], x[:, T + r * S_loc:T + (r + 1) * S_loc]], axis=1)
                   for x in (qg, kg, vg)]
            results[r] = ns_p["sequence_parallel_joint_self_attention"](*loc, T, "sp")

        threads = [threading.Thread(target=worker, args=(r,)) for r in range(P)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        out[f"{tag}_q"], out[f"{tag}_k"], out[f"{tag}_v"] = (x.astype(np.float32) for x in (qg, kg, vg))
        out[f"{tag}_text_len"] = np.array([T], np.int32)
        out[f"{tag}_o"] = np.stack([np.asarray(r).astype(np.float32) for r in results])
    return out


def gen_rope():
    """create_rope3d_freqs / apply_rope3d (src/vidax/core/rope3d.py) on small grids."""
    ns = make_namespace()
    jnp = ns["jnp"]
    jnp.power = np.power
    jnp.outer = np.outer
    jnp.cos = np.cos
    jnp.sin = np.sin
    jnp.stack = np.stack
    ns["Tuple"] = tuple
    load_functions("src/vidax/core/rope3d.py", ["_axis_freqs", "create_rope3d_freqs", "apply_rope3d"], ns)
    out = {}
    for i, (t, h, w, hd) in enumerate([(3, 4, 5, 128), (2, 3, 7, 64)]):
        cos, sin = ns["create_rope3d_freqs"](t, h, w, hd)
        x = seeded((1, t * h * w, 3, hd), 120 + i)
        y = ns["apply_rope3d"](x, (np.asarray(cos), np.asarray(sin)))
        assert y.dtype == BF16
        out[f"rope{i}_grid"] = np.array([t, h, w, hd], np.int32)
        out[f"rope{i}_cos"] = np.asarray(cos, np.float32)[0, :, 0, :]
        out[f"rope{i}_sin"] = np.asarray(sin, np.float32)[0, :, 0, :]
        out[f"rope{i}_x"] = x.astype(np.float32)
        out[f"rope{i}_y"] = y.astype(np.float32)
    return out


def load_method(relpath, cls, name, ns):
    """Executes method `name` of class `cls` as a plain function (first
    argument `self`); decorators such as nn.compact are dropped."""
    import textwrap
    path = os.path.join(REF, relpath)
    src = open(path).read()
    for node in ast.parse(src).body:
        if isinstance(node, ast.ClassDef) and node.name == cls:
            for fn in node.body:
                if isinstance(fn, ast.FunctionDef) and fn.name == name:
                    seg = textwrap.dedent(ast.get_source_segment(src, fn))
                    exec(compile("\n" * (fn.lineno - 1) + seg, path, "exec"), ns)
                    return ns[name]
    raise RuntimeError(f"{cls}.{name} not found in {path}")


def gen_rmsnorm():
    """RMSNorm.__call__ (src/vidax/core/attention.py:149-162): full-row (Wan)
    and per-head (HunyuanVideo / LTX-2.5) widths. jax.lax.rsqrt is shimmed as
    float32 1/sqrt; the fixture pins where the float32 / bf16 casts sit."""
    ns = make_namespace()
    jnp = ns["jnp"]
    jnp.mean = np.mean
    jnp.square = np.square
    ns["jax"].lax.rsqrt = lambda v: (np.float32(1.0) / np.sqrt(v)).astype(np.float32)
    ns["nn"] = types.SimpleNamespace(initializers=types.SimpleNamespace(ones=None))
    call = load_method("src/vidax/core/attention.py", "RMSNorm", "__call__", ns)
    out = {}
    for i, (rows, dim) in enumerate([(37, 1536), (29, 5120), (41, 128), (23, 64)]):
        rng = np.random.Generator(np.random.PCG64(140 + i))
        w = (1.0 + 0.25 * rng.standard_normal(dim)).astype(np.float32)
        x = seeded((rows, dim), 150 + i, scale=3.0)
        module = types.SimpleNamespace(dim=dim, eps=1e-6, param=lambda name, init, shape, w=w: w)
        y = call(module, x)
        assert y.dtype == BF16
        out[f"rms{i}_x"] = x.astype(np.float32)
        out[f"rms{i}_w"] = w
        out[f"rms{i}_y"] = y.astype(np.float32)
    return out


def gen_sinusoid():
    """sinusoidal_embedding_1d (src/vidax/core/rope3d.py:15-30), Wan's
    timestep embedding, at freq_dim 256 and a spread of timesteps."""
    ns = make_namespace()
    jnp = ns["jnp"]
    jnp.power = np.power
    jnp.outer = np.outer
    jnp.cos = np.cos
    jnp.sin = np.sin
    load_functions("src/vidax/core/rope3d.py", ["sinusoidal_embedding_1d"], ns)
    t = np.array([0.0, 1.0, 37.5, 500.0, 999.0], np.float32)
    return {"sinusoid_t": t,
            "sinusoid_emb": np.asarray(ns["sinusoidal_embedding_1d"](256, t), np.float32)}


def _ltx_namespace():
    """Namespace holding diffusion_vae.py's abs-RoPE helpers and the NA
    primitive, run under the numpy shim (jnp.cos / sin in float32)."""
    ns = make_namespace()
    jnp = ns["jnp"]
    jnp.cos = np.cos
    jnp.sin = np.sin
    jnp.stack = np.stack
    jnp.mean = np.mean
    jnp.square = np.square
    ns["math"] = __import__("math")
    load_functions("src/vidax/models/ltx2_5/diffusion_vae.py",
                   ["_default_rope_dim_split", "_rope_inv_freqs", "_apply_abs_rope_axis",
                    "_apply_abs_rope", "_window_start", "_gather_window",
                    "neighborhood_attention_3d"], ns)
    return ns


def gen_ltx_rope():
    """LTX-2.5's absolute split RoPE (diffusion_vae.py:96-150): the default
    split, the inverse frequencies, and `_apply_abs_rope` on small grids at
    head_dim 64 (the checkpoint's) and 128; also each axis's float32 angle
    tables cos / sin(position * inv_freq), the product's table entries."""
    ns = _ltx_namespace()
    out = {}
    for i, (t, h, w, hd, split) in enumerate([(3, 4, 5, 64, None), (2, 3, 6, 128, None),
                                             (4, 2, 3, 64, (8, 28, 28))]):
        split = tuple(int(x) for x in (split or ns["_default_rope_dim_split"](hd)))
        invs = [np.asarray(ns["_rope_inv_freqs"](d, 10000.0), np.float32) for d in split]
        pos = [np.arange(n, dtype=np.float32) for n in (t, h, w)]
        x = seeded((1, t, h, w, 3, hd), 250 + i)
        y = ns["_apply_abs_rope"](x, split, tuple(invs), tuple(pos))
        assert y.dtype == BF16 and y.shape == x.shape
        out[f"ltxrope{i}_grid"] = np.array([t, h, w, hd], np.int32)
        out[f"ltxrope{i}_split"] = np.array(split, np.int32)
        for a, (p_a, inv) in enumerate(zip(pos, invs)):
            ang = p_a[:, None] * inv[None, :]
            out[f"ltxrope{i}_cos{a}"] = np.cos(ang).astype(np.float32)
            out[f"ltxrope{i}_sin{a}"] = np.sin(ang).astype(np.float32)
        out[f"ltxrope{i}_x"] = x.astype(np.float32)
        out[f"ltxrope{i}_y"] = y.astype(np.float32)
    return out


class _WeakScalarBF16(np.ndarray):
    """A bf16 array whose product with a Python scalar follows JAX's weak
    typing: the scalar takes the array's dtype (bf16) and the result stays
    bf16, bf16(f32(x) * f32(bf16(c))). numpy with ml_dtypes would promote to
    float32 instead. Any other operation returns a plain ndarray."""

    def __array_ufunc__(self, ufunc, method, *inputs, **kw):
        plain = [np.asarray(x) if isinstance(x, _WeakScalarBF16) else x for x in inputs]
        if (ufunc is np.multiply and method == "__call__" and len(plain) == 2 and not kw
                and isinstance(plain[1], (float, int)) and plain[0].dtype == BF16):
            c = np.float32(np.asarray(plain[1], np.float32).astype(BF16))
            return (plain[0].astype(np.float32) * c).astype(BF16)
        return getattr(ufunc, method)(*plain, **kw)


def gen_ltx_na_block():
    """The NA caller contract: `NeighborhoodAttention3D.__call__`
    (diffusion_vae.py:252-284) run as a plain function whose `to_q` / `to_k`
    / `to_v` Dense layers return given projections and whose `to_out` is the
    identity, so the reference's own per-head RMSNorm (attention.py:149-162),
    bf16 q scaling (:265), absolute RoPE (:267-275) and NA call (:277) run on
    them. Head_dim 64 (the checkpoint's) and 128."""
    ns = _ltx_namespace()
    ns["jax"].lax.rsqrt = lambda v: (np.float32(1.0) / np.sqrt(v)).astype(np.float32)
    rms_ns = make_namespace()
    rms_ns["jnp"].mean = np.mean
    rms_ns["jnp"].square = np.square
    rms_ns["jax"].lax.rsqrt = ns["jax"].lax.rsqrt
    rms_ns["nn"] = types.SimpleNamespace(initializers=types.SimpleNamespace(ones=None))
    rms_call = load_method("src/vidax/core/attention.py", "RMSNorm", "__call__", rms_ns)
    out = {}
    cases = [((1, 3, 4, 6, 2, 64), (3, 3, 5)), ((1, 2, 5, 7, 2, 64), (3, 5, 5)),
             ((1, 3, 4, 5, 1, 128), (3, 3, 3))]
    for i, (shape, kernel) in enumerate(cases):
        B, T, H, W, NH, HD = shape
        proj = {n: seeded(shape, 260 + 3 * i + j, scale=2.0) for j, n in enumerate(("to_q", "to_k", "to_v"))}
        rng = np.random.Generator(np.random.PCG64(270 + i))
        weights = {n: (1.0 + 0.25 * rng.standard_normal(HD)).astype(np.float32)
                   for n in ("q_norm", "k_norm")}

        class Dense:
            def __init__(self, features, name):
                self.name = name

            def __call__(self, x):
                if self.name == "to_out":
                    return x
                return proj[self.name].reshape(x.shape[:4] + (NH * HD,))

        def rmsnorm(dim, eps=1e-6, name=None):
            module = types.SimpleNamespace(dim=dim, eps=eps,
                                           param=lambda pname, init, shp: weights[name])
            return lambda x: np.asarray(rms_call(module, x)).view(_WeakScalarBF16)

        ns["nn"] = types.SimpleNamespace(Dense=Dense)
        ns["RMSNorm"] = rmsnorm
        seen = {}
        na_fn = ns.get("_na_primitive", ns["neighborhood_attention_3d"])
        ns["_na_primitive"] = na_fn

        def recording_na(q, k, v, kernel_size, na_fn=na_fn, seen=seen):
            # the primitive's inputs: q / k after norm, scale and RoPE
            seen["q"], seen["k"] = q, k
            return na_fn(q, k, v, kernel_size)

        ns["neighborhood_attention_3d"] = recording_na
        call = load_method("src/vidax/models/ltx2_5/diffusion_vae.py", "NeighborhoodAttention3D",
                           "__call__", ns)
        module = types.SimpleNamespace(dim=NH * HD, kernel_size=kernel, head_dim=HD,
                                       rope_dim_split=None, rope_base=10000.0, eps=1e-6)
        x = np.zeros((B, T, H, W, NH * HD), BF16)
        o = call(module, x)
        assert o.dtype == BF16
        for n, tag in (("to_q", "q"), ("to_k", "k"), ("to_v", "v")):
            out[f"ltxna{i}_{tag}"] = proj[n].astype(np.float32)
        out[f"ltxna{i}_wq"] = weights["q_norm"]
        out[f"ltxna{i}_wk"] = weights["k_norm"]
        out[f"ltxna{i}_kernel"] = np.array(kernel, np.int32)
        out[f"ltxna{i}_o"] = np.asarray(o, np.float32).reshape(shape)
        assert seen["q"].dtype == BF16 and seen["k"].dtype == BF16
        out[f"ltxna{i}_qr"] = seen["q"].astype(np.float32)
        out[f"ltxna{i}_kr"] = seen["k"].astype(np.float32)
    return out


def main():
    if not REF or not os.path.isdir(REF):
        sys.exit("usage: make_golden.py <path-to-vidax-checkout>")
    na = gen_na3d()
    np.savez_compressed(os.path.join(OUT_DIR, "na3d_reference.npz"), **na)
    at = gen_attention()
    np.savez_compressed(os.path.join(OUT_DIR, "attention_reference.npz"), **at)
    ro = gen_rope()
    ro.update(gen_rmsnorm())
    ro.update(gen_sinusoid())
    np.savez_compressed(os.path.join(OUT_DIR, "rope_reference.npz"), **ro)
    ltx = gen_ltx_rope()
    ltx.update(gen_ltx_na_block())
    np.savez_compressed(os.path.join(OUT_DIR, "ltx_reference.npz"), **ltx)
    for f in ("na3d_reference.npz", "attention_reference.npz", "rope_reference.npz",
              "ltx_reference.npz"):
        print(f, os.path.getsize(os.path.join(OUT_DIR, f)), "bytes")


if __name__ == "__main__":
    main()
