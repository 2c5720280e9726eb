"""ctypes binding of the CPU oracle (oracle/_build/libbonsai_oracle.so) and of
the reference's own kernels compiled into oracle/_ref.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product code path.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "libbonsai_oracle.so"
REF_SO = HERE / "_ref" / "libbonsai_ref.so"
REF_SCALAR_SO = HERE / "_ref" / "libbonsai_ref_scalar.so"

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float


class Dims(ctypes.Structure):
    _fields_ = [("preset", _i), ("hidden", _i), ("heads", _i), ("head_dim", _i), ("mlp", _i)]


_sigs = {
    "orc_set_threads": [_i],
    "orc_b1_linear": [_vp, _i, _i, _vp, _i, _vp],
    "orc_linear_f32": [_vp, _i, _i, _vp, _vp, _i, _vp],
    "orc_rope_freqs": [_vp, _i, _f, _vp, _i],
    "orc_rope_cos_sin": [_vp, _i, _vp, _i, _f, _vp, _vp],
    "orc_rope_apply": [_vp, _vp, _vp, _i, _i, _i, _vp],
    "orc_rms_norm": [_vp, _vp, _i, _i, _f, _vp],
    "orc_ln_modulate": [_vp, _i, _i, _vp, _vp, _f, _vp],
    "orc_swiglu": [_vp, _i, _i, _vp, _i],
    "orc_gelu": [_vp, _i, _i, _vp, _i],
    "orc_attention": [_vp, _vp, _vp, _i, _i, _i, _f, _vp],
    "orc_timestep_embedding": [_f, _i, _f, _vp],
    "orc_qk_norm_rope_heads": [_vp, _i, _i, _i, _vp, _vp, _i, _f, _vp, _vp],
    "orc_double_block": [ctypes.POINTER(Dims), _i, _i, _vp] + [_vp] * 16,
    "orc_single_block": [ctypes.POINTER(Dims), _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "orc_silu": [_vp, _i, _vp],
}

_lib = None
_ref = {}


def _build():
    subprocess.run(["make", "-C", str(HERE)], check=True, capture_output=True)


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            _build()
        L = ctypes.CDLL(str(ORACLE_SO))
        for n, a in _sigs.items():
            getattr(L, n).argtypes = a
            getattr(L, n).restype = None
        _lib = L
    return _lib


def ref(scalar: bool = False):
    """The reference's own b1_linear_f32_f32 / rope_2d_fwd_f32 (oracle/_ref), or None."""
    path = REF_SCALAR_SO if scalar else REF_SO
    if path not in _ref:
        if not path.exists():
            _ref[path] = None
        else:
            L = ctypes.CDLL(str(path))
            L.ref_b1_linear.argtypes = [_vp, _i, _i, _vp, _i, _vp, _i]
            L.ref_rope_2d.argtypes = [_vp, _vp, _vp, _i, _i, _i, _vp, _i]
            L.ref_has_avx2.restype = _i
            _ref[path] = L
    return _ref[path]


def P(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def b1_linear(act: np.ndarray, packed: np.ndarray, out_dim: int) -> np.ndarray:
    act = f32(act)
    T, K = act.shape
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros((T, out_dim), np.float32)
    lib().orc_b1_linear(P(act), T, K, P(packed), out_dim, P(out))
    return out


def ref_b1_linear(act: np.ndarray, packed: np.ndarray, out_dim: int, nthreads: int = 4,
                  scalar: bool = False) -> np.ndarray:
    L = ref(scalar)
    assert L is not None, "oracle/_ref not built"
    act = f32(act)
    T, K = act.shape
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros((T, out_dim), np.float32)
    L.ref_b1_linear(P(act), T, K, P(packed), out_dim, P(out), nthreads)
    return out


def rope_cos_sin(ids: np.ndarray, axes, theta: float):
    ids = f32(ids)
    seq, n_axes = ids.shape
    ax = np.ascontiguousarray(axes, dtype=np.int32)
    half = int(ax.sum()) // 2
    c = np.zeros((seq, half), np.float32)
    s = np.zeros((seq, half), np.float32)
    lib().orc_rope_cos_sin(P(ids), seq, P(ax), n_axes, theta, P(c), P(s))
    return c, s


def rope_freqs(axes, theta: float):
    ax = np.ascontiguousarray(axes, dtype=np.int32)
    mh = int(ax.max()) // 2
    v = np.zeros((len(ax), mh), np.float32)
    lib().orc_rope_freqs(P(ax), len(ax), theta, P(v), mh)
    return v


def rope_apply(x: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
    x = f32(x)
    seq, nh, hd = x.shape
    out = np.zeros_like(x)
    lib().orc_rope_apply(P(x), P(f32(c)), P(f32(s)), hd, nh, seq, P(out))
    return out


def rms_norm(x, w, eps=1e-6):
    x = f32(x)
    rows, dim = x.shape
    y = np.zeros_like(x)
    lib().orc_rms_norm(P(x), P(f32(w)), rows, dim, eps, P(y))
    return y


def ln_modulate(x, shift, scale, eps=1e-6):
    x = f32(x)
    rows, dim = x.shape
    y = np.zeros_like(x)
    lib().orc_ln_modulate(P(x), rows, dim, P(f32(shift)), P(f32(scale)), eps, P(y))
    return y


def attention(q, k, v, scale):
    """q, k, v f32 [seq][heads][hd] -> out f32 [seq][heads*hd]."""
    q, k, v = f32(q), f32(k), f32(v)
    seq, nh, hd = q.shape
    out = np.zeros((seq, nh * hd), np.float32)
    lib().orc_attention(P(q), P(k), P(v), seq, nh, hd, scale, P(out))
    return out


def qk_norm_rope_heads(x, w_lo, w_hi, split, cos_t, sin_t, eps=1e-6):
    x = np.array(x, dtype=np.float32, copy=True, order="C")
    nh, seq, hd = x.shape
    lib().orc_qk_norm_rope_heads(P(x), nh, seq, hd, P(f32(w_lo)), P(f32(w_hi)), split, eps,
                                 P(f32(cos_t)), P(f32(sin_t)))
    return x


def timestep_embedding(t: float, dim: int = 256, max_period: float = 10000.0):
    out = np.zeros(dim, np.float32)
    lib().orc_timestep_embedding(t, dim, max_period, P(out))
    return out


def swiglu(x):
    x = f32(x)
    rows, n2 = x.shape
    y = np.zeros((rows, n2 // 2), np.float32)
    lib().orc_swiglu(P(x), rows, n2 // 2, P(y), n2 // 2)
    return y


def gelu(x):
    x = f32(x)
    rows, n = x.shape
    y = np.zeros_like(x)
    lib().orc_gelu(P(x), rows, n, P(y), n)
    return y


# ------------------------------------------------------------- blocks / step
_sigs_extra = {"orc_use_reference_b1": [_vp, _i], "orc_set_attention_f16": [_i]}


def _extra():
    L = lib()
    for n, a in _sigs_extra.items():
        getattr(L, n).argtypes = a
        getattr(L, n).restype = None
    return L


def use_reference_b1(on: bool = True, nthreads: int = 8) -> bool:
    """Run the reference's own b1_linear_f32_f32 (oracle/_ref AVX2 build)
    for every B1_0 linear inside the oracle blocks.  Returns False when
    oracle/_ref is not available (the C restatement is used instead)."""
    L = _extra()
    R = ref()
    if on and R is not None:
        L.orc_use_reference_b1(ctypes.cast(R.ref_b1_linear, _vp), nthreads)
        return True
    L.orc_use_reference_b1(None, 1)
    return False


def set_attention_f16(on: bool) -> None:
    """True: round q/k/v to f16 like the reference graph; False: fp32 oracle."""
    _extra().orc_set_attention_f16(1 if on else 0)


def dims(preset_swiglu: bool, mlp: int) -> Dims:
    return Dims(0 if preset_swiglu else 1, 3072, 24, 128, mlp)


def double_block(model, i: int, h: np.ndarray, mod_img, mod_txt, cos_t, sin_t) -> np.ndarray:
    """Run double block i of a bonsai_b200.Dit (weights exported by name) on h [L][3072]."""
    h = np.array(h, dtype=np.float32, copy=True, order="C")
    p = f"double.{i}."
    w = {n: model.weight(p + n) for n in
         ("img_qkv", "txt_qkv", "img_out", "txt_out", "img_mlp_in", "img_mlp_out", "txt_mlp_in",
          "txt_mlp_out")}
    nrm = {n: model.weight_f32(p + n) for n in ("img_norm_q", "img_norm_k", "txt_norm_q", "txt_norm_k")}
    D = dims(model.swiglu, model.mlp)
    lib().orc_double_block(ctypes.byref(D), model.txt, model.img, P(h), P(f32(mod_img)),
                           P(f32(mod_txt)), P(w["img_qkv"]), P(w["txt_qkv"]), P(w["img_out"]),
                           P(w["txt_out"]), P(w["img_mlp_in"]), P(w["img_mlp_out"]),
                           P(w["txt_mlp_in"]), P(w["txt_mlp_out"]), P(nrm["img_norm_q"]),
                           P(nrm["img_norm_k"]), P(nrm["txt_norm_q"]), P(nrm["txt_norm_k"]),
                           P(f32(cos_t)), P(f32(sin_t)))
    return h


def single_block(model, i: int, h: np.ndarray, mod, cos_t, sin_t) -> np.ndarray:
    h = np.array(h, dtype=np.float32, copy=True, order="C")
    p = f"single.{i}."
    wp, wo = model.weight(p + "proj"), model.weight(p + "out")
    nq, nk = model.weight_f32(p + "norm_q"), model.weight_f32(p + "norm_k")
    D = dims(model.swiglu, model.mlp)
    lib().orc_single_block(ctypes.byref(D), model.L, P(h), P(f32(mod)), P(wp), P(wo), P(nq), P(nk),
                           P(f32(cos_t)), P(f32(sin_t)))
    return h


def linear(x, W, b, out_dim):
    x = f32(x)
    T, K = x.shape
    y = np.zeros((T, out_dim), np.float32)
    lib().orc_linear_f32(P(x), T, K, P(f32(W)), P(f32(b)) if b is not None else None, out_dim, P(y))
    return y


def silu(x):
    x = f32(x)
    return x / (1.0 + np.exp(-x.astype(np.float64))).astype(np.float32)


def modulations(model, vec: np.ndarray):
    """Every modulation vector from vec, as the engine computes them:
    ({'double': [(img6H, txt6H)], 'single': [3H]}, final 2H)."""
    H = 3072
    vs = np.empty(H, np.float32)
    lib().orc_silu(P(f32(vec)), H, P(vs))
    out = {"double": [], "single": []}
    for i in range(model.depth):
        if model.per_block_mod:
            mi = b1_linear(vs[None], model.weight(f"double.{i}.img_mod"), 6 * H)[0]
            mt = b1_linear(vs[None], model.weight(f"double.{i}.txt_mod"), 6 * H)[0]
        else:
            mi = linear(vs[None], model.weight_f32("mod_img.w"), None, 6 * H)[0]
            mt = linear(vs[None], model.weight_f32("mod_txt.w"), None, 6 * H)[0]
        out["double"].append((mi, mt))
    for i in range(model.depth_single):
        if model.per_block_mod:
            ms = b1_linear(vs[None], model.weight(f"single.{i}.mod"), 3 * H)[0]
        else:
            ms = linear(vs[None], model.weight_f32("mod_single.w"), None, 3 * H)[0]
        out["single"].append(ms)
    nb = model.weight_f32("norm_out.b") if model.per_block_mod else None
    fin = linear(vs[None], model.weight_f32("norm_out.w"), nb, 2 * H)[0]
    return out, fin


def dit_forward(model, img, txt, pooled, t: float) -> np.ndarray:
    """The whole denoise-step forward (build_diffuser_graph) on the CPU."""
    H = 3072
    bias = (lambda n: model.weight_f32(n)) if model.per_block_mod else (lambda n: None)
    h = np.zeros((model.L, H), np.float32)
    h[:model.txt] = linear(txt, model.weight_f32("txt_in.w"), bias("txt_in.b"), H)
    h[model.txt:] = linear(img, model.weight_f32("img_in.w"), bias("img_in.b"), H)
    te = timestep_embedding(t)
    h1 = linear(te[None], model.weight_f32("time.w1"), bias("time.b1"), H)
    vec = linear(silu(h1), model.weight_f32("time.w2"), bias("time.b2"), H)[0]
    if model.pooled:
        v1 = linear(f32(pooled)[None], model.weight_f32("vec.w1"), bias("vec.b1"), H)
        vec = vec + linear(silu(v1), model.weight_f32("vec.w2"), bias("vec.b2"), H)[0]
    mods, fin = modulations(model, vec)
    c, s = rope_cos_sin(model.rope_ids(), model.axes, model.theta)
    for i in range(model.depth):
        h = double_block(model, i, h, mods["double"][i][0], mods["double"][i][1], c, s)
    for i in range(model.depth_single):
        h = single_block(model, i, h, mods["single"][i], c, s)
    xm = ln_modulate(h[model.txt:], fin[H:], fin[:H])
    return linear(xm, model.weight_f32("proj_out.w"), bias("proj_out.b"), model.in_ch)
