"""ctypes binding of libbonsai_cuda.so (include/bonsai_cuda.h).

This is the Python-side view of the C ABI that tests and the benchmark use.
It mirrors the reference's operator surface: ``b1_linear_f32`` is the
drop-in for ``b1_linear_f32_f32`` (src/b1_0_kernel.h:37-288), ``rope_2d_f32``
for ``rope_2d_fwd_f32`` (src/b1_0_kernel.h:309-361), and the model entry
points for one pass of ``build_diffuser_graph`` (src/diffuser_graph.cpp:231-561).

Device tensors are passed as raw pointers (``tensor.data_ptr()``); PyTorch is
used only to own device memory and streams.  There is no CPU fallback: if the
shared library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR.parent / "lib" / "libbonsai_cuda.so"

BONSAI_EPI_F32 = 0
BONSAI_EPI_F16 = 1
BONSAI_EPI_GELU = 2
BONSAI_EPI_RESID = 3
BONSAI_EPI_SWIGLU = 5

PRESET_KLEIN4B = 0
PRESET_FLUX1 = 1

_lib = None

_c_int = ctypes.c_int
_c_ll = ctypes.c_longlong
_vp = ctypes.c_void_p
_fp = ctypes.c_float

# name -> (restype, argtypes); every symbol declared in include/bonsai_cuda.h
SIGNATURES = {
    "bonsai_last_error": (ctypes.c_char_p, []),
    "bonsai_init": (_c_int, [_c_int]),
    "bonsai_device_error": (_c_int, []),
    "bonsai_shutdown": (_c_int, []),
    "bonsai_count_nonfinite": (_c_int, [_vp, _c_ll, ctypes.POINTER(_c_ll), _vp]),
    "bonsai_launch_count": (_c_ll, []),
    "bonsai_debug_stall_next_gemm": (_c_int, []),
    "bonsai_profile_start": (_c_int, []),
    "bonsai_profile_stop": (_c_int, [ctypes.c_char_p, _c_int]),
    "bonsai_b1_upload": (_c_int, [_vp, _c_int, _c_int, _c_int, ctypes.POINTER(_vp)]),
    "bonsai_b1_free": (_c_int, [_vp]),
    "bonsai_b1_shape": (_c_int, [_vp, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "bonsai_b1_linear_f32": (_c_int, [_vp, _c_int, _vp, _vp, _vp]),
    "bonsai_b1_linear_f32_noalloc": (_c_int, [_vp, _c_int, _vp, _vp, _vp]),
    "bonsai_b1_gemm": (_c_int, [_vp, _c_ll, _c_int, _vp, _c_int, _vp, _c_ll, _vp, _vp]),
    "bonsai_rope_2d_f32": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _vp, _vp]),
    "bonsai_rope_tables": (_c_int, [_vp, _c_int, _c_int, _vp, _fp, _vp, _vp, _vp]),
    "bonsai_rms_norm_f32": (_c_int, [_vp, _vp, _c_int, _c_int, _fp, _vp, _vp]),
    "bonsai_linear_f32": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _c_int, _vp, _vp]),
    "bonsai_ln_modulate": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _fp, _vp, _c_ll, _vp]),
    "bonsai_ln_modulate_f32": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _fp, _vp, _vp]),
    "bonsai_joint_attention": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _fp, _vp, _c_ll, _vp]),
    "bonsai_qk_norm_rope": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _vp, _c_int, _fp, _vp, _vp, _vp]),
    "bonsai_dit_create": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "bonsai_dit_destroy": (_c_int, [_vp]),
    "bonsai_dit_forward": (_c_int, [_vp, _vp, _vp, _vp, _fp, _vp, _vp]),
    "bonsai_dit_forward_host": (_c_int, [_vp, _vp, _vp, _vp, _fp, _vp, _vp]),
    "bonsai_dit_set_state": (_c_int, [_vp, _vp, _vp, _vp]),
    "bonsai_dit_get_state": (_c_int, [_vp, _vp, _vp]),
    "bonsai_dit_double_block": (_c_int, [_vp, _c_int, _vp]),
    "bonsai_dit_single_block": (_c_int, [_vp, _c_int, _vp]),
    "bonsai_dit_weight": (_c_ll, [_vp, ctypes.c_char_p, _vp, _c_ll]),
    "bonsai_dit_set_weight": (_c_int, [_vp, ctypes.c_char_p, _vp, _c_ll]),
    "bonsai_dit_load_safetensors": (_c_int, [_vp, ctypes.c_char_p]),
    "bonsai_safetensors_list": (_c_int, [ctypes.c_char_p, ctypes.c_char_p, _c_int]),
    "bonsai_dit_sample": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _vp, _vp]),
    "bonsai_dit_set_partition": (_c_int, [_vp, _c_int, _c_int]),
    "bonsai_dit_buffer": (_c_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(_c_ll)]),
    "bonsai_dit_begin": (_c_int, [_vp, _vp, _vp, _vp, _fp, _vp]),
    "bonsai_dit_phase": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp]),
    "bonsai_dit_end": (_c_int, [_vp, _vp, _vp]),
    "bonsai_dit_set_peers": (_c_int, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp), _c_int]),
    "bonsai_dit_ipc_handles": (_c_int, [_vp, _vp]),
    "bonsai_dit_open_peers": (_c_int, [_vp, _vp, _c_int]),
    "bonsai_dit_set_qkv_peers": (_c_int, [_vp, ctypes.POINTER(_vp), _c_int]),
    "bonsai_dit_ipc_handle": (_c_int, [_vp, ctypes.c_char_p, _vp]),
    "bonsai_dit_open_qkv_peers": (_c_int, [_vp, _vp, _c_int]),
    "bonsai_dit_set_flag_peers": (_c_int, [_vp, ctypes.POINTER(_vp), _c_int]),
    "bonsai_dit_open_flag_peers": (_c_int, [_vp, _vp, _c_int]),
    "bonsai_dit_barrier": (_c_int, [_vp, _vp]),
    "bonsai_vae_create": (_c_int, [_c_int, _c_int, ctypes.c_ulonglong, ctypes.POINTER(_vp)]),
    "bonsai_vae_destroy": (_c_int, [_vp]),
    "bonsai_vae_load_safetensors": (_c_int, [_vp, ctypes.c_char_p]),
    "bonsai_vae_decode": (_c_int, [_vp, _vp, _vp, _vp]),
    "bonsai_vae_decode_host": (_c_int, [_vp, _vp, _vp, _vp]),
    "bonsai_vae_rgb8": (_c_int, [_vp, _c_int, _c_int, _vp, _vp]),
    "bonsai_vae_info": (_c_int, [_vp, ctypes.POINTER(_c_int), ctypes.POINTER(_c_int)]),
    "bonsai_conv2d_nhwc": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _vp, _c_int, _c_int, _vp, _vp,
                                    _vp, _vp]),
}


class BonsaiError(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load the shared library (raises if it is absent: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise BonsaiError(
                f"{LIB_PATH} not found: build it with `make -C bonsai.cpp_b200` "
                "(or __graft_entry__.build())")
        L = ctypes.CDLL(str(LIB_PATH))
        missing = []
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(L, name)
            except AttributeError:
                missing.append(name)
                continue
            fn.restype = res
            fn.argtypes = args
        L.missing_symbols = missing
        _lib = L
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib().bonsai_last_error().decode(errors="replace")
        raise BonsaiError(f"{what or 'bonsai call'} failed with {rc}: {msg}")


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def init(device: int = 0) -> None:
    check(lib().bonsai_init(device), "bonsai_init")


def device_error() -> int:
    return int(lib().bonsai_device_error())


def launch_count() -> int:
    return int(lib().bonsai_launch_count())


def profile_start() -> None:
    check(lib().bonsai_profile_start(), "bonsai_profile_start")


def profile_stop() -> dict:
    import json
    buf = ctypes.create_string_buffer(1 << 16)
    n = lib().bonsai_profile_stop(buf, len(buf))
    if n < 0:
        check(n, "bonsai_profile_stop")
    return json.loads(buf.value.decode())


class B1Weight:
    """Device B1_0 weight uploaded from the reference's packed bytes."""

    def __init__(self, packed: np.ndarray, out_dim: int, in_dim: int, swiglu_from: int = -1):
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        assert packed.size == out_dim * (in_dim // 32) * 6, "packed size mismatch"
        h = _vp()
        check(lib().bonsai_b1_upload(packed.ctypes.data, out_dim, in_dim, swiglu_from,
                                     ctypes.byref(h)), "bonsai_b1_upload")
        self.handle = h
        self.out_dim = out_dim
        self.in_dim = in_dim

    def free(self):
        if self.handle:
            lib().bonsai_b1_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def b1_linear_f32(act, w: B1Weight, out, stream=None) -> None:
    """Drop-in b1_linear_f32_f32: act f32 [T][K] -> out f32 [T][N] (device tensors)."""
    assert act.is_contiguous() and out.is_contiguous()
    T = act.shape[0]
    check(lib().bonsai_b1_linear_f32(act.data_ptr(), T, w.handle, out.data_ptr(),
                                     stream_ptr(stream)), "bonsai_b1_linear_f32")


def b1_gemm(x16, w: B1Weight, mode: int, out, gate=None, stream=None) -> None:
    """Fused-epilogue GEMM on f16 activations x16 [T][ldx]."""
    T = x16.shape[0]
    check(lib().bonsai_b1_gemm(x16.data_ptr(), x16.stride(0), T, w.handle, mode,
                               out.data_ptr(), out.stride(0),
                               gate.data_ptr() if gate is not None else None,
                               stream_ptr(stream)), "bonsai_b1_gemm")


def linear_f32(x, W, bias, out, stream=None) -> None:
    """f32 edge linear: out[t][o] = x[t] . W[o] (+ bias[o]); device tensors."""
    T, K = x.shape
    N = W.shape[0]
    assert x.is_contiguous() and W.is_contiguous() and out.is_contiguous()
    check(lib().bonsai_linear_f32(x.data_ptr(), T, K, W.data_ptr(),
                                  bias.data_ptr() if bias is not None else None, N,
                                  out.data_ptr(), stream_ptr(stream)), "bonsai_linear_f32")


def count_nonfinite(x, stream=None) -> int:
    """Number of NaN / Inf values in a device f32 tensor."""
    n = _c_ll()
    check(lib().bonsai_count_nonfinite(x.data_ptr(), x.numel(), ctypes.byref(n), stream_ptr(stream)),
          "bonsai_count_nonfinite")
    return int(n.value)


def safetensors_list(path) -> list:
    """[(name, dtype, shape tuple, begin, end)] of a .safetensors file (host only)."""
    p = str(path).encode()
    n = lib().bonsai_safetensors_list(p, None, 0)
    if n < 0:
        check(n, "bonsai_safetensors_list")
    buf = ctypes.create_string_buffer(n + 1)
    check(0 if lib().bonsai_safetensors_list(p, buf, n + 1) == n else -1, "bonsai_safetensors_list")
    out = []
    for line in buf.value.decode().splitlines():
        name, dtype, shape, b, e = line.split("\t")
        out.append((name, dtype, tuple(int(d) for d in shape.split(",") if d), int(b), int(e)))
    return out


def shutdown() -> None:
    check(lib().bonsai_shutdown(), "bonsai_shutdown")


def joint_attention(q, k, v, out, scale=None, stream=None) -> None:
    """softmax(Q K^T * scale) V per head: q/k/v f16 [H][L][128] head-major,
    out f16 [L][ld >= H*128] token-major (head h at columns h*128)."""
    H, L, D = q.shape
    check(lib().bonsai_joint_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), H, L, D,
                                       float(scale if scale is not None else D ** -0.5),
                                       out.data_ptr(), out.stride(0), stream_ptr(stream)),
          "bonsai_joint_attention")


# ----------------------------------------------------------------- host side
def random_b1_packed(out_dim: int, in_dim: int, rng: np.random.Generator,
                     scale_std: float = 0.02) -> np.ndarray:
    """Seeded random packed B1_0 matrix [out_dim][in_dim/32*6] (uint8): signs
    Bernoulli(0.5), scales |N(0, scale_std)| rounded to f16, in the layout of
    convert_to_b1_0_packed.py:21-43."""
    nb = in_dim // 32
    signs = rng.integers(0, 2, size=(out_dim, nb, 32), dtype=np.uint8)
    scales = np.abs(rng.standard_normal((out_dim, nb)) * scale_std).astype(np.float16)
    raw = np.zeros((out_dim, nb, 6), dtype=np.uint8)
    raw[:, :, 0:2] = scales.view(np.uint8).reshape(out_dim, nb, 2)
    raw[:, :, 2:6] = np.packbits(signs, axis=-1, bitorder="little")
    return raw.reshape(out_dim, nb * 6)


def dequant_b1(packed: np.ndarray, out_dim: int, in_dim: int) -> np.ndarray:
    """f32 [out_dim][in_dim] = +-scale per the B1_0 block rule
    (tests/test_diffuser.py:24-33 dequant of the reference)."""
    nb = in_dim // 32
    raw = np.ascontiguousarray(packed, dtype=np.uint8).reshape(out_dim, nb, 6)
    scales = raw[:, :, 0:2].copy().view(np.float16).reshape(out_dim, nb).astype(np.float32)
    bits = np.unpackbits(raw[:, :, 2:6], axis=-1, bitorder="little").astype(np.float32)
    return ((bits * 2.0 - 1.0) * scales[:, :, None]).reshape(out_dim, in_dim)


# ----------------------------------------------------------------- model
class DitConfig(ctypes.Structure):
    _fields_ = [("preset", ctypes.c_int), ("depth", ctypes.c_int), ("depth_single", ctypes.c_int),
                ("img_tokens", ctypes.c_int), ("txt_tokens", ctypes.c_int),
                ("grid_h", ctypes.c_int), ("grid_w", ctypes.c_int), ("seed", ctypes.c_ulonglong)]


PRESET_DIMS = {
    # preset: (depth, depth_single, mlp, swiglu, in_ch, ctx_dim, pooled, axes, theta, per_block_mod)
    PRESET_KLEIN4B: (5, 20, 9216, True, 128, 7680, 0, (32, 32, 32, 32), 2000.0, False),
    PRESET_FLUX1: (19, 38, 12288, False, 64, 4096, 768, (16, 56, 56), 10000.0, True),
}
HIDDEN, HEADS, HEAD_DIM = 3072, 24, 128


class Dit:
    """One diffuser transformer on the device (bonsai_dit_* entry points)."""

    def __init__(self, preset: int, img_tokens: int, txt_tokens: int, grid_h: int, grid_w: int,
                 depth: int = 0, depth_single: int = 0, seed: int = 1234):
        d = PRESET_DIMS[preset]
        self.preset = preset
        self.depth = depth or d[0]
        self.depth_single = depth_single or d[1]
        self.mlp, self.swiglu, self.in_ch, self.ctx_dim, self.pooled = d[2], d[3], d[4], d[5], d[6]
        self.axes, self.theta, self.per_block_mod = d[7], d[8], d[9]
        self.img, self.txt, self.L = img_tokens, txt_tokens, img_tokens + txt_tokens
        self.grid_h, self.grid_w = grid_h, grid_w
        cfg = DitConfig(preset, depth, depth_single, img_tokens, txt_tokens, grid_h, grid_w, seed)
        h = _vp()
        check(lib().bonsai_dit_create(ctypes.byref(cfg), ctypes.byref(h)), "bonsai_dit_create")
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            lib().bonsai_dit_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight(self, name: str) -> np.ndarray:
        n = lib().bonsai_dit_weight(self.handle, name.encode(), None, 0)
        if n < 0:
            check(int(n), f"bonsai_dit_weight({name})")
        buf = np.empty(n, np.uint8)
        check(0 if lib().bonsai_dit_weight(self.handle, name.encode(), buf.ctypes.data, n) == n
              else -1, f"bonsai_dit_weight({name})")
        return buf

    def set_weight(self, name: str, data: np.ndarray):
        """Replace a weight from host bytes in the layout weight() returns."""
        buf = np.ascontiguousarray(data)
        check(lib().bonsai_dit_set_weight(self.handle, name.encode(), buf.ctypes.data, buf.nbytes),
              f"bonsai_dit_set_weight({name})")

    def load_safetensors(self, path):
        """Load a checkpoint in the reference's packed safetensors layout (klein4b)."""
        check(lib().bonsai_dit_load_safetensors(self.handle, str(path).encode()),
              "bonsai_dit_load_safetensors")

    def sample(self, latents, txt, pooled, n_steps: int, stream=None) -> np.ndarray:
        """Whole Euler loop on the device (latents updated in place); returns the
        per-step stats [n_steps][5] = NaN count, Inf count, min, max, mean."""
        stats = np.zeros((n_steps, 5), np.float32)
        check(lib().bonsai_dit_sample(self.handle, latents.data_ptr(),
                                      txt.data_ptr() if txt is not None else None,
                                      pooled.data_ptr() if pooled is not None else None,
                                      n_steps, stats.ctypes.data, stream_ptr(stream)),
              "bonsai_dit_sample")
        return stats

    def weight_f32(self, name: str) -> np.ndarray:
        return self.weight(name).view(np.float32)

    def rope_ids(self) -> np.ndarray:
        """Token ids [L][n_axes] (src/diffuser.cpp:240-249): text 0, image (.., y, x)."""
        na = len(self.axes)
        ids = np.zeros((self.L, na), np.float32)
        for y in range(self.grid_h):
            for x in range(self.grid_w):
                ids[self.txt + y * self.grid_w + x, na - 2] = y
                ids[self.txt + y * self.grid_w + x, na - 1] = x
        return ids

    def forward(self, img, txt, pooled, t: float, out, stream=None):
        check(lib().bonsai_dit_forward(self.handle, img.data_ptr(),
                                       txt.data_ptr() if txt is not None else None,
                                       pooled.data_ptr() if pooled is not None else None,
                                       float(t), out.data_ptr(), stream_ptr(stream)),
              "bonsai_dit_forward")

    def forward_host(self, img: np.ndarray, txt: np.ndarray, pooled, t: float,
                     out: np.ndarray, stream=None):
        check(lib().bonsai_dit_forward_host(self.handle, img.ctypes.data,
                                            txt.ctypes.data if txt is not None else None,
                                            pooled.ctypes.data if pooled is not None else None,
                                            float(t), out.ctypes.data, stream_ptr(stream)),
              "bonsai_dit_forward_host")

    def set_state(self, hidden, vec, stream=None):
        check(lib().bonsai_dit_set_state(self.handle, hidden.data_ptr(), vec.data_ptr(),
                                         stream_ptr(stream)), "bonsai_dit_set_state")

    def get_state(self, hidden, stream=None):
        check(lib().bonsai_dit_get_state(self.handle, hidden.data_ptr(), stream_ptr(stream)),
              "bonsai_dit_get_state")

    # ---- partitioned (multi-GPU) driving, see bonsai_b200.headsplit
    def set_partition(self, rank: int, world: int):
        check(lib().bonsai_dit_set_partition(self.handle, rank, world), "bonsai_dit_set_partition")

    def set_peers(self, xm_ptrs, cat_ptrs):
        """Fused exchanges: every rank's xm / cat device pointers as seen
        from this GPU ([rank] = this model's own); None switches back."""
        if xm_ptrs is None:
            check(lib().bonsai_dit_set_peers(self.handle, None, None, 0), "bonsai_dit_set_peers")
            return
        n = len(xm_ptrs)
        xa = (_vp * n)(*xm_ptrs)
        ca = (_vp * n)(*cat_ptrs)
        check(lib().bonsai_dit_set_peers(self.handle, xa, ca, n), "bonsai_dit_set_peers")

    def set_qkv_peers(self, qkv_ptrs):
        """QKV scatter: every rank's qkv device pointer as seen from this GPU
        ([rank] = this model's own); None switches back to the xm broadcast."""
        if qkv_ptrs is None:
            check(lib().bonsai_dit_set_qkv_peers(self.handle, None, 0), "bonsai_dit_set_qkv_peers")
            return
        n = len(qkv_ptrs)
        check(lib().bonsai_dit_set_qkv_peers(self.handle, (_vp * n)(*qkv_ptrs), n),
              "bonsai_dit_set_qkv_peers")

    def ipc_handle(self, name: str) -> bytes:
        buf = ctypes.create_string_buffer(64)
        check(lib().bonsai_dit_ipc_handle(self.handle, name.encode(), buf), "bonsai_dit_ipc_handle")
        return buf.raw

    def open_qkv_peers(self, handles: bytes, world: int):
        assert len(handles) == 64 * world
        check(lib().bonsai_dit_open_qkv_peers(self.handle, handles, world),
              "bonsai_dit_open_qkv_peers")

    def open_flag_peers(self, handles: bytes, world: int):
        """Every rank's "flags" IPC handle (world x 64 bytes): enables
        barrier(); order the ranks once (host barrier) before the first."""
        assert len(handles) == 64 * world
        check(lib().bonsai_dit_open_flag_peers(self.handle, handles, world),
              "bonsai_dit_open_flag_peers")

    def barrier(self, stream=None):
        """Stream-ordered barrier of the partitioned ranks over peer flags."""
        check(lib().bonsai_dit_barrier(self.handle, stream_ptr(stream)), "bonsai_dit_barrier")

    def ipc_handles(self) -> bytes:
        buf = ctypes.create_string_buffer(128)
        check(lib().bonsai_dit_ipc_handles(self.handle, buf), "bonsai_dit_ipc_handles")
        return buf.raw

    def open_peers(self, handles: bytes, world: int):
        assert len(handles) == 128 * world
        check(lib().bonsai_dit_open_peers(self.handle, handles, world), "bonsai_dit_open_peers")

    def buffer(self, name: str, dtype, shape):
        """Engine buffer as a torch tensor view (no copy)."""
        import torch
        ptr, nbytes = _vp(), _c_ll()
        check(lib().bonsai_dit_buffer(self.handle, name.encode(), ctypes.byref(ptr),
                                      ctypes.byref(nbytes)), f"bonsai_dit_buffer({name})")
        return _wrap_device(ptr.value, nbytes.value, dtype, shape)

    def begin(self, img, txt, pooled, t: float, stream=None):
        check(lib().bonsai_dit_begin(self.handle, img.data_ptr(),
                                     txt.data_ptr() if txt is not None else None,
                                     pooled.data_ptr() if pooled is not None else None,
                                     float(t), stream_ptr(stream)), "bonsai_dit_begin")

    def phase(self, kind: int, block: int, phase: int, stream=None):
        check(lib().bonsai_dit_phase(self.handle, kind, block, phase, stream_ptr(stream)),
              "bonsai_dit_phase")

    def end(self, out, stream=None):
        check(lib().bonsai_dit_end(self.handle, out.data_ptr(), stream_ptr(stream)), "bonsai_dit_end")

    def double_block(self, i: int, stream=None):
        check(lib().bonsai_dit_double_block(self.handle, i, stream_ptr(stream)), "double_block")

    def single_block(self, i: int, stream=None):
        check(lib().bonsai_dit_single_block(self.handle, i, stream_ptr(stream)), "single_block")


class Vae:
    """The Flux VAE decoder on the device (bonsai_vae_* entry points), the
    reference's bonsai_vae program (src/vae_decoder.cpp) for one encoded
    latent size: latent f32 [128][h][w] -> raw image f32 [3][16h][16w]."""

    def __init__(self, latent_h: int, latent_w: int, seed: int = 0):
        h = _vp()
        check(lib().bonsai_vae_create(latent_h, latent_w, seed, ctypes.byref(h)), "bonsai_vae_create")
        self.handle = h
        self.latent_h, self.latent_w = latent_h, latent_w
        self.image_h, self.image_w = 16 * latent_h, 16 * latent_w

    def close(self):
        if getattr(self, "handle", None):
            lib().bonsai_vae_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_safetensors(self, path) -> None:
        check(lib().bonsai_vae_load_safetensors(self.handle, str(path).encode()),
              "bonsai_vae_load_safetensors")

    def decode(self, latent, image, stream=None) -> None:
        """latent: cuda f32 [128][h][w]; image: cuda f32 [3][16h][16w]."""
        assert latent.is_contiguous() and image.is_contiguous()
        assert latent.numel() == 128 * self.latent_h * self.latent_w
        assert image.numel() == 3 * self.image_h * self.image_w
        check(lib().bonsai_vae_decode(self.handle, latent.data_ptr(), image.data_ptr(),
                                      stream_ptr(stream)), "bonsai_vae_decode")

    def decode_host(self, latent: np.ndarray, stream=None) -> np.ndarray:
        lat = np.ascontiguousarray(latent, dtype=np.float32)
        assert lat.size == 128 * self.latent_h * self.latent_w
        out = np.empty((3, self.image_h, self.image_w), np.float32)
        check(lib().bonsai_vae_decode_host(self.handle, lat.ctypes.data, out.ctypes.data,
                                           stream_ptr(stream)), "bonsai_vae_decode_host")
        return out


def conv2d_nhwc(x, w, bias, out, resid=None, stream=None) -> None:
    """x: cuda f16/bf16 NHWC [H][W][cin]; w: cuda f32 [cout][cin][k][k];
    bias: cuda f32 [cout] or None; out (and resid): cuda f32 NHWC [H][W][cout]."""
    import torch
    hh, ww, cin = x.shape
    cout, _, k, _ = w.shape
    assert x.is_contiguous() and w.is_contiguous() and out.is_contiguous()
    check(lib().bonsai_conv2d_nhwc(x.data_ptr(), hh, ww, cin, int(x.dtype == torch.bfloat16),
                                   w.data_ptr(), cout, k, bias.data_ptr() if bias is not None else None,
                                   resid.data_ptr() if resid is not None else None, out.data_ptr(),
                                   stream_ptr(stream)), "bonsai_conv2d_nhwc")


def vae_rgb8(image, rgb, stream=None) -> None:
    """image: cuda f32 [3][H][W]; rgb: cuda u8 [H][W][3] (sigmoid, x255, clamp)."""
    _, hh, ww = image.shape
    check(lib().bonsai_vae_rgb8(image.data_ptr(), hh, ww, rgb.data_ptr(), stream_ptr(stream)),
          "bonsai_vae_rgb8")


def _wrap_device(ptr: int, nbytes: int, dtype, shape):
    """A torch tensor aliasing device memory owned by the engine (no copy)."""
    import torch

    class _Holder:
        def __init__(self, p, n):
            self.__cuda_array_interface__ = {
                "shape": (n,), "typestr": "|u1", "data": (p, False), "version": 3}

    flat = torch.as_tensor(_Holder(ptr, nbytes), device="cuda")
    return flat.view(dtype).view(shape)
