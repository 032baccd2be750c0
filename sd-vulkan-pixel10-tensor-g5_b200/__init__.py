"""Python host binding of ``libsdg.so`` — the B200 SD1.5 UNet engine.

Mirrors the reference's host surface (``sd/VulkanBench.kt:10-27``, the JNI
entry points of ``app/src/main/cpp/vk_engine.cpp``) over the C ABI declared in
``include/sdg.h``:

=========================  ==========================================
reference (Kotlin/JNI)     here
=========================  ==========================================
``unetInit(shaders, dir)`` ``Engine(device, weights_dir)``
``unetForward(...)``       ``Engine.forward_tproj`` / ``Engine.forward``
``unetForward2(...)``      ``Engine.forward_cfg``
``unetProfile()``          ``Engine.profile``
``unetRelease()``          ``Engine.release``
op wrappers (C++ static)   ``conv2d``, ``linear``, ``groupnorm``, ...
=========================  ==========================================

Import the package with ``importlib.import_module`` (the directory name
contains dashes) or through ``sdg_b200 = load_package()`` helpers in tests.
There is no CPU fallback: every call goes through the CUDA library, and
loading fails loudly when ``libsdg.so`` is missing.
"""
from __future__ import annotations

import ctypes
import os
import re
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from . import multigpu  # noqa: E402,F401  (batch sharding + latent gather across GPUs)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsdg.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "sdg.h")

SDG_OK = 0
STATUS = {0: "SDG_OK", 1: "SDG_ERR_CUDA", 2: "SDG_ERR_ARG", 3: "SDG_ERR_SHAPE", 4: "SDG_ERR_MISSING_WEIGHT",
          5: "SDG_ERR_TIMEOUT", 6: "SDG_ERR_IO", 7: "SDG_ERR_NOT_INIT", 8: "SDG_ERR_DEVICE", 9: "SDG_ERR_NCCL",
          10: "SDG_ERR_UNSUPPORTED"}


class SdgError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class LaunchRow(ctypes.Structure):
    _fields_ = [("label", ctypes.c_char * 128), ("category", ctypes.c_char * 8), ("ms", ctypes.c_double),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


class ProfileRow(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("ms", ctypes.c_double), ("launches", ctypes.c_int),
                ("flops", ctypes.c_double), ("bytes", ctypes.c_double)]


_lib: Optional[ctypes.CDLL] = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_SIGS = {
    "sdg_init": (_I, [_I, ctypes.c_char_p, ctypes.POINTER(_P)]),
    "sdg_upload_weight": (_I, [_P, ctypes.c_char_p, _P, ctypes.POINTER(ctypes.c_int64), _I]),
    "sdg_load_dir": (_I, [_P, ctypes.c_char_p]),
    "sdg_prepare": (_I, [_P]),
    "sdg_quantize_wo8": (_I, [_P]),
    "sdg_release": (_I, [_P]),
    "sdg_last_error": (_I, [ctypes.c_char_p, _I]),
    "sdg_unet_forward": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "sdg_unet_forward_tproj": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "sdg_unet_forward_device": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _P, _P]),
    "sdg_unet_forward_cfg": (_I, [_P, _P, _F, _P, _P, _I, _I, _P]),
    "sdg_lcm_denoise": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P]),
    "sdg_lcm_denoise_ex": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P]),
    "sdg_profile": (_I, [_P, _I, _I, _I, ctypes.POINTER(ProfileRow), _I]),
    "sdg_forward_launches": (_I, [_P, _I, _I, _I]),
    "sdg_profile_launches": (_I, [_P, _I, _I, _I, ctypes.c_char_p, _I, ctypes.POINTER(LaunchRow), _I]),
    "sdg_profile_category": (_I, [_P, _I, _I, _I, ctypes.c_char_p, _I, ctypes.POINTER(ctypes.c_double),
                                  ctypes.POINTER(_I), ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
    "sdg_gemm_plan": (_I, [_I, _I, _I, _I, _I, _P]),
    "sdg_selftest_stalled_gemm": (_I, [_P, _P, _I, _I, _I, _P, _I, _I, _P, _P]),
    "sdg_conv2d": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _I, _I, _P, _P, _I, _P, _P, _P, ctypes.c_size_t, _P,
                        _P]),
    "sdg_linear": (_I, [_P, _I, _I, _P, _P, _I, _P, _I, _P, _P, ctypes.c_size_t, _P, _P]),
    "sdg_linear_wo8": (_I, [_P, _I, _I, _P, _P, _P, _I, _P, _I, _P, _P, ctypes.c_size_t, _P, _P]),
    "sdg_groupnorm": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _F, _I, _P, _P, _P]),
    "sdg_groupnorm_scratch_bytes": (ctypes.c_size_t, [_I, _I, _I, _I]),
    "sdg_groupnorm_noalloc": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _F, _I, _P, _P]),
    "sdg_groupnorm_noalloc_max_scratch_bytes": (ctypes.c_size_t, []),
    "sdg_layernorm": (_I, [_P, _I, _I, _P, _P, _F, _P, _P]),
    "sdg_attention": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "sdg_add": (_I, [_P, _P, ctypes.c_size_t, _P, _P]),
    "sdg_concat": (_I, [_P, _I, _P, _I, _I, _P, _P]),
    "sdg_upsample2x": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "sdg_pack_upsample_conv_weights": (_I, [_P, _I, _I, _P]),
    "sdg_upsample_conv3x3": (_I, [_P, _I, _I, _I, _I, _P, _P, _I, _P, _P, ctypes.c_size_t, _P, _P]),
}


def lib() -> ctypes.CDLL:
    """Load ``libsdg.so`` (build it with ``build.py``); raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: run `python {os.path.join(HERE, 'build.py')}`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def header_symbols() -> List[str]:
    """Every entry point declared in ``include/sdg.h``."""
    txt = open(HEADER).read()
    return re.findall(r"SDG_API\s+\w+\s+(sdg_\w+)\s*\(", txt)


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    lib().sdg_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(code: int) -> None:
    if code != SDG_OK:
        raise SdgError(code, last_error())


def _ptr(a) -> Optional[int]:
    """Device pointer of a torch tensor, host pointer of a numpy array, or None."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"]
        return a.ctypes.data
    assert a.is_contiguous(), "tensor must be contiguous"
    return a.data_ptr()


def _stream(stream) -> Optional[int]:
    if stream is not None:
        return stream
    try:
        import torch
        if torch.cuda.is_available():
            return torch.cuda.current_stream().cuda_stream or None
    except Exception:
        pass
    return None


# ------------------------------------------------------------------ engine
class Engine:
    """One UNet engine on one CUDA device (``unetInit`` ... ``unetRelease``)."""

    def __init__(self, device: int = 0, weights_dir: Optional[str] = None):
        h = ctypes.c_void_p()
        check(lib().sdg_init(device, weights_dir.encode() if weights_dir else None, ctypes.byref(h)))
        self._h = h
        self.device = device

    # weights -------------------------------------------------------------
    def upload_weight(self, key: str, ref_layout_fp16: np.ndarray, torch_shape: Sequence[int]) -> None:
        """One weight in the reference on-disk layout (Linear ``[in,out]``)."""
        a = np.ascontiguousarray(ref_layout_fp16, dtype=np.float16)
        shape = (ctypes.c_int64 * len(torch_shape))(*torch_shape)
        check(lib().sdg_upload_weight(self._h, key.encode(), a.ctypes.data, shape, len(torch_shape)))

    def upload_weights(self, blobs: Iterable[Tuple[str, np.ndarray]]) -> None:
        for k, a in blobs:
            self.upload_weight(k, a, a.shape)

    def load_dir(self, d: str) -> None:
        check(lib().sdg_load_dir(self._h, d.encode()))

    def prepare(self) -> None:
        check(lib().sdg_prepare(self._h))

    def quantize_wo8(self) -> None:
        """Use weight-only int8 weights (per output channel, scale fp16(max|w|/127));
        must precede ``prepare`` / the first forward."""
        check(lib().sdg_quantize_wo8(self._h))

    # forward -------------------------------------------------------------
    def forward(self, latent: np.ndarray, timesteps, context: np.ndarray) -> np.ndarray:
        """Host buffers in, host buffer out: latent [B,4,H,W], timesteps [1|B], context [B,77,768]."""
        lat = np.ascontiguousarray(latent, dtype=np.float32)
        t = np.ascontiguousarray(np.atleast_1d(np.asarray(timesteps, dtype=np.float32)))
        ctx = np.ascontiguousarray(context, dtype=np.float32)
        B, _, H, W = lat.shape
        out = np.empty_like(lat)
        check(lib().sdg_unet_forward(self._h, lat.ctypes.data, t.ctypes.data, t.size, ctx.ctypes.data, B, H, W,
                                     out.ctypes.data, None))
        return out

    def forward_tproj(self, latent: np.ndarray, temb_proj: np.ndarray, context: np.ndarray) -> np.ndarray:
        lat = np.ascontiguousarray(latent, dtype=np.float32)
        tp = np.ascontiguousarray(np.atleast_2d(temb_proj), dtype=np.float32)
        ctx = np.ascontiguousarray(context, dtype=np.float32)
        B, _, H, W = lat.shape
        out = np.empty_like(lat)
        check(lib().sdg_unet_forward_tproj(self._h, lat.ctypes.data, tp.ctypes.data, tp.shape[0], ctx.ctypes.data, B,
                                           H, W, out.ctypes.data, None))
        return out

    def forward_device(self, latent, timesteps, context, out, stream=None) -> None:
        """torch CUDA tensors (fp32), asynchronous on ``stream``."""
        B, _, H, W = latent.shape
        check(lib().sdg_unet_forward_device(self._h, _ptr(latent), _ptr(timesteps), timesteps.numel(), _ptr(context),
                                            B, H, W, _ptr(out), _stream(stream)))

    def forward_cfg(self, latent: np.ndarray, timestep: float, cond: np.ndarray, uncond: np.ndarray) -> np.ndarray:
        lat = np.ascontiguousarray(latent, dtype=np.float32)
        _, H, W = lat.shape
        out = np.empty((2,) + lat.shape, dtype=np.float32)
        check(lib().sdg_unet_forward_cfg(self._h, lat.ctypes.data, float(timestep),
                                         np.ascontiguousarray(cond, dtype=np.float32).ctypes.data,
                                         np.ascontiguousarray(uncond, dtype=np.float32).ctypes.data, H, W,
                                         out.ctypes.data))
        return out

    def lcm_denoise(self, latents: np.ndarray, cond: np.ndarray, uncond: Optional[np.ndarray],
                    step_noise: Optional[np.ndarray], steps: int = 4, cfg: float = 1.5,
                    cfg_steps: Optional[int] = None) -> np.ndarray:
        """LCM loop on the device; guidance on the first ``cfg_steps`` steps (all when None)."""
        lat = np.ascontiguousarray(latents, dtype=np.float32)
        n, _, H, W = lat.shape
        out = np.empty_like(lat)
        noise = None if step_noise is None else np.ascontiguousarray(step_noise, dtype=np.float32)
        unc = None if uncond is None else np.ascontiguousarray(uncond, np.float32)
        check(lib().sdg_lcm_denoise_ex(self._h, lat.ctypes.data, np.ascontiguousarray(cond, np.float32).ctypes.data,
                                       None if unc is None else unc.ctypes.data,
                                       None if noise is None else noise.ctypes.data, n, H, W, steps, float(cfg),
                                       steps if cfg_steps is None else int(cfg_steps), out.ctypes.data))
        return out

    def profile(self, B: int = 2, H: int = 64, W: int = 64) -> Dict[str, Tuple[float, int, float, float]]:
        """{category: (device ms, launches, algorithmic FLOPs, algorithmic bytes)} of one eager forward."""
        rows = (ProfileRow * 16)()
        n = lib().sdg_profile(self._h, B, H, W, rows, 16)
        if n < 0:
            raise SdgError(-n, last_error())
        return {rows[i].name.decode(): (rows[i].ms, rows[i].launches, rows[i].flops, rows[i].bytes) for i in range(n)}

    def profile_category(self, categories: str, B: int = 2, H: int = 64, W: int = 64,
                         reps: int = 20) -> Tuple[float, int, float, float]:
        """(device ms per forward, launches per forward, algorithmic FLOPs, algorithmic bytes) of the
        forward's launches of the given categories ("CONV3+GEMM", "GN", ...) replayed alone as a graph."""
        ms, n, fl, by = ctypes.c_double(), _I(), ctypes.c_double(), ctypes.c_double()
        check(lib().sdg_profile_category(self._h, B, H, W, categories.encode(), reps, ctypes.byref(ms),
                                         ctypes.byref(n), ctypes.byref(fl), ctypes.byref(by)))
        return ms.value, n.value, fl.value, by.value

    def profile_launches(self, categories: str, B: int = 2, H: int = 64, W: int = 64, reps: int = 10) -> List[dict]:
        """Per-launch device times of the forward's launches of the given categories, in forward order."""
        rows = (LaunchRow * 1024)()
        n = lib().sdg_profile_launches(self._h, B, H, W, categories.encode(), reps, rows, 1024)
        if n < 0:
            raise SdgError(-n, last_error())
        return [{"label": rows[i].label.decode(), "category": rows[i].category.decode(), "ms": rows[i].ms,
                 "flops": rows[i].flops, "bytes": rows[i].bytes} for i in range(n)]

    def forward_launches(self, B: int, H: int, W: int) -> int:
        return lib().sdg_forward_launches(self._h, B, H, W)

    def release(self) -> None:
        if self._h:
            check(lib().sdg_release(self._h))
            self._h = None

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


# ------------------------------------------------------------------ op surface (torch CUDA tensors)
def conv2d(x, w, bias, Co: int, k: int = 3, stride: int = 1, x2=None, rowbias=None, residual=None, act: int = 0,
           out=None, col_scratch=None, workspace=None, err_word=None, stream=None):
    """x [B,H,W,Ci1] fp16 (x2 [B,H,W,Ci2] concatenated after it), w [Co][k*k][Ci] fp16.
    col_scratch is accepted and ignored (stride 2 runs as an implicit GEMM)."""
    import torch
    B, H, W, Ci1 = x.shape
    Ci2 = 0 if x2 is None else x2.shape[3]
    Ho, Wo = (H, W) if stride == 1 else ((H - 1) // 2 + 1, (W - 1) // 2 + 1)
    if out is None:
        out = torch.empty((B, Ho, Wo, Co), dtype=torch.float16, device=x.device)
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().sdg_conv2d(_ptr(x), _ptr(x2), B, H, W, Ci1, Ci2, _ptr(w), _ptr(bias), Co, k, stride, _ptr(rowbias),
                           _ptr(residual), act, _ptr(out), _ptr(col_scratch), _ptr(workspace), wsb, _ptr(err_word),
                           _stream(stream)))
    return out


def gemm_plan(M: int, N: int, K: int, taps: int = 1, workspace: bool = True) -> Dict[str, int]:
    """The tile chooser's plan for an M x N x K GEMM (taps=9: 3x3 conv, K = 9*Cin) on the current device."""
    out = (ctypes.c_int * 4)()
    check(lib().sdg_gemm_plan(M, N, K, taps, 1 if workspace else 0, ctypes.addressof(out)))
    return {"bn": out[0], "pair": out[1], "splits": out[2], "csplit": out[3]}


def linear(x, w, bias=None, residual=None, act: int = 0, out=None, workspace=None, err_word=None, stream=None):
    """x [M,K] fp16, w [N,K] fp16 -> [M,N] (act 2 = GEGLU, w packed by pack_geglu_weight -> [M,N/2])."""
    import torch
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N // 2 if act == 2 else N), dtype=torch.float16, device=x.device)
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().sdg_linear(_ptr(x), M, K, _ptr(w), _ptr(bias), N, _ptr(residual), act, _ptr(out), _ptr(workspace),
                           wsb, _ptr(err_word), _stream(stream)))
    return out


def linear_wo8(x, w8, wscale, bias=None, residual=None, act: int = 0, out=None, workspace=None, err_word=None,
               stream=None):
    """x [M,K] fp16, w8 [N,K] int8, wscale [N] fp32 -> [M,N] fp16 (weight = w8 * wscale per row)."""
    import torch
    M, K = x.shape
    N = w8.shape[0]
    if out is None:
        out = torch.empty((M, N // 2 if act == 2 else N), dtype=torch.float16, device=x.device)
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().sdg_linear_wo8(_ptr(x), M, K, _ptr(w8), _ptr(wscale), _ptr(bias), N, _ptr(residual), act, _ptr(out),
                               _ptr(workspace), wsb, _ptr(err_word), _stream(stream)))
    return out


def quantize_wo8_rows(w):
    """Per-row symmetric int8 of a [N,K] weight (torch tensor): (q int8, scale fp32), the
    same rule the engine applies (scale = fp16(max|w|/127), 1 for a zero row,
    q = clamp(round_half_even(w/scale), +-127))."""
    import torch
    wf = w.float()
    s = (wf.abs().amax(dim=1) / 127.0).half().float()
    s = torch.where(s == 0, torch.ones_like(s), s)
    q = torch.clamp(torch.round(wf / s[:, None]), -127, 127).to(torch.int8)
    return q, s


def groupnorm(x, gamma, beta, eps: float, silu: bool, x2=None, groups: int = 32, out=None, stats=None, stream=None):
    """x [B,HW,C1] (x2 [B,HW,C2] concatenated after it) fp16 -> [B,HW,C1+C2]."""
    import torch
    B, HW, C1 = x.shape
    C2 = 0 if x2 is None else x2.shape[2]
    if out is None:
        out = torch.empty((B, HW, C1 + C2), dtype=torch.float16, device=x.device)
    if stats is None:
        nbytes = lib().sdg_groupnorm_scratch_bytes(B, HW, C1 + C2, groups)
        stats = torch.empty((nbytes // 4 + 1,), dtype=torch.float32, device=x.device)
    check(lib().sdg_groupnorm(_ptr(x), _ptr(x2), B, HW, C1, C2, groups, _ptr(gamma), _ptr(beta), eps, int(silu),
                              _ptr(out), _ptr(stats), _stream(stream)))
    return out


def groupnorm_noalloc(x, gamma, beta, eps: float, silu: bool, x2=None, groups: int = 32, out=None, stream=None):
    """Same as :func:`groupnorm` but through the entry point that allocates
    nothing (its scratch is a fixed array inside the library)."""
    import torch
    B, HW, C1 = x.shape
    C2 = 0 if x2 is None else x2.shape[2]
    if out is None:
        out = torch.empty((B, HW, C1 + C2), dtype=torch.float16, device=x.device)
    check(lib().sdg_groupnorm_noalloc(_ptr(x), _ptr(x2), B, HW, C1, C2, groups, _ptr(gamma), _ptr(beta), eps,
                                      int(silu), _ptr(out), _stream(stream)))
    return out


def layernorm(x, gamma, beta, eps: float = 1e-5, out=None, stream=None):
    import torch
    M, C = x.shape
    if out is None:
        out = torch.empty_like(x)
    check(lib().sdg_layernorm(_ptr(x), M, C, _ptr(gamma), _ptr(beta), eps, _ptr(out), _stream(stream)))
    return out


def attention(q, k, vt, B: int, heads: int, Sq: int, Sk: int, d: int, vt_ld: int, out=None, err_word=None,
              stream=None):
    """q [B*heads,Sq,dp], k [B*heads,Sk,dp], vt [B*heads,d16,vt_ld] -> o [B,Sq,heads*d]."""
    import torch
    if out is None:
        out = torch.empty((B, Sq, heads * d), dtype=torch.float16, device=q.device)
    check(lib().sdg_attention(_ptr(q), _ptr(k), _ptr(vt), B, heads, Sq, Sk, d, vt_ld, _ptr(out), _ptr(err_word),
                              _stream(stream)))
    return out


def add(a, b, out=None, stream=None):
    import torch
    if out is None:
        out = torch.empty_like(a)
    check(lib().sdg_add(_ptr(a), _ptr(b), a.numel(), _ptr(out), _stream(stream)))
    return out


def concat(a, b, out=None, stream=None):
    import torch
    rows = a.numel() // a.shape[-1]
    Ca, Cb = a.shape[-1], b.shape[-1]
    if out is None:
        out = torch.empty(a.shape[:-1] + (Ca + Cb,), dtype=a.dtype, device=a.device)
    check(lib().sdg_concat(_ptr(a), Ca, _ptr(b), Cb, rows, _ptr(out), _stream(stream)))
    return out


def upsample2x(x, out=None, stream=None):
    import torch
    B, H, W, C = x.shape
    if out is None:
        out = torch.empty((B, 2 * H, 2 * W, C), dtype=x.dtype, device=x.device)
    check(lib().sdg_upsample2x(_ptr(x), B, H, W, C, _ptr(out), _stream(stream)))
    return out


def pack_upsample_conv_weight(w3):
    """3x3 conv weight [Co,Ci,3,3] (fp16 numpy array or CPU tensor) -> the folded phase weights
    [4 phases][Co][4 taps][Ci] of ``upsample_conv3x3`` (host-side, through the C ABI)."""
    import numpy as np
    w = np.ascontiguousarray(np.asarray(w3, dtype=np.float16))
    Co, Ci = w.shape[0], w.shape[1]
    assert w.shape == (Co, Ci, 3, 3), w.shape
    out = np.empty((4, Co, 4, Ci), dtype=np.float16)
    check(lib().sdg_pack_upsample_conv_weights(w.ctypes.data, Co, Ci, out.ctypes.data))
    return out


def upsample_conv3x3(x, wp, bias4, out=None, workspace=None, err_word=None, stream=None):
    """conv3x3(upsample2x(x)) + bias without the upsampled copy: x [B,H,W,Ci] fp16, wp the folded phase
    weights [4,Co,4,Ci] fp16 (pack_upsample_conv_weight, on the device), bias4 fp32 [4*Co] (the conv bias
    repeated per phase) or None; returns [B,2H,2W,Co]."""
    import torch
    B, H, W, Ci = x.shape
    Co = wp.shape[1]
    if out is None:
        out = torch.empty((B, 2 * H, 2 * W, Co), dtype=torch.float16, device=x.device)
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().sdg_upsample_conv3x3(_ptr(x), B, H, W, Ci, _ptr(wp), _ptr(bias4), Co, _ptr(out), _ptr(workspace), wsb,
                                     _ptr(err_word), _stream(stream)))
    return out


# ------------------------------------------------------------------ engine weight layouts (for the op surface)
def pack_conv_weight(w_torch):
    """PyTorch conv weight [Co,Ci,k,k] -> engine layout [Co][k*k][Ci] (same dtype/device)."""
    Co, Ci, kh, kw = w_torch.shape
    return w_torch.permute(0, 2, 3, 1).reshape(Co, kh * kw * Ci).contiguous()


def pack_geglu_weight(w_torch, b_torch=None, group: int = 16):
    """FF-proj [8C, C] (rows: value half then gate half) -> rows interleaved in groups of 16:
    [16 value rows ; the matching 16 gate rows] repeated (the layout the GEGLU epilogue reads)."""
    import torch
    N = w_torch.shape[0]
    half = N // 2
    idx = []
    for t in range(half // group):
        idx += list(range(t * group, (t + 1) * group))
        idx += list(range(half + t * group, half + (t + 1) * group))
    idx_t = torch.tensor(idx, device=w_torch.device)
    wp = w_torch.index_select(0, idx_t).contiguous()
    bp = None if b_torch is None else b_torch.index_select(0, idx_t).contiguous()
    return wp, bp


def heads_layout(x_tokens, B: int, S: int, heads: int, d: int, transpose: bool = False, s_pad: Optional[int] = None):
    """Token-major [B*S, heads*d] -> padded per-head layout used by the attention kernel:
    [B*heads, S, dp] (dp = d rounded up to 64) or, transposed, [B*heads, d16, s_pad]."""
    import torch
    dp = (d + 63) // 64 * 64
    d16 = (d + 15) // 16 * 16
    x = x_tokens.reshape(B, S, heads, d).permute(0, 2, 1, 3)  # [B, heads, S, d]
    if not transpose:
        out = torch.zeros((B * heads, S, dp), dtype=x.dtype, device=x.device)
        out[:, :, :d] = x.reshape(B * heads, S, d)
        return out
    s_pad = s_pad or S
    out = torch.zeros((B * heads, d16, s_pad), dtype=x.dtype, device=x.device)
    out[:, :d, :S] = x.reshape(B * heads, S, d).transpose(1, 2)
    return out
