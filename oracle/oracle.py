"""ctypes wrapper around liboasr_oracle.so -- the CPU restatement of ggml
semantics.  TEST INFRASTRUCTURE ONLY: imported by tests/, by
__graft_entry__.smoke() and by bench.py's cpu_baseline leg, never by the
product package (openasr_b200).

Every helper takes/returns numpy arrays in ggml's dimension order written
fastest-first: a tensor with ne = [ne0, ne1, ne2, ne3] is a C-contiguous numpy
array of shape (ne3, ne2, ne1, ne0).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboasr_oracle.so")

F32, F16, Q4_0, Q8_0, Q4_K, Q8_K, I32 = 0, 1, 2, 8, 12, 15, 26
FA_GGML, FA_F32, FA_TC128 = 0, 1, 2
# decode-attention kernels whose arithmetic oo_fa_device restates (fattn.cu)
FAK_SPLIT, FAK_HEADS, FAK_GQA = 0, 1, 2
# norm reduction layouts (elementwise.cu): one warp per 32E-element chunk, or the 256-thread row kernel
NORM_E8, NORM_E4, NORM_ROW = 8, 4, 0
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q8_K: (256, 292)}


class OoTensor(ctypes.Structure):
    _fields_ = [
        ("type", ctypes.c_int32),
        ("_pad", ctypes.c_int32),
        ("data", ctypes.c_void_p),
        ("ne", ctypes.c_int64 * 4),
        ("nb", ctypes.c_int64 * 4),
    ]


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        src_mtime = max(os.path.getmtime(os.path.join(HERE, f)) for f in ("oracle.c", "oracle.h"))
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < src_mtime:
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, F, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        L.oo_f32_to_f16.argtypes, L.oo_f32_to_f16.restype = [F], ctypes.c_uint16
        L.oo_f16_to_f32.argtypes, L.oo_f16_to_f32.restype = [ctypes.c_uint16], F
        L.oo_synth_normal.argtypes, L.oo_synth_normal.restype = [ctypes.c_uint64, ctypes.c_uint64, P, I64, F, F], None
        L.oo_row_size.argtypes, L.oo_row_size.restype = [I, I64], I64
        L.oo_quantize_rows.argtypes, L.oo_quantize_rows.restype = [I, P, P, I64, I64], I
        L.oo_dequantize_row.argtypes, L.oo_dequantize_row.restype = [I, P, P, I64], I
        TP = ctypes.POINTER(OoTensor)
        L.oo_mul_mat.argtypes, L.oo_mul_mat.restype = [TP, TP, TP], I
        L.oo_flash_attn_ext.argtypes, L.oo_flash_attn_ext.restype = [TP, TP, TP, TP, F, I, TP], I
        L.oo_set_rows.argtypes, L.oo_set_rows.restype = [TP, TP, P, I64], I
        L.oo_argmax_first.argtypes, L.oo_argmax_first.restype = [P, I64, I64, P], None
        for name in ("oo_norm", "oo_rms_norm"):
            getattr(L, name).argtypes, getattr(L, name).restype = [P, P, I64, I64, F], None
        for name in ("oo_gelu", "oo_silu"):
            getattr(L, name).argtypes, getattr(L, name).restype = [P, P, I64], None
        L.oo_rope_neox.argtypes, L.oo_rope_neox.restype = [P, I64, I64, I64, P, F], None
        L.oo_expf.argtypes, L.oo_expf.restype = [F], F
        L.oo_norm_dev.argtypes, L.oo_norm_dev.restype = [P, P, I64, I64, F, I, I], None
        L.oo_fa_device.argtypes, L.oo_fa_device.restype = [TP, TP, TP, TP, F, I, I64, TP], I
        L.oo_fa_device_splits.argtypes, L.oo_fa_device_splits.restype = [I, I64, I64], I
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def tensor(a: np.ndarray, ggml_type: int, ne: list[int] | tuple[int, ...] | None = None) -> OoTensor:
    """Describe a C-contiguous numpy buffer as a contiguous ggml tensor."""
    assert a.flags["C_CONTIGUOUS"]
    if ne is None:
        shape = list(a.shape)[::-1]
        if ggml_type in (Q4_0, Q8_0, Q4_K, Q8_K):
            raise ValueError("quantized tensors need explicit ne")
        ne = shape + [1] * (4 - len(shape))
    ne = list(ne) + [1] * (4 - len(ne))
    be, bb = BLOCK[ggml_type]
    nb0 = bb
    nb1 = ne[0] // be * bb
    nb = [nb0, nb1, nb1 * ne[1], nb1 * ne[1] * ne[2]]
    t = OoTensor()
    t.type = ggml_type
    t.data = _ptr(a)
    t.ne[:] = ne
    t.nb[:] = nb
    return t


# ---- scalar / data helpers -------------------------------------------------
def synth_normal(seed: int, n: int, mean: float = 0.0, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().oo_synth_normal(seed & (2**64 - 1), offset, _ptr(out), n, mean, std)
    return out


def row_size(ggml_type: int, ne0: int) -> int:
    return int(lib().oo_row_size(ggml_type, ne0))


def quantize(ggml_type: int, x: np.ndarray) -> np.ndarray:
    """Quantize rows of a 2-D (rows, ne0) f32 array -> (rows, row_bytes) uint8."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    rows, ne0 = x.shape
    rs = row_size(ggml_type, ne0)
    if rs < 0:
        raise ValueError(f"ne0={ne0} not a multiple of the block size of type {ggml_type}")
    out = np.empty((rows, rs), np.uint8)
    rc = lib().oo_quantize_rows(ggml_type, _ptr(x), _ptr(out), rows, ne0)
    if rc != 0:
        raise RuntimeError(f"oo_quantize_rows failed ({rc})")
    return out


def dequantize(ggml_type: int, q: np.ndarray, ne0: int) -> np.ndarray:
    q = np.ascontiguousarray(q, np.uint8)
    rows = q.size // row_size(ggml_type, ne0)
    q = q.reshape(rows, -1)
    out = np.empty((rows, ne0), np.float32)
    for r in range(rows):
        rc = lib().oo_dequantize_row(ggml_type, _ptr(q[r]), _ptr(out[r]), ne0)
        if rc != 0:
            raise RuntimeError("oo_dequantize_row failed")
    return out


# ---- ops ---------------------------------------------------------------------
def mul_mat(w: np.ndarray, w_type: int, K: int, N: int, x: np.ndarray, x_type: int = F32,
            w_batch: tuple[int, int] = (1, 1)) -> np.ndarray:
    """ggml mul_mat: w is (w_ne3, w_ne2, N, row_bytes) blocks, x is (ne3, ne2, M, K).
    Returns (ne3, ne2, M, N) f32."""
    x = np.ascontiguousarray(x)
    xs = x.shape
    while len(xs) < 4:
        xs = (1,) + xs
    ne3, ne2, M, Kx = xs
    assert Kx == K
    w = np.ascontiguousarray(w)
    tw = tensor(w, w_type, [K, N, w_batch[1], w_batch[0]])
    tx = tensor(x, x_type, [K, M, ne2, ne3])
    out = np.zeros((ne3, ne2, M, N), np.float32)
    to = tensor(out, F32, [N, M, ne2, ne3])
    rc = lib().oo_mul_mat(ctypes.byref(tw), ctypes.byref(tx), ctypes.byref(to))
    if rc != 0:
        raise RuntimeError(f"oo_mul_mat failed ({rc})")
    return out.reshape(x.shape[:-1] + (N,)) if x.ndim < 4 else out


def flash_attn_ext(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray | None,
                   scale: float, mode: int = FA_GGML) -> np.ndarray:
    """q f32 (S, H, NQ, D); k/v f16|f32 (S, HKV, NKV, D); mask f16-bits uint16 (.., NQp, NKVp).
    Returns (S, NQ, H, DV) f32 == ggml dst ne [DV, H, NQ, S]."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    kt = F16 if k.dtype == np.float16 else F32
    S, H, NQ, D = q.shape
    DV = v.shape[-1]
    tq = tensor(q, F32)
    tk = tensor(k.view(np.uint16) if kt == F16 else k, kt)
    tv = tensor(v.view(np.uint16) if kt == F16 else v, kt)
    tm = None
    if mask is not None:
        mask = np.ascontiguousarray(mask.view(np.uint16) if mask.dtype == np.float16 else mask)
        tm = tensor(mask, F16)
        tm.nb[:] = [2, mask.shape[-1] * 2, mask.shape[-1] * 2 * mask.shape[-2],
                    mask.shape[-1] * 2 * mask.shape[-2] * (mask.shape[-3] if mask.ndim >= 3 else 1)]
    out = np.zeros((S, NQ, H, DV), np.float32)
    to = tensor(out, F32)
    rc = lib().oo_flash_attn_ext(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                 ctypes.byref(tm) if tm is not None else None, scale, mode, ctypes.byref(to))
    if rc != 0:
        raise RuntimeError(f"oo_flash_attn_ext failed ({rc})")
    return out


def set_rows(dst: np.ndarray, src: np.ndarray, rows: np.ndarray) -> None:
    """dst (ne3, ne2, R, D) f32|f16 updated in place; src (ne3, ne2, n, D) f32."""
    dt = F16 if dst.dtype == np.float16 else F32
    td = tensor(dst.view(np.uint16) if dt == F16 else dst, dt)
    ts = tensor(np.ascontiguousarray(src, np.float32), F32)
    r = np.ascontiguousarray(rows, np.int64)
    rc = lib().oo_set_rows(ctypes.byref(td), ctypes.byref(ts), _ptr(r), r.size)
    if rc != 0:
        raise RuntimeError("oo_set_rows failed")


def argmax_first(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    out = np.empty(x.shape[0], np.int32)
    lib().oo_argmax_first(_ptr(x), x.shape[-1], x.shape[0], _ptr(out))
    return out


def norm(x: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oo_norm(_ptr(x), _ptr(y), x.shape[-1], x.size // x.shape[-1], eps)
    return y


def rms_norm(x: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oo_rms_norm(_ptr(x), _ptr(y), x.shape[-1], x.size // x.shape[-1], eps)
    return y


def gelu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oo_gelu(_ptr(x), _ptr(y), x.size)
    return y


def silu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oo_silu(_ptr(x), _ptr(y), x.size)
    return y


def rope_neox(x: np.ndarray, pos: np.ndarray, freq_base: float) -> np.ndarray:
    """x (T, H, D) f32 -> rotated copy."""
    y = np.ascontiguousarray(x, np.float32).copy()
    T, H, D = y.shape
    p = np.ascontiguousarray(pos, np.int32)
    lib().oo_rope_neox(_ptr(y), D, H, T, _ptr(p), freq_base)
    return y


# ---- the decode path's canonical arithmetic (oracle.h) ------------------------------------
def expf(x) -> np.ndarray:
    """the decode path's e^x (oo_expf) elementwise"""
    x = np.asarray(x, np.float32)
    f = lib().oo_expf
    return np.array([f(float(v)) for v in x.ravel()], np.float32).reshape(x.shape)


def norm_dev(x: np.ndarray, eps: float, rms: bool, layout: int) -> np.ndarray:
    """LayerNorm / RMSNorm of the last axis with the device's reduction tree (oo_norm_dev)"""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oo_norm_dev(_ptr(x), _ptr(y), x.shape[-1], x.size // x.shape[-1], eps, 1 if rms else 0, layout)
    return y


def norm_layout(n: int, family: int | None) -> int:
    """the reduction layout the device's residual + norm (+ quantize) kernel uses for rows of n
    whose output feeds a mul_mat of activation family `family` (Q8_0 -> q8_0 planes, Q4_K ->
    q8_K planes, None -> f32 only): elementwise.cu launch_resid_norm_quant"""
    E = 4 if family == Q8_0 else 8
    if n % (32 * E) == 0 and n // (32 * E) <= 32 and (family != Q8_K or n % 256 == 0):
        return E
    return NORM_ROW


def fa_device(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray | None, scale: float,
              kind: int, nkv_max: int | None = None) -> np.ndarray:
    """Decode attention with the device kernels' arithmetic (oo_fa_device).  Shapes as
    flash_attn_ext; k / v hold the live prefix, nkv_max the cache length (split plan)."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    kt = F16 if k.dtype == np.float16 else F32
    S, H, NQ, D = q.shape
    tq = tensor(q, F32)
    tk = tensor(k.view(np.uint16) if kt == F16 else k, kt)
    tv = tensor(v.view(np.uint16) if kt == F16 else v, kt)
    tm = None
    if mask is not None:
        mask = np.ascontiguousarray(mask.view(np.uint16) if mask.dtype == np.float16 else mask)
        tm = tensor(mask, F16)
        tm.nb[:] = [2, mask.shape[-1] * 2, mask.shape[-1] * 2 * mask.shape[-2],
                    mask.shape[-1] * 2 * mask.shape[-2] * (mask.shape[-3] if mask.ndim >= 3 else 1)]
    out = np.zeros((S, NQ, H, D), np.float32)
    to = tensor(out, F32)
    nkv_max = k.shape[-2] if nkv_max is None else nkv_max
    rc = lib().oo_fa_device(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                            ctypes.byref(tm) if tm is not None else None, scale, kind, nkv_max, ctypes.byref(to))
    if rc != 0:
        raise RuntimeError(f"oo_fa_device failed ({rc})")
    return out


def fa_device_splits(kind: int, nkv_max: int, groups: int = 1) -> int:
    return int(lib().oo_fa_device_splits(kind, nkv_max, groups))
