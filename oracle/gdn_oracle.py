"""ctypes bindings for the CPU oracle (``libgdn_oracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` as the checker.  The product path
never imports this module.

Parity status: PARITY UNPINNED against the reference (its arithmetic lives in
closed CANN aclnn operators and absent Triton-Ascend binaries; its own tests
pin only self-consistency).  ``gdn_oracle.c`` restates the reference's
operator sequence (citations there); ``tests/test_oracle.py`` cross-checks it
against the PyTorch restatement in transformers 5.5.0 (Qwen3-Next) and against
the committed golden vectors in ``tests/golden/``.

bf16 arrays are passed as ``numpy.uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libgdn_oracle.so")
_lib = None

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile ``libgdn_oracle.so`` with ``oracle/Makefile`` if it is missing."""
    src = os.path.join(_HERE, "gdn_oracle.c")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        i64, i32, f32 = ctypes.c_int64, ctypes.c_int32, ctypes.c_float
        L.gdn_oracle_gating.argtypes = [_u16p, _u16p, _f32p, _f32p, i64, i32, _f32p, _u16p]
        L.gdn_oracle_l2norm.argtypes = [_u16p, i64, i32, _u16p]
        L.gdn_oracle_core.argtypes = [_u16p, _u16p, _u16p, _f32p, _u16p, _f32p, _u16p,
                                      _i32p, i32, i32, i32, i32, i32]
        L.gdn_oracle_tail_prologue.argtypes = [_u16p, _u16p, _u16p, i64, i32, i32, f32, i32, _u16p]
        L.gdn_oracle_gemm_bf16.argtypes = [_u16p, _u16p, i64, i64, i64, _u16p]
        L.gdn_oracle_output_tail.argtypes = [_u16p, _u16p, _u16p, _u16p, i64, i32, i32, i32,
                                             f32, i32, ctypes.c_void_p, _u16p]
        L.gdn_oracle_layer.argtypes = [_u16p, _u16p, _u16p, _u16p, _u16p, _u16p, _f32p, _f32p,
                                       _u16p, _u16p, _f32p, _u16p, _i32p, i32, i32, i32, i32,
                                       i32, i32, ctypes.c_void_p, ctypes.c_void_p]
        L.gdn_oracle_threads.restype = i32
        L.gdn_oracle_causal_conv1d.argtypes = [_u16p, _u16p, _u16p, _i32p, i32, i64, i32, _u16p]
        L.gdn_oracle_fill_synthetic.argtypes = [ctypes.c_uint64, ctypes.c_uint64,
                                                ctypes.c_uint64, i32, f32, f32, i32,
                                                ctypes.c_void_p]
        L.gdn_oracle_fill_synthetic.restype = i32
        _lib = L
    return _lib


# ------------------------------------------------------------------ bf16 --

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit pattern (uint16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------ synthetic inputs --

def fill(seed: int, tensor_id: int, shape, distribution: int, p0: float, p1: float,
         dtype: int) -> np.ndarray:
    """Seeded host tensor from the oracle's copy of the benchmark generator
    (bf16 as uint16 bit patterns when dtype is 1, float32 when 2); the same
    arguments and bits as ``gdn_b200.fill``, without the product library."""
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.uint16 if dtype == 1 else np.float32)
    if lib().gdn_oracle_fill_synthetic(seed, tensor_id, n, distribution, p0, p1, dtype,
                                       out.ctypes.data_as(ctypes.c_void_p)) != 0:
        raise ValueError("bad distribution or dtype")
    return out.reshape(shape)


# ------------------------------------------------------------ operators --

def threads() -> int:
    return int(lib().gdn_oracle_threads())


def gating(a, b, A_log, dt_bias):
    T, hv = a.shape
    g = np.empty((T, hv), np.float32)
    beta = np.empty((T, hv), np.uint16)
    lib().gdn_oracle_gating(np.ascontiguousarray(a), np.ascontiguousarray(b),
                            np.ascontiguousarray(A_log, np.float32),
                            np.ascontiguousarray(dt_bias, np.float32), T, hv, g, beta)
    return g, beta


def l2norm(x):
    d = x.shape[-1]
    out = np.empty_like(x, dtype=np.uint16)
    lib().gdn_oracle_l2norm(np.ascontiguousarray(x), x.size // d, d, out)
    return out


def core(qn, kn, v, g, beta, state, cu_seqlens, mode=0):
    """Runs the gated delta rule; ``state`` [S,Hv,D,D] f32 is updated in place.
    mode 0 = recurrent (ground truth), 1 = chunked exact, 2 = chunked with the
    reference chain's bf16 rounding points.  Returns o bf16 [T,Hv,D]."""
    T, hk, d = qn.shape
    hv = v.shape[1]
    o = np.empty((T, hv, d), np.uint16)
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    lib().gdn_oracle_core(np.ascontiguousarray(qn), np.ascontiguousarray(kn),
                          np.ascontiguousarray(v), np.ascontiguousarray(g, np.float32),
                          np.ascontiguousarray(beta), state, o, cu, len(cu) - 1, hk, hv, d, mode)
    return o


def tail_prologue(o, z, gamma, eps=1e-6, mode=0):
    rows, hv, d = o.shape
    gated = np.empty((rows, hv * d), np.uint16)
    lib().gdn_oracle_tail_prologue(np.ascontiguousarray(o), np.ascontiguousarray(z),
                                   np.ascontiguousarray(gamma), rows, hv, d, eps, mode, gated)
    return gated


def gemm_bf16(a, w):
    m, k = a.shape
    n = w.shape[0]
    out = np.empty((m, n), np.uint16)
    lib().gdn_oracle_gemm_bf16(np.ascontiguousarray(a), np.ascontiguousarray(w), m, n, k, out)
    return out


def output_tail(o, z, gamma, w, eps=1e-6, mode=0):
    """o, z bf16 [rows,Hv,D]; w bf16 [hidden, Hv*D].  Returns out bf16 [rows, hidden]."""
    rows, hv, d = o.shape
    hidden = w.shape[0]
    out = np.empty((rows, hidden), np.uint16)
    lib().gdn_oracle_output_tail(np.ascontiguousarray(o), np.ascontiguousarray(z),
                                 np.ascontiguousarray(gamma), np.ascontiguousarray(w),
                                 rows, hv, d, hidden, eps, mode, None, out)
    return out


def layer(q, k, v, a, b, z, A_log, dt_bias, gamma, w, state, cu_seqlens, mode=0,
          want_o=False, want_gated=False):
    """Whole post-projection layer.  ``state`` is updated in place.
    Returns ``out`` or a tuple ``(out, o, gated)`` when asked for them."""
    T, hk, d = q.shape
    hv = v.shape[1]
    hidden = w.shape[0]
    out = np.empty((T, hidden), np.uint16)
    o = np.empty((T, hv, d), np.uint16) if want_o else None
    gated = np.empty((T, hv * d), np.uint16) if want_gated else None
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    lib().gdn_oracle_layer(
        np.ascontiguousarray(q), np.ascontiguousarray(k), np.ascontiguousarray(v),
        np.ascontiguousarray(a), np.ascontiguousarray(b), np.ascontiguousarray(z),
        np.ascontiguousarray(A_log, np.float32), np.ascontiguousarray(dt_bias, np.float32),
        np.ascontiguousarray(gamma), np.ascontiguousarray(w), state, out, cu, len(cu) - 1,
        hk, hv, d, hidden, mode,
        o.ctypes.data if o is not None else None,
        gated.ctypes.data if gated is not None else None)
    if want_o or want_gated:
        return out, o, gated
    return out


# ------------------------------------------------------------ input side --

def causal_conv1d(x, w, state, cu_seqlens, use_state=True):
    """Depthwise causal conv (width 4) + SiLU over packed sequences.  x bf16
    [T, C]; w bf16 [4, C]; state bf16 [S, 3, C] (updated in place).  Returns
    bf16 [T, C]."""
    T, C = x.shape
    out = np.empty((T, C), np.uint16)
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    assert state.flags["C_CONTIGUOUS"] and state.dtype == np.uint16
    lib().gdn_oracle_causal_conv1d(np.ascontiguousarray(x), np.ascontiguousarray(w), state, cu,
                                   len(cu) - 1, C, 1 if use_state else 0, out)
    return out


def input_side(x, w_qkv, w_z, w_a, w_b, conv_w, conv_state, cu_seqlens, hk, hv, d=128,
               use_state=True):
    """Projections (qkv, z, a, b: x @ W^T, the reference's four aclnnMatmul
    calls, P:3101-3130), causal conv + SiLU over qkv with the conv-state update
    (P:3132-3179), and the q/k/v split (channels [0, hk d), [hk d, 2 hk d),
    [2 hk d, 2 hk d + hv d); P:3186-3247).  ``conv_state`` is updated in
    place.  Returns q, k, v, z (bf16 [T, heads, d]) and a, b (bf16 [T, hv])."""
    T = x.shape[0]
    qkv = gemm_bf16(x, w_qkv)
    z = gemm_bf16(x, w_z)
    a = gemm_bf16(x, w_a)
    b = gemm_bf16(x, w_b)
    conv = causal_conv1d(qkv, conv_w, conv_state, cu_seqlens, use_state)
    q = np.ascontiguousarray(conv[:, :hk * d]).reshape(T, hk, d)
    k = np.ascontiguousarray(conv[:, hk * d:2 * hk * d]).reshape(T, hk, d)
    v = np.ascontiguousarray(conv[:, 2 * hk * d:]).reshape(T, hv, d)
    return q, k, v, z.reshape(T, hv, d), a, b
