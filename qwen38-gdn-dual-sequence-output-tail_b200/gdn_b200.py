"""Python bindings (ctypes) for ``libgdn_b200.so``, the B200 GDN hot path.

The library is the product: C-ABI entry points declared in
``include/gdn_b200.h`` and ``include/statecentric_qwen38_provider_api_v1.h``.
This module only marshals arguments: torch tensors supply device memory and
the current CUDA stream.  There is no fallback path: if the shared library is
missing every call raises.

Workload generators (``synthetic``) produce the seeded inputs of the
benchmark configurations through ``gdn_b200_fill_synthetic`` so that host and
device harnesses see identical bits.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libgdn_b200.so")

HEAD_DIM = 128
CHUNK = 64
MAX_SEQUENCES = 1024

OK = 0
INVALID_ARGUMENT = 1
INTERNAL = 2
TIMEOUT = 3
NOT_READY = 4
UNSUPPORTED = 5
ABI_MISMATCH = 6

# Every exported symbol of include/gdn_b200.h and the provider header.
EXPORTED_SYMBOLS = (
    "gdn_b200_last_error",
    "gdn_b200_workspace_status",
    "gdn_b200_output_tail_workspace_bytes",
    "gdn_b200_output_tail",
    "gdn_b200_decode_step",
    "gdn_b200_chunk_prefill_workspace_bytes",
    "gdn_b200_chunk_prefill",
    "gdn_b200_layer_forward_workspace_bytes",
    "gdn_b200_layer_forward",
    "gdn_b200_fill_synthetic",
    "statecentric_qwen38_provider_query_v1",
)

_lib = None


class GdnError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"status {status}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Loads the shared library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `make -C {HERE}` "
                "(there is no CPU fallback for the GDN hot path)")
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, i64, u64, f32 = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                  ctypes.c_uint64, ctypes.c_float)
        i32p = ctypes.POINTER(ctypes.c_int32)
        L.gdn_b200_last_error.restype = ctypes.c_char_p
        L.gdn_b200_workspace_status.argtypes = [vp, vp]
        L.gdn_b200_workspace_status.restype = i32
        L.gdn_b200_output_tail_workspace_bytes.argtypes = [i64, i32, i32]
        L.gdn_b200_output_tail_workspace_bytes.restype = u64
        L.gdn_b200_output_tail.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, f32, vp, u64, vp]
        L.gdn_b200_output_tail.restype = i32
        L.gdn_b200_decode_step.argtypes = [vp] * 12 + [i32, i32, i32, vp]
        L.gdn_b200_decode_step.restype = i32
        L.gdn_b200_chunk_prefill_workspace_bytes.argtypes = [i32p, i32, i32, i32]
        L.gdn_b200_chunk_prefill_workspace_bytes.restype = u64
        L.gdn_b200_chunk_prefill.argtypes = [vp] * 9 + [i32p, i32, i32, i32, vp, u64, vp]
        L.gdn_b200_chunk_prefill.restype = i32
        L.gdn_b200_layer_forward_workspace_bytes.argtypes = [i32p, i32, i32, i32, i32]
        L.gdn_b200_layer_forward_workspace_bytes.restype = u64
        L.gdn_b200_layer_forward.argtypes = [vp] * 12 + [i32p, i32, i32, i32, i32, vp, u64, vp]
        L.gdn_b200_layer_forward.restype = i32
        L.gdn_b200_fill_synthetic.argtypes = [u64, u64, u64, i32, f32, f32, i32, vp]
        L.gdn_b200_fill_synthetic.restype = i32
        _lib = L
    return _lib


def last_error() -> str:
    return lib().gdn_b200_last_error().decode()


def _check(status: int) -> None:
    if status != OK:
        raise GdnError(status, last_error())


# ---------------------------------------------------------------- torch --

def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _cu_array(cu_seqlens):
    arr = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.int32))
    return arr, arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def _workspace(nbytes: int, device):
    import torch
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


def output_tail_workspace_bytes(rows: int, value_heads: int, hidden: int) -> int:
    return int(lib().gdn_b200_output_tail_workspace_bytes(rows, value_heads, hidden))


def output_tail(o, z, gamma, w_out, out=None, eps=1e-6, workspace=None, stream=None):
    """out[rows, hidden] = tail(o[rows, Hv, 128], z, gamma, w_out[hidden, Hv*128])."""
    import torch
    rows = o.shape[0]
    hv = o.shape[1]
    hidden = w_out.shape[0]
    if out is None:
        out = torch.empty(rows, hidden, dtype=torch.bfloat16, device=o.device)
    if workspace is None:
        workspace = _workspace(output_tail_workspace_bytes(rows, hv, hidden), o.device)
    _check(lib().gdn_b200_output_tail(_ptr(o), _ptr(z), _ptr(gamma), _ptr(w_out), _ptr(out),
                                      rows, hv, hidden, eps, _ptr(workspace),
                                      workspace.numel(), _stream(stream)))
    return out


def decode_step(q, k, v, a, b, A_log, dt_bias, state, o_out=None, z=None, gamma=None,
                gated_out=None, stream=None):
    batch, hk = q.shape[0], q.shape[1]
    hv = v.shape[1]
    _check(lib().gdn_b200_decode_step(_ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(A_log),
                                      _ptr(dt_bias), _ptr(state), _ptr(o_out), _ptr(z),
                                      _ptr(gamma), _ptr(gated_out), batch, hk, hv,
                                      _stream(stream)))


def chunk_prefill_workspace_bytes(cu_seqlens, qk_heads: int, value_heads: int) -> int:
    arr, p = _cu_array(cu_seqlens)
    return int(lib().gdn_b200_chunk_prefill_workspace_bytes(p, len(arr) - 1, qk_heads,
                                                            value_heads))


def chunk_prefill(q, k, v, a, b, A_log, dt_bias, state, cu_seqlens, o_out=None,
                  workspace=None, stream=None):
    import torch
    hk, hv = q.shape[1], v.shape[1]
    arr, p = _cu_array(cu_seqlens)
    if o_out is None:
        o_out = torch.empty_like(v)
    if workspace is None:
        workspace = _workspace(chunk_prefill_workspace_bytes(arr, hk, hv), q.device)
    _check(lib().gdn_b200_chunk_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b),
                                        _ptr(A_log), _ptr(dt_bias), _ptr(state), _ptr(o_out), p,
                                        len(arr) - 1, hk, hv, _ptr(workspace), workspace.numel(),
                                        _stream(stream)))
    return o_out


def layer_forward_workspace_bytes(cu_seqlens, qk_heads: int, value_heads: int,
                                  hidden: int) -> int:
    arr, p = _cu_array(cu_seqlens)
    return int(lib().gdn_b200_layer_forward_workspace_bytes(p, len(arr) - 1, qk_heads,
                                                            value_heads, hidden))


def layer_forward(q, k, v, a, b, z, A_log, dt_bias, gamma, w_out, state, cu_seqlens,
                  out=None, workspace=None, stream=None):
    import torch
    hk, hv = q.shape[1], v.shape[1]
    hidden = w_out.shape[0]
    arr, p = _cu_array(cu_seqlens)
    if out is None:
        out = torch.empty(q.shape[0], hidden, dtype=torch.bfloat16, device=q.device)
    if workspace is None:
        workspace = _workspace(layer_forward_workspace_bytes(arr, hk, hv, hidden), q.device)
    _check(lib().gdn_b200_layer_forward(_ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b), _ptr(z),
                                        _ptr(A_log), _ptr(dt_bias), _ptr(gamma), _ptr(w_out),
                                        _ptr(state), _ptr(out), p, len(arr) - 1, hk, hv, hidden,
                                        _ptr(workspace), workspace.numel(), _stream(stream)))
    return out


def workspace_status(workspace, stream=None) -> None:
    """Synchronises and raises if a kernel recorded a device-side error."""
    _check(lib().gdn_b200_workspace_status(_ptr(workspace), _stream(stream)))


# ------------------------------------------------------ synthetic inputs --

NORMAL, UNIFORM, LOG_UNIFORM = 0, 1, 2
BF16, F32 = 1, 2


def fill(seed: int, tensor_id: int, shape, distribution: int, p0: float, p1: float,
         dtype: int) -> np.ndarray:
    """Seeded host tensor (bf16 as uint16 bit patterns, or float32)."""
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.uint16 if dtype == BF16 else np.float32)
    _check(lib().gdn_b200_fill_synthetic(seed, tensor_id, n, distribution, p0, p1, dtype,
                                         out.ctypes.data_as(ctypes.c_void_p)))
    return out.reshape(shape)


@dataclass
class Geometry:
    qk_heads: int = 16
    value_heads: int = 32
    hidden: int = 2048

    @property
    def value(self) -> int:
        return self.value_heads * HEAD_DIM


# Tensor ids of the seeded generator.
TID = dict(q=1, k=2, v=3, a=4, b=5, z=6, A_log=7, dt_bias=8, gamma=9, w_out=10, state=11, o=12)


def synthetic_layer_inputs(cu_seqlens, geom: Geometry, seed: int = 0, state_std: float = 0.0,
                           a_log_hi: float = 16.0, shard=None):
    """Host inputs with the benchmark distributions: q, k, v, z ~ N(0,1);
    a ~ N(0,1); dt_bias ~ N(0,0.1); A_log = log U(0, a_log_hi); b ~ N(0,1);
    gamma = 1 + N(0, 0.02); w_out ~ N(0, 0.02); state ~ N(0, state_std) (zero
    when state_std is 0).  ``shard = (rank, world)`` slices the head-parallel
    shard of rank ``rank`` out of the full-geometry tensors."""
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    T = int(cu[-1])
    S = len(cu) - 1
    hk, hv, H, D = geom.qk_heads, geom.value_heads, geom.hidden, HEAD_DIM
    x = dict(
        q=fill(seed, TID["q"], (T, hk, D), NORMAL, 0.0, 1.0, BF16),
        k=fill(seed, TID["k"], (T, hk, D), NORMAL, 0.0, 1.0, BF16),
        v=fill(seed, TID["v"], (T, hv, D), NORMAL, 0.0, 1.0, BF16),
        a=fill(seed, TID["a"], (T, hv), NORMAL, 0.0, 1.0, BF16),
        b=fill(seed, TID["b"], (T, hv), NORMAL, 0.0, 1.0, BF16),
        z=fill(seed, TID["z"], (T, hv, D), NORMAL, 0.0, 1.0, BF16),
        A_log=fill(seed, TID["A_log"], (hv,), LOG_UNIFORM, 0.0, a_log_hi, F32),
        dt_bias=fill(seed, TID["dt_bias"], (hv,), NORMAL, 0.0, 0.1, F32),
        gamma=fill(seed, TID["gamma"], (D,), NORMAL, 1.0, 0.02, BF16),
        w_out=fill(seed, TID["w_out"], (H, hv * D), NORMAL, 0.0, 0.02, BF16),
    )
    if state_std > 0:
        x["state"] = fill(seed, TID["state"], (S, hv, D, D), NORMAL, 0.0, state_std, F32)
    else:
        x["state"] = np.zeros((S, hv, D, D), np.float32)
    if shard is not None:
        rank, world = shard
        hk_r, hv_r = hk // world, hv // world
        ks = slice(rank * hk_r, (rank + 1) * hk_r)
        vs = slice(rank * hv_r, (rank + 1) * hv_r)
        x["q"] = np.ascontiguousarray(x["q"][:, ks])
        x["k"] = np.ascontiguousarray(x["k"][:, ks])
        for n in ("v", "a", "b", "z"):
            x[n] = np.ascontiguousarray(x[n][:, vs])
        x["A_log"] = np.ascontiguousarray(x["A_log"][vs])
        x["dt_bias"] = np.ascontiguousarray(x["dt_bias"][vs])
        x["w_out"] = np.ascontiguousarray(x["w_out"][:, rank * hv_r * D:(rank + 1) * hv_r * D])
        x["state"] = np.ascontiguousarray(x["state"][:, vs])
    return x


def to_device(x: dict, device="cuda"):
    """Host dict of numpy arrays -> torch tensors (bf16 for uint16)."""
    import torch
    out = {}
    for n, arr in x.items():
        if arr.dtype == np.uint16:
            t = torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
        else:
            t = torch.from_numpy(np.ascontiguousarray(arr))
        out[n] = t.to(device)
    return out


def bf16_bits(t) -> np.ndarray:
    """torch bf16 tensor -> numpy uint16 bit patterns (host)."""
    import torch
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)
