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
import struct
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
    "gdn_b200_kernel_launches",
    "gdn_b200_workspace_status",
    "gdn_b200_output_tail_workspace_bytes",
    "gdn_b200_output_tail",
    "gdn_b200_decode_step",
    "gdn_b200_chunk_prefill_workspace_bytes",
    "gdn_b200_chunk_prefill",
    "gdn_b200_layer_forward_workspace_bytes",
    "gdn_b200_layer_forward",
    "gdn_b200_fill_synthetic",
    "gdn_b200_decode_step_rows",
    "gdn_b200_copy_graph_rows",
    "gdn_b200_input_side_workspace_bytes",
    "gdn_b200_input_side",
    "gdn_b200_layer_forward_x_workspace_bytes",
    "gdn_b200_layer_forward_x",
    "gdn_b200_tail_exchange_bytes",
    "gdn_b200_exchange_alloc",
    "gdn_b200_exchange_free",
    "gdn_b200_exchange_export",
    "gdn_b200_exchange_open",
    "gdn_b200_exchange_close",
    "gdn_b200_output_tail_allreduce_workspace_bytes",
    "gdn_b200_output_tail_allreduce",
    "gdn_b200_rank_sum_bytes",
    "gdn_b200_rank_sum_part",
    "gdn_b200_rank_sum_acquire",
    "gdn_b200_rank_sum",
    "gdn_b200_output_tail_no_alloc",
    "gdn_b200_output_tail_no_alloc_status",
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
        L.gdn_b200_kernel_launches.restype = u64
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
        L.gdn_b200_decode_step_rows.argtypes = [vp] * 12 + [i32, i32, i32, vp]
        L.gdn_b200_decode_step_rows.restype = i32
        L.gdn_b200_copy_graph_rows.argtypes = [ctypes.POINTER(LayoutWorkspaceV1), u64, u64, u64,
                                               u64, u64, i32, vp]
        L.gdn_b200_copy_graph_rows.restype = i32
        L.gdn_b200_input_side_workspace_bytes.argtypes = [i32p, i32, i32, i32, i32]
        L.gdn_b200_input_side_workspace_bytes.restype = u64
        L.gdn_b200_input_side.argtypes = [vp] * 7 + [i32p, i32, i32, i32, i32, i32] + [vp] * 7 + [u64, vp]
        L.gdn_b200_input_side.restype = i32
        L.gdn_b200_layer_forward_x_workspace_bytes.argtypes = [i32p, i32, i32, i32, i32]
        L.gdn_b200_layer_forward_x_workspace_bytes.restype = u64
        L.gdn_b200_layer_forward_x.argtypes = [vp] * 13 + [i32p, i32, i32, i32, i32, i32, vp, u64, vp]
        L.gdn_b200_layer_forward_x.restype = i32
        L.gdn_b200_tail_exchange_bytes.argtypes = [i64, i32, i32]
        L.gdn_b200_tail_exchange_bytes.restype = u64
        L.gdn_b200_exchange_alloc.argtypes = [u64, ctypes.POINTER(vp)]
        L.gdn_b200_exchange_alloc.restype = i32
        L.gdn_b200_exchange_free.argtypes = [vp]
        L.gdn_b200_exchange_free.restype = i32
        L.gdn_b200_exchange_export.argtypes = [vp, vp]
        L.gdn_b200_exchange_export.restype = i32
        L.gdn_b200_exchange_open.argtypes = [vp, ctypes.POINTER(vp)]
        L.gdn_b200_exchange_open.restype = i32
        L.gdn_b200_exchange_close.argtypes = [vp]
        L.gdn_b200_exchange_close.restype = i32
        L.gdn_b200_output_tail_allreduce_workspace_bytes.argtypes = [i64, i32]
        L.gdn_b200_output_tail_allreduce_workspace_bytes.restype = u64
        L.gdn_b200_output_tail_allreduce.argtypes = [vp, vp, vp, vp, i64, i32, i32, f32,
                                                     ctypes.POINTER(TailGroupV1), ctypes.c_uint32,
                                                     vp, u64, vp]
        L.gdn_b200_output_tail_allreduce.restype = i32
        L.gdn_b200_rank_sum_bytes.argtypes = [i64, i32, i32]
        L.gdn_b200_rank_sum_bytes.restype = u64
        L.gdn_b200_rank_sum_part.argtypes = [ctypes.POINTER(TailGroupV1), ctypes.c_uint32]
        L.gdn_b200_rank_sum_part.restype = vp
        L.gdn_b200_rank_sum_acquire.argtypes = [ctypes.POINTER(TailGroupV1), ctypes.c_uint32,
                                                vp, vp]
        L.gdn_b200_rank_sum_acquire.restype = i32
        L.gdn_b200_rank_sum.argtypes = [ctypes.POINTER(TailGroupV1), ctypes.c_uint32, i64, vp,
                                        vp, vp, vp]
        L.gdn_b200_rank_sum.restype = i32
        L.gdn_b200_output_tail_no_alloc.argtypes = [vp] * 5 + [i64, i32, i32, f32, vp]
        L.gdn_b200_output_tail_no_alloc.restype = i32
        L.gdn_b200_output_tail_no_alloc_status.argtypes = [vp]
        L.gdn_b200_output_tail_no_alloc_status.restype = i32
        _lib = L
    return _lib


def last_error() -> str:
    return lib().gdn_b200_last_error().decode()


def kernel_launches() -> int:
    """Kernels this library has launched in this process so far."""
    return int(lib().gdn_b200_kernel_launches())


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


def output_tail_no_alloc(o, z, gamma, w_out, out=None, eps=1e-6, stream=None):
    """The output tail with the library's static scratch instead of a
    workspace (``gdn_b200_output_tail_no_alloc``): rows <= 128,
    Hv*128 <= 4096, hidden <= 2048."""
    import torch
    rows, hv, hidden = o.shape[0], o.shape[1], w_out.shape[0]
    if out is None:
        out = torch.empty(rows, hidden, dtype=torch.bfloat16, device=o.device)
    _check(lib().gdn_b200_output_tail_no_alloc(_ptr(o), _ptr(z), _ptr(gamma), _ptr(w_out),
                                               _ptr(out), rows, hv, hidden, eps,
                                               _stream(stream)))
    return out


def output_tail_no_alloc_status(stream=None) -> None:
    """Synchronises and raises if the last no-alloc tail recorded a device error."""
    _check(lib().gdn_b200_output_tail_no_alloc_status(_stream(stream)))


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


# ------------------------------------------------------ graph binding --

def decode_step_rows(q, k, v, a, b, A_log, dt_bias, state_rows, o_out=None, z=None, gamma=None,
                     gated_out=None, stream=None):
    """Decode with sequence i's state at the device address state_rows[i]
    (``state_rows``: int64 tensor on the device)."""
    batch, hk = q.shape[0], q.shape[1]
    hv = v.shape[1]
    _check(lib().gdn_b200_decode_step_rows(_ptr(q), _ptr(k), _ptr(v), _ptr(a), _ptr(b),
                                           _ptr(A_log), _ptr(dt_bias), _ptr(state_rows),
                                           _ptr(o_out), _ptr(z), _ptr(gamma), _ptr(gated_out),
                                           batch, hk, hv, _stream(stream)))


BINDING_COPY_V1, BINDING_DIRECT_V1, GRAPH_MAX_ROWS = 1, 2, 4


class LayoutWorkspaceV1(ctypes.Structure):
    """statecentric_qwen38_gdn_layout_workspace_v1 of the provider header."""
    _fields_ = [("size", ctypes.c_uint32), ("abi_version", ctypes.c_uint32),
                ("batch_size", ctypes.c_uint32), ("binding_mode", ctypes.c_uint32),
                ("arena", ctypes.c_size_t), ("arena_bytes", ctypes.c_uint64),
                ("required_arena_bytes", ctypes.c_uint64),
                ("conv_bytes_per_row", ctypes.c_uint64),
                ("recurrent_bytes_per_row", ctypes.c_uint64),
                ("conv_row_addresses", ctypes.c_size_t * GRAPH_MAX_ROWS),
                ("recurrent_row_addresses", ctypes.c_size_t * GRAPH_MAX_ROWS)]


def copy_graph_rows(layout, batch_size, conv_bytes, recurrent_bytes, packed_conv,
                    packed_recurrent, gather, stream=None):
    _check(lib().gdn_b200_copy_graph_rows(ctypes.byref(layout), batch_size, conv_bytes,
                                          recurrent_bytes, packed_conv, packed_recurrent,
                                          1 if gather else 0, _stream(stream)))


# ------------------------------------------------------------ input side --

def input_side_workspace_bytes(cu_seqlens, qk_heads: int, value_heads: int, hidden: int) -> int:
    arr, p = _cu_array(cu_seqlens)
    return int(lib().gdn_b200_input_side_workspace_bytes(p, len(arr) - 1, qk_heads, value_heads,
                                                         hidden))


def input_side(x, w_qkv, w_z, w_a, w_b, conv_w, conv_state, cu_seqlens, qk_heads: int,
               use_conv_state=True, out=None, workspace=None, stream=None):
    """x bf16 [T, hidden] -> (q, k, v, z, a, b) on the device (into ``out``
    when given); conv_state is updated in place."""
    import torch
    T, hidden = x.shape
    hv = w_z.shape[0] // HEAD_DIM
    arr, p = _cu_array(cu_seqlens)
    dev = x.device
    if out is not None:
        q, k, v, z, a, b = out
    else:
        q = torch.empty(T, qk_heads, HEAD_DIM, dtype=torch.bfloat16, device=dev)
        k = torch.empty_like(q)
        v = torch.empty(T, hv, HEAD_DIM, dtype=torch.bfloat16, device=dev)
        z = torch.empty_like(v)
        a = torch.empty(T, hv, dtype=torch.bfloat16, device=dev)
        b = torch.empty_like(a)
    if workspace is None:
        workspace = _workspace(input_side_workspace_bytes(arr, qk_heads, hv, hidden), dev)
    _check(lib().gdn_b200_input_side(_ptr(x), _ptr(w_qkv), _ptr(w_z), _ptr(w_a), _ptr(w_b),
                                     _ptr(conv_w), _ptr(conv_state), p, len(arr) - 1, qk_heads,
                                     hv, hidden, 1 if use_conv_state else 0, _ptr(q), _ptr(k),
                                     _ptr(v), _ptr(z), _ptr(a), _ptr(b), _ptr(workspace),
                                     workspace.numel(), _stream(stream)))
    return q, k, v, z, a, b


def layer_forward_x_workspace_bytes(cu_seqlens, qk_heads: int, value_heads: int,
                                    hidden: int) -> int:
    arr, p = _cu_array(cu_seqlens)
    return int(lib().gdn_b200_layer_forward_x_workspace_bytes(p, len(arr) - 1, qk_heads,
                                                              value_heads, hidden))


def layer_forward_x(x, w_qkv, w_z, w_a, w_b, conv_w, conv_state, A_log, dt_bias, gamma, w_out,
                    state, cu_seqlens, qk_heads: int, use_conv_state=True, out=None,
                    workspace=None, stream=None):
    """The whole layer from x; conv_state and state are updated in place.
    The projections' input width and the output width are both ``hidden``."""
    import torch
    T, hidden = x.shape
    if w_out.shape[0] != hidden:
        raise GdnError(INVALID_ARGUMENT, "w_out rows must equal the hidden size of x")
    hv = w_z.shape[0] // HEAD_DIM
    arr, p = _cu_array(cu_seqlens)
    if out is None:
        out = torch.empty(T, w_out.shape[0], dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = _workspace(layer_forward_x_workspace_bytes(arr, qk_heads, hv, hidden),
                               x.device)
    _check(lib().gdn_b200_layer_forward_x(
        _ptr(x), _ptr(w_qkv), _ptr(w_z), _ptr(w_a), _ptr(w_b), _ptr(conv_w), _ptr(conv_state),
        _ptr(A_log), _ptr(dt_bias), _ptr(gamma), _ptr(w_out), _ptr(state), _ptr(out), p,
        len(arr) - 1, qk_heads, hv, hidden,
        1 if use_conv_state else 0, _ptr(workspace), workspace.numel(), _stream(stream)))
    return out


# ------------------------------------------------- head-parallel tail --

MAX_RANKS = 8
EXCHANGE_HANDLE_BYTES = 64


class TailGroupV1(ctypes.Structure):
    """gdn_b200_tail_group_v1 of include/gdn_b200.h."""
    _fields_ = [("rank", ctypes.c_int32), ("world_size", ctypes.c_int32),
                ("max_rows", ctypes.c_int64), ("hidden", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("region", ctypes.c_void_p * MAX_RANKS)]


class _DeviceArray:
    """A raw device allocation presented to torch through
    ``__cuda_array_interface__`` (the tensor keeps this object alive)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(int(d) for d in shape),
                                         "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3}


def tail_exchange_bytes(max_rows: int, hidden: int, world_size: int) -> int:
    return int(lib().gdn_b200_tail_exchange_bytes(max_rows, hidden, world_size))


def output_tail_allreduce_workspace_bytes(rows: int, value_heads: int) -> int:
    return int(lib().gdn_b200_output_tail_allreduce_workspace_bytes(rows, value_heads))


class TailGroup:
    """One rank of a head-parallel output-tail group
    (``gdn_b200_output_tail_allreduce``): the rank's exchange region, the
    other ranks' regions mapped into this process, and the call epoch.

    ``exchange(payload: bytes) -> list[bytes]`` returns every rank's payload
    in rank order (for example around ``torch.distributed.all_gather_object``);
    it is called once, here, when ``world_size > 1``.  ``out`` is this rank's
    output ``[max_rows, hidden]`` bf16 inside its region.  Every rank must
    call :meth:`output_tail` the same number of times with the same rows, and
    :meth:`close` only after every rank's last call has finished (a barrier).
    """

    def __init__(self, max_rows: int, hidden: int, rank: int, world_size: int, device,
                 exchange=None):
        import torch
        self.device = torch.device(device)
        self.max_rows, self.hidden = int(max_rows), int(hidden)
        self.rank, self.world_size = int(rank), int(world_size)
        nbytes = tail_exchange_bytes(max_rows, hidden, world_size)
        if nbytes == 0:
            raise GdnError(INVALID_ARGUMENT, "invalid tail group geometry")
        self._opened = []
        region = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _check(lib().gdn_b200_exchange_alloc(nbytes, ctypes.byref(region)))
        self._own = region.value
        regions = [None] * world_size
        regions[rank] = self._own
        if world_size > 1:
            handle = (ctypes.c_uint8 * EXCHANGE_HANDLE_BYTES)()
            _check(lib().gdn_b200_exchange_export(ctypes.c_void_p(self._own), handle))
            # The geometry travels with the handle: regions laid out for
            # different sizes would put a peer's flags outside this region.
            geometry = struct.pack("<qii", max_rows, hidden, world_size)
            payloads = exchange(bytes(handle) + geometry)
            if len(payloads) != world_size:
                raise GdnError(INVALID_ARGUMENT, "exchange returned the wrong number of handles")
            if any(bytes(pl[EXCHANGE_HANDLE_BYTES:]) != geometry for pl in payloads):
                self.close()
                raise GdnError(INVALID_ARGUMENT, "ranks disagree on max_rows, hidden or world size")
            for i, payload in enumerate(payloads):
                if i == rank:
                    continue
                h = (ctypes.c_uint8 * EXCHANGE_HANDLE_BYTES).from_buffer_copy(
                    bytes(payload[:EXCHANGE_HANDLE_BYTES]))
                peer = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    _check(lib().gdn_b200_exchange_open(h, ctypes.byref(peer)))
                regions[i] = peer.value
                self._opened.append(peer.value)
        self.group = TailGroupV1(rank, world_size, max_rows, hidden, 0,
                                 (ctypes.c_void_p * MAX_RANKS)(*regions))
        self.out = torch.as_tensor(_DeviceArray(self._own, (max_rows, hidden), "<i2"),
                                   device=self.device).view(torch.bfloat16)
        self.epoch = 0

    def output_tail(self, o, z, gamma, w_out, eps=1e-6, workspace=None, stream=None):
        """Fused tail of this rank's heads plus the rank sum; returns the
        first ``rows`` rows of :attr:`out` (the same values on every rank)."""
        rows, hv = o.shape[0], o.shape[1]
        if workspace is None:
            workspace = _workspace(output_tail_allreduce_workspace_bytes(rows, hv), o.device)
        self.epoch += 1
        _check(lib().gdn_b200_output_tail_allreduce(
            _ptr(o), _ptr(z), _ptr(gamma), _ptr(w_out), rows, hv, self.hidden, eps,
            ctypes.byref(self.group), self.epoch, _ptr(workspace), workspace.numel(),
            _stream(stream)))
        return self.out[:rows]

    def close(self) -> None:
        for p in self._opened:
            lib().gdn_b200_exchange_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own is not None:
            self.out = None
            lib().gdn_b200_exchange_free(ctypes.c_void_p(self._own))
            self._own = None


class RankSum:
    """One rank of a copy-engine rank sum (``gdn_b200_rank_sum``): the
    rank's region (two partial-output buffers, staging, flags), the other
    ranks' regions mapped into this process, and the epoch.

    Per step: :meth:`part` gives the buffer the layer writes its rank-partial
    output into; call :meth:`acquire` before the layer and :meth:`reduce`
    after it, on the layer's stream; the shard is written on ``comm_stream``.
    ``exchange(payload: bytes) -> list[bytes]`` as for :class:`TailGroup`."""

    def __init__(self, max_rows: int, hidden: int, rank: int, world_size: int, device,
                 exchange=None):
        import torch
        self.device = torch.device(device)
        self.max_rows, self.hidden = int(max_rows), int(hidden)
        self.rank, self.world_size = int(rank), int(world_size)
        nbytes = int(lib().gdn_b200_rank_sum_bytes(max_rows, hidden, world_size))
        if nbytes == 0:
            raise GdnError(INVALID_ARGUMENT, "invalid rank-sum geometry")
        self._opened = []
        region = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _check(lib().gdn_b200_exchange_alloc(nbytes, ctypes.byref(region)))
        self._own = region.value
        regions = [None] * world_size
        regions[rank] = self._own
        if world_size > 1:
            handle = (ctypes.c_uint8 * EXCHANGE_HANDLE_BYTES)()
            _check(lib().gdn_b200_exchange_export(ctypes.c_void_p(self._own), handle))
            geometry = struct.pack("<qii", max_rows, hidden, world_size)
            payloads = exchange(bytes(handle) + geometry)
            if any(bytes(pl[EXCHANGE_HANDLE_BYTES:]) != geometry for pl in payloads):
                self.close()
                raise GdnError(INVALID_ARGUMENT, "ranks disagree on max_rows, hidden or world size")
            for i, payload in enumerate(payloads):
                if i == rank:
                    continue
                h = (ctypes.c_uint8 * EXCHANGE_HANDLE_BYTES).from_buffer_copy(
                    bytes(payload[:EXCHANGE_HANDLE_BYTES]))
                peer = ctypes.c_void_p()
                with torch.cuda.device(self.device):
                    _check(lib().gdn_b200_exchange_open(h, ctypes.byref(peer)))
                regions[i] = peer.value
                self._opened.append(peer.value)
        self.group = TailGroupV1(rank, world_size, max_rows, hidden, 0,
                                 (ctypes.c_void_p * MAX_RANKS)(*regions))
        self._err = torch.zeros(64, dtype=torch.int32, device=self.device)
        self.epoch = 0

    def part(self, epoch: int, rows: int):
        """The [rows, hidden] bf16 buffer of this rank's partial for ``epoch``."""
        import torch
        ptr = lib().gdn_b200_rank_sum_part(ctypes.byref(self.group), epoch)
        return torch.as_tensor(_DeviceArray(ptr, (rows, self.hidden), "<i2"),
                               device=self.device).view(torch.bfloat16)

    def acquire(self, epoch: int, stream=None) -> None:
        _check(lib().gdn_b200_rank_sum_acquire(ctypes.byref(self.group), epoch,
                                               _ptr(self._err), _stream(stream)))

    def reduce(self, epoch: int, rows: int, shard_out, stream=None, comm_stream=None) -> None:
        _check(lib().gdn_b200_rank_sum(ctypes.byref(self.group), epoch, rows, _ptr(shard_out),
                                       _ptr(self._err), _stream(stream), _stream(comm_stream)))

    def status(self, stream=None) -> None:
        """Synchronises and raises if a wait of the exchange ran out."""
        _check(lib().gdn_b200_workspace_status(_ptr(self._err), _stream(stream)))

    def close(self) -> None:
        for p in self._opened:
            lib().gdn_b200_exchange_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own is not None:
            lib().gdn_b200_exchange_free(ctypes.c_void_p(self._own))
            self._own = None


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
TID = dict(q=1, k=2, v=3, a=4, b=5, z=6, A_log=7, dt_bias=8, gamma=9, w_out=10, state=11, o=12,
           x=13, w_qkv=14, w_z=15, w_a=16, w_b=17, conv_w=18, conv_state=19)


def synthetic_layer_inputs(cu_seqlens, geom: Geometry, seed: int = 0, state_std: float = 0.0,
                           a_log_hi: float = 16.0, shard=None, fill=fill):
    """Host inputs with the benchmark distributions: q, k, v, z ~ N(0,1);
    a ~ N(0,1); dt_bias ~ N(0,0.1); A_log = log U(0, a_log_hi); b ~ N(0,1);
    gamma = 1 + N(0, 0.02); w_out ~ N(0, 0.02); state ~ N(0, state_std) (zero
    when state_std is 0).  ``shard = (rank, world)`` slices the head-parallel
    shard of rank ``rank`` out of the full-geometry tensors.  ``fill`` is the
    generator (this module's, or any function with its signature and bits)."""
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


def synthetic_input_side(cu_seqlens, geom: Geometry, seed: int = 0, conv_state_std: float = 0.0):
    """Host inputs of the input side: x ~ N(0,1) [T, hidden]; w_qkv, w_z,
    w_a, w_b ~ N(0, 0.02) [N, hidden] (so the projections are ~N(0, 0.9));
    conv_w ~ N(0, 0.5) [4, channels]; conv_state ~ N(0, conv_state_std)
    [S, 3, channels] bf16 (zero when the std is 0)."""
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    T = int(cu[-1])
    S = len(cu) - 1
    hk, hv, H, D = geom.qk_heads, geom.value_heads, geom.hidden, HEAD_DIM
    C = (2 * hk + hv) * D
    x = dict(
        x=fill(seed, TID["x"], (T, H), NORMAL, 0.0, 1.0, BF16),
        w_qkv=fill(seed, TID["w_qkv"], (C, H), NORMAL, 0.0, 0.02, BF16),
        w_z=fill(seed, TID["w_z"], (hv * D, H), NORMAL, 0.0, 0.02, BF16),
        w_a=fill(seed, TID["w_a"], (hv, H), NORMAL, 0.0, 0.02, BF16),
        w_b=fill(seed, TID["w_b"], (hv, H), NORMAL, 0.0, 0.02, BF16),
        conv_w=fill(seed, TID["conv_w"], (4, C), NORMAL, 0.0, 0.5, BF16),
    )
    if conv_state_std > 0:
        x["conv_state"] = fill(seed, TID["conv_state"], (S, 3, C), NORMAL, 0.0, conv_state_std,
                               BF16)
    else:
        x["conv_state"] = np.zeros((S, 3, C), np.uint16)
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


# ------------------------------------------------------------ provider --
# ctypes mirror of include/statecentric_qwen38_provider_api_v1.h.

ABI_V1 = 1
SCALAR_BF16, SCALAR_F32 = 1, 2
MEMORY_DEVICE = 1
STAGE_GDN = 1
EVENT_PENDING, EVENT_COMPLETE = 0, 1
GDN_FORWARD_V1 = 1 << 0
GDN_PREFILL_SPLIT_V2 = 1 << 1
GDN_PREFILL_SPLIT_V3 = 1 << 2
GDN_PREFILL_STRIDED_QKV_V4 = 1 << 3
GDN_PREFILL_POST_CONV_PACK_V5 = 1 << 4
GDN_POST_PROJECTION_V6 = 1 << 5
GDN_OUTPUT_TAIL_V7 = 1 << 6
MAX_RANK = 8

_c = ctypes


class HostV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("context", _c.c_void_p),
                ("monotonic_time_ns", _c.CFUNCTYPE(_c.c_uint64, _c.c_void_p))]


class CreateV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("world_size", _c.c_uint32),
                ("rank", _c.c_uint32), ("device_ordinal", _c.c_int32),
                ("assembly_fingerprint_length", _c.c_uint32),
                ("assembly_fingerprint_sha256", _c.POINTER(_c.c_uint8)),
                ("configuration", _c.c_void_p), ("configuration_length", _c.c_uint64)]


class GdnCreateConfigV1(_c.Structure):
    _fields_ = [(n, _c.c_uint32) for n in (
        "size", "abi_version", "hidden_size", "qkv_size_per_rank", "value_size_per_rank",
        "gate_heads_per_rank", "query_heads_per_rank", "value_heads_per_rank", "head_dim",
        "max_tokens_per_submission", "prefill_qkv_split_variant", "reserved")]


class TensorV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("data", _c.c_uint64),
                ("scalar_type", _c.c_uint32), ("memory_kind", _c.c_uint32),
                ("device_ordinal", _c.c_int32), ("rank", _c.c_uint32),
                ("dimensions", _c.c_uint64 * MAX_RANK), ("strides", _c.c_int64 * MAX_RANK),
                ("byte_length", _c.c_uint64)]


class StateRegionV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("layer_index", _c.c_uint32),
                ("reserved", _c.c_uint32), ("state_kind", _c.c_char_p), ("tensor", TensorV1)]


class ExecutionV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("rank", _c.c_uint32),
                ("world_size", _c.c_uint32), ("device_ordinal", _c.c_int32),
                ("stage", _c.c_uint32), ("flags", _c.c_uint32), ("layer_index", _c.c_uint32),
                ("token_count", _c.c_uint64), ("context_tokens", _c.c_uint64),
                ("stream", _c.c_uint64), ("input_count", _c.c_uint32),
                ("output_count", _c.c_uint32), ("inputs", _c.POINTER(TensorV1)),
                ("outputs", _c.POINTER(TensorV1)), ("mutable_state_count", _c.c_uint32),
                ("reserved", _c.c_uint32), ("mutable_state", _c.POINTER(StateRegionV1)),
                ("workspace", _c.c_uint64), ("workspace_length", _c.c_uint64)]


class GdnBatchV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("state_count", _c.c_uint64),
                ("reserved", _c.c_uint32), ("reserved1", _c.c_uint32),
                ("token_offsets", _c.POINTER(_c.c_uint32)),
                ("token_counts", _c.POINTER(_c.c_uint32))]


class ErrorV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("status", _c.c_int32),
                ("reserved", _c.c_uint32), ("message", _c.c_char_p),
                ("reserved_pointer", _c.c_void_p)]


class CompletionV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32), ("phase", _c.c_uint32),
                ("reserved", _c.c_uint32), ("elapsed_ns", _c.c_uint64),
                ("completed_ns", _c.c_uint64)]


_ErrPP = _c.POINTER(_c.POINTER(ErrorV1))


class DescriptorV1(_c.Structure):
    _fields_ = [("size", _c.c_uint32), ("abi_version", _c.c_uint32),
                ("provider_id", _c.c_char_p), ("provider_version", _c.c_char_p),
                ("operator_name", _c.c_char_p), ("operator_version", _c.c_uint32),
                ("stage", _c.c_uint32), ("flags", _c.c_uint32), ("reserved_flags", _c.c_uint32),
                ("create", _c.CFUNCTYPE(_c.c_int32, _c.POINTER(HostV1), _c.POINTER(CreateV1),
                                        _c.POINTER(_c.c_void_p), _ErrPP)),
                ("destroy", _c.CFUNCTYPE(None, _c.c_void_p)),
                ("submit", _c.CFUNCTYPE(_c.c_int32, _c.c_void_p, _c.POINTER(ExecutionV1),
                                        _c.c_uint64, _c.POINTER(_c.c_void_p), _ErrPP)),
                ("poll", _c.CFUNCTYPE(_c.c_int32, _c.c_void_p, _c.c_void_p,
                                      _c.POINTER(CompletionV1), _ErrPP)),
                ("wait", _c.CFUNCTYPE(_c.c_int32, _c.c_void_p, _c.c_void_p, _c.c_uint64,
                                      _c.POINTER(CompletionV1), _ErrPP)),
                ("cancel", _c.CFUNCTYPE(_c.c_int32, _c.c_void_p, _c.c_void_p, _ErrPP)),
                ("release_event", _c.CFUNCTYPE(None, _c.c_void_p, _c.c_void_p)),
                ("release_error", _c.CFUNCTYPE(None, _c.POINTER(ErrorV1))),
                ("reserved0", _c.c_void_p), ("reserved1", _c.c_void_p),
                ("reserved2", _c.c_void_p)]


def query_descriptor(abi_version=ABI_V1, size=None):
    """Calls statecentric_qwen38_provider_query_v1; returns (status, descriptor, message)."""
    L = lib()
    fn = L.statecentric_qwen38_provider_query_v1
    fn.argtypes = [_c.c_uint32, _c.c_uint32, _c.POINTER(DescriptorV1), _ErrPP]
    fn.restype = _c.c_int32
    d = DescriptorV1()
    err = _c.POINTER(ErrorV1)()
    st = fn(abi_version, _c.sizeof(DescriptorV1) if size is None else size, _c.byref(d),
            _c.byref(err))
    msg = ""
    if st != OK and err:
        msg = err.contents.message.decode()
        if d.release_error:
            d.release_error(err)
    return st, d, msg


def tensor_view(t, dims=None, strides=None, device=0) -> TensorV1:
    """TensorV1 describing torch tensor ``t`` (dims/strides in elements)."""
    import torch
    dims = list(t.shape) if dims is None else list(dims)
    strides = list(t.stride()) if strides is None else list(strides)
    v = TensorV1()
    v.size = _c.sizeof(TensorV1)
    v.abi_version = ABI_V1
    v.data = t.data_ptr()
    v.scalar_type = SCALAR_BF16 if t.dtype == torch.bfloat16 else SCALAR_F32
    v.memory_kind = MEMORY_DEVICE
    v.device_ordinal = device
    v.rank = len(dims)
    for i, (d, s) in enumerate(zip(dims, strides)):
        v.dimensions[i] = d
        v.strides[i] = s
    n = 1
    for d in dims:
        n *= d
    v.byte_length = n * t.element_size()
    return v


class ProviderError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"provider status {status}: {message}")
        self.status = status


class Provider:
    """Drives the library only through the descriptor's function pointers,
    the way a host engine that dlopen()s the provider does."""

    def __init__(self, geom: Geometry, max_tokens: int, world_size=1, rank=0, device=0,
                 fingerprint=bytes(32)):
        import time as _time
        st, d, msg = query_descriptor()
        if st != OK:
            raise ProviderError(st, msg)
        self.d = d
        self.geom = geom
        self.device = device
        self.rank = rank
        self.world_size = world_size
        self._clock = HostV1._fields_[3][1](lambda ctx: _time.monotonic_ns())
        self.host = HostV1(_c.sizeof(HostV1), ABI_V1, None, self._clock)
        cfg = GdnCreateConfigV1()
        cfg.size = _c.sizeof(cfg)
        cfg.abi_version = ABI_V1
        cfg.hidden_size = geom.hidden
        cfg.qkv_size_per_rank = 2 * geom.qk_heads * HEAD_DIM + geom.value
        cfg.value_size_per_rank = geom.value
        cfg.gate_heads_per_rank = geom.value_heads
        cfg.query_heads_per_rank = geom.qk_heads
        cfg.value_heads_per_rank = geom.value_heads
        cfg.head_dim = HEAD_DIM
        cfg.max_tokens_per_submission = max_tokens
        self.cfg = cfg
        self.fp = (_c.c_uint8 * 32)(*fingerprint[:32])
        cr = CreateV1(_c.sizeof(CreateV1), ABI_V1, world_size, rank, device, 32,
                      _c.cast(self.fp, _c.POINTER(_c.c_uint8)), _c.cast(_c.byref(cfg), _c.c_void_p),
                      _c.sizeof(cfg))
        self.create_args = cr
        self.handle = _c.c_void_p()
        err = _c.POINTER(ErrorV1)()
        st = d.create(_c.byref(self.host), _c.byref(cr), _c.byref(self.handle), _c.byref(err))
        self._raise(st, err)
        self._keep = []

    def _raise(self, st, err):
        if st != OK:
            msg = ""
            if err:
                msg = err.contents.message.decode()
                self.d.release_error(err)
            raise ProviderError(st, msg)

    def _execution(self, flags, inputs, output, states, tokens, stream, batch=None):
        ins = (TensorV1 * len(inputs))(*inputs)
        outs = (TensorV1 * 1)(output)
        st = (StateRegionV1 * max(len(states), 1))(*states) if states else None
        ex = ExecutionV1()
        ex.size = _c.sizeof(ex)
        ex.abi_version = ABI_V1
        ex.rank = self.rank
        ex.world_size = self.world_size
        ex.device_ordinal = self.device
        ex.stage = STAGE_GDN
        ex.flags = flags
        ex.layer_index = 0
        ex.token_count = tokens
        ex.stream = stream
        ex.input_count = len(inputs)
        ex.output_count = 1
        ex.inputs = _c.cast(ins, _c.POINTER(TensorV1))
        ex.outputs = _c.cast(outs, _c.POINTER(TensorV1))
        ex.mutable_state_count = len(states)
        ex.mutable_state = _c.cast(st, _c.POINTER(StateRegionV1)) if st is not None else None
        if batch is not None:
            ex.workspace = _c.addressof(batch)
            ex.workspace_length = _c.sizeof(batch)
        self._keep.append((ins, outs, st, batch))
        return ex

    @staticmethod
    def batch_metadata(cu_seqlens):
        cu = [int(x) for x in cu_seqlens]
        n = len(cu) - 1
        offs = (_c.c_uint32 * n)(*cu[:-1])
        cnts = (_c.c_uint32 * n)(*[cu[i + 1] - cu[i] for i in range(n)])
        b = GdnBatchV1(_c.sizeof(GdnBatchV1), ABI_V1, n, 0, 0,
                       _c.cast(offs, _c.POINTER(_c.c_uint32)),
                       _c.cast(cnts, _c.POINTER(_c.c_uint32)))
        b._arrays = (offs, cnts)
        return b

    def submit_layer(self, t, state, out, cu_seqlens, stream=None, deadline_s=60.0,
                     conv_state=None):
        """Post-projection GDN layer (GDN_FORWARD_V1 | GDN_POST_PROJECTION_V6).
        ``t`` holds q, k, v, a, b, z, A_log, dt_bias, gamma, w_out as torch tensors."""
        import time as _time
        g = self.geom
        T = t["q"].shape[0]
        D = HEAD_DIM
        dv = self.device
        inputs = [
            tensor_view(t["q"], [T, g.qk_heads * D], [g.qk_heads * D, 1], dv),
            tensor_view(t["k"], [T, g.qk_heads * D], [g.qk_heads * D, 1], dv),
            tensor_view(t["v"], [T, g.value], [g.value, 1], dv),
            tensor_view(t["a"], [T, g.value_heads], [g.value_heads, 1], dv),
            tensor_view(t["b"], [T, g.value_heads], [g.value_heads, 1], dv),
            tensor_view(t["z"], [T, g.value], [g.value, 1], dv),
            tensor_view(t["A_log"], [g.value_heads], [1], dv),
            tensor_view(t["dt_bias"], [g.value_heads], [1], dv),
            tensor_view(t["gamma"], [D], [1], dv),
            tensor_view(t["w_out"], [g.value, g.hidden], [1, g.value], dv),
        ]
        S = state.shape[0]
        rs = StateRegionV1(_c.sizeof(StateRegionV1), ABI_V1, 0, 0, b"gdn.recurrent",
                           tensor_view(state, device=dv))
        states = [rs]
        if conv_state is not None:
            states = [StateRegionV1(_c.sizeof(StateRegionV1), ABI_V1, 0, 0, b"gdn.conv",
                                    tensor_view(conv_state, device=dv)), rs]
        batch = self.batch_metadata(cu_seqlens) if S > 1 else None
        ex = self._execution(GDN_FORWARD_V1 | GDN_POST_PROJECTION_V6, inputs,
                             tensor_view(out, device=dv), states, T,
                             _stream(stream).value or 0, batch)
        return self.submit(ex, deadline_s)

    def submit_layer_x(self, xs, t, conv_state, state, out, cu_seqlens, context_tokens=0,
                       flags=None, stream=None, deadline_s=60.0):
        """The reference's x-based GDN layer (GDN_FORWARD_V1, optionally with
        a split-variant flag): ``xs`` holds x, w_qkv, w_z, w_a, w_b, conv_w and
        ``t`` holds A_log, dt_bias, gamma, w_out as torch tensors; conv_state
        and state are the gdn.conv / gdn.recurrent regions (updated in place).
        ``context_tokens`` 0 means no earlier context: zero conv history."""
        g = self.geom
        T, H = xs["x"].shape
        D = HEAD_DIM
        dv = self.device
        C = (2 * g.qk_heads + g.value_heads) * D
        inputs = [
            tensor_view(xs["x"], [T, H], [H, 1], dv),
            tensor_view(xs["w_qkv"], [H, C], [1, H], dv),
            tensor_view(xs["w_z"], [H, g.value], [1, H], dv),
            tensor_view(xs["w_a"], [H, g.value_heads], [1, H], dv),
            tensor_view(xs["w_b"], [H, g.value_heads], [1, H], dv),
            tensor_view(xs["conv_w"], [4, C], [C, 1], dv),
            tensor_view(t["A_log"], [g.value_heads], [1], dv),
            tensor_view(t["dt_bias"], [g.value_heads], [1], dv),
            tensor_view(t["gamma"], [D], [1], dv),
            tensor_view(t["w_out"], [g.value, g.hidden], [1, g.value], dv),
        ]
        S = state.shape[0]
        states = [StateRegionV1(_c.sizeof(StateRegionV1), ABI_V1, 0, 0, b"gdn.conv",
                                tensor_view(conv_state, device=dv)),
                  StateRegionV1(_c.sizeof(StateRegionV1), ABI_V1, 0, 0, b"gdn.recurrent",
                                tensor_view(state, device=dv))]
        batch = self.batch_metadata(cu_seqlens) if S > 1 else None
        ex = self._execution(GDN_FORWARD_V1 if flags is None else flags, inputs,
                             tensor_view(out, device=dv), states, T,
                             _stream(stream).value or 0, batch)
        ex.context_tokens = context_tokens
        return self.submit(ex, deadline_s)

    def submit_tail(self, o, z, gamma, w_out, out, stream=None, deadline_s=60.0):
        g = self.geom
        rows = o.shape[0]
        dv = self.device
        inputs = [tensor_view(o, [rows, g.value], [g.value, 1], dv),
                  tensor_view(z, [rows, g.value], [g.value, 1], dv),
                  tensor_view(gamma, [HEAD_DIM], [1], dv),
                  tensor_view(w_out, [g.value, g.hidden], [1, g.value], dv)]
        ex = self._execution(GDN_FORWARD_V1 | GDN_OUTPUT_TAIL_V7, inputs,
                             tensor_view(out, device=dv), [], rows, _stream(stream).value or 0)
        return self.submit(ex, deadline_s)

    def submit(self, ex, deadline_s=60.0, deadline_ns=None):
        import time as _time
        if deadline_ns is None:
            deadline_ns = _time.monotonic_ns() + int(deadline_s * 1e9)
        ev = _c.c_void_p()
        err = _c.POINTER(ErrorV1)()
        st = self.d.submit(self.handle, _c.byref(ex), deadline_ns, _c.byref(ev), _c.byref(err))
        self._keep.clear()
        self._raise(st, err)
        return ev

    def wait(self, ev, timeout_s=60.0):
        import time as _time
        c = CompletionV1()
        err = _c.POINTER(ErrorV1)()
        st = self.d.wait(self.handle, ev, _time.monotonic_ns() + int(timeout_s * 1e9),
                         _c.byref(c), _c.byref(err))
        self._raise(st, err)
        return c

    def poll(self, ev):
        c = CompletionV1()
        err = _c.POINTER(ErrorV1)()
        st = self.d.poll(self.handle, ev, _c.byref(c), _c.byref(err))
        if st == NOT_READY:
            return None
        self._raise(st, err)
        return c

    def release(self, ev):
        self.d.release_event(self.handle, ev)

    def close(self):
        if self.handle:
            self.d.destroy(self.handle)
            self.handle = _c.c_void_p()
