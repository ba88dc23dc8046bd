"""C-ABI argument validation and provider contract checks that need no GPU:
every malformed call must be rejected with a status and a message before any
device work, and the library must fail loudly (never fall back) when no CUDA
device is present."""
import ctypes

import numpy as np
import pytest

import gdn_b200 as G

vp = ctypes.c_void_p
FAKE = vp(0x10000)          # 16-byte aligned, never dereferenced: calls fail earlier
ODD = vp(0x10002)


def lib():
    return G.lib()


def tail(o=FAKE, z=FAKE, gamma=FAKE, w=FAKE, out=FAKE, rows=128, hv=32, hidden=2048,
         eps=1e-6, ws=FAKE, ws_bytes=1 << 40, stream=None):
    return lib().gdn_b200_output_tail(o, z, gamma, w, out, rows, hv, hidden, eps, ws, ws_bytes,
                                      stream)


@pytest.mark.parametrize("kwargs,fragment", [
    (dict(rows=-1), "positive"),
    (dict(hv=0), "positive"),
    (dict(hidden=100), "multiple of 128"),
    (dict(eps=0.0), "eps"),
    (dict(o=None), "null"),
    (dict(ws=None), "null"),
    (dict(o=ODD), "aligned"),
    (dict(gamma=vp(0x10008)), "aligned"),
    (dict(ws_bytes=100), "workspace too small"),
])
def test_output_tail_rejects(kwargs, fragment):
    assert tail(**kwargs) == G.INVALID_ARGUMENT
    assert fragment in G.last_error()


def test_output_tail_workspace_size():
    # error word + gated activations (+ f32 split-K partials when K is split
    # across separate CTAs; up to 128 rows the split is reduced inside a
    # thread-block cluster and needs no partials)
    n = G.output_tail_workspace_bytes(8192, 32, 2048)
    assert n == 256 + 8192 * 4096 * 2
    small = G.output_tail_workspace_bytes(128, 32, 2048)
    assert small == 256 + 128 * 4096 * 2
    mid = G.output_tail_workspace_bytes(512, 32, 2048)
    assert mid > 256 + 512 * 4096 * 2


def _cu(values):
    arr = np.asarray(values, np.int32)
    return arr, arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


@pytest.mark.parametrize("cu,nseq,fragment", [
    ([1, 5], 1, "cu_seqlens[0]"),
    ([0, 5, 3], 2, "non-decreasing"),
    ([0], 0, "num_seqs"),
    (list(range(1026)), 1025, "num_seqs"),
])
def test_chunk_prefill_rejects_bad_seqlens(cu, nseq, fragment):
    arr, p = _cu(cu)
    st = lib().gdn_b200_chunk_prefill(*([FAKE] * 9), p, nseq, 16, 32, FAKE, 1 << 40, None)
    assert st == G.INVALID_ARGUMENT
    assert fragment in G.last_error()


def test_chunk_prefill_rejects_bad_heads_and_workspace():
    arr, p = _cu([0, 64, 128])
    assert lib().gdn_b200_chunk_prefill(*([FAKE] * 9), p, 2, 16, 30, FAKE, 1 << 40, None) == \
        G.INVALID_ARGUMENT
    assert lib().gdn_b200_chunk_prefill(*([FAKE] * 9), p, 2, 16, 32, FAKE, 1024, None) == \
        G.INVALID_ARGUMENT
    assert "workspace too small" in G.last_error()


def test_chunk_workspace_size_counts_records():
    cu = [0, 4096, 8192]
    # 128 chunks x (16 [K;Q] images of 32 KB + 32 per-v-head records)
    expect = 256 + 128 * (16 * 32768 + 32 * 25856)
    assert G.chunk_prefill_workspace_bytes(cu, 16, 32) == expect
    assert G.chunk_prefill_workspace_bytes([0, 1, 66], 16, 32) == 256 + 3 * (16 * 32768 + 32 * 25856)


def test_layer_forward_rejects():
    arr, p = _cu([0, 64, 128])
    args = [FAKE] * 12
    assert lib().gdn_b200_layer_forward(*args, p, 2, 16, 32, 1000, FAKE, 1 << 40, None) == \
        G.INVALID_ARGUMENT
    args[5] = None  # z
    assert lib().gdn_b200_layer_forward(*args, p, 2, 16, 32, 2048, FAKE, 1 << 40, None) == \
        G.INVALID_ARGUMENT
    assert "null" in G.last_error()


def test_decode_rejects():
    args = [FAKE] * 12
    assert lib().gdn_b200_decode_step(*args, -1, 16, 32, None) == G.INVALID_ARGUMENT
    assert lib().gdn_b200_decode_step(*args, 4, 16, 24 + 1, None) == G.INVALID_ARGUMENT
    args[11] = FAKE
    args[9] = None  # gated_out without z
    assert lib().gdn_b200_decode_step(*args, 4, 16, 32, None) == G.INVALID_ARGUMENT
    assert "z and gamma" in G.last_error()


def test_valid_call_without_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st = tail(rows=0 + 128)
    assert st == G.INTERNAL
    assert G.last_error() != ""


# --------------------------------------------------------------- provider --

def test_query_descriptor_fields():
    st, d, _ = G.query_descriptor()
    assert st == G.OK
    assert d.provider_id == b"org.statecentric.qwen38.gdn"
    assert d.provider_version == b"1.0.0"
    assert d.operator_name == b"operator.qwen38.gdn"
    assert d.operator_version == 1 and d.stage == G.STAGE_GDN and d.flags == 1
    assert d.abi_version == G.ABI_V1 and d.size == ctypes.sizeof(G.DescriptorV1)
    for f in ("create", "destroy", "submit", "poll", "wait", "cancel", "release_event",
              "release_error"):
        assert getattr(d, f)
    assert not d.reserved0 and not d.reserved1 and not d.reserved2


@pytest.mark.parametrize("abi,size", [(2, None), (1, 16)])
def test_query_abi_mismatch(abi, size):
    st, _, msg = G.query_descriptor(abi_version=abi, size=size)
    assert st == G.ABI_MISMATCH and "ABI mismatch" in msg


def _create(mutate_create=None, mutate_cfg=None):
    st, d, _ = G.query_descriptor()
    clock = G.HostV1._fields_[3][1](lambda ctx: 1)
    host = G.HostV1(ctypes.sizeof(G.HostV1), 1, None, clock)
    cfg = G.GdnCreateConfigV1()
    cfg.size = ctypes.sizeof(cfg)
    cfg.abi_version = 1
    cfg.hidden_size = 2048
    cfg.qkv_size_per_rank = 2 * 16 * 128 + 4096
    cfg.value_size_per_rank = 4096
    cfg.gate_heads_per_rank = 32
    cfg.query_heads_per_rank = 16
    cfg.value_heads_per_rank = 32
    cfg.head_dim = 128
    cfg.max_tokens_per_submission = 8192
    if mutate_cfg:
        mutate_cfg(cfg)
    fp = (ctypes.c_uint8 * 32)()
    cr = G.CreateV1(ctypes.sizeof(G.CreateV1), 1, 1, 0, 0, 32,
                    ctypes.cast(fp, ctypes.POINTER(ctypes.c_uint8)),
                    ctypes.cast(ctypes.byref(cfg), ctypes.c_void_p), ctypes.sizeof(cfg))
    if mutate_create:
        mutate_create(cr)
    handle = ctypes.c_void_p()
    err = ctypes.POINTER(G.ErrorV1)()
    st = d.create(ctypes.byref(host), ctypes.byref(cr), ctypes.byref(handle), ctypes.byref(err))
    msg = err.contents.message.decode() if err else ""
    if err:
        d.release_error(err)
    return st, msg, handle, d


@pytest.mark.parametrize("what,mc,mf", [
    ("world 3", lambda c: setattr(c, "world_size", 3), None),
    ("rank >= world", lambda c: setattr(c, "rank", 1), None),
    ("fingerprint", lambda c: setattr(c, "assembly_fingerprint_length", 31), None),
    ("abi", lambda c: setattr(c, "abi_version", 2), None),
    ("hidden", None, lambda f: setattr(f, "hidden_size", 2000)),
    ("head dim", None, lambda f: setattr(f, "head_dim", 64)),
    ("gqa", None, lambda f: setattr(f, "query_heads_per_rank", 12)),
    ("value size", None, lambda f: setattr(f, "value_size_per_rank", 4000)),
    ("max tokens", None, lambda f: setattr(f, "max_tokens_per_submission", 0)),
    ("reserved", None, lambda f: setattr(f, "reserved", 1)),
    ("variant", None, lambda f: setattr(f, "prefill_qkv_split_variant", 8)),
])
def test_create_rejects_invalid_contract(what, mc, mf):
    st, msg, _, _ = _create(mc, mf)
    assert st == G.INVALID_ARGUMENT, what
    assert "invalid" in msg


def test_create_without_gpu_reports_internal():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st, msg, _, _ = _create()
    assert st == G.INTERNAL and "CUDA device" in msg


def test_cancel_is_unsupported():
    st, d, _ = G.query_descriptor()
    err = ctypes.POINTER(G.ErrorV1)()
    assert d.cancel(None, None, ctypes.byref(err)) == G.UNSUPPORTED
    assert b"cannot be cancelled" in err.contents.message
    d.release_error(err)


# ------------------------------------------------- head-parallel fused tail --

def _group(rank=0, world=2, max_rows=256, hidden=2048, reserved=0, regions=None):
    if regions is None:
        regions = [0x100000 * (i + 1) for i in range(world)]
    arr = (ctypes.c_void_p * G.MAX_RANKS)(*(regions + [None] * (G.MAX_RANKS - len(regions))))
    return G.TailGroupV1(rank, world, max_rows, hidden, reserved, arr)


def tail_ar(group, rows=128, hv=16, hidden=2048, eps=1e-6, epoch=1, ws=FAKE, ws_bytes=1 << 40,
            o=FAKE):
    return lib().gdn_b200_output_tail_allreduce(o, FAKE, FAKE, FAKE, rows, hv, hidden, eps,
                                                ctypes.byref(group) if group is not None else None,
                                                epoch, ws, ws_bytes, None)


@pytest.mark.parametrize("gkw,ckw,fragment", [
    ({}, dict(hidden=2176), "multiple of 256"),
    ({}, dict(rows=-1), "positive"),
    (dict(world=3, regions=[0x100000, 0x200000, 0x300000]), {}, "world_size"),
    (dict(rank=2), {}, "rank"),
    (dict(reserved=1), {}, "reserved"),
    (dict(hidden=1024), {}, "hidden differs"),
    ({}, dict(rows=257), "max_rows"),
    (dict(regions=[0x100000, None]), {}, "region is null"),
    (dict(regions=[0x100000, 0x100010]), {}, "256-byte aligned"),
    ({}, dict(epoch=0), "epoch"),
    ({}, dict(ws_bytes=100), "workspace too small"),
    ({}, dict(o=ODD), "aligned"),
])
def test_output_tail_allreduce_rejects(gkw, ckw, fragment):
    assert tail_ar(_group(**gkw), **ckw) == G.INVALID_ARGUMENT
    assert fragment in G.last_error()


def test_output_tail_allreduce_rejects_null_group():
    assert tail_ar(None) == G.INVALID_ARGUMENT
    assert "null" in G.last_error()


def test_tail_exchange_layout_sizes():
    # [max_rows, hidden] bf16 output, then per owned tile slot one 64 KB
    # staging tile per rank, per-(tile, rank, warp) flags, per-(CTA, rank)
    # done flags (148 CTAs).
    def expect(rows, hidden, world):
        r256 = lambda x: (x + 255) // 256 * 256
        tiles = -(-rows // 128) * (hidden // 256)
        grid = min(tiles, 148)
        rounds = -(-tiles // grid)
        slots = -(-rounds // world) * grid
        total = r256(rows * hidden * 2)
        if world > 1:
            total += slots * world * 128 * 512 + r256(tiles * world * 16) + r256(148 * world * 4)
        return total
    for rows, hidden, world in [(16384, 2048, 2), (65536, 2048, 8), (8192, 2048, 1),
                                (100, 1024, 4), (32768, 2048, 4)]:
        assert G.tail_exchange_bytes(rows, hidden, world) == expect(rows, hidden, world)
    assert G.tail_exchange_bytes(128, 1000, 2) == 0
    assert G.tail_exchange_bytes(128, 2048, 3) == 0
    assert G.tail_exchange_bytes(0, 2048, 2) == 0
    assert G.output_tail_allreduce_workspace_bytes(100, 16) == 256 + 100 * 16 * 128 * 2


def test_exchange_entry_points_without_gpu_fail_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    region = ctypes.c_void_p()
    assert lib().gdn_b200_exchange_alloc(1 << 20, ctypes.byref(region)) == G.INTERNAL
    assert region.value is None
    assert tail_ar(_group()) == G.INTERNAL
    assert lib().gdn_b200_exchange_export(None, None) == G.INVALID_ARGUMENT


# ------------------------------------------------------------ input side --

def _input_side(x=FAKE, conv_state=FAKE, cu=(0, 64, 128), hk=16, hv=32, hidden=2048, ws=FAKE,
                ws_bytes=1 << 40, q=FAKE):
    arr, p = _cu(list(cu))
    return lib().gdn_b200_input_side(x, FAKE, FAKE, FAKE, FAKE, FAKE, conv_state, p,
                                     len(arr) - 1, hk, hv, hidden, 1, q, FAKE, FAKE, FAKE, FAKE,
                                     FAKE, ws, ws_bytes, None)


@pytest.mark.parametrize("kwargs,fragment", [
    (dict(hidden=1000), "multiple of 128"),
    (dict(hv=30), "multiple of qk_heads"),
    (dict(x=None), "null"),
    (dict(conv_state=None), "null"),
    (dict(q=None), "null"),
    (dict(x=ODD), "aligned"),
    (dict(cu=(1, 5)), "cu_seqlens[0]"),
    (dict(ws_bytes=100), "workspace too small"),
])
def test_input_side_rejects(kwargs, fragment):
    assert _input_side(**kwargs) == G.INVALID_ARGUMENT
    assert fragment in G.last_error()


def test_layer_forward_x_rejects_and_sizes():
    arr, p = _cu([0, 64, 128])
    args = [FAKE] * 13
    assert lib().gdn_b200_layer_forward_x(*args, p, 2, 16, 32, 2048, 1, FAKE, 100, None) == \
        G.INVALID_ARGUMENT
    assert "workspace too small" in G.last_error()
    args[7] = None  # A_log
    assert lib().gdn_b200_layer_forward_x(*args, p, 2, 16, 32, 2048, 1, FAKE, 1 << 40, None) == \
        G.INVALID_ARGUMENT
    assert "null" in G.last_error()
    # the layer-from-x workspace holds the input side's buffers and scratch
    # plus the post-projection layer's
    cu = [0, 4096, 8192]
    assert G.layer_forward_x_workspace_bytes(cu, 16, 32, 2048) > \
        G.layer_forward_workspace_bytes(cu, 16, 32, 2048) + \
        G.input_side_workspace_bytes(cu, 16, 32, 2048) - 256


def test_rank_sum_layout_and_rejections():
    # two partial buffers + 2 x world staging slots + 256 bytes of flags
    part = 8192 * 2048 * 2
    slot = 8192 // 8 * 2048 * 2
    assert G.lib().gdn_b200_rank_sum_bytes(8192, 2048, 8) == 2 * part + 2 * 8 * slot + 256
    assert G.lib().gdn_b200_rank_sum_bytes(8190, 2048, 8) == 0      # rows % world
    assert G.lib().gdn_b200_rank_sum_bytes(64, 2048, 9) == 0        # at most 8 ranks
    assert G.lib().gdn_b200_rank_sum_bytes(64, 100, 2) == 0         # hidden % 8
    grp = G.TailGroupV1(0, 2, 64, 2048, 0, (ctypes.c_void_p * G.MAX_RANKS)())
    st = G.lib().gdn_b200_rank_sum(ctypes.byref(grp), 1, 64, ctypes.c_void_p(256),
                                   ctypes.c_void_p(256), None, None)
    assert st == G.INVALID_ARGUMENT and "group" in G.last_error()
    assert G.lib().gdn_b200_rank_sum_part(ctypes.byref(grp), 1) is None
    regions = (ctypes.c_void_p * G.MAX_RANKS)(4096, 8192)
    grp = G.TailGroupV1(0, 2, 64, 2048, 0, regions)
    assert G.lib().gdn_b200_rank_sum(ctypes.byref(grp), 0, 64, ctypes.c_void_p(256),
                                     ctypes.c_void_p(256), None, None) == G.INVALID_ARGUMENT
    assert G.lib().gdn_b200_rank_sum(ctypes.byref(grp), 1, 63, ctypes.c_void_p(256),
                                     ctypes.c_void_p(256), None, None) == G.INVALID_ARGUMENT
    assert "multiple of world_size" in G.last_error()
    assert G.lib().gdn_b200_rank_sum_part(ctypes.byref(grp), 3) == 4096 + 64 * 2048 * 2
