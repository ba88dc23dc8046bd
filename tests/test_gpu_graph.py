"""CUDA-graph capture and state-slot binding of the decode step: the B200
counterpart of the reference's graph binding (native/include/statecentric/
qwen38_gdn_graph_binding.h:15-73) and capture-lifetime events
(qwen38_gdn_graph_event_policy.h:70-74; a CUDA graph owns its own
dependencies, so no event pool is involved).

* gdn_b200_decode_step_rows on rows scattered through a state pool equals
  gdn_b200_decode_step on the same rows packed contiguously, bit for bit, and
  leaves every other row untouched.
* A CUDA graph of one decode step (decode + output tail), captured once and
  replayed against other slots by rewriting the device row table, equals
  eager calls bit for bit (DIRECT binding without the exact-address
  restriction).
* COPY binding: rows gathered into packed buffers with
  gdn_b200_copy_graph_rows, a graph captured on the packed buffers, the rows
  scattered back: equal to eager calls; a refused binding copies nothing.
"""
import numpy as np
import pytest

import gdn_b200 as G

pytestmark = pytest.mark.gpu

GEOM = G.Geometry(16, 32, 2048)
ROW_BYTES = 32 * 128 * 128 * 4


def _decode_inputs(B, seed, cuda):
    cu = np.arange(B + 1, dtype=np.int32)
    x = G.synthetic_layer_inputs(cu, GEOM, seed=seed)
    return G.to_device({n: x[n] for n in ("q", "k", "v", "a", "b", "z", "A_log", "dt_bias",
                                          "gamma", "w_out")}, cuda)


def _row_table(pool, slots, device):
    import torch
    base = pool.data_ptr()
    stride = pool[0].numel() * pool.element_size()
    return torch.tensor([base + s * stride for s in slots], dtype=torch.int64, device=device)


def test_decode_rows_equal_contiguous_decode(cuda):
    import torch
    B, P = 8, 20
    t = _decode_inputs(B, 12, cuda)
    gen = torch.Generator(device=cuda).manual_seed(3)
    pool = torch.randn(P, 32, 128, 128, device=cuda, generator=gen) * 0.05
    before = pool.clone()
    slots = [7, 3, 19, 0, 11, 5, 16, 2]
    packed = pool[slots].clone()
    o_rows = torch.empty_like(t["v"])
    o_cont = torch.empty_like(t["v"])
    G.decode_step_rows(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"],
                       _row_table(pool, slots, cuda), o_out=o_rows)
    G.decode_step(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"], packed,
                  o_out=o_cont)
    torch.cuda.synchronize()
    assert torch.equal(o_rows, o_cont)
    assert torch.equal(pool[slots], packed)
    others = [i for i in range(P) if i not in slots]
    assert torch.equal(pool[others], before[others])


def _step(t, rows, o, out, ws):
    G.decode_step_rows(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"], rows,
                       o_out=o)
    G.output_tail(o, t["z"], t["gamma"], t["w_out"], out=out, workspace=ws)


def test_graph_replay_rebinds_slots(cuda):
    import torch
    B, P = 8, 24
    t = _decode_inputs(B, 13, cuda)
    gen = torch.Generator(device=cuda).manual_seed(4)
    pool = torch.randn(P, 32, 128, 128, device=cuda, generator=gen) * 0.05
    rows = torch.empty(B, dtype=torch.int64, device=cuda)   # the table the graph reads
    o = torch.empty_like(t["v"])
    out = torch.empty(B, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    ws = torch.empty(G.output_tail_workspace_bytes(B, 32, GEOM.hidden), dtype=torch.uint8,
                     device=cuda)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):          # warm-up outside the capture
        scratch = pool.clone()
        rows.copy_(_row_table(scratch, list(range(B)), cuda))
        _step(t, rows, o, out, ws)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _step(t, rows, o, out, ws)
    rng = np.random.default_rng(5)
    for trial in range(3):
        slots = [int(s) for s in rng.permutation(P)[:B]]
        ref_pool = pool.clone()
        o_e = torch.empty_like(o)
        out_e = torch.empty_like(out)
        ws_e = torch.empty_like(ws)
        _step(t, _row_table(ref_pool, slots, cuda), o_e, out_e, ws_e)
        rows.copy_(_row_table(pool, slots, cuda))
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, out_e), f"trial {trial}: output"
        assert torch.equal(pool, ref_pool), f"trial {trial}: state pool"
    G.workspace_status(ws)


def test_copy_binding_gathers_and_scatters(cuda):
    import torch
    B, P = 4, 9
    C = (2 * 16 + 32) * 128
    conv_bytes, rec_bytes = 3 * C * 2, ROW_BYTES
    t = _decode_inputs(B, 14, cuda)
    # One arena: P conv rows, then P recurrent rows.
    arena = torch.zeros(P * (conv_bytes + rec_bytes), dtype=torch.uint8, device=cuda)
    conv_pool = arena[:P * conv_bytes].view(torch.int16).view(P, 3, C)
    rec_pool = arena[P * conv_bytes:].view(torch.float32).view(P, 32, 128, 128)
    gen = torch.Generator(device=cuda).manual_seed(6)
    rec_pool.copy_(torch.randn(P, 32, 128, 128, device=cuda, generator=gen) * 0.05)
    conv_pool.copy_(torch.randint(-2000, 2000, (P, 3, C), device=cuda, dtype=torch.int16,
                                  generator=gen))
    packed_conv = torch.empty(B, 3, C, dtype=torch.int16, device=cuda)
    packed_rec = torch.empty(B, 32, 128, 128, dtype=torch.float32, device=cuda)
    o = torch.empty_like(t["v"])
    out = torch.empty(B, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    ws = torch.empty(G.output_tail_workspace_bytes(B, 32, GEOM.hidden), dtype=torch.uint8,
                     device=cuda)

    def packed_step(o_, out_, ws_):
        G.decode_step(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"],
                      packed_rec, o_out=o_)
        G.output_tail(o_, t["z"], t["gamma"], t["w_out"], out=out_, workspace=ws_)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        packed_step(o, out, ws)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        packed_step(o, out, ws)

    def layout(slots):
        lay = G.LayoutWorkspaceV1()
        lay.size = G.ctypes.sizeof(lay)
        lay.abi_version = G.ABI_V1
        lay.batch_size = B
        lay.binding_mode = G.BINDING_COPY_V1
        lay.arena = arena.data_ptr()
        lay.arena_bytes = arena.numel()
        lay.required_arena_bytes = arena.numel()
        lay.conv_bytes_per_row = conv_bytes
        lay.recurrent_bytes_per_row = rec_bytes
        for i, s in enumerate(slots):
            lay.conv_row_addresses[i] = conv_pool[s].data_ptr()
            lay.recurrent_row_addresses[i] = rec_pool[s].data_ptr()
        return lay

    for slots in ([2, 7, 0, 5], [8, 1, 4, 3]):
        lay = layout(slots)
        ref_rec = rec_pool.clone()
        ref_conv = conv_pool.clone()
        o_e, out_e, ws_e = torch.empty_like(o), torch.empty_like(out), torch.empty_like(ws)
        G.decode_step_rows(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"],
                           _row_table(ref_rec, slots, cuda), o_out=o_e)
        G.output_tail(o_e, t["z"], t["gamma"], t["w_out"], out=out_e, workspace=ws_e)
        stream = torch.cuda.current_stream()
        G.copy_graph_rows(lay, B, conv_bytes, rec_bytes, packed_conv.data_ptr(),
                          packed_rec.data_ptr(), True, stream)
        graph.replay()
        G.copy_graph_rows(lay, B, conv_bytes, rec_bytes, packed_conv.data_ptr(),
                          packed_rec.data_ptr(), False, stream)
        torch.cuda.synchronize()
        assert torch.equal(out, out_e)
        assert torch.equal(rec_pool, ref_rec)
        assert torch.equal(conv_pool, ref_conv)
        assert torch.equal(packed_conv, conv_pool[slots])

    # A row outside the arena: refused, nothing copied.
    lay = layout([0, 1, 2, 3])
    lay.recurrent_row_addresses[3] = arena.data_ptr() + arena.numel() - rec_bytes + 256
    snapshot = packed_rec.clone()
    with pytest.raises(G.GdnError) as e:
        G.copy_graph_rows(lay, B, conv_bytes, rec_bytes, packed_conv.data_ptr(),
                          packed_rec.data_ptr(), True)
    assert e.value.status == G.INVALID_ARGUMENT and "out of bounds" in str(e.value)
    torch.cuda.synchronize()
    assert torch.equal(packed_rec, snapshot)
