"""The provider C ABI on the GPU: the same results as the direct entry points
(bit for bit), and the reference provider's validation, deadline, poll/wait,
cancel and release behaviour."""
import ctypes
import time

import numpy as np
import pytest

import gdn_b200 as G

pytestmark = pytest.mark.gpu

GEOM = G.Geometry(16, 32, 2048)


@pytest.fixture()
def setup(cuda):
    import torch
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    prov = G.Provider(GEOM, max_tokens=4096)
    yield prov, stream
    prov.close()
    torch.cuda.set_stream(torch.cuda.default_stream())


def _inputs(cu, cuda, seed=31):
    x = G.synthetic_layer_inputs(np.asarray(cu, np.int32), GEOM, seed=seed, state_std=0.05)
    return x, G.to_device(x, cuda)


@pytest.mark.parametrize("cu", [[0, 64, 128], [0, 130], [0, 1, 2, 3, 4], [0, 1, 70, 200]])
def test_provider_layer_matches_direct_entry_point(setup, cuda, cu):
    import torch
    prov, stream = setup
    x, t = _inputs(cu, cuda)
    T = cu[-1]
    state_p = t["state"].clone()
    out_p = torch.empty(T, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    ev = prov.submit_layer(t, state_p, out_p, cu, stream=stream)
    c = prov.wait(ev)
    assert c.phase == G.EVENT_COMPLETE
    prov.release(ev)
    state_d = t["state"].clone()
    out_d = G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                            t["dt_bias"], t["gamma"], t["w_out"], state_d, cu, stream=stream)
    torch.cuda.synchronize()
    assert torch.equal(out_p, out_d)
    assert torch.equal(state_p, state_d)


def test_provider_tail_matches_direct_entry_point(setup, cuda):
    import torch
    prov, stream = setup
    x, t = _inputs([0, 64, 128], cuda)
    o = torch.randn(128, GEOM.value_heads, 128, device=cuda).to(torch.bfloat16)
    out_p = torch.empty(128, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    ev = prov.submit_tail(o, t["z"], t["gamma"], t["w_out"], out_p, stream=stream)
    prov.wait(ev)
    prov.release(ev)
    out_d = G.output_tail(o, t["z"], t["gamma"], t["w_out"], stream=stream)
    torch.cuda.synchronize()
    assert torch.equal(out_p, out_d)


def _expect(status, fn, fragment=None):
    with pytest.raises(G.ProviderError) as e:
        fn()
    assert e.value.status == status
    if fragment:
        assert fragment in str(e.value)


def test_provider_rejections(setup, cuda):
    import torch
    prov, stream = setup
    cu = [0, 64, 128]
    x, t = _inputs(cu, cuda)
    out = torch.empty(128, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    st = t["state"]
    base = dict(t)

    # Null stream (the reference requires a stream too).
    _expect(G.INVALID_ARGUMENT,
            lambda: prov.submit_layer(base, st, out, cu, stream=torch.cuda.default_stream()))
    # Wrong v geometry, wrong dtype, wrong state kind.
    def narrow_v(ins, rs):
        ins[2].dimensions[1] = GEOM.value // 2
        ins[2].byte_length //= 2

    def f32_gamma(ins, rs):
        ins[8].scalar_type = G.SCALAR_F32

    def conv_kind(ins, rs):
        rs.state_kind = b"gdn.conv"

    for mutate in (narrow_v, f32_gamma, conv_kind):
        _expect(G.INVALID_ARGUMENT,
                lambda: _submit_raw(prov, base, st, out, cu, stream, mutate=mutate), "geometry")
    # Ranges not packed / not covering the tokens.
    _expect(G.INVALID_ARGUMENT,
            lambda: _submit_raw(prov, base, st, out, [0, 64, 128], stream, offsets=[0, 63]),
            "not packed")
    _expect(G.INVALID_ARGUMENT,
            lambda: _submit_raw(prov, base, st, out, [0, 64, 128], stream, counts=[64, 63]),
            "cover")
    # Expired deadline.
    _expect(G.TIMEOUT, lambda: prov.submit_layer(base, st, out, cu, stream=stream,
                                                 deadline_s=-1.0), "deadline")
    # Too many tokens for the configured maximum.
    big = G.Provider(GEOM, max_tokens=64)
    try:
        _expect(G.INVALID_ARGUMENT, lambda: big.submit_layer(base, st, out, cu, stream=stream))
    finally:
        big.close()


def _submit_raw(prov, t, state, out, cu, stream, offsets=None, counts=None, flags=None,
                layer=0, mutate=None):
    """Builds an execution by hand to reach the individual validation clauses."""
    batch = G.Provider.batch_metadata(cu)
    if offsets is not None:
        for i, v in enumerate(offsets):
            batch._arrays[0][i] = v
    if counts is not None:
        for i, v in enumerate(counts):
            batch._arrays[1][i] = v
    g = GEOM
    T = cu[-1]
    D = 128
    ins = [G.tensor_view(t["q"], [T, g.qk_heads * D], [g.qk_heads * D, 1]),
           G.tensor_view(t["k"], [T, g.qk_heads * D], [g.qk_heads * D, 1]),
           G.tensor_view(t["v"], [T, g.value], [g.value, 1]),
           G.tensor_view(t["a"], [T, g.value_heads], [g.value_heads, 1]),
           G.tensor_view(t["b"], [T, g.value_heads], [g.value_heads, 1]),
           G.tensor_view(t["z"], [T, g.value], [g.value, 1]),
           G.tensor_view(t["A_log"]), G.tensor_view(t["dt_bias"]), G.tensor_view(t["gamma"]),
           G.tensor_view(t["w_out"], [g.value, g.hidden], [1, g.value])]
    rs = G.StateRegionV1(ctypes.sizeof(G.StateRegionV1), 1, layer, 0, b"gdn.recurrent",
                         G.tensor_view(state))
    if mutate is not None:
        mutate(ins, rs)
    ex = prov._execution(flags if flags is not None else (G.GDN_FORWARD_V1 | G.GDN_POST_PROJECTION_V6),
                         ins, G.tensor_view(out), [rs], T, stream.cuda_stream, batch)
    ex.layer_index = layer
    return prov.submit(ex)


def test_reference_flags_and_layer_rules(setup, cuda):
    import torch
    prov, stream = setup
    cu = [0, 64, 128]
    x, t = _inputs(cu, cuda)
    out = torch.empty(128, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    # x-based flags need the x-based inputs and both state regions
    for flags in (G.GDN_FORWARD_V1, G.GDN_FORWARD_V1 | G.GDN_PREFILL_POST_CONV_PACK_V5,
                  G.GDN_FORWARD_V1 | G.GDN_PREFILL_SPLIT_V2):
        _expect(G.INVALID_ARGUMENT, lambda: _submit_raw(prov, t, t["state"], out, cu, stream,
                                                        flags=flags))
    _expect(G.INVALID_ARGUMENT, lambda: _submit_raw(prov, t, t["state"], out, cu, stream,
                                                    flags=G.GDN_POST_PROJECTION_V6))
    # Full-attention layers (layer_index % 4 == 3) are not GDN layers.
    _expect(G.INVALID_ARGUMENT, lambda: _submit_raw(prov, t, t["state"], out, cu, stream,
                                                    layer=3))


def test_poll_wait_release(setup, cuda):
    import torch
    prov, stream = setup
    cu = [0, 4096]
    x, t = _inputs(cu, cuda)
    out = torch.empty(4096, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    ev = prov.submit_layer(t, t["state"], out, cu, stream=stream)
    first = prov.poll(ev)          # None (NOT_READY) or a completion
    assert first is None or first.phase == G.EVENT_COMPLETE
    c = prov.wait(ev, timeout_s=30.0)
    assert c.phase == G.EVENT_COMPLETE and c.elapsed_ns > 0
    assert prov.poll(ev).phase == G.EVENT_COMPLETE
    prov.release(ev)
    # Releasing an event that has not been waited for synchronises first.
    ev = prov.submit_layer(t, t["state"], out, cu, stream=stream)
    prov.release(ev)
    # An expired wait deadline is TIMEOUT.
    ev = prov.submit_layer(t, t["state"], out, cu, stream=stream)
    _expect(G.TIMEOUT, lambda: prov.wait(ev, timeout_s=-1.0))
    prov.wait(ev)
    prov.release(ev)


def test_pool_reuses_workspace_and_reports(cuda, capfd, monkeypatch):
    import torch
    monkeypatch.setenv("STATECENTRIC_QWEN38_GDN_POOL_TELEMETRY", "1")
    stream = torch.cuda.Stream()
    prov = G.Provider(GEOM, max_tokens=256)
    cu = [0, 64, 128]
    x, t = _inputs(cu, cuda)
    out = torch.empty(128, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    for _ in range(3):
        ev = prov.submit_layer(t, t["state"], out, cu, stream=stream)
        prov.wait(ev)
        prov.release(ev)
    prov.close()
    err = capfd.readouterr().err
    assert '"allocations":1' in err and '"reuses":2' in err and '"drained":true' in err


@pytest.mark.parametrize("flags_name,context", [("GDN_FORWARD_V1", 0),
                                                ("GDN_PREFILL_POST_CONV_PACK_V5", 64),
                                                ("GDN_PREFILL_SPLIT_V2", 0)])
def test_provider_x_based_layer_matches_direct_entry_point(setup, cuda, flags_name, context):
    """The reference's x-based submission runs the whole layer (projections,
    causal conv with the gdn.conv state, core, tail) and gives the same bits
    as gdn_b200_layer_forward_x; context_tokens 0 means zero conv history."""
    import torch
    prov, stream = setup
    cu = [0, 100, 164]
    xs = G.synthetic_input_side(cu, GEOM, seed=11, conv_state_std=1.0)
    lx = G.synthetic_layer_inputs(cu, GEOM, seed=11, state_std=0.05)
    tx = G.to_device(xs, cuda)
    t = G.to_device({n: lx[n] for n in ("A_log", "dt_bias", "gamma", "w_out", "state")}, cuda)
    flags = G.GDN_FORWARD_V1 | (0 if flags_name == "GDN_FORWARD_V1" else getattr(G, flags_name))
    out_p = torch.empty(164, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    cs_p, st_p = tx["conv_state"].clone(), t["state"].clone()
    with torch.cuda.stream(stream):
        ev = prov.submit_layer_x(tx, t, cs_p, st_p, out_p, cu, context_tokens=context,
                                 flags=flags, stream=stream)
    prov.wait(ev)
    prov.release(ev)
    cs_d, st_d = tx["conv_state"].clone(), t["state"].clone()
    out_d = G.layer_forward_x(tx["x"], tx["w_qkv"], tx["w_z"], tx["w_a"], tx["w_b"],
                              tx["conv_w"], cs_d, t["A_log"], t["dt_bias"], t["gamma"],
                              t["w_out"], st_d, cu, GEOM.qk_heads, use_conv_state=context > 0)
    torch.cuda.synchronize()
    assert torch.equal(out_p, out_d)
    assert torch.equal(st_p, st_d)
    assert torch.equal(cs_p, cs_d)


def test_first_admission_telemetry(cuda, capfd):
    """One line per executed path at its first admission (the reference's
    first-admission telemetry, P:590-723): packed decode (V12) and its flat
    output projection (V18) in the reference's format, and the B200 chunked
    prefill path."""
    import torch
    stream = torch.cuda.Stream()
    prov = G.Provider(GEOM, max_tokens=4096)
    dec = [0, 1, 2, 3, 4]
    _, td = _inputs(dec, cuda)
    out_d = torch.empty(4, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    for _ in range(2):
        ev = prov.submit_layer(td, td["state"], out_d, dec, stream=stream)
        prov.wait(ev)
        prov.release(ev)
    pre = [0, 64, 128]
    _, tp = _inputs(pre, cuda)
    out_p = torch.empty(128, GEOM.hidden, dtype=torch.bfloat16, device=cuda)
    ev = prov.submit_layer(tp, tp["state"], out_p, pre, stream=stream)
    prov.wait(ev)
    prov.release(ev)
    prov.close()
    err = capfd.readouterr().err.splitlines()
    decode = [l for l in err if l.startswith("STATECENTRIC_QWEN38_GDN_PACKED_DECODE_TELEMETRY_V12=")]
    flat = [l for l in err if l.startswith("STATECENTRIC_QWEN38_GDN_DECODE_FLAT_OUTPUT_PROJECTION_V18=")]
    chunk = [l for l in err if l.startswith("STATECENTRIC_QWEN38_GDN_B200_CHUNK_PREFILL_TELEMETRY_V1=")]
    assert decode == ['STATECENTRIC_QWEN38_GDN_PACKED_DECODE_TELEMETRY_V12='
                      '{"rank":0,"submit_calls":1,"admitted_calls":1}']
    assert flat == ['STATECENTRIC_QWEN38_GDN_DECODE_FLAT_OUTPUT_PROJECTION_V18='
                    '{"rank":0,"admitted_calls":1,"rows":4}']
    assert chunk == ['STATECENTRIC_QWEN38_GDN_B200_CHUNK_PREFILL_TELEMETRY_V1='
                     '{"rank":0,"submit_calls":3,"admitted_calls":1,"sequences":2,"chunks":2}']
