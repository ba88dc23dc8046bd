"""gdn_b200_output_tail_no_alloc: the output tail for callers that cannot
allocate device scratch (an operator interface that passes only inputs and
outputs, or a serving loop bound to a memory plan frozen at start-up).  Its
scratch is a static device array inside the library.

Called twice in a row through the C ABI, each result must equal the
workspace-taking entry point bit for bit (both run the same kernels on the
same sizes), must match the CPU oracle within the output tolerance of the
other parity tests, and the second call must leave the device's free memory
unchanged.  The status query must report no device error after the calls.
This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes when run alone in a fresh
process.
"""
import ctypes

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

pytestmark = pytest.mark.gpu

OUT_MAX_ABS = 2e-2
OUT_MEAN_REL = 5e-3


def _no_alloc(o, z, gamma, w, out, rows, hv, hidden, stream, eps=1e-6):
    fn = G.lib().gdn_b200_output_tail_no_alloc
    return fn(o.data_ptr(), z.data_ptr(), gamma.data_ptr(), w.data_ptr(), out.data_ptr(), rows,
              hv, hidden, eps, ctypes.c_void_p(stream.cuda_stream))


def _status(stream):
    return G.lib().gdn_b200_output_tail_no_alloc_status(ctypes.c_void_p(stream.cuda_stream))


def _close(a_bits, b_bits):
    a = O.bf16_to_f32(a_bits).astype(np.float64)
    b = O.bf16_to_f32(b_bits).astype(np.float64)
    d = np.abs(a - b)
    return d.max() <= OUT_MAX_ABS and d.mean() / max(np.abs(b).mean(), 1e-30) <= OUT_MEAN_REL


@pytest.mark.parametrize("rows,hv,hidden", [(128, 32, 2048), (64, 32, 2048), (1, 8, 512)])
def test_no_alloc_tail_matches_workspace_entry_point_and_oracle(cuda, rows, hv, hidden):
    import torch
    D = G.HEAD_DIM
    o = G.fill(41, 1, (rows, hv, D), G.NORMAL, 0.0, 1.0, G.BF16)
    z = G.fill(41, 2, (rows, hv, D), G.NORMAL, 0.0, 1.0, G.BF16)
    gamma = G.fill(41, 3, (D,), G.NORMAL, 1.0, 0.02, G.BF16)
    w = G.fill(41, 4, (hidden, hv * D), G.NORMAL, 0.0, 0.02, G.BF16)
    t = G.to_device(dict(o=o, z=z, gamma=gamma, w=w), cuda)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        ref = G.output_tail(t["o"], t["z"], t["gamma"], t["w"], stream=stream)
        outs = [torch.empty(rows, hidden, dtype=torch.bfloat16, device=cuda) for _ in range(2)]
    torch.cuda.synchronize()
    assert _no_alloc(t["o"], t["z"], t["gamma"], t["w"], outs[0], rows, hv, hidden, stream) == G.OK
    assert _status(stream) == G.OK, G.last_error()
    free_before = torch.cuda.mem_get_info()[0]
    assert _no_alloc(t["o"], t["z"], t["gamma"], t["w"], outs[1], rows, hv, hidden, stream) == G.OK
    assert _status(stream) == G.OK, G.last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    ref_bits = G.bf16_bits(ref)
    oracle_bits = O.output_tail(o, z, gamma, w)
    for out in outs:
        bits = G.bf16_bits(out)
        assert np.array_equal(bits, ref_bits)
        assert _close(bits, oracle_bits)


def test_no_alloc_tail_rejects_sizes_beyond_its_scratch(cuda):
    import torch
    x = torch.zeros(256, 32, 128, dtype=torch.bfloat16, device=cuda)
    w = torch.zeros(4096, 32 * 128, dtype=torch.bfloat16, device=cuda)
    out = torch.empty(256, 4096, dtype=torch.bfloat16, device=cuda)
    g = torch.ones(128, dtype=torch.bfloat16, device=cuda)
    s = torch.cuda.current_stream()
    assert _no_alloc(x, x, g, w, out, 129, 32, 2048, s) == G.INVALID_ARGUMENT
    assert "static scratch" in G.last_error()
    assert _no_alloc(x, x, g, w, out, 128, 33, 2048, s) == G.INVALID_ARGUMENT
    assert _no_alloc(x, x, g, w, out, 128, 32, 4096, s) == G.INVALID_ARGUMENT
    assert _no_alloc(x, x, g, w, out, 128, 32, 2048, s, eps=float("inf")) == G.INVALID_ARGUMENT
    assert "eps" in G.last_error()
    # a valid call clears the message, as every other entry point does
    assert _no_alloc(x, x, g, w, out, 2, 32, 2048, s) == G.OK
    assert G.last_error() == ""
    assert _status(s) == G.OK
