"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle on
identical seeded inputs.

Tolerances (the bar for bf16 outputs with f32 accumulation and for the f32
recurrent state):
  outputs: max |gpu - ref| <= 2e-2 and mean|gpu - ref| / mean|ref| <= 5e-3
  state:   ||S_gpu - S_ref||_F / ||S_ref||_F <= 1e-3
The oracle reference for the core is the token-serial recurrence in double
precision (``gdn_oracle.core(mode=0)``).
"""
import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

OUT_MAX_ABS = 2e-2
OUT_MEAN_REL = 5e-3
STATE_REL = 1e-3

pytestmark = pytest.mark.gpu


def out_metrics(gpu_bits, ref_bits):
    g = O.bf16_to_f32(gpu_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    d = np.abs(g - r)
    return float(d.max()), float(d.mean() / max(np.abs(r).mean(), 1e-30))


def assert_out_close(gpu_bits, ref_bits, what):
    mx, mr = out_metrics(gpu_bits, ref_bits)
    assert mx <= OUT_MAX_ABS and mr <= OUT_MEAN_REL, f"{what}: max_abs={mx:.3e} mean_rel={mr:.3e}"


def assert_state_close(gpu, ref, what):
    rel = float(np.linalg.norm((gpu - ref).astype(np.float64)) /
                max(np.linalg.norm(ref.astype(np.float64)), 1e-30))
    assert rel <= STATE_REL, f"{what}: state rel={rel:.3e}"


def oracle_core(x, cu):
    g, beta = O.gating(x["a"], x["b"], x["A_log"], x["dt_bias"])
    qn, kn = O.l2norm(x["q"]), O.l2norm(x["k"])
    st = x["state"].copy()
    o = O.core(qn, kn, x["v"], g, beta, st, cu, mode=0)
    return o, st


# ------------------------------------------------------------------ tail --

# 2400 rows: 19 x 8 tiles of 128 x 256 on 148 SMs leave a last wave of 4
# tiles, which run as 8 half-width tiles, one of them in the partial last
# row tile.
@pytest.mark.parametrize("rows,hv,hidden", [(128, 32, 2048), (1, 32, 2048), (64, 32, 2048),
                                            (130, 32, 2048), (1000, 32, 2048),
                                            (2400, 32, 2048),
                                            (256, 4, 2048), (96, 8, 384),
                                            (64, 4, 2048), (32, 2, 2048)])
def test_output_tail_matches_oracle(cuda, rows, hv, hidden):
    import torch
    D = G.HEAD_DIM
    o = G.fill(0, 21, (rows, hv, D), G.NORMAL, 0.0, 1.0, G.BF16)
    z = G.fill(0, 22, (rows, hv, D), G.NORMAL, 0.0, 1.0, G.BF16)
    gamma = G.fill(0, 23, (D,), G.NORMAL, 1.0, 0.02, G.BF16)
    w = G.fill(0, 24, (hidden, hv * D), G.NORMAL, 0.0, 0.02, G.BF16)
    ref = O.output_tail(o, z, gamma, w)
    t = G.to_device(dict(o=o, z=z, gamma=gamma, w=w), cuda)
    ws = torch.empty(G.output_tail_workspace_bytes(rows, hv, hidden), dtype=torch.uint8,
                     device=cuda)
    out = G.output_tail(t["o"], t["z"], t["gamma"], t["w"], workspace=ws)
    G.workspace_status(ws)
    assert_out_close(G.bf16_bits(out), ref, f"tail rows={rows}")


def test_flat_tail_equals_per_sequence_tails(cuda):
    """The reference's dual-tail benchmark invariant: the flattened 2x64 tail
    is bit-identical to the two per-sequence tails."""
    D, hv, hidden = G.HEAD_DIM, 32, 2048
    o = G.fill(0, 31, (128, hv, D), G.NORMAL, 0.0, 1.0, G.BF16)
    z = G.fill(0, 32, (128, hv, D), G.NORMAL, 0.0, 1.0, G.BF16)
    gamma = G.fill(0, 33, (D,), G.NORMAL, 1.0, 0.02, G.BF16)
    w = G.fill(0, 34, (hidden, hv * D), G.NORMAL, 0.0, 0.02, G.BF16)
    t = G.to_device(dict(o=o, z=z, gamma=gamma, w=w), cuda)
    flat = G.bf16_bits(G.output_tail(t["o"], t["z"], t["gamma"], t["w"]))
    s0 = G.bf16_bits(G.output_tail(t["o"][:64], t["z"][:64], t["gamma"], t["w"]))
    s1 = G.bf16_bits(G.output_tail(t["o"][64:], t["z"][64:], t["gamma"], t["w"]))
    assert np.array_equal(flat, np.concatenate([s0, s1])), "flat tail differs from per-sequence"


# ---------------------------------------------------------------- decode --

@pytest.mark.parametrize("batch", [1, 4, 64, 100])
def test_decode_step_matches_oracle(cuda, batch):
    import torch
    geom = G.Geometry(16, 32, 2048)
    cu = np.arange(batch + 1, dtype=np.int32)
    x = G.synthetic_layer_inputs(cu, geom, seed=2, state_std=0.05)
    ref_o, ref_state = oracle_core(x, cu)
    ref_gated = O.tail_prologue(ref_o, x["z"], x["gamma"])
    t = G.to_device(x, cuda)
    o = torch.empty_like(t["v"])
    gated = torch.empty(batch, geom.value, dtype=torch.bfloat16, device=cuda)
    G.decode_step(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"], t["state"],
                  o_out=o, z=t["z"], gamma=t["gamma"], gated_out=gated)
    torch.cuda.synchronize()
    assert_out_close(G.bf16_bits(o), ref_o, "decode o")
    assert_out_close(G.bf16_bits(gated), ref_gated, "decode gated")
    assert_state_close(t["state"].cpu().numpy(), ref_state, "decode state")


# ----------------------------------------------------------------- chunk --

CHUNK_CASES = [
    ([0, 1], 16.0, 0.05),
    ([0, 9], 16.0, 0.05),
    ([0, 64], 16.0, 0.0),
    ([0, 65], 16.0, 0.05),
    ([0, 130], 0.05, 0.05),
    ([0, 200], 1.0, 0.05),
    ([0, 1, 10, 74, 200, 457], 16.0, 0.05),
    ([0, 300, 600], 0.05, 0.05),
]


@pytest.mark.parametrize("cu,a_log_hi,state_std", CHUNK_CASES)
def test_chunk_prefill_matches_oracle(cuda, cu, a_log_hi, state_std):
    import torch
    geom = G.Geometry(16, 32, 2048)
    cu = np.asarray(cu, np.int32)
    x = G.synthetic_layer_inputs(cu, geom, seed=3, state_std=state_std, a_log_hi=a_log_hi)
    ref_o, ref_state = oracle_core(x, cu)
    t = G.to_device(x, cuda)
    ws = torch.empty(G.chunk_prefill_workspace_bytes(cu, geom.qk_heads, geom.value_heads), dtype=torch.uint8,
                     device=cuda)
    o = G.chunk_prefill(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"],
                        t["state"], cu, workspace=ws)
    G.workspace_status(ws)
    assert_out_close(G.bf16_bits(o), ref_o, f"chunk o {cu.tolist()}")
    assert_state_close(t["state"].cpu().numpy(), ref_state, f"chunk state {cu.tolist()}")


# ----------------------------------------------------------------- layer --

@pytest.mark.parametrize("cu,state_std", [([0, 64, 128], 0.0), ([0, 100, 356], 0.05),
                                          (list(range(9)), 0.05)])
def test_layer_forward_matches_oracle(cuda, cu, state_std):
    import torch
    geom = G.Geometry(16, 32, 2048)
    cu = np.asarray(cu, np.int32)
    x = G.synthetic_layer_inputs(cu, geom, seed=4, state_std=state_std)
    st = x["state"].copy()
    ref_out = O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"], x["dt_bias"],
                      x["gamma"], x["w_out"], st, cu, mode=0)
    t = G.to_device(x, cuda)
    ws = torch.empty(G.layer_forward_workspace_bytes(cu, geom.qk_heads, geom.value_heads, geom.hidden),
                     dtype=torch.uint8, device=cuda)
    out = G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                          t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu, workspace=ws)
    G.workspace_status(ws)
    assert_out_close(G.bf16_bits(out), ref_out, f"layer out {cu.tolist()}")
    assert_state_close(t["state"].cpu().numpy(), st, f"layer state {cu.tolist()}")
