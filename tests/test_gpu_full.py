"""Full-size parity on the GPU: the benchmark workloads against the oracle,
plus size-independent invariants (chunk-aligned continuation, per-sequence
decode, golden vectors)."""
import os

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O
from test_gpu_parity import assert_out_close, assert_state_close

pytestmark = pytest.mark.gpu
GEOM = G.Geometry(16, 32, 2048)
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _layer_both(cu, cuda, seed, state_std):
    import torch
    x = G.synthetic_layer_inputs(cu, GEOM, seed=seed, state_std=state_std)
    st = x["state"].copy()
    ref = O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"], x["dt_bias"],
                  x["gamma"], x["w_out"], st, cu, mode=0)
    t = G.to_device(x, cuda)
    out = G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                          t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu)
    torch.cuda.synchronize()
    return G.bf16_bits(out), ref, t["state"].cpu().numpy(), st


def test_prefill_2x4096_matches_oracle(cuda):
    cu = np.array([0, 4096, 8192], np.int32)
    out, ref, st, st_ref = _layer_both(cu, cuda, seed=1, state_std=0.0)
    assert_out_close(out, ref, "2x4096 layer")
    assert_state_close(st, st_ref, "2x4096 state")


def varlen_lengths(seed=1, n=8, lo=64, hi=8192):
    u = G.fill(seed, 100, (n,), G.UNIFORM, float(lo), float(hi + 1), G.F32)
    return np.floor(u).astype(np.int64)


def test_varlen_8_sequences_matches_oracle(cuda):
    lens = varlen_lengths()
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    out, ref, st, st_ref = _layer_both(cu, cuda, seed=1, state_std=0.05)
    assert_out_close(out, ref, f"varlen {lens.tolist()}")
    assert_state_close(st, st_ref, "varlen state")


def test_chunk_aligned_continuation_is_bit_identical(cuda):
    """Prefill of 2 x 4096 tokens in one call equals two calls of 2 x 2048
    with the state carried (chunk boundaries coincide)."""
    import torch
    cu = np.array([0, 4096, 8192], np.int32)
    x = G.synthetic_layer_inputs(cu, GEOM, seed=5, state_std=0.05, a_log_hi=0.05)
    t = G.to_device(x, cuda)
    s1 = t["state"].clone()
    o1 = G.chunk_prefill(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"], s1, cu)
    s2 = t["state"].clone()
    halves = []
    for part in (0, 1):
        sl = [slice(s * 4096 + part * 2048, s * 4096 + (part + 1) * 2048) for s in (0, 1)]
        sub = {n: torch.cat([t[n][s] for s in sl]).contiguous() for n in ("q", "k", "v", "a", "b")}
        halves.append(G.chunk_prefill(sub["q"], sub["k"], sub["v"], sub["a"], sub["b"],
                                      t["A_log"], t["dt_bias"], s2, [0, 2048, 4096]))
    torch.cuda.synchronize()
    o2 = torch.cat([halves[0][:2048], halves[1][:2048], halves[0][2048:], halves[1][2048:]])
    assert torch.equal(o1, o2)
    assert torch.equal(s1, s2)


def test_decode_batch_equals_per_sequence_decode(cuda):
    import torch
    cu = np.arange(65, dtype=np.int32)
    x = G.synthetic_layer_inputs(cu, GEOM, seed=6, state_std=0.05)
    t = G.to_device(x, cuda)
    s_all = t["state"].clone()
    o_all = torch.empty_like(t["v"])
    G.decode_step(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"], s_all,
                  o_out=o_all)
    s_one = t["state"].clone()
    o_one = torch.empty_like(t["v"])
    for i in range(64):
        G.decode_step(t["q"][i:i + 1], t["k"][i:i + 1], t["v"][i:i + 1], t["a"][i:i + 1],
                      t["b"][i:i + 1], t["A_log"], t["dt_bias"], s_one[i:i + 1],
                      o_out=o_one[i:i + 1])
    torch.cuda.synchronize()
    assert torch.equal(o_all, o_one) and torch.equal(s_all, s_one)


def test_decode_steps_track_oracle(cuda):
    """Ten decode steps of 64 sequences (state in place) against the oracle."""
    import torch
    B = 64
    cu1 = np.arange(B + 1, dtype=np.int32)
    st_ref = G.synthetic_layer_inputs(cu1, GEOM, seed=8, state_std=0.05)["state"]
    state = torch.from_numpy(st_ref.copy()).to(cuda)
    st_ref = st_ref.copy()
    for step in range(10):
        x = G.synthetic_layer_inputs(cu1, GEOM, seed=100 + step)
        x["state"] = st_ref
        ref = O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"], x["dt_bias"],
                      x["gamma"], x["w_out"], st_ref, cu1, mode=0)
        t = G.to_device({k: v for k, v in x.items() if k != "state"}, cuda)
        out = G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                              t["dt_bias"], t["gamma"], t["w_out"], state, cu1)
        torch.cuda.synchronize()
        assert_out_close(G.bf16_bits(out), ref, f"decode step {step}")
    assert_state_close(state.cpu().numpy(), st_ref, "decode state after 10 steps")


def _golden_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden",
                                                  os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _golden_module()


@pytest.mark.parametrize("name", sorted(MG.CASES))
def test_cuda_path_matches_golden_vectors(cuda, name):
    import torch
    ref = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    cu, x = MG.inputs(name)
    t = G.to_device(x, cuda)
    out = G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                          t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu)
    torch.cuda.synchronize()
    assert_out_close(G.bf16_bits(out), ref["out"], f"golden {name}")
    assert_state_close(t["state"].cpu().numpy(), ref["final_state"], f"golden {name} state")
