"""Generates the golden vectors in this directory (run from the repo root):

    python tests/golden/make_golden.py

Each case is a small post-projection GDN layer (reduced head counts so the
files stay small) on seeded inputs with the benchmark distributions.  The
outputs come from the CPU oracle (oracle/gdn_oracle.c, recurrent mode in
double precision) and are cross-checked here, before being written, against
the independent PyTorch restatement of the gated delta rule in transformers
(models/qwen3_next/modeling_qwen3_next.py: torch_recurrent_gated_delta_rule and
torch_chunk_gated_delta_rule), so a fixture is only written when two
independent implementations agree.  The reference repository itself ships no
golden vectors and its arithmetic runs in closed Ascend operators.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "qwen38-gdn-dual-sequence-output-tail_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import gdn_b200 as G  # noqa: E402
import gdn_oracle as O  # noqa: E402

# name: (cu_seqlens, qk_heads, value_heads, hidden, a_log_hi, state_std, seed)
# Inputs are not stored: they are regenerated from these parameters by the
# seeded generator (gdn_b200.synthetic_layer_inputs); the files hold outputs.
CASES = {
    "t1": ([0, 1], 1, 2, 128, 16.0, 0.05, 11),
    "t9": ([0, 9], 1, 2, 128, 16.0, 0.05, 12),
    "t64": ([0, 64], 1, 2, 128, 16.0, 0.0, 13),
    "t65": ([0, 65], 1, 2, 128, 1.0, 0.05, 14),
    "t130_weak_decay": ([0, 130], 1, 2, 128, 0.05, 0.05, 15),
    "dual_2x64": ([0, 64, 128], 1, 2, 128, 16.0, 0.0, 16),
    "varlen_4": ([0, 1, 10, 74, 139], 1, 2, 128, 16.0, 0.05, 17),
    "decode_b4": ([0, 1, 2, 3, 4], 1, 2, 128, 16.0, 0.05, 18),
}


def inputs(name):
    cu, hk, hv, hidden, a_hi, s_std, seed = CASES[name]
    cu = np.asarray(cu, np.int32)
    x = G.synthetic_layer_inputs(cu, G.Geometry(hk, hv, hidden), seed=seed, state_std=s_std,
                                 a_log_hi=a_hi)
    return cu, x


def torch_reference(x, cu, hk, hv):
    """Core output and final state from the transformers restatement."""
    import torch
    from transformers.models.qwen3_next.modeling_qwen3_next import (
        torch_chunk_gated_delta_rule, torch_recurrent_gated_delta_rule)
    g, beta = O.gating(x["a"], x["b"], x["A_log"], x["dt_bias"])
    qn = O.bf16_to_f32(O.l2norm(x["q"])).astype(np.float64)
    kn = O.bf16_to_f32(O.l2norm(x["k"])).astype(np.float64)
    v = O.bf16_to_f32(x["v"]).astype(np.float64)
    b = O.bf16_to_f32(beta).astype(np.float64)
    rep = hv // hk
    outs, states_r, states_c = [], [], []
    for s in range(len(cu) - 1):
        sl = slice(cu[s], cu[s + 1])
        q_t = torch.from_numpy(np.repeat(qn[sl], rep, axis=1))[None]
        k_t = torch.from_numpy(np.repeat(kn[sl], rep, axis=1))[None]
        v_t = torch.from_numpy(v[sl])[None]
        g_t = torch.from_numpy(g[sl].astype(np.float64))[None]
        b_t = torch.from_numpy(b[sl])[None]
        # transformers keeps the state as [key, value]; ours is [value, key].
        s0 = torch.from_numpy(x["state"][s].astype(np.float64).transpose(0, 2, 1).copy())[None]
        o_r, st_r = torch_recurrent_gated_delta_rule(q_t, k_t, v_t, g_t, b_t, s0, True)
        o_c, st_c = torch_chunk_gated_delta_rule(q_t, k_t, v_t, g_t, b_t, 64, s0, True)
        outs.append(o_r[0].numpy())
        states_r.append(st_r[0].numpy().transpose(0, 2, 1))
        states_c.append(st_c[0].numpy().transpose(0, 2, 1))
    return np.concatenate(outs), np.stack(states_r), np.stack(states_c)


def make(name):
    _, hk, hv, hidden, _, _, _ = CASES[name]
    cu, x = inputs(name)
    st = x["state"].copy()
    out, o, gated = O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"],
                            x["dt_bias"], x["gamma"], x["w_out"], st, cu, mode=0,
                            want_o=True, want_gated=True)
    o_ref, st_r, st_c = torch_reference(x, cu, hk, hv)
    f = O.bf16_to_f32(o).astype(np.float64)
    scale = np.abs(o_ref).max() + 1e-30
    assert np.abs(f - o_ref).max() <= 2 ** -7 * scale, f"{name}: core output disagrees"
    den = np.linalg.norm(st_r) + 1e-30
    assert np.linalg.norm(st - st_r) / den < 1e-6, f"{name}: state disagrees (recurrent)"
    # torch_chunk_gated_delta_rule rounds its decay mask to float32, which
    # limits its agreement to about 1e-6.
    assert np.linalg.norm(st - st_c) / den < 1e-4, f"{name}: state disagrees (chunked)"
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), cu=cu,
                        geometry=np.array([hk, hv, hidden], np.int32),
                        out=out, o=o, gated=gated, final_state=st)
    print(f"{name}: ok ({int(cu[-1])} tokens)")


if __name__ == "__main__":
    for n in CASES:
        make(n)
