"""CPU tests of the oracle: golden vectors, agreement with the independent
PyTorch restatement in transformers, internal consistency of its modes and
the reference's constants."""
import glob
import os

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _golden_cases():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden",
                                                  os.path.join(GOLDEN, "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _golden_cases()


@pytest.mark.parametrize("name", sorted(MG.CASES))
def test_oracle_reproduces_golden_vectors(name):
    ref = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    cu, x = MG.inputs(name)
    assert np.array_equal(cu, ref["cu"])
    st = x["state"].copy()
    out, o, gated = O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"],
                            x["dt_bias"], x["gamma"], x["w_out"], st, cu, mode=0,
                            want_o=True, want_gated=True)
    assert np.array_equal(out, ref["out"])
    assert np.array_equal(o, ref["o"])
    assert np.array_equal(gated, ref["gated"])
    assert np.array_equal(st, ref["final_state"])


def test_every_golden_file_has_a_case():
    files = {os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "*.npz"))}
    assert files == set(MG.CASES)


@pytest.mark.parametrize("name", ["t65", "t130_weak_decay", "varlen_4"])
def test_oracle_agrees_with_transformers_restatement(name):
    cu, x = MG.inputs(name)
    hk, hv = MG.CASES[name][1], MG.CASES[name][2]
    g, beta = O.gating(x["a"], x["b"], x["A_log"], x["dt_bias"])
    st = x["state"].copy()
    o = O.core(O.l2norm(x["q"]), O.l2norm(x["k"]), x["v"], g, beta, st, cu, mode=0)
    o_ref, st_r, _ = MG.torch_reference(x, cu, hk, hv)
    f = O.bf16_to_f32(o).astype(np.float64)
    assert np.abs(f - o_ref).max() <= 2 ** -7 * np.abs(o_ref).max()
    assert np.linalg.norm(st - st_r) / np.linalg.norm(st_r) < 1e-6


@pytest.mark.parametrize("a_log_hi", [16.0, 0.05])
def test_chunked_form_equals_recurrent_form(a_log_hi):
    cu = np.array([0, 1, 70, 200], np.int32)
    x = G.synthetic_layer_inputs(cu, G.Geometry(2, 4, 128), seed=5, state_std=0.05,
                                 a_log_hi=a_log_hi)
    g, beta = O.gating(x["a"], x["b"], x["A_log"], x["dt_bias"])
    qn, kn = O.l2norm(x["q"]), O.l2norm(x["k"])
    s0 = x["state"].copy()
    s1 = x["state"].copy()
    s2 = x["state"].copy()
    o0 = O.core(qn, kn, x["v"], g, beta, s0, cu, mode=0)
    o1 = O.core(qn, kn, x["v"], g, beta, s1, cu, mode=1)
    o2 = O.core(qn, kn, x["v"], g, beta, s2, cu, mode=2)
    f0, f1, f2 = (O.bf16_to_f32(v).astype(np.float64) for v in (o0, o1, o2))
    assert np.abs(f0 - f1).max() <= 2 ** -7 * np.abs(f0).max()
    assert np.linalg.norm(s0 - s1) / np.linalg.norm(s0) < 1e-6
    # The reference chain's bf16 rounding points (T, W, U, h, v_new) cost
    # accuracy: this is why the B200 kernels keep those operands as hi/lo
    # pairs.  The outputs stay inside the output tolerance.
    assert np.abs(f0 - f2).mean() / np.abs(f0).mean() < 5e-3
    assert np.linalg.norm(s0 - s2) / np.linalg.norm(s0) < 2e-2


def test_gating_formula():
    a = G.fill(3, 1, (50, 4), G.NORMAL, 0.0, 3.0, G.BF16)
    b = G.fill(3, 2, (50, 4), G.NORMAL, 0.0, 3.0, G.BF16)
    A_log = np.log(np.array([0.5, 1.0, 8.0, 15.9], np.float32))
    dt = np.array([0.1, -0.2, 25.0, 0.0], np.float32)
    g, beta = O.gating(a, b, A_log, dt)
    x = O.bf16_to_f32(a).astype(np.float64) + dt
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    g_ref = -np.exp(A_log.astype(np.float64)) * sp
    assert np.allclose(g, g_ref, rtol=1e-6, atol=0)
    b_ref = 1.0 / (1.0 + np.exp(-O.bf16_to_f32(b).astype(np.float64)))
    assert np.array_equal(beta, O.f32_to_bf16(b_ref.astype(np.float32)))


def test_l2norm_matches_reference_rmsnorm_constants():
    # gamma = bf16(1/sqrt(128)) rounded to nearest even, eps = 1e-6 / 128
    gamma = O.bf16_to_f32(O.f32_to_bf16(np.array([1.0 / np.sqrt(128.0)], np.float32)))[0]
    assert gamma == np.float32(0.08837890625)
    x = G.fill(4, 1, (10, 128), G.NORMAL, 0.0, 1.0, G.BF16)
    y = O.l2norm(x)
    xf = O.bf16_to_f32(x).astype(np.float64)
    ref = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-6 / 128) * gamma
    assert np.array_equal(y, O.f32_to_bf16(ref.astype(np.float32)))


def test_tail_prologue_rounding_modes():
    o = G.fill(5, 1, (16, 4, 128), G.NORMAL, 0.0, 1.0, G.BF16)
    z = G.fill(5, 2, (16, 4, 128), G.NORMAL, 0.0, 1.0, G.BF16)
    gamma = G.fill(5, 3, (128,), G.NORMAL, 1.0, 0.02, G.BF16)
    ref_round = O.tail_prologue(o, z, gamma, mode=0)
    fused = O.tail_prologue(o, z, gamma, mode=1)
    of = O.bf16_to_f32(o).astype(np.float64).reshape(16, 4, 128)
    zf = O.bf16_to_f32(z).astype(np.float64).reshape(16, 4, 128)
    gf = O.bf16_to_f32(gamma).astype(np.float64)
    n = of / np.sqrt((of * of).mean(-1, keepdims=True) + 1e-6) * gf
    s = zf / (1.0 + np.exp(-zf))
    exact = (n * s).reshape(16, -1)
    for v in (ref_round, fused):
        assert np.abs(O.bf16_to_f32(v) - exact).max() <= 2 ** -6 * np.abs(exact).max()
    # mode 0 rounds n and s to bf16 before the product, like the reference's
    # RmsNorm -> Silu -> Mul operator chain.
    nb = O.bf16_to_f32(O.f32_to_bf16(n.astype(np.float32))).astype(np.float64)
    sb = O.bf16_to_f32(O.f32_to_bf16(s.astype(np.float32))).astype(np.float64)
    chain = O.f32_to_bf16((nb * sb).reshape(16, -1).astype(np.float32))
    assert np.mean(chain != ref_round) < 1e-3


def test_gemm_matches_float64():
    a = G.fill(6, 1, (9, 256), G.NORMAL, 0.0, 1.0, G.BF16)
    w = G.fill(6, 2, (128, 256), G.NORMAL, 0.0, 0.02, G.BF16)
    out = O.gemm_bf16(a, w)
    ref = O.bf16_to_f32(a).astype(np.float64) @ O.bf16_to_f32(w).astype(np.float64).T
    assert np.array_equal(out, O.f32_to_bf16(ref.astype(np.float32)))


def test_bf16_rounding_matches_torch():
    import torch
    x = np.concatenate([G.fill(7, 1, (4096,), G.NORMAL, 0.0, 100.0, G.F32),
                        np.array([0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 65504.0,
                                  3.0e38, 1e-40], np.float32)])
    ours = O.f32_to_bf16(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


# ------------------------------------------------------------ input side --

def test_causal_conv_matches_transformers_update():
    """The conv oracle against transformers 5.5.0's torch_causal_conv1d_update
    (models/qwen3_next/modeling_qwen3_next.py: state rows concatenated before
    the tokens, depthwise conv of width 4, SiLU, state <- the last rows), per
    sequence, with and without a carried state, for sequences shorter and
    longer than the three-row history."""
    import torch
    from transformers.models.qwen3_next.modeling_qwen3_next import torch_causal_conv1d_update
    rng = np.random.default_rng(5)
    C = 96
    cu = np.array([0, 1, 3, 40, 41], np.int32)
    x = O.f32_to_bf16(rng.normal(0, 1, (int(cu[-1]), C)).astype(np.float32))
    w = O.f32_to_bf16(rng.normal(0, 0.5, (4, C)).astype(np.float32))
    st0 = O.f32_to_bf16(rng.normal(0, 1, (4, 3, C)).astype(np.float32))
    wt = torch.from_numpy(O.bf16_to_f32(w).T.copy())
    for use_state in (True, False):
        st = st0.copy()
        out = O.causal_conv1d(x, w, st, cu, use_state)
        same = total = 0
        for s in range(len(cu) - 1):
            hs = torch.from_numpy(O.bf16_to_f32(x[cu[s]:cu[s + 1]]).T.copy())[None]
            cs = (torch.from_numpy(O.bf16_to_f32(st0[s]).T.copy())[None] if use_state
                  else torch.zeros(1, C, 3))
            ref = O.f32_to_bf16(torch_causal_conv1d_update(hs, cs, wt)[0].T.contiguous().numpy())
            got = out[cu[s]:cu[s + 1]]
            g, r = O.bf16_to_f32(got), O.bf16_to_f32(ref)
            ulp = np.spacing(np.abs(r).astype(np.float32)) * 65536.0
            assert (np.abs(g - r) <= ulp).all(), f"sequence {s}: beyond one bf16 ulp"
            same += int((got == ref).sum())
            total += got.size
            assert np.array_equal(st[s], O.f32_to_bf16(cs[0].T.contiguous().numpy())), \
                f"sequence {s}: conv state differs"
        assert same / total > 0.97


def test_causal_conv_continuation_is_exact():
    """Splitting a sequence and carrying the conv state gives the same bits."""
    rng = np.random.default_rng(6)
    C = 64
    x = O.f32_to_bf16(rng.normal(0, 1, (50, C)).astype(np.float32))
    w = O.f32_to_bf16(rng.normal(0, 0.5, (4, C)).astype(np.float32))
    st = O.f32_to_bf16(rng.normal(0, 1, (1, 3, C)).astype(np.float32))
    st_a = st.copy()
    whole = O.causal_conv1d(x, w, st_a, np.array([0, 50], np.int32))
    st_b = st.copy()
    parts = [O.causal_conv1d(x[i:j], w, st_b, np.array([0, j - i], np.int32))
             for i, j in ((0, 2), (2, 3), (3, 29), (29, 50))]
    assert np.array_equal(whole, np.concatenate(parts))
    assert np.array_equal(st_a, st_b)


@pytest.mark.parametrize("dist,p0,p1", [(G.NORMAL, 0.0, 1.0), (G.NORMAL, 1.0, 0.02),
                                        (G.NORMAL, 0.0, 0.05), (G.UNIFORM, -2.0, 3.0),
                                        (G.LOG_UNIFORM, 0.0, 16.0)])
@pytest.mark.parametrize("dtype", [G.BF16, G.F32])
def test_oracle_generator_matches_product_generator(dist, p0, p1, dtype):
    # The CPU baseline builds its inputs with the oracle's generator so that
    # it never loads the product library; both must give the same bits.
    a = G.fill(3, 11, (65537,), dist, p0, p1, dtype)
    b = O.fill(3, 11, (65537,), dist, p0, p1, dtype)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_benchmark_inputs_from_the_oracle_generator_are_identical():
    cu = np.array([0, 70, 200], np.int32)
    geom = G.Geometry(4, 8, 256)
    a = G.synthetic_layer_inputs(cu, geom, seed=1, state_std=0.05)
    b = G.synthetic_layer_inputs(cu, geom, seed=1, state_std=0.05, fill=O.fill)
    assert a.keys() == b.keys()
    for name in a:
        assert np.array_equal(a[name].view(np.uint8), b[name].view(np.uint8)), name
