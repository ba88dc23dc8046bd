"""The provider's threading contract on the GPU: one handle shared by several
host threads, each submitting, waiting for and releasing its own events on its
own stream, concurrently (the reference guards its shared state with mutexes
and atomics so that concurrent Submit calls on one handle are allowed,
native/src/qwen38_geometry_normalized_gdn_provider.cpp:162-201).

Four threads run three chained submissions each (the recurrent state carries
from one to the next) on different packed batches.  Every result must equal
the same submissions run one after another on one thread bit for bit, and
must match the CPU oracle within the output and state tolerances."""
import threading

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

pytestmark = pytest.mark.gpu

GEOM = G.Geometry(16, 32, 2048)
OUT_MAX_ABS = 2e-2
OUT_MEAN_REL = 5e-3
STATE_REL = 1e-3
CASES = [[0, 64, 128], [0, 130], [0, 1, 2, 3, 4], [0, 1, 70, 200]]
ROUNDS = 3


def _oracle_rounds(x, cu):
    st = x["state"].copy()
    outs = []
    for _ in range(ROUNDS):
        outs.append(O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"],
                            x["dt_bias"], x["gamma"], x["w_out"], st, np.asarray(cu, np.int32),
                            mode=0))
    return outs, st


def _run(prov, t, state, cu, stream):
    import torch
    outs = []
    for _ in range(ROUNDS):
        out = torch.empty(cu[-1], GEOM.hidden, dtype=torch.bfloat16, device=state.device)
        ev = prov.submit_layer(t, state, out, cu, stream=stream)
        c = prov.wait(ev, timeout_s=60.0)
        assert c.phase == G.EVENT_COMPLETE
        prov.release(ev)
        outs.append(out)
    return outs


def test_one_handle_driven_from_four_threads(cuda):
    import torch
    prov = G.Provider(GEOM, max_tokens=4096)
    try:
        inputs = [G.synthetic_layer_inputs(np.asarray(cu, np.int32), GEOM, seed=50 + i,
                                           state_std=0.05) for i, cu in enumerate(CASES)]
        dev = [G.to_device(x, cuda) for x in inputs]
        streams = [torch.cuda.Stream() for _ in CASES]

        # Serial: the same submissions on this thread.
        serial_states = [t["state"].clone() for t in dev]
        serial = [_run(prov, t, st, cu, s)
                  for t, st, cu, s in zip(dev, serial_states, CASES, streams)]
        torch.cuda.synchronize()

        # Concurrent: one thread per batch, all started together.
        states = [t["state"].clone() for t in dev]
        results = [None] * len(CASES)
        errors = []
        start = threading.Barrier(len(CASES))

        def worker(i):
            try:
                torch.cuda.set_device(cuda)
                start.wait(timeout=60)
                results[i] = _run(prov, dev[i], states[i], CASES[i], streams[i])
            except Exception as e:          # reported below, on the main thread
                errors.append((i, repr(e)))

        threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(CASES))]
        for th in threads:
            th.start()
        for th in threads:
            th.join(timeout=300)
        torch.cuda.synchronize()
        assert not errors, errors
        assert all(not th.is_alive() for th in threads)

        for i, cu in enumerate(CASES):
            assert torch.equal(states[i], serial_states[i]), f"state of batch {cu}"
            ref_outs, ref_state = _oracle_rounds(inputs[i], cu)
            for r in range(ROUNDS):
                assert torch.equal(results[i][r], serial[i][r]), f"batch {cu}, round {r}"
                g = O.bf16_to_f32(G.bf16_bits(results[i][r])).astype(np.float64)
                o = O.bf16_to_f32(ref_outs[r]).astype(np.float64)
                d = np.abs(g - o)
                assert d.max() <= OUT_MAX_ABS, (cu, r, d.max())
                assert d.mean() / max(np.abs(o).mean(), 1e-30) <= OUT_MEAN_REL, (cu, r)
            st = states[i].cpu().numpy()
            rel = np.linalg.norm(st - ref_state) / np.linalg.norm(ref_state)
            assert rel <= STATE_REL, (cu, rel)
    finally:
        prov.close()
