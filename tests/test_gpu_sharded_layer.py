"""Head-parallel layer on 2, 4 and 8 GPUs: a ragged packed prefill with
nonzero initial states, then a 256-sequence decode step, the 32 v-heads and
16 q/k heads split evenly over the ranks (one process per GPU), each rank
holding its own state shard and out_proj column slice.  The rank-partial
outputs are summed by the fused tail kernel
(``gdn_b200_output_tail_allreduce``).

Checks, for the prefill and for the decode step:
* every rank's state shard equals the same heads of a single-GPU run over all
  heads, bit for bit (heads never interact inside the core);
* the core run alone and the unfused layer over a rank's heads (whose output
  is the rank-partial that the reference hands to its engine, P:3541-3547)
  leave the same state;
* every rank holds the same output, equal bit for bit to the f32 rank-order
  sum of the ranks' bf16 partial tails (same prologue and GEMM main loop);
* that output meets the output tolerance in the mean against the
  single-GPU layer over all heads and stays within the rounding a bf16 rank
  sum may add, element by element.
Tolerance: mean|gpu - ref| / mean|ref| <= 5e-3.
"""
import os
import socket

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

OUT_MEAN_REL = 5e-3
PREFILL_LENS = (3000, 4096, 1000, 5000)
DECODE_BATCH = 256

pytestmark = pytest.mark.gpu


def _bf16_ulp(bits):
    return np.spacing(np.abs(O.bf16_to_f32(bits)).astype(np.float32)).astype(np.float64) * 65536.0


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, outdir):
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=300))
    try:
        geom = G.Geometry(16, 32, 2048)

        def exchange(payload):
            got = [None] * world
            dist.all_gather_object(got, payload)
            return got

        cu_p = np.concatenate([[0], np.cumsum(PREFILL_LENS)]).astype(np.int32)
        cu_d = np.arange(DECODE_BATCH + 1, dtype=np.int32)
        grp = G.TailGroup(int(cu_p[-1]), geom.hidden, rank, world, dev, exchange=exchange)
        solo = G.TailGroup(int(cu_p[-1]), geom.hidden, 0, 1, dev)
        stream = torch.cuda.Stream(device=dev)
        for tag, cu, seed in (("prefill", cu_p, 31), ("decode", cu_d, 32)):
            x = G.synthetic_layer_inputs(cu, geom, seed=seed, state_std=0.05,
                                         shard=(rank, world))
            t = G.to_device(x, dev)
            # the unfused layer over this rank's heads (its rank-partial output)
            st_part = t["state"].clone()
            G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                            t["dt_bias"], t["gamma"], t["w_out"], st_part, cu, stream=stream)
            # core, then the fused tail with the rank sum
            st = t["state"].clone()
            o = torch.empty_like(t["v"])
            if tag == "decode":
                G.decode_step(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"], t["dt_bias"],
                              st, o_out=o, stream=stream)
            else:
                G.chunk_prefill(t["q"], t["k"], t["v"], t["a"], t["b"], t["A_log"],
                                t["dt_bias"], st, cu, o_out=o, stream=stream)
            out = grp.output_tail(o, t["z"], t["gamma"], t["w_out"], stream=stream)
            # this rank's bf16 partial from the same prologue and GEMM main loop
            part = solo.output_tail(o, t["z"], t["gamma"], t["w_out"], stream=stream)
            stream.synchronize()
            assert torch.equal(st, st_part), f"{tag}: state differs between the two paths"
            np.save(os.path.join(outdir, f"{tag}_out{rank}.npy"), G.bf16_bits(out))
            np.save(os.path.join(outdir, f"{tag}_part{rank}.npy"), G.bf16_bits(part))
            np.save(os.path.join(outdir, f"{tag}_state{rank}.npy"), st.cpu().numpy())
            if rank == 0:
                xf = G.synthetic_layer_inputs(cu, geom, seed=seed, state_std=0.05)
                tf = G.to_device(xf, dev)
                full = G.layer_forward(tf["q"], tf["k"], tf["v"], tf["a"], tf["b"], tf["z"],
                                       tf["A_log"], tf["dt_bias"], tf["gamma"], tf["w_out"],
                                       tf["state"], cu, stream=stream)
                stream.synchronize()
                np.save(os.path.join(outdir, f"{tag}_full_out.npy"), G.bf16_bits(full))
                np.save(os.path.join(outdir, f"{tag}_full_state.npy"), tf["state"].cpu().numpy())
                del tf
            del t
        torch.cuda.synchronize()
        dist.barrier()
        grp.close()
        solo.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_parallel_layer_matches_single_gpu(cuda, tmp_path, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    hv_r = 32 // world
    for tag in ("prefill", "decode"):
        full_state = np.load(tmp_path / f"{tag}_full_state.npy")
        for r in range(world):
            st = np.load(tmp_path / f"{tag}_state{r}.npy")
            assert np.array_equal(st, full_state[:, r * hv_r:(r + 1) * hv_r]), \
                f"{tag}: rank {r} state shard differs from the single-GPU heads"
        outs = [np.load(tmp_path / f"{tag}_out{r}.npy") for r in range(world)]
        for r in range(1, world):
            assert np.array_equal(outs[0], outs[r]), f"{tag}: rank {r} output differs"
        parts = [np.load(tmp_path / f"{tag}_part{r}.npy") for r in range(world)]
        acc = O.bf16_to_f32(parts[0]).astype(np.float32)
        for p in parts[1:]:
            acc = acc + O.bf16_to_f32(p)
        assert np.array_equal(outs[0], O.f32_to_bf16(acc)), f"{tag}: output != bf16 rank sum"
        full = np.load(tmp_path / f"{tag}_full_out.npy")
        g = O.bf16_to_f32(outs[0]).astype(np.float64)
        ref = O.bf16_to_f32(full).astype(np.float64)
        assert np.abs(g - ref).mean() / np.abs(ref).mean() <= OUT_MEAN_REL, tag
        bound = 0.5 * sum(_bf16_ulp(p) for p in parts)
        bound = bound + np.maximum(_bf16_ulp(outs[0]), _bf16_ulp(full))
        bound = bound + 2.0 ** -20 * sum(np.abs(O.bf16_to_f32(p)).astype(np.float64)
                                         for p in parts)
        bad = np.abs(g - ref) > bound
        assert not bad.any(), f"{tag}: {int(bad.sum())} elements beyond the rank-sum bound"
