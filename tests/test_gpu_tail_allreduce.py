"""Head-parallel output tail with the rank sum fused into the tail GEMM
(``gdn_b200_output_tail_allreduce``).

* World size 1 (one GPU): no exchange; the fused kernel's epilogue (staged
  through shared memory, row-contiguous stores) must give the same bits as
  the single-GPU tail wherever that one does not split K.
* World sizes 2, 4 and 8 (one process per GPU, exchange regions mapped by CUDA
  IPC), over several calls in a row (growing epochs): both ranks must hold
  the same bits, equal to the sum of the ranks' bf16 partial tails (each
  rank's tail over its own heads from the same GEMM main loop, added in f32
  in rank order and rounded: what the reference's engine gets from the
  rank-partial outputs, P:3541-3547, with a bf16 all-reduce); against the
  single-GPU full-width tail every element must be within the rounding a
  bf16 rank sum may add; and the output must meet the tolerance below
  against the oracle's full-width tail (small cases) and in the mean against
  the single-GPU tail.

Tolerances: max |gpu - ref| <= 2e-2 and mean|gpu - ref| / mean|ref| <= 5e-3.
A bf16 rank sum adds up to one bf16 ulp to the result (0.03 for outputs of
magnitude 4 to 8), so against the full-size single-GPU tail the maximum is
bounded element by element instead (half an ulp of each partial + one ulp of
the result).
"""
import os
import socket

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

OUT_MAX_ABS = 2e-2
OUT_MEAN_REL = 5e-3

pytestmark = pytest.mark.gpu


def _inputs(rows, hv, hidden, seed=0):
    D = G.HEAD_DIM
    return dict(o=G.fill(seed, 41, (rows, hv, D), G.NORMAL, 0.0, 1.0, G.BF16),
                z=G.fill(seed, 42, (rows, hv, D), G.NORMAL, 0.0, 1.0, G.BF16),
                gamma=G.fill(seed, 43, (D,), G.NORMAL, 1.0, 0.02, G.BF16),
                w=G.fill(seed, 44, (hidden, hv * D), G.NORMAL, 0.0, 0.02, G.BF16))


def _assert_close(gpu_bits, ref_bits, what):
    g = O.bf16_to_f32(gpu_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    d = np.abs(g - r)
    mx, mr = float(d.max()), float(d.mean() / max(np.abs(r).mean(), 1e-30))
    assert mx <= OUT_MAX_ABS and mr <= OUT_MEAN_REL, f"{what}: max_abs={mx:.3e} mean_rel={mr:.3e}"


def _bf16_ulp(bits):
    """Spacing of bf16 numbers at each value (bf16 keeps 8 of f32's 24
    significand bits)."""
    return np.spacing(np.abs(O.bf16_to_f32(bits)).astype(np.float32)).astype(np.float64) * 65536.0


def _assert_rank_sum_bound(gpu_bits, ref_bits, partials, what):
    """|gpu - ref| <= half a bf16 ulp of every rank partial (the rounding a
    bf16 rank sum may apply to each) + one ulp of the result (the final
    roundings).  Relative to the result this is loose only where the
    partials cancel."""
    g = O.bf16_to_f32(gpu_bits).astype(np.float64)
    r = O.bf16_to_f32(ref_bits).astype(np.float64)
    bound = 0.5 * sum(_bf16_ulp(p) for p in partials)
    bound = bound + np.maximum(_bf16_ulp(gpu_bits), _bf16_ulp(ref_bits))
    # f32 accumulation-order differences between kernels (K <= 4096)
    bound = bound + 2.0 ** -20 * sum(np.abs(O.bf16_to_f32(p)).astype(np.float64)
                                     for p in partials)
    bad = np.abs(g - r) > bound
    assert not bad.any(), f"{what}: {int(bad.sum())} elements beyond the rank-sum bound"


def _single_gpu_tail_splits_k(rows, hidden):
    """The single-GPU tail splits K over CTAs (another f32 summation order)
    when it has fewer than 75 output tiles."""
    return -(-rows // 128) * (hidden // 256) * 2 <= 148


@pytest.mark.parametrize("rows,hv,hidden,max_rows", [(8192, 32, 2048, 8192),
                                                     (4000, 16, 2048, 4096),
                                                     (1000, 8, 1024, 1000),
                                                     (130, 16, 2048, 4096),
                                                     (1, 4, 256, 1)])
def test_world1_matches_single_gpu_tail(cuda, rows, hv, hidden, max_rows):
    import torch
    x = _inputs(rows, hv, hidden)
    t = G.to_device(x, cuda)
    ref = G.bf16_bits(G.output_tail(t["o"], t["z"], t["gamma"], t["w"]))
    grp = G.TailGroup(max_rows, hidden, 0, 1, cuda)
    try:
        ws = torch.empty(G.output_tail_allreduce_workspace_bytes(rows, hv), dtype=torch.uint8,
                         device=cuda)
        for _ in range(2):
            out = grp.output_tail(t["o"], t["z"], t["gamma"], t["w"], workspace=ws)
            G.workspace_status(ws)
            if _single_gpu_tail_splits_k(rows, hidden):
                _assert_close(G.bf16_bits(out), ref, f"world 1 vs single-GPU rows={rows}")
            else:
                assert np.array_equal(G.bf16_bits(out), ref), "fused tail (world 1) differs"
        if rows <= 1000:
            _assert_close(G.bf16_bits(out), O.output_tail(x["o"], x["z"], x["gamma"], x["w"]),
                          f"world 1 rows={rows}")
    finally:
        torch.cuda.synchronize()
        grp.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, rows, hv_total, hidden, calls, outdir):
    """One rank: its share of the heads and of w_out's columns, the fused tail
    `calls` times, then its output bits (and, at rank 0, the single-GPU
    full-width tail) written to `outdir`."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=120))
    try:
        x = _inputs(rows, hv_total, hidden)
        hv = hv_total // world
        K = hv * G.HEAD_DIM
        mine = dict(o=np.ascontiguousarray(x["o"][:, rank * hv:(rank + 1) * hv]),
                    z=np.ascontiguousarray(x["z"][:, rank * hv:(rank + 1) * hv]),
                    gamma=x["gamma"],
                    w=np.ascontiguousarray(x["w"][:, rank * K:(rank + 1) * K]))
        t = G.to_device(mine, dev)

        def exchange(payload):
            got = [None] * world
            dist.all_gather_object(got, payload)
            return got

        grp = G.TailGroup(rows, hidden, rank, world, dev, exchange=exchange)
        ws = torch.empty(G.output_tail_allreduce_workspace_bytes(rows, hv), dtype=torch.uint8,
                         device=dev)
        stream = torch.cuda.Stream(device=dev)
        for _ in range(calls):
            out = grp.output_tail(t["o"], t["z"], t["gamma"], t["w"], workspace=ws,
                                  stream=stream)
        G.workspace_status(ws, stream)
        np.save(os.path.join(outdir, f"rank{rank}.npy"), G.bf16_bits(out))
        # This rank's bf16 partial from the same GEMM main loop (a one-rank
        # group), i.e. exactly what the exchange rounded and sent.
        solo = G.TailGroup(rows, hidden, 0, 1, dev)
        partial = solo.output_tail(t["o"], t["z"], t["gamma"], t["w"], workspace=ws,
                                   stream=stream)
        G.workspace_status(ws, stream)
        np.save(os.path.join(outdir, f"partial{rank}.npy"), G.bf16_bits(partial))
        solo.close()
        if rank == 0:
            full = G.to_device(x, dev)
            ref = G.output_tail(full["o"], full["z"], full["gamma"], full["w"])
            np.save(os.path.join(outdir, "single.npy"), G.bf16_bits(ref))
        torch.cuda.synchronize()
        dist.barrier()
        grp.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows,hv_total,hidden,calls", [(2, 1000, 32, 2048, 3),
                                                              (2, 16384, 32, 2048, 4),
                                                              (2, 200, 8, 512, 2),
                                                              (4, 1000, 32, 2048, 3),
                                                              (4, 32768, 32, 2048, 2),
                                                              (8, 1000, 32, 2048, 3),
                                                              (8, 8192, 32, 2048, 2)])
def test_ranks_agree_and_match_full_tail(cuda, tmp_path, world, rows, hv_total, hidden, calls):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_rank_main, args=(world, _free_port(), rows, hv_total, hidden, calls,
                                         str(tmp_path)),
                       nprocs=world, start_method="spawn")
    outs = [np.load(tmp_path / f"rank{r}.npy") for r in range(world)]
    r0 = outs[0]
    single = np.load(tmp_path / "single.npy")
    assert r0.shape == (rows, hidden)
    for r in range(1, world):
        assert np.array_equal(r0, outs[r]), f"rank {r} holds a different output"
    partials = [np.load(tmp_path / f"partial{r}.npy") for r in range(world)]
    acc = O.bf16_to_f32(partials[0]).astype(np.float32)
    for part in partials[1:]:
        acc = acc + O.bf16_to_f32(part)
    rank_sum = O.f32_to_bf16(acc)
    assert np.array_equal(r0, rank_sum), "fused sum differs from the bf16 rank sum"
    _assert_rank_sum_bound(r0, single, partials, f"world {world} vs single-GPU rows={rows}")
    g = O.bf16_to_f32(r0).astype(np.float64)
    ref = O.bf16_to_f32(single).astype(np.float64)
    assert np.abs(g - ref).mean() / np.abs(ref).mean() <= OUT_MEAN_REL
    if rows <= 1000:
        x = _inputs(rows, hv_total, hidden)
        _assert_close(r0, O.output_tail(x["o"], x["z"], x["gamma"], x["w"]),
                      f"world {world} vs oracle rows={rows}")
