"""Copy-engine rank sum of the head-parallel layer's rank-partial outputs
(``gdn_b200_rank_sum``: a reduce-scatter whose rows move as peer copies).

World sizes 1, 2, 4 and 8 (one process per GPU, regions mapped by CUDA IPC),
several epochs in a row with different data per epoch, so that both partial
buffers and both staging sets are reused: every rank's shard must equal, bit
for bit, the f32 sum in rank order of all ranks' bf16 partial rows, rounded
once to bf16 (what the reference's engine computes from the rank-partial
outputs, P:3541-3547).  A second part checks the layer path itself: the
layer's rank-partial written straight into the exchange buffer and summed
across ranks must match the single-GPU layer within the output tolerance.
"""
import os
import socket

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial(rank, epoch, rows, hidden):
    return G.fill(100 + epoch, 7 + rank, (rows, hidden), G.NORMAL, 0.0, 1.0, G.BF16)


def _rank_main(rank, world, port, rows, hidden, epochs, outdir):
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=120))
    try:
        def exchange(payload):
            got = [None] * world
            dist.all_gather_object(got, payload)
            return got

        rs = G.RankSum(rows, hidden, rank, world, dev, exchange=exchange)
        stream = torch.cuda.Stream(device=dev)
        comm = torch.cuda.Stream(device=dev)
        shards = [torch.empty(rows // world, hidden, dtype=torch.bfloat16, device=dev)
                  for _ in range(epochs)]
        for e in range(1, epochs + 1):
            rs.acquire(e, stream)
            src = G.to_device({"p": _partial(rank, e, rows, hidden)}, dev)["p"]
            with torch.cuda.stream(stream):
                rs.part(e, rows).copy_(src)
            rs.reduce(e, rows, shards[e - 1], stream, comm)
        torch.cuda.synchronize()
        rs.status(comm)
        rs.status(stream)
        for e in range(epochs):
            np.save(os.path.join(outdir, f"rank{rank}_e{e + 1}.npy"), G.bf16_bits(shards[e]))
        dist.barrier()
        rs.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,rows,hidden,epochs", [(1, 64, 2048, 3), (2, 1000, 2048, 5),
                                                      (2, 16384, 2048, 3), (4, 4096, 512, 4),
                                                      (8, 8192, 2048, 3)])
def test_rank_sum_is_the_rank_order_f32_sum(cuda, tmp_path, world, rows, hidden, epochs):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_rank_main, args=(world, _free_port(), rows, hidden, epochs,
                                         str(tmp_path)),
                       nprocs=world, start_method="spawn")
    sr = rows // world
    for e in range(1, epochs + 1):
        parts = [O.bf16_to_f32(_partial(r, e, rows, hidden)) for r in range(world)]
        acc = parts[0].copy()
        for p in parts[1:]:
            acc = acc + p
        want = O.f32_to_bf16(acc)
        for r in range(world):
            got = np.load(tmp_path / f"rank{r}_e{e}.npy")
            assert np.array_equal(got, want[r * sr:(r + 1) * sr]), f"rank {r} epoch {e}"


def _layer_rank_main(rank, world, port, outdir):
    """The layer's rank-partial written into the exchange buffer and summed:
    2 sequences of 300 tokens, this rank's share of the heads."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=120))
    try:
        cu = np.array([0, 300, 600], np.int32)
        full = G.Geometry(16, 32, 2048)
        x = G.synthetic_layer_inputs(cu, full, seed=9, state_std=0.05, shard=(rank, world))
        geom = G.Geometry(16 // world, 32 // world, 2048)
        t = G.to_device(x, dev)

        def exchange(payload):
            got = [None] * world
            dist.all_gather_object(got, payload)
            return got

        rows = int(cu[-1])
        rs = G.RankSum(rows, 2048, rank, world, dev, exchange=exchange)
        stream = torch.cuda.Stream(device=dev)
        comm = torch.cuda.Stream(device=dev)
        shard = torch.empty(rows // world, 2048, dtype=torch.bfloat16, device=dev)
        rs.acquire(1, stream)
        G.layer_forward(t["q"], t["k"], t["v"], t["a"], t["b"], t["z"], t["A_log"],
                        t["dt_bias"], t["gamma"], t["w_out"], t["state"], cu,
                        out=rs.part(1, rows), stream=stream)
        rs.reduce(1, rows, shard, stream, comm)
        torch.cuda.synchronize()
        rs.status(comm)
        np.save(os.path.join(outdir, f"shard{rank}.npy"), G.bf16_bits(shard))
        dist.barrier()
        rs.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_layer_rank_sum_matches_oracle(cuda, tmp_path, world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_layer_rank_main, args=(world, _free_port(), str(tmp_path)),
                       nprocs=world, start_method="spawn")
    got = np.concatenate([np.load(tmp_path / f"shard{r}.npy") for r in range(world)])
    cu = np.array([0, 300, 600], np.int32)
    x = G.synthetic_layer_inputs(cu, G.Geometry(16, 32, 2048), seed=9, state_std=0.05)
    st = x["state"].copy()
    ref = O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"], x["dt_bias"],
                  x["gamma"], x["w_out"], st, cu, mode=0)
    g = O.bf16_to_f32(got).astype(np.float64)
    r = O.bf16_to_f32(ref).astype(np.float64)
    d = np.abs(g - r)
    assert d.max() <= 2e-2 and d.mean() / np.abs(r).mean() <= 5e-3, (d.max(), d.mean())
