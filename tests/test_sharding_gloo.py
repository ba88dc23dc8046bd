"""Head-parallel sharding on CPU ranks (gloo, world size 2): each rank runs
the layer on its v-head / q-k head shard with its out_proj column slice, the
rank-partial outputs are summed with an all-reduce, and the sum must match the
unsharded layer.  This is the exchange the multi-GPU path performs with NCCL
(the reference leaves the rank-partial out_proj to the engine's all-reduce,
qwen38_geometry_normalized_gdn_provider.cpp:3541-3547)."""
import os
import sys

import numpy as np
import pytest

import gdn_b200 as G
import gdn_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))


def _rank_main(rank, world, port, cu, result_path):
    import torch
    import torch.distributed as dist
    sys.path[:0] = [os.path.join(os.path.dirname(HERE), "qwen38-gdn-dual-sequence-output-tail_b200"),
                    os.path.join(os.path.dirname(HERE), "oracle")]
    import gdn_b200 as G2
    import gdn_oracle as O2
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    geom = G2.Geometry(4, 8, 256)
    x = G2.synthetic_layer_inputs(cu, geom, seed=21, state_std=0.05, shard=(rank, world))
    st = x["state"].copy()
    out = O2.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"], x["dt_bias"],
                   x["gamma"], x["w_out"], st, cu, mode=0)
    part = torch.from_numpy(O2.bf16_to_f32(out).copy())
    dist.all_reduce(part)
    if rank == 0:
        np.save(result_path, part.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_head_parallel_partials_sum_to_full_layer(tmp_path):
    import socket
    import torch.multiprocessing as mp
    cu = np.array([0, 37, 100], np.int32)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "sum.npy")
    mp.start_processes(_rank_main, args=(2, port, cu, path), nprocs=2, join=True,
                       start_method="spawn")
    summed = np.load(path)
    geom = G.Geometry(4, 8, 256)
    x = G.synthetic_layer_inputs(cu, geom, seed=21, state_std=0.05)
    st = x["state"].copy()
    full = O.bf16_to_f32(O.layer(x["q"], x["k"], x["v"], x["a"], x["b"], x["z"], x["A_log"],
                                 x["dt_bias"], x["gamma"], x["w_out"], st, cu, mode=0))
    d = np.abs(summed - full)
    # Each rank rounds its partial to bf16 before the reduction.
    assert d.max() <= 2e-2 and d.mean() / np.abs(full).mean() <= 5e-3


def test_shard_slices_are_gqa_aligned():
    cu = np.array([0, 5], np.int32)
    geom = G.Geometry(16, 32, 2048)
    full = G.synthetic_layer_inputs(cu, geom, seed=3)
    for world in (2, 4, 8):
        for rank in range(world):
            x = G.synthetic_layer_inputs(cu, geom, seed=3, shard=(rank, world))
            hk, hv = 16 // world, 32 // world
            assert x["q"].shape == (5, hk, 128) and x["v"].shape == (5, hv, 128)
            # v-head h of the shard uses q/k head h // 2 of the shard, i.e. the
            # global heads keep their group: global v = rank*hv + h, global k =
            # rank*hk + h//2 = (rank*hv + h)//2.
            assert np.array_equal(x["k"], full["k"][:, rank * hk:(rank + 1) * hk])
            assert np.array_equal(x["w_out"],
                                  full["w_out"][:, rank * hv * 128:(rank + 1) * hv * 128])
            assert np.array_equal(x["A_log"], full["A_log"][rank * hv:(rank + 1) * hv])


def test_synthetic_generator_is_deterministic_and_distributed():
    a = G.fill(9, 3, (1 << 16,), G.NORMAL, 0.0, 1.0, G.F32)
    b = G.fill(9, 3, (1 << 16,), G.NORMAL, 0.0, 1.0, G.F32)
    c = G.fill(9, 4, (1 << 16,), G.NORMAL, 0.0, 1.0, G.F32)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1.0) < 0.02
    u = G.fill(9, 5, (1 << 16,), G.UNIFORM, 0.0, 16.0, G.F32)
    assert u.min() >= 0.0 and u.max() < 16.0 and abs(u.mean() - 8.0) < 0.1
    la = G.fill(9, 6, (1 << 16,), G.LOG_UNIFORM, 0.0, 16.0, G.F32)
    assert np.all(np.exp(la) <= 16.0) and abs(np.exp(la).mean() - 8.0) < 0.1
    h = G.fill(9, 3, (1 << 16,), G.NORMAL, 0.0, 1.0, G.BF16)
    assert np.array_equal(h, O.f32_to_bf16(a))
