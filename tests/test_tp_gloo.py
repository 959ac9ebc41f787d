"""Tensor-parallel sharding (nebula_b200.tp) checked on CPU with two gloo ranks.

Each rank builds the same full layer weights from a seed, takes its shard with
tp.shard_spec / tp.slice_weights, and computes its local product with the CPU
oracle.  Column-parallel layers (QKV, gate_up with its two halves) are gathered
and must equal the full product's columns; row-parallel layers (O, down) are
summed with an all-reduce and must equal the full product (fp32, up to the
order of the k summation: relative 1e-5).  This covers the host-side index
logic that the NCCL path on the GPUs uses with the same functions.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nebula_b200 import tp

# Small stand-ins for the 27B layer shapes with the same divisibility rules.
LAYERS = [("qkv", 256, 128), ("o", 256, 128), ("gate_up", 256, 256), ("down", 512, 128)]
GROUP = 128
M = 5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    from oracle import oracle as o
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        errs = {}
        for i, (name, K, N) in enumerate(LAYERS):
            A, q, S = o.gen_int4_case(M, K, N, group=GROUP, seed=40 + i)
            lin = o.pack_linear_u4(q)
            full = o.w4_gemm(A, lin, S, group=GROUP)
            spec = tp.shard_spec(name, K, N, world, rank, group=GROUP)
            lw, ls = tp.slice_weights(lin, S, spec, wbits=4, group=GROUP)
            xa = tp.slice_activations(A, spec)
            assert lw.shape == (spec.K // 8, spec.N) and ls.shape == (spec.K // GROUP, spec.N)
            y = o.w4_gemm(np.ascontiguousarray(xa), lw, ls, group=GROUP)
            t = torch.from_numpy(np.ascontiguousarray(y))
            if spec.row_parallel:
                dist.all_reduce(t)
                got = t.numpy()
            else:
                parts = [torch.empty_like(t) for _ in range(world)]
                dist.all_gather(parts, t)
                specs = [tp.shard_spec(name, K, N, world, r, group=GROUP) for r in range(world)]
                got = tp.gather_columns([p.numpy() for p in parts], specs)
            errs[name] = float(np.max(np.abs(got - full)) / max(np.max(np.abs(full)), 1e-30))
        np.save(os.path.join(out_dir, f"errs_{rank}.npy"), np.array([errs[n] for n, _, _ in LAYERS]))
    finally:
        dist.destroy_process_group()


def test_tp_shards_reproduce_the_full_layer_two_ranks(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        errs = np.load(tmp_path / f"errs_{r}.npy")
        assert (errs <= 1e-5).all(), dict(zip([n for n, _, _ in LAYERS], errs))


def test_shard_spec_shapes_for_the_27b_layer():
    for world in (1, 2, 4, 8):
        for name, K, N in tp.LAYER_SHAPES:
            specs = [tp.shard_spec(name, K, N, world, r) for r in range(world)]
            if name in tp.ROW_PARALLEL:
                assert sum(s.K for s in specs) == K and all(s.N == N for s in specs)
                assert all(s.K % 128 == 0 for s in specs)
            else:
                assert sum(s.N for s in specs) == N and all(s.K == K for s in specs)
                assert all(s.N % 16 == 0 for s in specs)
                cols = sorted(c for s in specs for a, b in s.col_ranges for c in (a, b))
                assert cols[0] == 0 and cols[-1] == N
    gate_up = tp.shard_spec("gate_up", 5120, 34816, 8, 3)
    assert gate_up.col_ranges == ((3 * 2176, 4 * 2176), (17408 + 3 * 2176, 17408 + 4 * 2176))


def test_shard_spec_rejects_shapes_that_do_not_divide():
    with pytest.raises(ValueError):
        tp.shard_spec("down", 17408, 5120, 3, 0)  # 17408 / 3 is not whole 128-groups
    with pytest.raises(ValueError):
        tp.shard_spec("qkv", 5120, 7168, 128, 0)  # 7168 / 128 = 56 columns is not whole 16-strips
    with pytest.raises(ValueError):
        tp.shard_spec("qkv", 5120, 7168, 2, 2)
