"""Tensor-parallel layer stack (BASELINE configs[4] at reduced depth) on two GPUs against the oracle.

Two processes (one per GPU) run two layers of the 27B linear stack, sharded as
nebula_b200.tp plans it: QKV and gate_up column-parallel (every rank computes
its slice of the output columns), O and down row-parallel (every rank computes a
partial sum over its slice of K, then an all-reduce: this library's
hq_allreduce_sum over NVLink peer loads after O, NCCL after down).  The
per-rank GEMMs are hq_gemm on tile-order shards repacked on each GPU.

Layer l's input x_l [M, 5120] feeds QKV, O and gate_up; down reads the gate half
of gate_up's gathered output; down's output is x_{l+1}.  Rank 0 checks every
GEMM's assembled output against the fp32 oracle applied to the same (bf16)
input and the unsharded weights: max relative error <= 2e-2 (bf16 output), the
tolerance of every bf16 parity test here.  Rows: M = 8 (the decode kernel) and
M = 48 (the tensor-core kernel).  Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2
LAYERS = 2
TOL = 2e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer_weights(layer, name, K, N):
    """Seeded full-size weights of one projection (identical on every rank)."""
    from oracle import oracle as o
    _, q, S = o.gen_int4_case(1, K, N, group=128, seed=9000 + 10 * layer + ["qkv", "o", "gate_up", "down"].index(name),
                              a_dtype="bf16")
    return o.pack_linear_u4(q), S


def _worker(rank, port, out_dir):
    import ctypes
    import datetime

    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm

    from nebula_b200 import _lib, hq, tp
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            device_id=dev, timeout=datetime.timedelta(seconds=120))
    try:
        L = _lib.lib()
        shapes = {n: (K, N) for n, K, N in tp.LAYER_SHAPES}
        specs = {n: tp.shard_spec(n, K, N, WORLD, rank) for n, K, N in tp.LAYER_SHAPES}
        flags = symm.empty(32, dtype=torch.int32, device=dev)
        flags.zero_()
        hf = symm.rendezvous(flags, dist.group.WORLD)
        fptrs = (ctypes.c_void_p * WORLD)(*hf.buffer_ptrs)
        epoch = 0
        shards = []
        for layer in range(LAYERS):
            per = {}
            for name, (K, N) in shapes.items():
                lin, S = _layer_weights(layer, name, K, N)
                wl, sl = tp.slice_weights(lin, S, specs[name])
                Wt = hq.repack(torch.from_numpy(wl.view(np.uint8).reshape(-1)).to(dev), _lib.HQ_WFMT_LINEAR_U4,
                               _lib.HQ_WFMT_TILE_U4, specs[name].K, specs[name].N)
                per[name] = (Wt, torch.from_numpy(sl).to(dev).bfloat16())
            shards.append(per)
        torch.cuda.synchronize()
        dist.barrier()
        record = {}
        for M in (8, 48):
            g = np.random.default_rng(77 + M)
            x = torch.from_numpy(g.standard_normal((M, 5120)).astype(np.float32)).to(dev).bfloat16()
            ws = hq.make_workspace(M, 34816, 17408, 128, _lib.HQ_WFMT_TILE_U4, dev)
            # row-parallel outputs live in symmetric memory for hq_allreduce_sum
            ybuf = symm.empty((M, 5120), dtype=torch.bfloat16, device=dev)
            hb = symm.rendezvous(ybuf, dist.group.WORLD)
            bptrs = (ctypes.c_void_p * WORLD)(*hb.buffer_ptrs)
            for layer in range(LAYERS):
                ins = {}

                def col_parallel(name, inp):
                    sp = specs[name]
                    y = hq.gemm(inp, shards[layer][name][0], shards[layer][name][1], N=sp.N, workspace=ws)
                    parts = [torch.empty_like(y) for _ in range(WORLD)]
                    dist.all_gather(parts, y)
                    all_specs = [tp.shard_spec(name, *shapes[name], WORLD, r) for r in range(WORLD)]
                    return torch.from_numpy(tp.gather_columns([p.float().cpu().numpy() for p in parts],
                                                              all_specs)).to(dev).bfloat16()

                ins["qkv"] = x
                y_qkv = col_parallel("qkv", x)
                # O: row-parallel, hq_allreduce_sum (peer loads) on the partial sums
                ins["o"] = x
                sp = specs["o"]
                hq.gemm(tp.slice_activations(x, sp), shards[layer]["o"][0], shards[layer]["o"][1], N=sp.N,
                        out=ybuf, workspace=ws)
                epoch += 1
                _lib.check(L.hq_allreduce_sum(bptrs, fptrs, None, WORLD, rank, _lib.HQ_BF16, ybuf.numel(), epoch, 32,
                                              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
                torch.cuda.synchronize()
                _lib.check(L.hq_check_device_error())
                y_o = ybuf.clone()
                ins["gate_up"] = x
                y_gu = col_parallel("gate_up", x)
                a_down = y_gu[:, :17408].contiguous()
                ins["down"] = a_down
                sp = specs["down"]
                y_down = hq.gemm(tp.slice_activations(a_down, sp), shards[layer]["down"][0],
                                 shards[layer]["down"][1], N=sp.N, workspace=ws)
                dist.all_reduce(y_down)  # NCCL
                outs = {"qkv": y_qkv, "o": y_o, "gate_up": y_gu, "down": y_down}
                for name in shapes:
                    record[f"M{M}_L{layer}_{name}_in"] = ins[name].float().cpu().numpy()
                    record[f"M{M}_L{layer}_{name}_out"] = outs[name].float().cpu().numpy()
                # next layer's input: the down output, rescaled to unit variance
                x = (y_down.float() / y_down.float().std()).bfloat16()
            dist.barrier()
            del ybuf, hb
        if rank == 0:
            np.savez(os.path.join(out_dir, "stack.npz"), **record)
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_tp_stack_matches_oracle(tmp_path):
    import torch.multiprocessing as mp

    from nebula_b200 import tp
    from oracle import oracle as o
    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    rec = np.load(tmp_path / "stack.npz")
    worst = {}
    for layer in range(LAYERS):
        for name, K, N in tp.LAYER_SHAPES:
            lin, S = _layer_weights(layer, name, K, N)
            for M in (8, 48):
                A = rec[f"M{M}_L{layer}_{name}_in"]
                ref = o.w4_gemm(A, lin, S, group=128)
                err = o.max_rel_err(rec[f"M{M}_L{layer}_{name}_out"], ref)
                worst[f"M{M} L{layer} {name}"] = err
    assert max(worst.values()) <= TOL, worst
