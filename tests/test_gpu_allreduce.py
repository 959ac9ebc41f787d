"""hq_allreduce_sum (peer-memory all-reduce over NVLink) on two GPUs.

Two processes (one per GPU, NCCL process group for the rendezvous) hold seeded
random bf16 / fp16 partials in PyTorch symmetric-memory buffers; the kernel
sums them in place.  Reference: the partials gathered with NCCL, summed in fp32
in rank order and rounded once, which is exactly what the kernel computes, so
the results are compared bit for bit, on every rank, over several calls in a row
(each call a new epoch on the same flags), alternating the NVLS multicast path
(when the GPUs support it) and the peer-load path, then with epoch 0 inside a
CUDA graph replayed five times.  Skipped when fewer than two
GPUs are visible.  Peer-load path: bit for bit against the gathered fp32 sum.  NVLS
path: the switch rounds its fp32 sum its own way (it differs from round-to-
nearest in about a fifth of the elements), so within one ulp of the reference
and identical on every rank.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, out_dir):
    import datetime

    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm

    from nebula_b200 import _lib
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        L = _lib.lib()
        flags = symm.empty(32, dtype=torch.int32, device=dev)
        flags.zero_()
        hf = symm.rendezvous(flags, dist.group.WORLD)
        fptrs = (ctypes.c_void_p * WORLD)(*hf.buffer_ptrs)
        torch.cuda.synchronize()
        dist.barrier()
        errs, epoch = [], 0
        for dt, hdt in ((torch.bfloat16, _lib.HQ_BF16), (torch.float16, _lib.HQ_F16)):
            for n in (8, 4096, 5 * 2304 * 64 + 8, 2304 * 5120):
                buf = symm.empty(n, dtype=dt, device=dev)
                hb = symm.rendezvous(buf, dist.group.WORLD)
                bptrs = (ctypes.c_void_p * WORLD)(*hb.buffer_ptrs)
                mc = int(hb.multicast_ptr or 0)
                for call in range(4):
                    use_mc = bool(mc) and call % 2 == 1  # alternate the NVLS and peer-load paths
                    g = torch.Generator(device=dev)
                    g.manual_seed(1000 * rank + 17 * call + n)
                    x = torch.randn(n, device=dev, generator=g).to(dt)
                    buf.copy_(x)
                    parts = [torch.empty_like(x) for _ in range(WORLD)]
                    dist.all_gather(parts, x)
                    ref = torch.zeros(n, device=dev, dtype=torch.float32)
                    for p_ in parts:
                        ref += p_.float()
                    ref = ref.to(dt)
                    epoch += 1
                    st = L.hq_allreduce_sum(bptrs, fptrs, ctypes.c_void_p(mc if use_mc else 0), WORLD, rank, hdt, n,
                                            epoch, 64,
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
                    assert st == 0, L.hq_last_error_string()
                    torch.cuda.synchronize()
                    assert L.hq_check_device_error() == 0
                    if not use_mc:
                        errs.append(int((buf.view(torch.int16) != ref.view(torch.int16)).sum().item()))
                    else:
                        # The switch's own rounding of the fp32 sum: within one ulp of the
                        # reference, and the same bits on every rank.
                        ulp = (2.0 ** -7) if dt == torch.bfloat16 else (2.0 ** -10)
                        d = (buf.float() - ref.float()).abs()
                        bound = ulp * ref.float().abs() + 1e-30
                        errs.append(int((d > bound).sum().item()))
                        others = [torch.empty_like(buf) for _ in range(WORLD)]
                        dist.all_gather(others, buf)
                        errs.append(int(sum((o.view(torch.int16) != buf.view(torch.int16)).sum().item()
                                            for o in others)))
                dist.barrier()
                del buf, hb
        # epoch 0 (the kernel reads the call count from the flag area), captured in a CUDA
        # graph with the copy of the partial and replayed: bit for bit on every replay.
        n = 2304 * 64
        buf = symm.empty(n, dtype=torch.bfloat16, device=dev)
        hb = symm.rendezvous(buf, dist.group.WORLD)
        bptrs = (ctypes.c_void_p * WORLD)(*hb.buffer_ptrs)
        g = torch.Generator(device=dev)
        g.manual_seed(777 + rank)
        x = torch.randn(n, device=dev, generator=g).bfloat16()
        parts = [torch.empty_like(x) for _ in range(WORLD)]
        dist.all_gather(parts, x)
        ref = sum(p_.float() for p_ in parts).bfloat16()
        side = torch.cuda.Stream(device=dev)
        torch.cuda.synchronize()
        dist.barrier()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            buf.copy_(x)
            st = L.hq_allreduce_sum(bptrs, fptrs, None, WORLD, rank, _lib.HQ_BF16, n, 0, 64,
                                    ctypes.c_void_p(side.cuda_stream))
        assert st == 0, L.hq_last_error_string()
        for _ in range(5):
            dist.barrier()
            gr.replay()
            torch.cuda.synchronize()
            assert L.hq_check_device_error() == 0
            errs.append(int((buf.view(torch.int16) != ref.view(torch.int16)).sum().item()))
        del gr
        torch.cuda.synchronize()
        dist.barrier()
        np.save(os.path.join(out_dir, f"mismatch_{rank}.npy"), np.array(errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_allreduce_matches_gathered_sum_bit_for_bit(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    for r in range(WORLD):
        m = np.load(tmp_path / f"mismatch_{r}.npy")
        assert m.size >= 32 and (m == 0).all(), m
