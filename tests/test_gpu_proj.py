"""Output projection and embedding lookup over GGML F32 / BF16 / Q8_0 / TQ1_0 weights against the oracle's
restatement of kernel_output_projection / kernel_embedding_lookup (forward_baseline.cu:55-109, 178-257)."""
import os

import numpy as np
import pytest
import torch

from nebula_b200 import _lib, hq
from oracle import oracle as o

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden.npz")
TOL = 1e-5  # max |y - y_ref| / max |y_ref|, fp32 sums in a different order


def dev_bytes(a, offset=0):
    """Raw bytes on cuda:0, starting `offset` bytes into a 256-byte aligned allocation."""
    b = np.ascontiguousarray(a).view(np.uint8).ravel()
    buf = torch.zeros(b.size + offset, dtype=torch.uint8, device="cuda:0")
    buf[offset:] = torch.from_numpy(b).to("cuda:0")
    return buf[offset:]


def check_close(y, ref):
    y = np.asarray(y)
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    fin = ~np.isnan(ref)
    assert o.max_rel_err(y[fin], ref[fin]) <= TOL


@pytest.mark.parametrize("prefix", ["pf32", "pbf16", "pq8", "ptq1"])
def test_projection_and_embedding_golden(prefix):
    g = np.load(GOLDEN)
    w_type, K, N, _ = (int(v) for v in g[f"{prefix}_meta"])
    w = dev_bytes(g[f"{prefix}_w"])
    x = torch.from_numpy(g[f"{prefix}_x"]).to("cuda:0")
    check_close(hq.output_projection(x, w, w_type, N).cpu().numpy(), g[f"{prefix}_y"])
    for tk, row in zip(g[f"{prefix}_tokens"], g[f"{prefix}_emb"]):
        e = hq.embedding_lookup(w, w_type, int(tk), K, N).cpu().numpy()
        assert np.array_equal(e, row)


def make_weights(w_type, K, N, rng):
    if w_type == o.GGML_F32:
        return rng.standard_normal((N, K), dtype=np.float32)
    if w_type == o.GGML_BF16:
        return (rng.standard_normal((N, K), dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
    if w_type == o.GGML_Q8_0:
        q = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
        d = rng.uniform(0.005, 0.02, size=(N, K // 32)).astype(np.float16).view(np.uint16)
        return o.pack_q8_0(q, d)
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    return o.pack_tq1_0(t, d)


@pytest.mark.parametrize("w_type,K,N,offset", [
    (o.GGML_F32, 1024, 517, 0),   # stream kernel
    (o.GGML_F32, 1022, 33, 0),    # K % 4 != 0: the reference's loop
    (o.GGML_BF16, 5120, 1003, 0),  # stream kernel, ragged last 4-row group
    (o.GGML_BF16, 5120, 64, 2),   # W 2-byte aligned only: the reference's loop
    (o.GGML_BF16, 100, 45, 0),    # K % 8 != 0
    (o.GGML_Q8_0, 5120, 999, 0),  # stream kernel
    (o.GGML_Q8_0, 4096, 70, 2),   # W 2-byte aligned only
    (o.GGML_Q8_0, 96, 50, 0),     # K % 64 != 0
    (o.GGML_TQ1_0, 2048, 300, 0),  # tensor-core TQ1_0 kernel
])
def test_projection_paths(w_type, K, N, offset):
    rng = np.random.default_rng(K * 7 + N)
    w = make_weights(w_type, K, N, rng)
    x = rng.standard_normal(K).astype(np.float32)
    y = hq.output_projection(torch.from_numpy(x).to("cuda:0"), dev_bytes(w, offset), w_type, N)
    torch.cuda.synchronize()
    check_close(y.cpu().numpy(), o.output_projection(x, w, w_type, K, N))


def test_q8_0_nan_scale_propagates():
    """Q8_0 applies d unchecked (forward_baseline.cu:211): a NaN d makes that row's logit NaN."""
    rng = np.random.default_rng(5)
    K, N = 1024, 40
    q = rng.integers(-128, 128, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.005, 0.02, size=(N, K // 32)).astype(np.float16).view(np.uint16)
    d[7, 3] = 0x7E00
    w = o.pack_q8_0(q, d)
    x = rng.standard_normal(K).astype(np.float32)
    y = hq.output_projection(torch.from_numpy(x).to("cuda:0"), dev_bytes(w), o.GGML_Q8_0, N).cpu().numpy()
    ref = o.output_projection(x, w, o.GGML_Q8_0, K, N)
    assert np.isnan(y[7]) and np.isnan(ref[7])
    check_close(y, ref)


@pytest.mark.parametrize("w_type", [o.GGML_BF16, o.GGML_Q8_0])
def test_output_projection_full_size(w_type):
    """The output projection at vocab 248320 x hidden 5120 (native_decoder.hpp:180); 512 sampled rows
    against the oracle."""
    K, N = 5120, 248320
    g = torch.Generator(device="cuda:0")
    g.manual_seed(w_type)
    if w_type == o.GGML_BF16:
        w = (torch.randn((N, K), device="cuda:0", generator=g)).bfloat16().view(torch.uint8).view(N, -1)
    else:
        blk = torch.randint(-128, 128, (N, K // 32, 34), dtype=torch.int8, device="cuda:0", generator=g).view(torch.uint8)
        d = (torch.rand((N, K // 32), device="cuda:0", generator=g) * 0.015 + 0.005).half()
        blk[..., 0:2] = d.view(torch.uint8).view(N, K // 32, 2)
        w = blk.view(N, -1)
    x = torch.randn(K, device="cuda:0", generator=g)
    y = hq.output_projection(x, w.reshape(-1), w_type, N).cpu().numpy()
    rows = np.sort(np.random.default_rng(1).choice(N, 512, replace=False))
    ref = o.output_projection(x.cpu().numpy(), w[torch.from_numpy(rows).cuda()].cpu().numpy(), w_type, K, len(rows))
    check_close(y[rows], ref)


def test_shared_memory_attribute_not_lowered():
    """One kernel launched with shrinking then growing staged-x sizes: a smaller launch must not lower the
    kernel's dynamic shared-memory limit under a later, larger one."""
    rng = np.random.default_rng(9)
    for K in (4096, 1024, 4096, 2048):
        w = make_weights(o.GGML_Q8_0, K, 64, rng)
        x = rng.standard_normal(K).astype(np.float32)
        y = hq.output_projection(torch.from_numpy(x).to("cuda:0"), dev_bytes(w), o.GGML_Q8_0, 64).cpu().numpy()
        check_close(y, o.output_projection(x, w, o.GGML_Q8_0, K, 64))


def test_q8_0_nonfinite_x_takes_float_loop():
    """x holding Inf/NaN: the Q8_0 kernel switches to the reference's float loop, so the non-finite pattern of
    the logits is the reference's."""
    rng = np.random.default_rng(12)
    K, N = 1024, 48
    w = make_weights(o.GGML_Q8_0, K, N, rng)
    x = rng.standard_normal(K).astype(np.float32)
    x[17] = np.inf
    y = hq.output_projection(torch.from_numpy(x).to("cuda:0"), dev_bytes(w), o.GGML_Q8_0, N).cpu().numpy()
    ref = o.output_projection(x, w, o.GGML_Q8_0, K, N)
    assert np.array_equal(np.isnan(y), np.isnan(ref)) and np.array_equal(np.isinf(y), np.isinf(ref))
    assert np.array_equal(np.sign(y[np.isinf(ref)]), np.sign(ref[np.isinf(ref)]))
