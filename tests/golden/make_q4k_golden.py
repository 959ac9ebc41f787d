"""Generate tests/golden/q4_k.npz: GGUF Q4_K blocks and their dequantised weights.

The reference names Q4_K only as a GGUF block type (hydrogen/include/gguf_parser.hpp:44,
:130: 256 weights in 144 bytes); the field layout and the dequantisation are llama.cpp's.
The expected weights here come from gguf-py 0.19.0 (``gguf.quants.dequantize``), llama.cpp's
own Python implementation of the format, so they pin the oracle's independent restatement
(oracle/oracle.py ``unpack_q4_k`` / ``dequant_q4_k``) to the published format.  CPU only.

    python tests/golden/make_q4k_golden.py           # (re)write q4_k.npz
    python tests/golden/make_q4k_golden.py --check   # regenerate in memory, compare

Cases
  * ``rand_*``: K=512, N=32, seeded random scale / min / code bytes, fp16 d and dmin in
    [1e-3, 4e-3];
  * ``edge_*``: K=256, N=16 with every 6-bit scale and min at its maximum (0xFF bytes), a
    zero d, the smallest subnormal d, a negative d and dmin, the largest finite fp16 d,
    and Inf / NaN d and dmin in single blocks.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as o  # noqa: E402

OUT = os.path.join(HERE, "q4_k.npz")


def _f16_bytes(v: float) -> np.ndarray:
    return np.frombuffer(np.float16(v).tobytes(), np.uint8)


def edge_blocks() -> np.ndarray:
    K, N = 256, 16
    blk = o.gen_q4_k_blocks(K, N, seed=7).reshape(N, 1, o.Q4K_BLOCK_BYTES).copy()
    blk[0, 0, 4:16] = 0xFF                           # sc = m = 63 for all eight sub-blocks
    blk[1, 0, 0:2] = _f16_bytes(0.0)                 # d = 0
    blk[2, 0, 0:2] = np.array([1, 0], np.uint8)      # smallest subnormal d
    blk[3, 0, 0:2] = _f16_bytes(-2.5e-3)             # negative d
    blk[3, 0, 2:4] = _f16_bytes(-1.5e-3)             # negative dmin
    blk[4, 0, 0:2] = _f16_bytes(65504.0)             # largest finite d
    blk[5, 0, 0:2] = _f16_bytes(np.inf)
    blk[6, 0, 2:4] = _f16_bytes(np.nan)
    blk[7, 0, 16:] = 0xFF                            # every code 15
    blk[8, 0, 16:] = 0x00                            # every code 0
    return blk.reshape(-1)


def build() -> dict:
    from gguf import GGMLQuantizationType, quants

    cases = {"rand": (512, 32, o.gen_q4_k_blocks(512, 32, seed=3)), "edge": (256, 16, edge_blocks())}
    out = {}
    for name, (K, N, blob) in cases.items():
        w = quants.dequantize(blob.reshape(N, -1), GGMLQuantizationType.Q4_K)  # [N][K]
        out[f"{name}_K"] = np.int32(K)
        out[f"{name}_N"] = np.int32(N)
        out[f"{name}_blocks"] = blob
        out[f"{name}_w_nk"] = np.ascontiguousarray(w, np.float32)
    return out


def main() -> int:
    data = build()
    if "--check" in sys.argv:
        old = np.load(OUT)
        bad = [k for k in data if not np.array_equal(old[k], data[k], equal_nan=True)]
        print("q4_k.npz matches" if not bad else f"q4_k.npz differs in {bad}")
        return 1 if bad else 0
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
