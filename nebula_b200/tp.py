"""Megatron-style tensor parallelism for the quantized linear layers.

A 27B-class decoder layer has four quantized GEMMs.  Across `world` ranks
(one process and one GPU each):
  * column-parallel QKV and gate_up: every rank holds a slice of the output
    columns N (gate_up's gate and up halves are sliced separately so that each
    rank holds matching gate and up columns); no communication;
  * row-parallel O and down: every rank holds a slice of the input rows K, cut
    on scale-group boundaries, and produces a partial sum of the full output;
    the partial outputs are summed with an all-reduce (NCCL over NVLink on the
    GPU box, gloo in the CPU tests).
The reference engine has no multi-GPU code (it runs replicas only); the split
follows the plan for its layer shapes: QKV 5120x7168, O 5120x5120, gate_up
5120x34816, down 17408x5120.

The slicing helpers work on the reference's linear int4 layout (uint32
[K/8][N], marlin_gemm.cu:495-510), the ternary linear layout (uint32
[K/16][N]) and the scales [K/group][N]; each shard is then repacked to tile
order on its own GPU (hq.repack).
"""
from __future__ import annotations

from dataclasses import dataclass

LAYER_SHAPES = (("qkv", 5120, 7168), ("o", 5120, 5120), ("gate_up", 5120, 34816), ("down", 17408, 5120))
COLUMN_PARALLEL = {"qkv": 1, "gate_up": 2}  # value = number of independently sliced halves along N
ROW_PARALLEL = ("o", "down")


@dataclass(frozen=True)
class Shard:
    """Local problem of one rank: K_local x N_local, plus where it sits in the full matrix."""
    name: str
    K: int
    N: int
    row_parallel: bool
    k0: int          # first input row of this rank (row-parallel)
    col_ranges: tuple  # ((n_begin, n_end), ...) of the full matrix held by this rank, in local order


def shard_spec(name: str, K: int, N: int, world: int, rank: int, group: int = 128) -> Shard:
    """The slice of layer `name` that rank `rank` of `world` holds.

    Column-parallel: N split into `world` equal parts per half (each a multiple
    of 16, the tile strip width).  Row-parallel: K split into `world` equal
    parts that are whole scale groups.  Raises ValueError when the shape does
    not divide."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if name in ROW_PARALLEL:
        if K % (world * group):
            raise ValueError(f"{name}: K={K} does not split into {world} parts of whole {group}-groups")
        kl = K // world
        return Shard(name, kl, N, True, rank * kl, ((0, N),))
    halves = COLUMN_PARALLEL.get(name)
    if halves is None:
        raise ValueError(f"unknown layer {name}")
    if N % (halves * world * 16):
        raise ValueError(f"{name}: N={N} does not split into {world} parts of whole 16-column strips")
    hw = N // halves
    part = hw // world
    ranges = tuple((h * hw + rank * part, h * hw + (rank + 1) * part) for h in range(halves))
    return Shard(name, K, part * halves, False, 0, ranges)


def _k_per_word(wbits: int) -> int:
    return 32 // wbits


def slice_weights(linear, scales, spec: Shard, wbits: int = 4, group: int = 128):
    """(linear, scales) of the full layer -> this rank's (linear, scales), both
    contiguous.  Works for numpy arrays and torch tensors alike."""
    kpw = _k_per_word(wbits)
    if spec.row_parallel:
        w = linear[spec.k0 // kpw:(spec.k0 + spec.K) // kpw]
        s = scales[spec.k0 // group:(spec.k0 + spec.K) // group]
        return _contig(w), _contig(s)
    ws = [linear[:, a:b] for a, b in spec.col_ranges]
    ss = [scales[:, a:b] for a, b in spec.col_ranges]
    return _cat(ws), _cat(ss)


def slice_activations(x, spec: Shard):
    """Row-parallel layers read the matching K slice of the (replicated) input."""
    if spec.row_parallel:
        return _contig(x[:, spec.k0:spec.k0 + spec.K])
    return x


def _contig(a):
    if hasattr(a, "contiguous"):
        return a.contiguous()
    import numpy as np
    return np.ascontiguousarray(a)


def _cat(parts):
    if len(parts) == 1:
        return _contig(parts[0])
    if hasattr(parts[0], "contiguous"):
        import torch
        return torch.cat(parts, dim=1).contiguous()
    import numpy as np
    return np.ascontiguousarray(np.concatenate(parts, axis=1))


def gather_columns(local_outputs, specs):
    """Column-parallel outputs of all ranks (rank order) -> the full output, by
    placing each rank's columns at their ranges (host-side check helper)."""
    import numpy as np
    N = max(b for s in specs for _, b in s.col_ranges)
    M = local_outputs[0].shape[0]
    out = np.zeros((M, N), dtype=np.asarray(local_outputs[0]).dtype)
    for y, s in zip(local_outputs, specs):
        o = 0
        for a, b in s.col_ranges:
            out[:, a:b] = np.asarray(y)[:, o:o + (b - a)]
            o += b - a
    return out
