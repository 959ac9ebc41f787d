"""CPU checks of the index arithmetic the integer-pipe kernels rest on (no GPU): the exact int8 pieces of x, the
TQ1_0 tensor-core kernel's operand layout (csrc/hq_tq1.cu), emulated fragment by fragment against the oracle,
and the Q8_0 projection kernel's block-pair layout and shared-memory swizzles (csrc/hq_proj.cu)."""
import numpy as np
import pytest

from oracle import oracle as o


# ------------------------------------------------------------ x as int8 pieces

def x_pieces(x, e):
    """X = rint(x * 2^(27-e)) as balanced base-128 digits q0..q3 (the kernels' x_pieces)."""
    X = np.rint(np.ldexp(x.astype(np.float64), 27 - e)).astype(np.int64)
    q3 = ((X + 64) & 127) - 64
    X1 = (X - q3) >> 7
    q2 = ((X1 + 64) & 127) - 64
    X2 = (X1 - q2) >> 7
    q1 = ((X2 + 64) & 127) - 64
    q0 = (X2 - q1) >> 7
    return X, np.stack([q0, q1, q2, q3], -1)


def test_x_pieces_are_exact_and_fit_int8():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100_000).astype(np.float32),
                        np.array([0, 1, -1, 0.5, -0.5, 0.999999, -0.999999], np.float32)])
    m = np.max(np.abs(x))
    e = int(np.frexp(m)[1])
    X, q = x_pieces(x, e)
    assert np.all(np.abs(X) <= 2 ** 27)
    assert np.all(np.abs(q) <= 65)  # int8 with room
    assert np.array_equal(((q[:, 0] * 128 + q[:, 1]) * 128 + q[:, 2]) * 128 + q[:, 3], X)
    # the fixed-point copy is within half a unit of 2^(e-27) of x
    assert np.max(np.abs(np.ldexp(X.astype(np.float64), e - 27) - x)) <= 2.0 ** (e - 28)


# ------------------------------------------------ TQ1_0 tensor-core kernel

def digit_word(v):
    d = [(v // 3 ** s) % 3 for s in range(5)]
    return d[0] | (d[4] << 2) | (d[1] << 8) | (d[2] << 16) | (d[3] << 24)


def slot_k(ob, r, i):
    """tq1_slot_k: the block offset of A slot i of register r of a lane whose 8 bytes start at block byte ob."""
    beta = r if r < 8 else 4 * (r - 8) + i
    s = i if r < 8 else 4
    p = ob + beta - 2
    if 0 <= p < 50:
        return 5 * p + s
    if p in (50, 51) and s < 3:
        return 250 + 3 * (p - 50) + s
    return -1


def test_tq1_slots_cover_each_weight_once():
    """Over a 4-block group (7 windows x 4 lane pieces x 10 registers x 4 slots), every weight of every block
    appears in exactly one slot; the empty slots are the d bytes, pad bytes and digits 3-4 of bytes 50-51."""
    seen = np.zeros((4, 256), np.int64)
    empty = 0
    for win in range(7):
        for t in range(4):
            o_ = 32 * win + 8 * t
            blk, ob = divmod(o_, 56)
            assert ob + 8 <= 56  # a lane's 8 bytes never straddle blocks
            for r in range(10):
                for i in range(4):
                    k = slot_k(ob, r, i)
                    if k < 0:
                        empty += 1
                    else:
                        seen[blk, k] += 1
    assert np.all(seen == 1)
    assert empty == 7 * 4 * 40 - 4 * 256
    # blocks start in windows 0, 1, 3, 5 (lanes 0, 3, 2, 1) and end in windows 1, 3, 5, 6
    starts = [divmod(56 * b, 32) for b in range(4)]
    assert [(w, off // 8) for w, off in starts] == [(0, 0), (1, 3), (3, 2), (5, 1)]
    assert [(56 * b + 55) // 32 for b in range(4)] == [1, 3, 5, 6]


def emulate_tq1(x, blob, K, N):
    """The kernel's arithmetic with numpy: per window the A (digits) and B (x pieces per parity) operands built
    exactly as the kernel builds them, integer products, the per-block flush with the piece-sum correction."""
    nb = K // 256
    W = blob.reshape(N, nb * 56)
    e = int(np.frexp(np.max(np.abs(x)))[1]) if np.max(np.abs(x)) > 0 else 0
    _, q = x_pieces(x, e)
    qsum = q.reshape(nb, 256, 4).sum(1)  # per block piece sums (the "- 1" of every trit)
    lut = np.array([digit_word(v) for v in range(256)], np.int64)
    y = np.zeros(N)
    for G in range(nb // 4):
        acc = np.zeros((N, 8), np.int64)   # columns (parity, piece)
        dsc = np.zeros((N, 2))
        for win in range(7):
            for t in range(4):
                base = G * 224 + 32 * win + 8 * t
                blk_in_g, ob = divmod(32 * win + 8 * t, 56)
                b = 4 * G + blk_in_g
                P = blk_in_g & 1
                if ob == 0:  # the block's d: taken when it starts
                    d = W[:, base:base + 2].copy().view(np.float16).astype(np.float64).ravel()
                    dsc[:, P] = np.where(np.isfinite(d), d, 0.0)
                T = lut[W[:, base:base + 8]]                      # [N, 8] table words
                for r in range(10):
                    for i in range(4):
                        k = slot_k(ob, r, i)
                        if k < 0:
                            continue
                        if r < 8:
                            a = (T[:, r] >> (8 * i)) & 3 if i else T[:, r] & 3
                        else:
                            a = ((T[:, 4 * (r - 8) + i] & 0xFF) >> 2) & 3
                        acc[:, 4 * P:4 * P + 4] += a[:, None] * q[256 * b + k][None, :]
            for blk_in_g, end_win in enumerate((1, 3, 5, 6)):
                if win == end_win:
                    P = blk_in_g & 1
                    b = 4 * G + blk_in_g
                    dc = acc[:, 4 * P:4 * P + 4] - qsum[b][None, :]
                    v = ((dc[:, 0] * 128 + dc[:, 1]) * 128 + dc[:, 2]) * 128 + dc[:, 3]
                    y += dsc[:, P] * v
                    acc[:, 4 * P:4 * P + 4] = 0
        assert not acc.any()
    return np.ldexp(y, e - 27)


@pytest.mark.parametrize("K,N", [(1024, 24), (2048, 9)])
def test_tq1_tensor_core_layout_matches_oracle(K, N):
    rng = np.random.default_rng(K + N)
    t = rng.integers(-1, 2, size=(N, K), dtype=np.int8)
    d = rng.uniform(0.01, 0.05, size=(N, K // 256)).astype(np.float16).view(np.uint16)
    d[1, 0] = 0x7C00  # Inf d: the block is skipped
    blob = o.pack_tq1_0(t, d).reshape(N, -1)
    blob[:, 2:54:11] = 247  # bytes outside 0..242 follow the same digit arithmetic
    blob = blob.ravel()
    x = rng.standard_normal(K).astype(np.float32)
    assert o.max_rel_err(emulate_tq1(x, blob, K, N), o.gemv_tq1_0(x, blob, K, N)) < 1e-6


# --------------------------------------------------- Q8_0 projection kernel

def q8_chunk_pos(c):
    return (c & ~7) | ((c & 7) ^ ((c >> 3) & 7))


def stage_swizzle(c):
    return (c & ~15) | ((c & 15) ^ ((c >> 4) & 15))


def test_swizzles_are_bijections_and_spread_banks():
    for f, group in ((q8_chunk_pos, 8), (stage_swizzle, 16)):
        c = np.arange(1024)
        pos = np.array([f(int(v)) for v in c])
        assert sorted(pos) == list(c)
        assert np.all(pos // group == c // group)
    # the 32 lanes (block pairs pr) read chunk 4 pr + r of a piece array: all eight 16-byte bank groups, 4 each
    for r in range(4):
        groups = [q8_chunk_pos(4 * pr + r) % 8 for pr in range(32)]
        assert sorted(np.bincount(groups, minlength=8)) == [4] * 8


def test_q8_pair_layout_and_dp4a_sums():
    """A 68-byte block pair: d0 in bytes 0-1, the first block's int8 at 2..33 (read as words funnel-shifted by 16
    bits), d1 in 34-35, the second block's at 36..67 (aligned words 9..16); four exact piece dot products per
    block reproduce d * sum(q * x) to fp32 rounding."""
    rng = np.random.default_rng(4)
    q = rng.integers(-128, 128, size=64, dtype=np.int8)
    d = rng.uniform(0.005, 0.02, size=2).astype(np.float16)
    pair = np.empty(68, np.uint8)
    pair[0:2] = d[:1].view(np.uint8)
    pair[2:34] = q[:32].view(np.uint8)
    pair[34:36] = d[1:].view(np.uint8)
    pair[36:68] = q[32:].view(np.uint8)
    Wd = pair.view(np.uint32)
    for g in range(8):  # block 0 groups: (W[g] >> 16) | (W[g+1] << 16)
        word = (int(Wd[g]) >> 16) | ((int(Wd[g + 1]) << 16) & 0xFFFFFFFF)
        assert np.array_equal(np.frombuffer(np.uint32(word).tobytes(), np.int8), q[4 * g:4 * g + 4])
        assert np.array_equal(np.frombuffer(Wd[9 + g].tobytes(), np.int8), q[32 + 4 * g:36 + 4 * g])
    assert np.uint16(Wd[0] & 0xFFFF).view(np.float16) == d[0]
    assert np.uint16(Wd[8] >> 16).view(np.float16) == d[1]
    x = rng.standard_normal(64).astype(np.float32)
    e = int(np.frexp(np.max(np.abs(x)))[1])
    _, xp = x_pieces(x, e)
    for blk in range(2):
        S = (q[32 * blk:32 * blk + 32, None].astype(np.int64) * xp[32 * blk:32 * blk + 32]).sum(0)
        v = np.ldexp(float((S[0] * 128 + S[1]) * 2 ** 14 + (S[2] * 128 + S[3])), e - 27) * float(d[blk])
        ref = float(d[blk]) * float(q[32 * blk:32 * blk + 32].astype(np.float64) @ x[32 * blk:32 * blk + 32])
        assert abs(v - ref) <= 1e-6 * (abs(ref) + 1e-3)


# ---------------------------------------------------------------------------
# Integer-MMA decode (csrc/hq_decode_i8.cu): tile-order codes -> signed bytes
# 16 q, activation pieces in the prep kernel's order, m16n8k32 s8 fragments.

_PIECE_POS = [0, 2, 1, 3, 8, 10, 9, 11, 4, 6, 5, 7, 12, 14, 13, 15]  # byte j of a lane's 16 B <- k offset


def _s8(words):
    return np.asarray(words, np.uint32).view(np.uint8).view(np.int8).astype(np.int64)


def _mma_m16n8k32(a, b):
    """a: 32 lanes x 4 regs (4 s8 each); b: 32 lanes x 2 regs -> D[16][8] (the PTX fragment layout)."""
    A = np.zeros((16, 32), np.int64)
    B = np.zeros((32, 8), np.int64)
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        for r, (row, k0) in enumerate([(g, 4 * t), (g + 8, 4 * t), (g, 16 + 4 * t), (g + 8, 16 + 4 * t)]):
            A[row, k0:k0 + 4] = _s8([a[lane][r]])
        B[4 * t:4 * t + 4, g] = _s8([b[lane][0]])
        B[16 + 4 * t:16 + 4 * t + 4, g] = _s8([b[lane][1]])
    return A @ B


@pytest.mark.parametrize("seed", range(3))
def test_int8_decode_fragments_give_16q_dot_x(seed):
    rng = np.random.default_rng(seed)
    K, N, M = 64, 16, 4
    q = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    tile = o.pack_tile(q, 4).view(np.uint32)  # one chunk: 16 columns x 64 k
    xf = rng.integers(-16384, 16385, size=(M, K))  # fixed-point activations
    h = (xf + 128) >> 8
    l = xf - 256 * h
    assert h.min() >= -128 and h.max() <= 127 and l.min() >= -128 and l.max() <= 127
    # prep kernel layout: [(m*2 + piece)*4 + t][16 bytes]
    pieces = np.zeros((M * 2 * 4, 16), np.int8)
    for m in range(M):
        for p, arr in enumerate((h, l)):
            for t in range(4):
                pieces[(m * 2 + p) * 4 + t] = [arr[m, 16 * t + _PIECE_POS[j]] for j in range(16)]
    xbytes = pieces.reshape(-1).view(np.uint32).reshape(32, 4)  # lane -> its 16 bytes
    lo = lambda w: (((w << 4) & 0xFFFFFFFF) & 0xF0F0F0F0) ^ 0x80808080  # noqa: E731
    hi = lambda w: (w & 0xF0F0F0F0) ^ 0x80808080  # noqa: E731
    a_lo, a_hi = [], []
    for lane in range(32):
        x, y, z, w = (int(v) for v in tile[4 * lane:4 * lane + 4])
        a_lo.append([lo(x), lo(z), lo(y), lo(w)])
        a_hi.append([hi(x), hi(z), hi(y), hi(w)])
    D = _mma_m16n8k32(a_lo, [xbytes[lane][0:2] for lane in range(32)]) + \
        _mma_m16n8k32(a_hi, [xbytes[lane][2:4] for lane in range(32)])
    want = 16 * (q.astype(np.int64).T @ xf.T)  # [n][m]
    for m in range(M):
        assert np.array_equal(256 * D[:, 2 * m] + D[:, 2 * m + 1], want[:, m])


def _prmt(a, b, sel):
    """PTX prmt.b32 (default mode): byte i of the result is byte (sel >> 4i) & 7 of a (bytes 0-3)
    followed by b (bytes 4-7)."""
    src = list(int(a).to_bytes(4, "little")) + list(int(b).to_bytes(4, "little"))
    return sum(src[(sel >> (4 * i)) & 7] << (8 * i) for i in range(4))


def _t2_operands(w):
    """hq_decode_i8.cu t2_operands: one TILE_T2 word -> its four field classes (MMA 0 slots 4t..,
    MMA 0 slots 16+4t.., MMA 1 ...), one mask each."""
    return w & 0x03030303, (w >> 2) & 0x03030303, (w >> 4) & 0x03030303, (w >> 6) & 0x03030303


# Ternary activation pieces (x_prep_kernel<..., T2 = true>): byte j of lane t's 16 bytes holds element
# _T2_PIECE_POS[j] of its 16 k, the order of the field classes above.
_T2_PIECE_POS = [0, 8, 1, 9, 2, 10, 3, 11, 4, 12, 5, 13, 6, 14, 7, 15]


def _t2_prep_words(h_oct0, h_oct1):
    """The prep kernel's assembly of one lane's four words from its two octets' natural-order bytes
    (prmt 0x5140 / 0x7362 across the pair of neighbouring prep lanes)."""
    w = lambda v: int.from_bytes(bytes(int(x) & 0xFF for x in v), "little")  # noqa: E731
    e0a, e1a, e0b, e1b = w(h_oct0[0:4]), w(h_oct0[4:8]), w(h_oct1[0:4]), w(h_oct1[4:8])
    return [_prmt(e0a, e0b, 0x5140), _prmt(e0a, e0b, 0x7362), _prmt(e1a, e1b, 0x5140), _prmt(e1a, e1b, 0x7362)]


@pytest.mark.parametrize("seed", range(3))
def test_int8_decode_ternary_fragments_give_q_dot_x(seed):
    """The integer decode kernel's ternary operands: codes c = q + 1 as u8 field classes, with the
    ternary activation pieces in the matching order, give sum c x - sum x = sum q x (one 64-k block)."""
    rng = np.random.default_rng(100 + seed)
    K, N, M = 64, 16, 4
    t = rng.integers(-1, 2, size=(K, N), dtype=np.int8)
    tile = o.pack_tile(t, 2).view(np.uint32)  # one chunk: 16 columns x 64 k, 2 words per lane
    xf = rng.integers(-16384, 16385, size=(M, K))
    h = (xf + 128) >> 8
    l = xf - 256 * h
    pieces = np.zeros((M * 2 * 4, 16), np.int8)
    for m in range(M):
        for p, arr in enumerate((h, l)):
            for tt in range(4):
                pieces[(m * 2 + p) * 4 + tt] = [arr[m, 16 * tt + _T2_PIECE_POS[j]] for j in range(16)]
                # the prep kernel's two-lane assembly gives the same bytes
                words = _t2_prep_words(arr[m, 16 * tt:16 * tt + 8], arr[m, 16 * tt + 8:16 * tt + 16])
                assert np.array_equal(np.array(words, np.uint32).view(np.int8), pieces[(m * 2 + p) * 4 + tt])
    xbytes = pieces.reshape(-1).view(np.uint32).reshape(32, 4)
    a0, a1 = [], []
    for lane in range(32):
        x, y = int(tile[2 * lane]), int(tile[2 * lane + 1])  # columns g and g + 8
        l0, l2, h0, h2 = _t2_operands(x)
        l1, l3, h1, h3 = _t2_operands(y)
        a0.append([l0, l1, l2, l3])
        a1.append([h0, h1, h2, h3])
    D = _mma_m16n8k32(a0, [xbytes[lane][0:2] for lane in range(32)]) + \
        _mma_m16n8k32(a1, [xbytes[lane][2:4] for lane in range(32)])
    want = t.astype(np.int64).T @ xf.T  # [n][m]
    for m in range(M):
        assert np.array_equal(256 * D[:, 2 * m] + D[:, 2 * m + 1] - xf[m].sum(), want[:, m])
