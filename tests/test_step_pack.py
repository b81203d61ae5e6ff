"""Tile streams of the persistent decode-step kernel, checked on the CPU.

``spark_b200.step`` repacks the checkpoint tensors into tiles whose 16-byte
lane slices are MMA fragments. These tests replay, in NumPy, exactly what a
warp of ``csrc/sb_step.cu`` does with a tile - the byte permutes / LOP3 code
conversions, the staged activation layouts, and ``mma.sync.m16n8k16``
assembled from the per-lane fragments with the PTX ISA's documented layout
(A: a0 = row g cols 2c..2c+1, a1 = row g+8, a2 = row g cols 2c+8..2c+9, a3 =
row g+8; B: b0 = rows 2c..2c+1 of column g, b1 = rows 2c+8..2c+9; C: c0/c1 =
row g cols 2c/2c+1, c2/c3 = row g+8) - and compare each tile's partial sums
with the plain dot products of the unpacked weights. A layout mistake in the
packer or in the kernel's reading of it shows up here without a GPU.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import formats, quant  # noqa: E402
from spark_b200 import step  # noqa: E402


# ------------------------------------------------------------ bit helpers
def u32s(b16):
    """16 bytes -> 4 little-endian uint32 words."""
    return np.frombuffer(np.asarray(b16, np.uint8).tobytes(), "<u4")


def halves(word, kind):
    """uint32 -> (low, high) 16-bit values as float (kind 'f16' or 'bf16')."""
    lo, hi = np.uint16(word & 0xFFFF), np.uint16(word >> 16)
    if kind == "f16":
        return float(np.array(lo).view(np.float16)), float(np.array(hi).view(np.float16))
    return (float(formats.bf16_from_bits(np.array([lo]))[0]), float(formats.bf16_from_bits(np.array([hi]))[0]))


def prmt(a, b, sel):
    src = np.frombuffer(np.array([a, b], "<u4").tobytes(), np.uint8)
    out = [src[(sel >> (4 * i)) & 7] for i in range(4)]
    return int(np.frombuffer(bytes(out), "<u4")[0])


def lop_and_or(a, mask, bits):
    return (a & mask) | bits


def mma(acc, lanes_a, lanes_b):
    """acc [16, 8] += A @ B with A, B assembled from 32 lanes' fragments.

    lanes_a[L] = 4 pairs (a0..a3), lanes_b[L] = 2 pairs (b0, b1) of floats."""
    A = np.zeros((16, 16))
    B = np.zeros((16, 8))
    for L in range(32):
        g, c = L >> 2, L & 3
        a0, a1, a2, a3 = lanes_a[L]
        b0, b1 = lanes_b[L]
        for j in range(2):
            A[g, 2 * c + j] = a0[j]
            A[g + 8, 2 * c + j] = a1[j]
            A[g, 2 * c + 8 + j] = a2[j]
            A[g + 8, 2 * c + 8 + j] = a3[j]
            B[2 * c + j, g] = b0[j]
            B[2 * c + 8 + j, g] = b1[j]
    acc += A @ B


def fp16_bits(v):
    return int(np.array(v, np.float16).view(np.uint16))


def bf16_bits(v):
    return int(formats.bf16_bits(np.array([v], np.float32))[0])


# --------------------------------------------------------------------- W8
def emulate_w8_tile(tile, x_chunk):
    """sb_step.cu w8_tile: returns the 16 rows' partial sums."""
    kb_count = x_chunk.shape[0] // 32
    acc = np.zeros((16, 8))
    for kb in range(kb_count):
        lanes_a, lanes_b, lanes_a2, lanes_b2 = [], [], [], []
        for L in range(32):
            c = L & 3
            a = u32s(tile[kb * 512 + L * 16: kb * 512 + L * 16 + 16])
            xb = x_chunk[kb * 32 + c * 8: kb * 32 + c * 8 + 8].astype(np.float16)

            def code(word, sel):
                lo, hi = halves(prmt(int(word), 0x64646464, sel), "f16")
                return (lo - 1152.0, hi - 1152.0)  # sub.f16x2 with 1152 (exact)

            lanes_a.append([code(a[0], 0x4140), code(a[1], 0x4140), code(a[0], 0x4342), code(a[1], 0x4342)])
            lanes_b.append([(float(xb[0]), float(xb[1])), (float(xb[2]), float(xb[3]))])
            lanes_a2.append([code(a[2], 0x4140), code(a[3], 0x4140), code(a[2], 0x4342), code(a[3], 0x4342)])
            lanes_b2.append([(float(xb[4]), float(xb[5])), (float(xb[6]), float(xb[7]))])
        mma(acc, lanes_a, lanes_b)
        mma(acc, lanes_a2, lanes_b2)
    return acc[:, 0]


def test_w8_stream_tiles_reproduce_dot_products():
    rng = np.random.default_rng(0)
    n, k, ck = 32, 128, 64
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    x = rng.standard_normal(k).astype(np.float16).astype(np.float64)
    stream = step.pack_w8(torch.from_numpy(w), ck).numpy()
    tile_bytes = 16 * ck
    for rb in range(n // 16):
        for ch in range(k // ck):
            t = stream[(rb * (k // ck) + ch) * tile_bytes:][:tile_bytes]
            got = emulate_w8_tile(t, x[ch * ck:(ch + 1) * ck])
            ref = w[rb * 16:(rb + 1) * 16, ch * ck:(ch + 1) * ck].astype(np.float64) @ x[ch * ck:(ch + 1) * ck]
            np.testing.assert_allclose(got, ref, rtol=0, atol=1e-9)


def test_qkv_row_order_pairs_rope_partners():
    order = step.qkv_row_order(2, 1, 128).numpy()
    assert sorted(order.tolist()) == list(range(4 * 128))
    blocks = order.reshape(-1, 16)
    for b, rows in enumerate(blocks):
        hd, i = b // 8, b % 8
        np.testing.assert_array_equal(rows[:8], hd * 128 + 8 * i + np.arange(8))
        np.testing.assert_array_equal(rows[8:], hd * 128 + 64 + 8 * i + np.arange(8))


# --------------------------------------------------------------------- W4
def stage_w4(x):
    """sb_step.cu stage_w4: per 8-value word 16 bytes [bf16 (x0,x4) | bf16
    (x2,x6) | fp16 (x1,x5) | fp16 (x3,x7)] and per group (O, X)."""
    n = x.shape[0]
    xs = np.zeros(n * 2, np.uint8)
    om = []
    for v in range(n // 8):
        f = x[v * 8:(v + 1) * 8]
        words = [bf16_bits(f[0]) | (bf16_bits(f[4]) << 16), bf16_bits(f[2]) | (bf16_bits(f[6]) << 16),
                 fp16_bits(f[1]) | (fp16_bits(f[5]) << 16), fp16_bits(f[3]) | (fp16_bits(f[7]) << 16)]
        xs[v * 16:(v + 1) * 16] = np.frombuffer(np.array(words, "<u4").tobytes(), np.uint8)
    for gi in range(n // 64):
        f = x[gi * 64:(gi + 1) * 64]
        h = f.copy()
        h[1::2] = f[1::2].astype(np.float16)
        om.append((128.0 * h[0::2].sum() + 64.0 * h[1::2].sum(), f.sum()))
    return xs, om


def emulate_w4_tile(tile, mats, ngroups, xs, om):
    """sb_step.cu w4_tile: per matrix the 16 rows' partial sums."""
    zero = np.zeros(128, np.uint8)
    rounds = (ngroups + 7) // 8
    meta = tile[mats * ngroups * 512:]
    sc = np.frombuffer(meta[:rounds * mats * 256].tobytes(), "<u2")
    bi = np.frombuffer(meta[rounds * mats * 256:rounds * mats * 512].tobytes(), "<u2")
    res = np.zeros((mats, 16))
    for r in range(rounds):
        acc = np.zeros((mats, 16, 8))
        jn = min(8, ngroups - 8 * r)
        for j in range(jn):
            gi = 8 * r + j
            for m in range(mats):
                la = [[], []]
                lb = [[], []]
                for L in range(32):
                    g, c = L >> 2, L & 3
                    bp = xs[gi * 128:(gi + 1) * 128] if g == j else zero
                    b0 = u32s(bp[c * 16:c * 16 + 16])
                    b1 = u32s(bp[64 + c * 16:64 + c * 16 + 16])
                    a = u32s(tile[(gi * mats + m) * 512 + L * 16:][:16])

                    def conv(w):
                        s = int(w) >> 8
                        w = int(w)
                        return [lop_and_or(w, 0x000F000F, 0x43004300), lop_and_or(w, 0x00F000F0, 0x54005400),
                                lop_and_or(s, 0x000F000F, 0x43004300), lop_and_or(s, 0x00F000F0, 0x54005400)]

                    for half, (wg, wh, bb) in enumerate(((a[0], a[1], b0), (a[2], a[3], b1))):
                        tg, th = conv(wg), conv(wh)
                        # bf16 MMA of (n0,n4)/(n2,n6), fp16 MMA of (n1,n5)/(n3,n7)
                        lanes_bf = [halves(tg[0], "bf16"), halves(th[0], "bf16"), halves(tg[2], "bf16"),
                                    halves(th[2], "bf16")]
                        lanes_hf = [halves(tg[1], "f16"), halves(th[1], "f16"), halves(tg[3], "f16"),
                                    halves(th[3], "f16")]
                        la[half].append((lanes_bf, lanes_hf))
                        lb[half].append(((halves(bb[0], "bf16"), halves(bb[1], "bf16")),
                                         (halves(bb[2], "f16"), halves(bb[3], "f16"))))
                for half in range(2):
                    mma(acc[m], [la[half][L][0] for L in range(32)], [lb[half][L][0] for L in range(32)])
                    mma(acc[m], [la[half][L][1] for L in range(32)], [lb[half][L][1] for L in range(32)])
        for m in range(mats):
            base = (r * mats + m) * 128
            for row in range(16):
                for e in range(8):
                    if e >= jn:
                        continue
                    s = float(formats.bf16_from_bits(np.array([sc[base + row * 8 + e]]))[0])
                    b = float(formats.bf16_from_bits(np.array([bi[base + row * 8 + e]]))[0])
                    O, X = om[8 * r + e]
                    res[m, row] += s * (acc[m, row, e] - O) + b * X
    return res


@pytest.mark.parametrize("mats,ngroups,n,k", [(2, 8, 16, 512), (1, 3, 32, 384), (1, 19, 16, 1216)])
def test_w4_stream_tiles_reproduce_affine_dot_products(mats, ngroups, n, k):
    rng = np.random.default_rng(1 + ngroups)
    trip = []
    dense = []
    for _ in range(mats):
        wf = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        packed, s_bits, b_bits = quant.quantize_affine_minmax(wf, 64, 4)
        trip.append((torch.from_numpy(packed.view(np.int32)), torch.from_numpy(s_bits.view(np.int16)).view(torch.bfloat16),
                     torch.from_numpy(b_bits.view(np.int16)).view(torch.bfloat16)))
        dense.append(quant.dequantize_affine(packed, formats.bf16_from_bits(s_bits), formats.bf16_from_bits(b_bits), 64, 4))
    x = formats.round_bf16(rng.standard_normal(k).astype(np.float32)).astype(np.float64)
    stream = step.pack_w4(trip, ngroups).numpy()
    rounds = (ngroups + 7) // 8
    tile_bytes = mats * ngroups * 512 + 2 * rounds * mats * 256
    chunks = k // 64 // ngroups
    assert stream.size == (n // 16) * chunks * tile_bytes
    for rb in range(n // 16):
        for ch in range(chunks):
            t = stream[(rb * chunks + ch) * tile_bytes:][:tile_bytes]
            xc = x[ch * ngroups * 64:(ch + 1) * ngroups * 64]
            xs, om = stage_w4(xc)
            got = emulate_w4_tile(t, mats, ngroups, xs, om)
            for m in range(mats):
                ref = dense[m][rb * 16:(rb + 1) * 16, ch * ngroups * 64:(ch + 1) * ngroups * 64] @ xc
                np.testing.assert_allclose(got[m], ref, rtol=1e-6, atol=1e-6)


# ------------------------------------------------------------------- BF16
def test_bf16_stream_tiles_reproduce_dot_products():
    rng = np.random.default_rng(2)
    v, k, ck = 40, 128, 32  # 40 rows: padded to 48
    w = formats.round_bf16(rng.standard_normal((v, k)).astype(np.float32))
    x = formats.round_bf16(rng.standard_normal(k).astype(np.float32)).astype(np.float64)
    wt = torch.from_numpy(formats.bf16_bits(w).view(np.int16)).view(torch.bfloat16)
    stream = step.pack_bf16(wt, ck).numpy()
    tile_bytes = 16 * ck * 2
    assert stream.size == 3 * (k // ck) * tile_bytes
    wp = np.concatenate([w, np.zeros((8, k), np.float32)])
    for rb in range(3):
        for ch in range(k // ck):
            t = stream[(rb * (k // ck) + ch) * tile_bytes:][:tile_bytes]
            acc = np.zeros((16, 8))
            for j in range(ck // 16):
                la, lb = [], []
                for L in range(32):
                    c = L & 3
                    a = u32s(t[j * 512 + L * 16:][:16])
                    xb = x[ch * ck + 16 * j + 4 * c:][:4]
                    la.append([halves(a[0], "bf16"), halves(a[1], "bf16"), halves(a[2], "bf16"), halves(a[3], "bf16")])
                    lb.append([(xb[0], xb[1]), (xb[2], xb[3])])
                mma(acc, la, lb)
            ref = wp[rb * 16:(rb + 1) * 16, ch * ck:(ch + 1) * ck].astype(np.float64) @ x[ch * ck:(ch + 1) * ck]
            np.testing.assert_allclose(acc[:, 0], ref, rtol=0, atol=1e-9)
