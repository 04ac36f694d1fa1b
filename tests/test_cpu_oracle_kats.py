"""The CPU oracle pinned against the reference's own known-answer tests (no GPU).

Each test restates one reference unit test for this path (file:line of the test in the
reference crate) and runs it against the oracle (oracle/oracle.c), which the GPU parity
tests then use as the checker.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.cpu


def f16_bytes(bits):
    return [bits & 0xFF, bits >> 8]


def test_q8_0_block_decodes_gguf_layout(orc):
    """q8.rs:4486-4500: scale 0x3800 -> 0.5, values idx - 16."""
    L = orc.lib()
    blk = np.array(f16_bytes(0x3800) + [(i - 16) & 0xFF for i in range(32)], dtype=np.uint8)
    out = np.zeros(32, dtype=np.float32)
    L.orc_dequant_row(8, orc.ptr(blk), 32, orc.ptr(out))
    assert out[0] == -16 * 0.5 and out[31] == 15 * 0.5
    assert L.orc_f16_to_f32(0x3800) == 0.5


def test_q4_0_block_decodes_low_then_high_nibbles(orc):
    """q8.rs:4514-4530: byte i = i | (15 - i) << 4, scale 0x3c00 = 1.0."""
    blk = np.array(f16_bytes(0x3C00) + [i | ((15 - i) << 4) for i in range(16)], dtype=np.uint8)
    vals = np.zeros(32, dtype=np.int8)
    orc.lib().orc_q4_0_unpack(orc.ptr(blk), orc.ptr(vals))
    assert (vals[0], vals[15], vals[16], vals[31]) == (-8, 7, 7, -8)
    assert list(vals[:16]) == [i - 8 for i in range(16)]
    assert list(vals[16:]) == [7 - i for i in range(16)]


def test_q4_0_q8_0_dot_matches_unpacked(orc):
    """q8.rs:4533-4566: fixed nibble bytes, q8 = idx - 16; dot == sum(unpacked * q8)."""
    L = orc.lib()
    qs = [0x80, 0x91, 0xA2, 0xB3, 0xC4, 0xD5, 0xE6, 0xF7, 0x08, 0x19, 0x2A, 0x3B, 0x4C, 0x5D, 0x6E, 0x7F]
    blk = np.array(f16_bytes(0x3C00) + qs, dtype=np.uint8)
    q8 = np.array([i - 16 for i in range(32)], dtype=np.int8)
    unpacked = np.array([(b & 15) - 8 for b in qs] + [(b >> 4) - 8 for b in qs], dtype=np.int32)
    assert L.orc_block_dot(2, orc.ptr(blk), orc.ptr(q8)) == int(np.dot(unpacked, q8.astype(np.int32)))


def test_f16_decode_edges_and_exhaustive(orc):
    """q8.rs:5156-5175: edge values and all 65536 bit patterns (numpy's exact widening)."""
    L = orc.lib()
    assert L.orc_f16_to_f32(0x0000) == 0.0
    assert np.signbit(np.float32(L.orc_f16_to_f32(0x8000)))
    assert L.orc_f16_to_f32(0x3C00) == 1.0 and L.orc_f16_to_f32(0xBC00) == -1.0
    assert L.orc_f16_to_f32(0x0400) == np.float32(0.000061035156)
    assert L.orc_f16_to_f32(0x7C00) == np.inf
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([L.orc_f16_to_f32(int(b)) for b in bits], dtype=np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f32_to_f16_truncating_encode(orc):
    """q8.rs:5178-5195 representative values, NaN stays NaN."""
    L = orc.lib()
    cases = [(0.0, 0x0000), (-0.0, 0x8000), (1.0, 0x3C00), (-1.0, 0xBC00), (0.5, 0x3800), (2.0, 0x4000),
             (65504.0, 0x7BFF), (np.inf, 0x7C00), (-np.inf, 0xFC00)]
    for v, b in cases:
        assert L.orc_f32_to_f16(v) == b, v
    n = L.orc_f32_to_f16(float("nan"))
    assert n & 0x7C00 == 0x7C00 and n & 0x03FF != 0


def test_q4_0_matrix_quantizer_reconstructs_within_scale(orc):
    """q8.rs:4187-4245: 8 x 64 values (zero row, outlier block, mixed ramp)."""
    rows, cols = 8, 64
    v = np.zeros((rows, cols), dtype=np.float32)
    for r in range(rows):
        for c in range(cols):
            idx = r * cols + c
            if r == 0:
                v[r, c] = 0.0
            elif r == 1 and c // 32 == 0:
                v[r, c] = -12.5 if c == 0 else (0.25 * c if c % 2 == 0 else -0.125 * c)
            else:
                v[r, c] = (1.0 if (r + c) % 2 == 0 else -1.0) * (np.float32(0.03) * np.float32(idx) + np.float32(0.5))
    blocks = np.zeros(rows * (cols // 32) * 18, dtype=np.uint8)
    orc.lib().orc_quantize_matrix_q4_0(orc.ptr(v), rows, cols, orc.ptr(blocks))
    for r in range(rows):
        for b in range(cols // 32):
            blk = blocks[(r * 2 + b) * 18:(r * 2 + b + 1) * 18]
            d = np.frombuffer(blk[:2].tobytes(), dtype=np.float16)[0].astype(np.float32)
            q = np.zeros(32, dtype=np.int8)
            orc.lib().orc_q4_0_unpack(orc.ptr(np.ascontiguousarray(blk)), orc.ptr(q))
            err = np.abs(q.astype(np.float32) * d - v[r, 32 * b:32 * b + 32])
            assert np.all(err <= abs(d) + 1e-4), (r, b)
    # all-zero block: scale == 0.0 (the quantiser writes -0.0, which compares equal), values 0
    assert np.frombuffer(blocks[:2].tobytes(), dtype=np.float16)[0] == 0.0
    q = np.zeros(32, dtype=np.int8)
    orc.lib().orc_q4_0_unpack(orc.ptr(blocks[:18].copy()), orc.ptr(q))
    assert not q.any()


def k_scales(seed):
    return [(seed + i * 5) % 64 for i in range(12)]


def q4_k_block(scale_bits, min_bits, seed):
    """inference.rs:5519-5573 test helpers k_scales / q4_k_block."""
    vals = [((seed + i * 3) % 16) | (((seed + i * 7) % 16) << 4) for i in range(128)]
    return np.array(f16_bytes(scale_bits) + f16_bytes(min_bits) + k_scales(seed) + vals, dtype=np.uint8)


def test_q4_k_matmul_matches_dequantized(orc):
    """inference.rs:6517-6559: 2 rows x 512 columns, 1e-4 absolute."""
    L = orc.lib()
    rows, cols = 2, 512
    xq = np.array([((i * 5) % 61) - 30 for i in range(cols)], dtype=np.int8)
    xs = np.array([0.125 + i * 0.03125 for i in range(cols // 32)], dtype=np.float32)
    w = np.concatenate([q4_k_block(0x3800, 0x3000, 1), q4_k_block(0x3C00, 0x3400, 2),
                        q4_k_block(0x4000, 0x3800, 3), q4_k_block(0x4200, 0x3A00, 4)])
    got = orc.matmul(12, w, rows, cols, xq, xs)
    for r in range(rows):
        s = np.float32(0.0)
        for b in range(2):
            vals = np.zeros(256, dtype=np.float32)
            L.orc_dequant_row(12, orc.ptr(w[(r * 2 + b) * 144:(r * 2 + b + 1) * 144].copy()), 256, orc.ptr(vals))
            for i in range(256):
                s = np.float32(s + vals[i] * np.float32(xq[b * 256 + i]) * xs[(b * 256 + i) // 32])
        assert abs(got[r] - s) < 1e-4, (r, got[r], s)


def test_q4_k_scale_min_unpacking(orc):
    """q8.rs:4708-4727 preloaded == scalar: the dot over a fixed block equals a float64
    evaluation of the published Q4_K formula (d*sc_j*sum(q*x) - dmin*m_j*sum(x)) * x_s."""
    L = orc.lib()
    scales = [(i * 7 + 11) % 64 for i in range(12)]
    vals = [((i * 3 + 5) % 16) | (((i * 11 + 13) % 16) << 4) for i in range(128)]
    blk = np.array(f16_bytes(0x3C00) + f16_bytes(0x3800) + scales + vals, dtype=np.uint8)
    x = np.array([((i * 13 + 17) % 127) - 63 for i in range(256)], dtype=np.int8)
    xs = np.array([0.015625 * (1 + (i % 5)) for i in range(8)], dtype=np.float32)

    def scale_min(j):
        if j < 4:
            return scales[j] & 63, scales[j + 4] & 63
        return (scales[j + 4] & 0x0F) | ((scales[j - 4] >> 6) << 4), (scales[j + 4] >> 4) | ((scales[j] >> 6) << 4)

    ref = 0.0
    for j in range(8):
        sc, m = scale_min(j)
        chunk, half = j // 2, j % 2
        q = [(vals[32 * chunk + l] >> (4 * half)) & 15 for l in range(32)]
        xx = x[32 * j:32 * j + 32].astype(np.int64)
        ref += float(xs[j]) * (1.0 * sc * float(np.dot(q, xx)) - 0.5 * m * float(xx.sum()))
    got = L.orc_q4_k_dot(orc.ptr(blk), orc.ptr(x), orc.ptr(xs))
    assert abs(got - ref) <= 1e-5 * max(1.0, abs(ref))


def test_q4_matmul_kat(orc):
    """inference.rs:6028-6076: rows 3, cols 64, q4_block(scale, seed), x = (5i % 61) - 30."""
    def q4_block(scale_bits, seed):
        return np.array(f16_bytes(scale_bits) + [((seed + i * 3) % 16) | (((seed + (i + 16) * 3) % 16) << 4)
                                                  for i in range(16)], dtype=np.uint8)
    w = np.concatenate([q4_block(s, k + 1) for k, s in enumerate([0x3800, 0x3C00, 0x4000, 0x4200, 0x4400, 0x4600])])
    xq = np.array([((i * 5) % 61) - 30 for i in range(64)], dtype=np.int8)
    xs = np.array([0.25, 0.5], dtype=np.float32)
    got = orc.matmul(2, w, 3, 64, xq, xs)
    for r in range(3):
        s = np.float32(0.0)
        for b in range(2):
            blk = w[(r * 2 + b) * 18:(r * 2 + b + 1) * 18]
            d = np.frombuffer(blk[:2].tobytes(), dtype=np.float16)[0].astype(np.float32)
            q = [(int(v) & 15) - 8 for v in blk[2:]] + [(int(v) >> 4) - 8 for v in blk[2:]]
            for i in range(32):
                s = np.float32(s + np.float32(d * q[i]) * np.float32(xq[b * 32 + i]) * xs[b])
        assert abs(got[r] - s) <= 1e-5 * max(1.0, abs(s))


@pytest.mark.parametrize("qtype", [2, 8, 12])
def test_batch_rows_equal_single_rows(orc, qtype):
    """inference.rs:6866-6913 / 7282-7327: each batch row equals the single-token GEMV."""
    rng = np.random.default_rng(qtype)
    rows, cols, ntok = 37, 512, 4
    nb = rows * cols // (256 if qtype == 12 else 32)
    bb = {2: 18, 8: 34, 12: 144}[qtype]
    w = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    sc = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint16)
    w[:, 0], w[:, 1] = sc & 0xFF, sc >> 8
    w = w.reshape(-1)
    x = rng.standard_normal((ntok, cols)).astype(np.float32)
    qs = [orc.quantize_q8_0(x[t]) for t in range(ntok)]
    xq = np.concatenate([q for q, _ in qs])
    xs = np.concatenate([s for _, s in qs])
    batch = orc.matmul_batch(qtype, w, rows, cols, ntok, xq, xs)
    for t in range(ntok):
        single = orc.matmul(qtype, w, rows, cols, xq[t * cols:(t + 1) * cols], xs[t * cols // 32:(t + 1) * cols // 32])
        assert np.array_equal(batch[t].view(np.uint32), single.view(np.uint32))


def test_activation_quantizer_rules(orc):
    """inference.rs:991-1029: scale = amax/127 (f32), round half away from zero, zero
    block -> scale 0 and values 0."""
    x = np.zeros(96, dtype=np.float32)
    x[32:64] = np.arange(32, dtype=np.float32) * 0.5 - 8.0       # exact .5 ties after scaling
    x[64:96] = np.linspace(-3, 3, 32, dtype=np.float32)
    q, s = orc.quantize_q8_0(x)
    assert s[0] == 0 and not q[:32].any()
    for b in (1, 2):
        blk = x[32 * b:32 * b + 32]
        scale = np.float32(np.max(np.abs(blk)) / np.float32(127.0))
        assert s[b] == scale
        inv = np.float32(1.0) / scale
        ref = np.clip(np.sign(blk * inv) * np.floor(np.abs(blk * inv) + 0.5), -127, 127).astype(np.int8)
        assert np.array_equal(q[32 * b:32 * b + 32], ref)


def test_rope_partial_dimension(orc):
    """inference.rs:7423-7440: rope_dim 2 of head_dim 4 rotates only the first pair."""
    d = np.array([1.0, 0.0, 10.0, 20.0], dtype=np.float32)
    orc.lib().orc_apply_rope(orc.ptr(d), 1, 1, 4, 2, np.float32(10000.0))
    assert abs(d[0] - np.cos(np.float32(1.0))) < 1e-6 and abs(d[1] - np.sin(np.float32(1.0))) < 1e-6
    assert d[2] == 10.0 and d[3] == 20.0


def test_argmax_first_max(orc):
    """inference.rs:4834-4845: strict '>' scan keeps the first maximum."""
    x = np.array([1.0, 3.0, 2.0, 3.0, -1.0], dtype=np.float32)
    assert orc.lib().orc_argmax(orc.ptr(x), x.size) == 1


# ---------------------------------------------------------------- Q6_K (oracle ahead of the GPU kernel)
def _q6_k_block(scale_bits, seed):
    """inference.rs:5589-5603 q6_k_block: ql[i] = (seed + 5i) mod 256, qh[i] = (seed + 7i)
    mod 256, scales[i] = (seed + 3i) mod 15 - 7, d = scale_bits."""
    i = np.arange(128)
    ql = ((seed + i * 5) % 256).astype(np.uint8)
    qh = ((seed + np.arange(64) * 7) % 256).astype(np.uint8)
    sc = (((seed + np.arange(16) * 3) % 15) - 7).astype(np.int8)
    return np.concatenate([ql, qh, sc.view(np.uint8), np.array([scale_bits & 0xFF, scale_bits >> 8], np.uint8)])


def test_q6_k_dequant_layout(orc):
    """q8.rs:4646-4666: ql[0] = 0x10, ql[32] = 0x02, qh[0] = 0b11_10_01_00, scales 1,
    d = 1.0 -> values[0] = -32, [32] = -14, [64] = 1, [96] = 16."""
    blk = np.zeros(210, dtype=np.uint8)
    blk[0], blk[32], blk[128] = 0x10, 0x02, 0b11100100
    blk[192:208] = 1
    blk[208], blk[209] = 0x00, 0x3c
    out = np.zeros(256, dtype=np.float32)
    orc.lib().orc_q6_k_dequant(orc.ptr(blk), orc.ptr(out))
    assert (out[0], out[32], out[64], out[96]) == (-32.0, -14.0, 1.0, 16.0)


def test_q6_k_matmul_matches_dequantized(orc):
    """inference.rs:6605-6640: rows 2, cols 512, x = (5i % 61) - 30, x scales 0.125 +
    i/32; the row sums agree with the dequantized reference within 1e-4."""
    rows, cols = 2, 512
    w = np.concatenate([_q6_k_block(b, s) for b, s in ((0x3800, 1), (0x3c00, 2), (0x4000, 3), (0x4200, 4))])
    x = ((np.arange(cols) * 5) % 61 - 30).astype(np.int8)
    xs = (0.125 + np.arange(cols // 32) * 0.03125).astype(np.float32)
    got = orc.matmul(14, w, rows, cols, x, xs)
    for r in range(rows):
        s = np.float32(0.0)
        for b in range(2):
            vals = np.zeros(256, dtype=np.float32)
            orc.lib().orc_q6_k_dequant(orc.ptr(np.ascontiguousarray(w[(r * 2 + b) * 210:(r * 2 + b + 1) * 210])),
                                       orc.ptr(vals))
            for i in range(256):
                xi = b * 256 + i
                s = np.float32(s + np.float32(np.float32(vals[i] * np.float32(x[xi])) * xs[xi // 32]))
        assert abs(float(got[r]) - float(s)) < 1e-4, (r, got[r], s)


# ---------------------------------------------------------------- F16 / Q8_0 KV caches (oracle ahead of the GPU)
def _kv_case(hd):
    heads, kvh, ctx, pos = 4, 2, 5, 4
    kvw = kvh * hd
    q = (np.arange(heads * hd, dtype=np.float32) * np.float32(0.017) - np.float32(0.25)).astype(np.float32)
    k = (np.float32(0.5) - np.arange(ctx * kvw, dtype=np.float32) * np.float32(0.009)).astype(np.float32)
    v = (np.arange(ctx * kvw, dtype=np.float32) * np.float32(0.013) - np.float32(0.4)).astype(np.float32)
    return heads, kvh, kvw, pos, q, k, v


def _attn(orc, kind, q, kc, vc, pos, heads, kvh, hd, kvw):
    out = np.zeros(heads * hd, dtype=np.float32)
    orc.lib().orc_attention_kv(kind, orc.ptr(out), orc.ptr(q), orc.ptr(kc), orc.ptr(vc), pos, heads, kvh, hd, kvw)
    return out


def test_f16_kv_attention_matches_decoded_cache(orc):
    """inference.rs:5812-5880: attention over an F16 cache equals the f32 path over the
    explicitly decoded cache (within 1e-6)."""
    hd = 8
    heads, kvh, kvw, pos, q, k, v = _kv_case(hd)
    k16, v16 = np.zeros(k.size, np.uint16), np.zeros(v.size, np.uint16)
    orc.lib().orc_kv_store_f16(orc.ptr(k), k.size, orc.ptr(k16))
    orc.lib().orc_kv_store_f16(orc.ptr(v), v.size, orc.ptr(v16))
    kd = np.array([orc.lib().orc_f16_to_f32(int(b)) for b in k16], dtype=np.float32)
    vd = np.array([orc.lib().orc_f16_to_f32(int(b)) for b in v16], dtype=np.float32)
    got = _attn(orc, 1, q, k16, v16, pos, heads, kvh, hd, kvw)
    want = _attn(orc, 0, q, kd, vd, pos, heads, kvh, hd, kvw)
    assert float(np.max(np.abs(got - want))) < 1e-6


def test_q8_0_kv_attention_matches_dequantized_cache(orc):
    """inference.rs:5886-5983: attention over a Q8_0 cache against the f32 path over the
    dequantised cache; q is quantised too, so within 5e-2."""
    hd = 32
    heads, kvh, kvw, pos, q, k, v = _kv_case(hd)
    kq, vq = np.zeros(k.size // 32 * 34, np.uint8), np.zeros(v.size // 32 * 34, np.uint8)
    orc.lib().orc_kv_quantize_row_q8_0(orc.ptr(k), k.size, orc.ptr(kq))
    orc.lib().orc_kv_quantize_row_q8_0(orc.ptr(v), v.size, orc.ptr(vq))

    def deq(blocks):
        b = blocks.reshape(-1, 34)
        s = np.array([orc.lib().orc_f16_to_f32(int(x[0]) | (int(x[1]) << 8)) for x in b], dtype=np.float32)
        return (b[:, 2:].view(np.int8).astype(np.float32) * s[:, None]).reshape(-1).astype(np.float32)

    got = _attn(orc, 2, q, kq, vq, pos, heads, kvh, hd, kvw)
    want = _attn(orc, 0, q, deq(kq), deq(vq), pos, heads, kvh, hd, kvw)
    assert float(np.max(np.abs(got - want))) < 5e-2
    # the store keeps the truncating f16 scale and round-half-away values
    blk = kq[:34]
    s = np.float32(np.max(np.abs(k[:32])) / np.float32(127.0))
    assert (int(blk[0]) | (int(blk[1]) << 8)) == orc.lib().orc_f32_to_f16(s)
