"""GPU kernels vs the CPU oracle (restatement of the reference's scalar path).

Bars: integer block dots bit-exact (q8.rs:2699-2702, 505, 1350-1368); the activation
quantiser bit-exact (inference.rs:991-1029); f32 row sums bit-exact too: the GEMVs fold
the per-block terms in block order exactly as the reference's rows do
(inference.rs:1150-1160, 2659-2664, 3129-3133), so every output equals the oracle's f32
bits (stricter than the reference's own matmul tests, 1e-5 absolute on O(1) values,
inference.rs:6068-6075)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BB = {2: 18, 8: 34, 12: 144, 14: 210}
BE = {2: 32, 8: 32, 12: 256, 14: 256}


def random_blocks(qtype, rows, cols, seed):
    """Random raw GGUF blocks: arbitrary nibble / int8 / scale bytes, finite f16 scales."""
    rng = np.random.default_rng(seed)
    nb = rows * (cols // BE[qtype])
    raw = rng.integers(0, 256, size=(nb, BB[qtype]), dtype=np.uint8)
    scales = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint16)
    at = 208 if qtype == 14 else 0   # Q6_K keeps d at the end of its block
    raw[:, at] = scales & 0xFF
    raw[:, at + 1] = scales >> 8
    if qtype == 12:
        dmin = (np.abs(rng.standard_normal(nb)) * 0.003).astype(np.float16).view(np.uint16)
        raw[:, 2] = dmin & 0xFF
        raw[:, 3] = dmin >> 8
    return raw.reshape(-1)


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_quantizer_bit_exact(ncm, orc, cuda):
    torch = cuda
    rng = np.random.default_rng(1)
    for n in [32, 64, 2048, 14336]:
        x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 30.0])).astype(np.float32)
        x[:32] = 0.0                       # zero block -> scale 0, all-zero values
        if n >= 96:
            x[64:96] = 0.5 * np.arange(32) - 8.0   # exact .5 ties (round half away from zero)
        q_ref, s_ref = orc.quantize_q8_0(x)
        xd = dev(torch, x)
        qd = torch.zeros(n, dtype=torch.int8, device="cuda")
        sd = torch.zeros(n // 32, dtype=torch.float32, device="cuda")
        ncm.quantize_f32_to_q8_0(xd.data_ptr(), n, qd.data_ptr(), sd.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(qd.cpu().numpy(), q_ref)
        assert np.array_equal(sd.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))


@pytest.mark.parametrize("qtype", [2, 8, 12])
@pytest.mark.parametrize("rows,cols", [(5, 256), (64, 2048), (33, 14336), (9, 28672), (7, 96), (3, 32)])
def test_block_dots_bit_exact(ncm, orc, cuda, qtype, rows, cols):
    torch = cuda
    if cols % BE[qtype]:
        pytest.skip("Q4_K needs 256-aligned columns")
    w = random_blocks(qtype, rows, cols, seed=rows * 7 + qtype)
    x = np.random.default_rng(cols).standard_normal(cols).astype(np.float32)
    xq, xs = orc.quantize_q8_0(x)
    ref = orc.block_dots(qtype, w, rows, cols, xq)
    out = torch.zeros(ref.size, dtype=torch.int32, device="cuda")
    wd, xqd = dev(torch, w), dev(torch, xq)
    ncm.block_dots(out.data_ptr(), xqd.data_ptr(), wd.data_ptr(), rows, cols, qtype)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)


SHAPES = [(3, 64), (7, 256), (5, 32), (300, 96), (2049, 160), (64, 2080), (64, 2048), (2048, 2048), (4097, 3072), (1024, 4096), (512, 8192), (200, 14336),
          (96, 28672), (1, 8192)]


@pytest.mark.parametrize("qtype", [2, 8, 12, 14])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matmul_quantized_vs_oracle(ncm, orc, cuda, qtype, rows, cols):
    torch = cuda
    if cols % BE[qtype]:
        pytest.skip("K-quants need 256-aligned columns")
    w = random_blocks(qtype, rows, cols, seed=rows + cols + qtype)
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    xq, xs = orc.quantize_q8_0(x)
    ref = orc.matmul(qtype, w, rows, cols, xq, xs)
    out = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    wd, xqd, xsd = dev(torch, w), dev(torch, xq), dev(torch, xs)
    ncm.matmul_quantized(out.data_ptr(), xqd.data_ptr(), xsd.data_ptr(), wd.data_ptr(), rows, cols, qtype)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.all(np.isfinite(got))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), float(np.max(np.abs(got - ref)))


def test_matmul_reference_kat_shape(ncm, orc, cuda):
    """inference.rs:6028-6076: rows 3, cols 64, q4_block(scale, seed) weights, x = (5i % 61) - 30."""
    torch = cuda

    def q4_block(scale_bits, seed):
        b = np.zeros(18, dtype=np.uint8)
        b[0], b[1] = scale_bits & 0xFF, scale_bits >> 8
        for i in range(16):
            lo = (seed + i * 3) % 16
            hi = (seed + (i + 16) * 3) % 16
            b[2 + i] = lo | (hi << 4)
        return b

    w = np.concatenate([q4_block(s, k + 1) for k, s in enumerate([0x3800, 0x3C00, 0x4000, 0x4200, 0x4400, 0x4600])])
    xq = np.array([((i * 5) % 61) - 30 for i in range(64)], dtype=np.int8)
    xs = np.array([0.25, 0.5], dtype=np.float32)
    ref = orc.matmul(2, w, 3, 64, xq, xs)
    # the reference test's dequantised expectation
    exp = []
    for r in range(3):
        s = np.float32(0.0)
        for b in range(2):
            blk = w[(r * 2 + b) * 18:(r * 2 + b + 1) * 18]
            d = np.frombuffer(blk[:2].tobytes(), dtype=np.float16)[0].astype(np.float32)
            sc = np.float32(d * xs[b])
            nib = [int(v) for v in blk[2:18]]
            vals = [(b & 15) - 8 for b in nib] + [(b >> 4) - 8 for b in nib]
            for i in range(32):
                s = np.float32(s + np.float32(sc * np.float32(vals[i])) * np.float32(xq[b * 32 + i]))
        exp.append(s)
    assert np.allclose(ref, exp, atol=1e-5)
    out = torch.zeros(3, dtype=torch.float32, device="cuda")
    keep = [dev(torch, xq), dev(torch, xs), dev(torch, w)]   # device buffers must outlive the launch
    ncm.matmul_quantized(out.data_ptr(), keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), 3, 64, 2)
    torch.cuda.synchronize()
    assert np.allclose(out.cpu().numpy(), exp, atol=1e-5)


@pytest.mark.parametrize("qtype", [2, 8, 12])
@pytest.mark.parametrize("ntok,rows,cols", [(1, 300, 4096), (4, 300, 4096), (5, 300, 4096), (8, 64, 28672),
                                            (5, 40, 14336), (8, 100, 2048)])
def test_matmul_batch_vs_single(ncm, orc, cuda, qtype, ntok, rows, cols):
    """inference.rs:6866-6913 / 7282-7327: each batch row equals the single-token result,
    bit for bit; 8 rows of 28672 columns (the 70B down projection) are too wide for shared
    memory and are read in place from global memory."""
    torch = cuda
    w = random_blocks(qtype, rows, cols, seed=ntok + qtype)
    x = np.random.default_rng(ntok).standard_normal((ntok, cols)).astype(np.float32)
    qs = [orc.quantize_q8_0(x[t]) for t in range(ntok)]
    xq = np.concatenate([q for q, _ in qs])
    xs = np.concatenate([s for _, s in qs])
    ref = orc.matmul_batch(qtype, w, rows, cols, ntok, xq, xs)
    out = torch.zeros(ntok * rows, dtype=torch.float32, device="cuda")
    keep = [dev(torch, xq), dev(torch, xs), dev(torch, w)]
    ncm.matmul_quantized_batch(out.data_ptr(), keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), ntok,
                               rows, cols, qtype)
    torch.cuda.synchronize()
    got = out.cpu().numpy().reshape(ntok, rows)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), float(np.max(np.abs(got - ref)))
    for t in range(ntok):
        single = orc.matmul(qtype, w, rows, cols, xq[t * cols:(t + 1) * cols], xs[t * cols // 32:(t + 1) * cols // 32])
        assert np.array_equal(single, ref[t])


def test_rms_norm_silu_attention(ncm, orc, cuda):
    torch = cuda
    L = orc.lib()
    rng = np.random.default_rng(3)
    n = 3072
    x = rng.standard_normal(n).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    ref = np.zeros(n, dtype=np.float32)
    L.orc_rms_norm(orc.ptr(ref), orc.ptr(x), orc.ptr(w), n, np.float32(1e-5))
    out = torch.zeros(n, dtype=torch.float32, device="cuda")
    xd, wd = dev(torch, x), dev(torch, w)
    ncm.rms_norm(out.data_ptr(), xd.data_ptr(), wd.data_ptr(), n, 1e-5)
    torch.cuda.synchronize()
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-6)

    g = (rng.standard_normal(n) * 4).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    ref = np.zeros(n, dtype=np.float32)
    L.orc_silu_mul(orc.ptr(ref), orc.ptr(g), orc.ptr(u), n)
    gd, ud = dev(torch, g), dev(torch, u)
    ncm.fused_silu_mul(out.data_ptr(), gd.data_ptr(), ud.data_ptr(), n)
    torch.cuda.synchronize()
    assert np.allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-6)

    for heads, kvh, hd, pos in [(4, 2, 64, 0), (32, 8, 64, 47), (24, 8, 128, 200), (64, 8, 128, 1023)]:
        kvw = kvh * hd
        q = rng.standard_normal(heads * hd).astype(np.float32)
        kc = rng.standard_normal((pos + 1) * kvw).astype(np.float32)
        vc = rng.standard_normal((pos + 1) * kvw).astype(np.float32)
        ref = np.zeros(heads * hd, dtype=np.float32)
        L.orc_attention(orc.ptr(ref), orc.ptr(q), orc.ptr(kc), orc.ptr(vc), pos, heads, kvh, hd, kvw)
        o = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
        qd, kd, vd = dev(torch, q), dev(torch, kc), dev(torch, vc)
        ncm.attention(o.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pos, heads, kvh, hd)
        assert np.allclose(o.cpu().numpy(), ref, rtol=1e-4, atol=1e-5), (heads, kvh, hd, pos)


def test_peer_wait_times_out_cleanly(ncm, cuda):
    """Bounded device wait on a flag nobody sets returns NCM_ETIMEOUT; context stays usable."""
    import time
    t0 = time.time()
    st = ncm.peer_timeout_selftest(0, 200_000_000)
    dt = time.time() - t0
    assert st == 3
    assert dt < 5.0
    x = cuda.ones(4, device="cuda")
    assert float(x.sum()) == 4.0


def _rms_cases(rng):
    yield "normal", rng.standard_normal(3072).astype(np.float32)
    yield "normal_8192", rng.standard_normal(8192).astype(np.float32)
    yield "normal_odd", rng.standard_normal(3001).astype(np.float32)
    yield "segmented", rng.standard_normal(20011).astype(np.float32)
    yield "one", np.array([3.0], dtype=np.float32)
    yield "short", rng.standard_normal(33).astype(np.float32)
    yield "ints_ties", rng.integers(-4096, 4096, size=8192).astype(np.float32)
    yield "small_ints", rng.integers(-7, 8, size=4096).astype(np.float32)
    yield "powers_of_two", np.ldexp(1.0, rng.integers(-30, 20, size=4096)).astype(np.float32)
    yield "wide_range", (10.0 ** rng.uniform(-20, 5, size=4096) * rng.choice([-1, 1], size=4096)).astype(np.float32)
    x = np.zeros(4096, dtype=np.float32)
    x[1000::997] = 1.5
    yield "sparse", x
    x = rng.standard_normal(4096).astype(np.float32)
    x[:2000] = 1e-30
    yield "tiny_prefix", x
    x = rng.standard_normal(2048).astype(np.float32) * 1e-3
    x[0] = 1e4
    yield "big_first", x
    yield "quantised", (np.round(rng.standard_normal(3072) * 40) / 64).astype(np.float32)


def test_rms_norm_bit_exact_sequential_sum(ncm, orc, cuda):
    """The device sum of squares reproduces the reference's sequential f32 fold bit for bit
    (inference.rs:697-706) on adversarial inputs: exact ties, binade crossings, zeros,
    tiny and huge terms, lengths that are not multiples of 32 and beyond one segment."""
    torch = cuda
    L = orc.lib()
    rng = np.random.default_rng(17)
    for name, x in _rms_cases(rng):
        n = x.size
        w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        ref = np.zeros(n, dtype=np.float32)
        L.orc_rms_norm(orc.ptr(ref), orc.ptr(x), orc.ptr(w), n, np.float32(1e-5))
        out = torch.zeros(n, dtype=torch.float32, device="cuda")
        xd, wd = dev(torch, x), dev(torch, w)
        ncm.rms_norm(out.data_ptr(), xd.data_ptr(), wd.data_ptr(), n, 1e-5)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name


def test_attention_bit_exact(ncm, orc, cuda):
    """Scores, softmax (sequential denominator, glibc-exact exp) and the V accumulation
    follow inference.rs:4242-4292 term by term: outputs equal the oracle's bit for bit."""
    torch = cuda
    L = orc.lib()
    rng = np.random.default_rng(23)
    for heads, kvh, hd, pos in [(4, 2, 64, 0), (32, 8, 64, 47), (24, 8, 128, 200), (32, 8, 128, 2500)]:
        kvw = kvh * hd
        q = rng.standard_normal(heads * hd).astype(np.float32)
        kc = rng.standard_normal((pos + 1) * kvw).astype(np.float32) * 0.3
        vc = rng.standard_normal((pos + 1) * kvw).astype(np.float32)
        ref = np.zeros(heads * hd, dtype=np.float32)
        L.orc_attention(orc.ptr(ref), orc.ptr(q), orc.ptr(kc), orc.ptr(vc), pos, heads, kvh, hd, kvw)
        o = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
        qd, kd, vd = dev(torch, q), dev(torch, kc), dev(torch, vc)
        ncm.attention(o.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pos, heads, kvh, hd)
        torch.cuda.synchronize()
        assert np.array_equal(o.cpu().numpy().view(np.uint32), ref.view(np.uint32)), (heads, kvh, hd, pos)


@pytest.mark.parametrize("kind", [1, 2])
def test_attention_f16_q8_cache_bit_exact(ncm, orc, cuda, kind):
    """apply_attention_head_f16 / _q8_0 (inference.rs:4319-4458) over caches stored the
    reference's way (truncating f16 per value; Q8_0 blocks with a truncated f16 scale):
    outputs equal the oracle's bit for bit."""
    torch = cuda
    L = orc.lib()
    rng = np.random.default_rng(31 + kind)
    for heads, kvh, hd, pos in [(4, 2, 64, 0), (32, 8, 64, 47), (24, 8, 128, 200), (64, 8, 128, 1100)]:
        kvw = kvh * hd
        q = rng.standard_normal(heads * hd).astype(np.float32)
        kf = (rng.standard_normal((pos + 1) * kvw) * 0.3).astype(np.float32)
        vf = rng.standard_normal((pos + 1) * kvw).astype(np.float32)
        if kind == 1:
            kc = np.zeros((pos + 1) * kvw, dtype=np.uint16)
            vc = np.zeros((pos + 1) * kvw, dtype=np.uint16)
            L.orc_kv_store_f16(orc.ptr(kf), kf.size, orc.ptr(kc))
            L.orc_kv_store_f16(orc.ptr(vf), vf.size, orc.ptr(vc))
        else:
            kc = np.zeros((pos + 1) * kvw // 32 * 34, dtype=np.uint8)
            vc = np.zeros((pos + 1) * kvw // 32 * 34, dtype=np.uint8)
            L.orc_kv_quantize_row_q8_0(orc.ptr(kf), kf.size, orc.ptr(kc))
            L.orc_kv_quantize_row_q8_0(orc.ptr(vf), vf.size, orc.ptr(vc))
        ref = np.zeros(heads * hd, dtype=np.float32)
        L.orc_attention_kv(kind, orc.ptr(ref), orc.ptr(q), orc.ptr(kc), orc.ptr(vc), pos, heads, kvh, hd, kvw)
        o = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
        qd, kd, vd = dev(torch, q), dev(torch, kc), dev(torch, vc)
        ncm.attention_kv(kind, o.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), pos, heads, kvh, hd)
        torch.cuda.synchronize()
        assert np.array_equal(o.cpu().numpy().view(np.uint32), ref.view(np.uint32)), (kind, heads, kvh, hd, pos)
