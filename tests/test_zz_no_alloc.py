"""ncm_attention_noalloc: attention for callers that may not allocate device memory.

Such callers (hosts that hand out a fixed device-memory budget at start-up and forbid
allocation afterwards, or latency-critical loops that a device-synchronising cudaMalloc
would stall) get the same result as ncm_attention from a fixed in-library scratch array.  This file is
collected last so that a failure here does not hide the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _fn(ncm):
    f = ncm.lib().ncm_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    return f


def _case(torch, rng, heads, kvh, hd, pos):
    kvw = kvh * hd
    q = torch.from_numpy(rng.standard_normal(heads * hd).astype(np.float32)).cuda()
    kc = torch.from_numpy((rng.standard_normal((pos + 1) * kvw) * 0.3).astype(np.float32)).cuda()
    vc = torch.from_numpy(rng.standard_normal((pos + 1) * kvw).astype(np.float32)).cuda()
    return q, kc, vc


def test_noalloc_attention_matches_allocating_entry_point(ncm, cuda):
    """Bit-identical to ncm_attention (the same kernels), on two calls in a row that share
    the scratch (the second shorter than the first), and on the largest accepted request
    (heads * (pos + 1) = 262144 exactly).  The first call happens before any allocating
    entry point has run in a fresh process, so its own set-up must make exp glibc-exact."""
    torch = cuda
    noalloc = _fn(ncm)
    rng = np.random.default_rng(11)
    for heads, kvh, hd, pos in [(32, 8, 64, 300), (24, 8, 128, 47), (16, 8, 128, 16383)]:
        q, kc, vc = _case(torch, rng, heads, kvh, hd, pos)
        got = torch.full((heads * hd,), float("nan"), dtype=torch.float32, device="cuda")
        st = noalloc(got.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos, heads, kvh, hd, None)
        assert st == 0, ncm.lib().ncm_last_error().decode()
        torch.cuda.synchronize()
        ref = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
        ncm.attention(ref.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos, heads, kvh, hd)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.cpu().numpy().view(np.uint32)), (heads, pos)


def test_noalloc_attention_equals_oracle(ncm, orc, cuda):
    """The reference's apply_attention_heads (oracle restatement), bit for bit."""
    torch = cuda
    noalloc = _fn(ncm)
    rng = np.random.default_rng(5)
    heads, kvh, hd, pos = 32, 8, 128, 700
    q, kc, vc = _case(torch, rng, heads, kvh, hd, pos)
    got = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
    assert noalloc(got.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos, heads, kvh, hd, None) == 0
    torch.cuda.synchronize()
    ref = np.zeros(heads * hd, dtype=np.float32)
    qn, kn, vn = q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy()
    orc.lib().orc_attention(orc.ptr(ref), orc.ptr(qn), orc.ptr(kn), orc.ptr(vn), pos, heads, kvh, hd, kvh * hd)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_noalloc_attention_rejects_oversized_request(ncm, cuda):
    noalloc = _fn(ncm)
    x = cuda.zeros(64, dtype=cuda.float32, device="cuda")
    # 17 heads of 16384 positions: past the scratch
    st = noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 16383, 17, 17, 32, None)
    assert st == 1
    assert "exceeds the fixed scratch" in ncm.lib().ncm_last_error().decode()
    # positions past ncm_attention's limit are rejected even when the scratch would fit
    st = noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 16384, 8, 8, 32, None)
    assert st == 1
