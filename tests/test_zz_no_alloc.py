"""ncm_attention_noalloc: attention for callers that may not allocate device memory.

Such callers (work captured into CUDA graphs, hosts with a fixed memory budget) get the
same result as ncm_attention from a fixed in-library scratch array.  This file is
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


def test_noalloc_attention_matches_allocating_entry_point(ncm, cuda):
    torch = cuda
    noalloc = _fn(ncm)
    rng = np.random.default_rng(11)
    # two calls in a row on the shared scratch, the second shorter than the first
    for heads, kvh, hd, pos in [(32, 8, 64, 300), (24, 8, 128, 47)]:
        kvw = kvh * hd
        q = torch.from_numpy(rng.standard_normal(heads * hd).astype(np.float32)).cuda()
        kc = torch.from_numpy(rng.standard_normal((pos + 1) * kvw).astype(np.float32)).cuda()
        vc = torch.from_numpy(rng.standard_normal((pos + 1) * kvw).astype(np.float32)).cuda()
        ref = torch.zeros(heads * hd, dtype=torch.float32, device="cuda")
        got = torch.full((heads * hd,), float("nan"), dtype=torch.float32, device="cuda")
        ncm.attention(ref.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos, heads, kvh, hd)
        st = noalloc(got.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos, heads, kvh, hd, None)
        assert st == 0, ncm.lib().ncm_last_error().decode()
        torch.cuda.synchronize()
        assert np.allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=1e-4, atol=1e-5)


def test_noalloc_attention_rejects_oversized_request(ncm, cuda):
    noalloc = _fn(ncm)
    x = cuda.zeros(64, dtype=cuda.float32, device="cuda")
    st = noalloc(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 262144, 8, 8, 32, None)
    assert st == 1
    assert "exceeds the fixed scratch" in ncm.lib().ncm_last_error().decode()
