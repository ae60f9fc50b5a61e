"""The allocation-free matvec entry point.

f5_matvec_y32_host_noalloc serves callers that cannot call cudaMalloc
(device memory owned by another allocator's pool or arena, loops that cannot
take the device synchronisation of cudaMalloc/cudaFree).  It stages its buffers in one fixed device array the
library reserves at load time.  This test calls it through the C ABI twice
in a row with different inputs and requires exactly the results of the
allocating entry point f5_matvec_y32_host (bit-exact: the integer law has no
tolerance), and checks that a request above the array's size is refused.
The file sorts last so a failure here leaves every other test already run;
it passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest

from fable5_llm_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _call(fn, img, N, K, sh, x8, want_p):
    y = np.empty(N, dtype=np.int32)
    p = np.empty(N, dtype=np.int64) if want_p else None
    rc = fn(img.ctypes.data, N, K, 128, sh, x8.ctypes.data, y.ctypes.data,
            p.ctypes.data if p is not None else None)
    return rc, y, p


def _case(seed, N, K):
    rng = np.random.default_rng(seed)
    stride = (K // 128 + (K // 128 + 31) // 32) * 64
    img = rng.integers(0, 256, (N, stride), dtype=np.uint8)
    NG = K // 128
    img[:, K // 2:K // 2 + 2 * NG] = rng.integers(1, 65536, (N, NG)).astype("<u2").view(np.uint8)
    img[:, K // 2 + 2 * NG:] = 0
    x8 = rng.integers(-127, 128, K).astype(np.int8)
    sh = max(0, (NG * 65535 * (128 * 8 * 127)).bit_length() - 31)
    return np.ascontiguousarray(img), x8, sh


def test_noalloc_matches_allocating_entry_point():
    lib = L.lib()
    for call, (seed, N, K, want_p) in enumerate([(1, 3000, 4096, True), (2, 700, 12288, False)]):
        img, x8, sh = _case(seed, N, K)
        rc0, y0, p0 = _call(lib.f5_matvec_y32_host, img, N, K, sh, x8, want_p)
        assert rc0 == 0, L.last_error()
        rc1, y1, p1 = _call(lib.f5_matvec_y32_host_noalloc, img, N, K, sh, x8, want_p)
        assert rc1 == 0, L.last_error()
        assert np.array_equal(y1, y0), f"call {call}: y32 differs"
        if want_p:
            assert np.array_equal(p1, p0), f"call {call}: p differs"


def test_noalloc_rejects_oversize():
    lib = L.lib()
    N, K = 8200, 4096                      # 8200 * 2112 B > 16 MiB
    img = np.zeros((N, 2112), dtype=np.uint8)
    x8 = np.zeros(K, dtype=np.int8)
    y = np.empty(N, dtype=np.int32)
    rc = lib.f5_matvec_y32_host_noalloc(img.ctypes.data, N, K, 128, 7, x8.ctypes.data, y.ctypes.data, None)
    assert rc == L.F5_EINVAL
    assert "fixed scratch" in L.last_error()
