"""GPU parity of the batched decode path (B sequences sharing the weights):
the tcgen05 W4A8 GEMM against the oracle's matvec_y32, one sequence at a
time, bit-exact."""
import numpy as np
import pytest
import torch

import oracle as O
from fable5_llm_b200 import ops

pytestmark = pytest.mark.gpu


def rand_image(rng, N, K, m_lo=1, m_hi=65536):
    w4 = rng.integers(-8, 8, (N, K)).astype(np.int8)
    m = rng.integers(m_lo, m_hi, (N, K // 128)).astype(np.uint16)
    img, _ = O.pack_ddr_rows(w4, m, 128)
    return img


def check_batch(img, N, K, x8):
    sh = O.final_shift(K)
    d_img = ops.to_dev(img)
    y, err, p = ops.batch_matvec_y32(d_img, N, K, sh, ops.to_dev(x8), want_p=True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    y, p = y.cpu().numpy(), p.cpu().numpy()
    for b in range(x8.shape[0]):
        y_ref, p_ref = O.matvec_img(img, N, K, sh, x8[b], 128, want_p=True)
        assert np.array_equal(p[b], p_ref), f"p mismatch at sequence {b}"
        assert np.array_equal(y[b], y_ref), f"y32 mismatch at sequence {b}"


@pytest.mark.parametrize("B", [1, 8, 16, 17, 32, 40, 64])
def test_batch_matvec_4096(B):
    rng = np.random.default_rng(100 + B)
    N, K = 1000, 4096          # a ragged last tile (1000 = 7 * 128 + 104)
    img = rand_image(rng, N, K)
    x8 = rng.integers(-127, 128, (B, K)).astype(np.int8)
    check_batch(img, N, K, x8)


@pytest.mark.parametrize("N,K,B", [(4096, 4096, 64), (32, 4096, 8), (4096, 12288, 32), (300, 12288, 64),
                                   (12288, 4096, 16), (2048, 1024, 8)])
def test_batch_matvec_shapes(N, K, B):
    rng = np.random.default_rng(N + K + B)
    img = rand_image(rng, N, K)
    x8 = rng.integers(-127, 128, (B, K)).astype(np.int8)
    check_batch(img, N, K, x8)


def test_batch_matvec_extremes():
    """|acc_g| and |p| at their maxima: all -8 / 7 weights, m = 65535,
    x = +-127 (and the unsigned-weight correction at its largest)."""
    for K in (4096, 12288):
        N = 256
        w4 = np.full((N, K), -8, dtype=np.int8)
        w4[1::2] = 7
        m = np.full((N, K // 128), 65535, dtype=np.uint16)
        img, _ = O.pack_ddr_rows(w4, m)
        x8 = np.empty((16, K), dtype=np.int8)
        x8[0::2], x8[1::2] = 127, -127
        x8[3] = np.where(np.arange(K) % 2 == 0, 127, -127)
        check_batch(img, N, K, x8)
