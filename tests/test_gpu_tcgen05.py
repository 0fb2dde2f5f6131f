"""Tensor-core (tcgen05) layer self-test: descriptors, TMEM, commit/mbarrier,
and the 3-product bf16 split used by the mixed-precision kernels, against a
numpy fp64 matmul."""
import numpy as np
import pytest

import b200dp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (1, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("K,N", [(32, 64), (64, 112), (128, 16), (128, 256), (256, 64)])
def test_mma_layouts_and_split(a_mn, b_mn, K, N):
    rng = np.random.default_rng(K * 1000 + N + 7 * a_mn + 13 * b_mn)
    A = rng.normal(size=(128, K)).astype(np.float32)
    B = rng.normal(size=(N, K)).astype(np.float32)
    ref = A.astype(np.float64) @ B.astype(np.float64).T
    scale = np.abs(ref).max()
    c3 = b200dp.selftest_mma(A, B, passes=3, a_mn_major=a_mn, b_mn_major=b_mn)
    err3 = np.abs(c3 - ref).max() / scale
    assert err3 < 5e-5, err3
    c1 = b200dp.selftest_mma(A, B, passes=1, a_mn_major=a_mn, b_mn_major=b_mn)
    err1 = np.abs(c1 - ref).max() / scale
    assert 1e-4 < err1 < 2e-2, err1  # single bf16 product: bf16-level error


def test_mma_rejects_oversized_operands():
    A = np.zeros((128, 256), np.float32)
    B = np.zeros((256, 256), np.float32)
    with pytest.raises(b200dp.B200DPError) as e:
        b200dp.selftest_mma(A, B)
    assert e.value.status == 1
