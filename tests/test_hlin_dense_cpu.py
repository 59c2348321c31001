"""The algebra behind the dense tensor-core form of HadamardLinear(F, F), on
the CPU in float64: the matrix that walsh_hadamard_linear_dense_weights
writes (entry (h, o; p, i) = an integer sum over the 32 groups of
H[g, h] H[p, g] w[g, o, i], times alpha[p, i] / (32 q), row scale beta[h, o] q
with q the power of two at or above max |alpha|; unnormalised Sylvester H)
reproduces the reference's HadamardLinear.forward (src/model/fht_cuda.py:
489-519, restated by the oracle), and its entries are integers in [-32, 32]
before the alpha scaling, at most 1 in magnitude after it.  The device kernel
is checked against the same matrix on the GPU (test_gpu_parity.py)."""
import math

import numpy as np
import pytest

from oracle import walsh_oracle as O


def _dense(wq, alpha, beta):
    G, io, _ = wq.shape
    H = O.hadamard_matrix(G, normalize=False)
    # sums[h, o, p, i] = sum_g H[g, h] H[p, g] w[g, o, i]
    sums = np.einsum("gh,goi,pg->hopi", H, wq, H)
    q = 2.0 ** math.frexp(float(np.abs(alpha).max()))[1]
    M = sums * alpha[None, None] / (32.0 * q)
    scale = beta * q
    return sums, M.reshape(G * io, G * io), scale.reshape(G * io)


@pytest.mark.parametrize("F", [512, 2048])
def test_dense_matrix_reproduces_hadamard_linear(F):
    rng = np.random.default_rng(F)
    io = F // 32
    w = rng.normal(size=(32, io, io))
    alpha = rng.uniform(0.5, 3.0, (32, io)).astype(np.float32)
    beta = rng.uniform(0.1, 0.4, (32, io)).astype(np.float32)
    x = rng.normal(size=(7, F))
    sums, M, scale = _dense(O.quantize_ternary(w).astype(np.float64), alpha.astype(np.float64),
                            beta.astype(np.float64))
    assert np.array_equal(sums, np.round(sums)) and np.abs(sums).max() <= 32
    assert np.abs(M).max() <= 1.0
    y = (x @ M.T) * scale
    ref = O.hadamard_linear(x, w, alpha, beta)
    np.testing.assert_allclose(y, ref, rtol=0, atol=1e-12 * np.abs(ref).max())
