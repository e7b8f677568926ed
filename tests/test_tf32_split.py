"""CPU check of the operand split used by the tensor-core fp32 mm
(wgpu-executorch_b200/csrc/mm_tf32.cu): each fp32 value is a TF32 head (13
low mantissa bits cleared) plus an fp32 tail (value - head, exact), and the
product keeps head*head + head*tail + tail*head with every factor read as
TF32. This emulates that arithmetic in numpy (products summed in float64, so
only the operand rounding is modelled) and checks the claims the kernel's
accuracy rests on."""
import numpy as np
import pytest


def tf32(x):
    """What a TF32 multiply reads of an fp32 value: 13 low mantissa bits cleared."""
    return (np.asarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def split(x):
    x = np.asarray(x, np.float32)
    hi = tf32(x)
    lo = (x - hi).astype(np.float32)
    return hi, lo


def test_split_is_exact():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-20, 20, 100000))).astype(np.float32)
    hi, lo = split(x)
    # the tail is exact in fp32 and small against the value
    assert np.array_equal((hi.astype(np.float64) + lo.astype(np.float64)).astype(np.float32), x)
    nz = x != 0
    assert np.all(np.abs(lo[nz]) <= np.abs(x[nz]) * 2.0 ** -10)


@pytest.mark.parametrize("K", [64, 512, 4096])
@pytest.mark.parametrize("scale", [1.0, 1e3])
def test_three_products_keep_fp32_accuracy(K, scale):
    rng = np.random.default_rng(K)
    M = N = 64
    a = (rng.uniform(-1, 1, (M, K)) * scale).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    b[:, ::3] *= 1e-3
    exact = a.astype(np.float64) @ b.astype(np.float64)
    ah, al = split(a)
    bh, bl = split(b)
    f = lambda m: tf32(m).astype(np.float64)
    three = f(ah) @ f(bh) + f(ah) @ f(bl) + f(al) @ f(bh)
    one = f(a) @ f(b)  # plain TF32, for contrast
    denom = np.abs(exact).max()
    err3 = np.abs(three - exact).max() / denom
    err1 = np.abs(one - exact).max() / denom
    # operand rounding of the three-product form stays far inside the 1e-4
    # fp32 bound of the GPU tests; plain TF32 does not
    assert err3 <= 1e-6, err3
    assert err1 > 10 * err3
