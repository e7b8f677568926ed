"""CPU tests of the oracle: the restated WGSL arithmetic must reproduce the
reference's own known-answer tests (both modes), and its index math must
agree with an independent float64 numpy convolution."""
import numpy as np
import pytest

import oracle
from kat_cases import KATS, cases, run_oracle

CASES = cases()


def test_fixture_has_reference_cases():
    n = sum(len(v["cases"]) for v in KATS["files"].values())
    assert n >= 15


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
@pytest.mark.parametrize("mode", ["wgsl", "exact"])
def test_reference_kat_on_oracle(case, mode):
    case.check(run_oracle(case, mode))


def np_conv(x, w, b, s, p, d, g):
    """Independent float64 convolution (loops over taps, vectorised over
    output positions)."""
    x = x.astype(np.float64)
    w = w.astype(np.float64)
    B, IC, IH, IW = x.shape
    OC, icpg, KH, KW = w.shape
    OH = (IH + 2 * p[0] - d[0] * (KH - 1) - 1) // s[0] + 1
    OW = (IW + 2 * p[1] - d[1] * (KW - 1) - 1) // s[1] + 1
    xp = np.zeros((B, IC, IH + 2 * p[0], IW + 2 * p[1]))
    xp[:, :, p[0]:p[0] + IH, p[1]:p[1] + IW] = x
    out = np.zeros((B, OC, OH, OW))
    ocpg = OC // g
    for oc in range(OC):
        gi = oc // ocpg
        for c in range(icpg):
            ic = gi * icpg + c
            for kh in range(KH):
                for kw in range(KW):
                    patch = xp[:, ic, kh * d[0]: kh * d[0] + s[0] * (OH - 1) + 1: s[0],
                               kw * d[1]: kw * d[1] + s[1] * (OW - 1) + 1: s[1]]
                    out[:, oc] += patch * w[oc, c, kh, kw]
    if b is not None:
        out += b.astype(np.float64)[None, :, None, None]
    return out


GEOMS = [
    # B, IC, H, W, OC, K, s, p, d, g
    (2, 3, 11, 13, 5, 3, 1, 1, 1, 1),
    (1, 8, 9, 7, 4, 3, 2, 1, 1, 1),
    (2, 6, 10, 10, 6, 5, 1, 2, 1, 6),
    (1, 4, 12, 9, 8, 3, 1, 2, 2, 2),
    (3, 16, 5, 5, 1, 1, 1, 0, 1, 1),
]


@pytest.mark.parametrize("geom", GEOMS)
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_oracle_exact_matches_numpy(geom, dtype):
    B, IC, H, W, OC, K, s, p, d, g = geom
    x, w, b = oracle.make_inputs([(B, IC, H, W), (OC, IC // g, K, K), (OC,)], seed=1,
                                 dtype=dtype)
    ref = np_conv(x, w, b, (s, s), (p, p), (d, d), g)
    y = oracle.conv2d(x, w, b, s, p, d, g, mode="exact")
    np.testing.assert_allclose(y.astype(np.float64), ref.astype(dtype).astype(np.float64),
                               rtol=0, atol=np.finfo(dtype).eps * 4 * max(1, np.abs(ref).max()))


def test_oracle_wgsl_f16_accumulation_differs_but_bounded():
    # the reference's f16 kernels accumulate in f16: a K=576 dot product
    # drifts from the exact result by a few f16 ulps of the running sum
    x, w, b = oracle.make_inputs([(1, 64, 16, 16), (32, 64, 3, 3), (32,)], seed=2)
    w = (w.astype(np.float32) * np.sqrt(2 / 576)).astype(np.float16)
    ex = oracle.conv2d(x, w, b, 1, 1, 1, 1, mode="exact")
    wg = oracle.conv2d(x, w, b, 1, 1, 1, 1, mode="wgsl")
    err = oracle.rel_err(wg, ex)
    assert 0 < err < 2e-2


def test_oracle_silu_and_clamp_epilogues():
    x, w, b = oracle.make_inputs([(1, 8, 6, 6), (4, 8, 3, 3), (4,)], seed=3, dtype=np.float32)
    base = np_conv(x, w, b, (1, 1), (1, 1), (1, 1), 1)
    silu = oracle.conv2d(x, w, b, 1, 1, 1, 1, act=oracle.ACT_SILU, mode="exact")
    np.testing.assert_allclose(silu, oracle.silu_exact(base), rtol=1e-5, atol=1e-6)
    cl = oracle.conv2d(x, w, b, 1, 1, 1, 1, act=oracle.ACT_CLAMP, out_min=-0.5, out_max=0.25,
                       mode="exact")
    np.testing.assert_allclose(cl, np.clip(base, -0.5, 0.25), rtol=1e-5, atol=1e-6)


def test_oracle_tile32_layout_flag():
    # aten.convolution's tile32 kernel writes [OC, B, OH, OW]; with the flag
    # the oracle reproduces that layout, without it the result is NCHW
    x, w, _ = oracle.make_inputs([(2, 4, 8, 8), (16, 4, 3, 3), (16,)], seed=4)
    good = oracle.conv2d(x, w, None, 1, 1, 1, 1, mode="exact")
    bug = oracle.conv2d(x, w, None, 1, 1, 1, 1, mode="exact", bug_tile32=True)
    np.testing.assert_array_equal(bug.reshape(16, 2, 8, 8).transpose(1, 0, 2, 3), good)


def test_oracle_mm_modes():
    a, b = oracle.make_inputs([(33, 70), (70, 17)], seed=5, dist="uniform", dtype=np.float32)
    ex = oracle.mm(a, b, "exact")
    np.testing.assert_allclose(ex, (a.astype(np.float64) @ b).astype(np.float32), rtol=1e-6)
    wg = oracle.mm(a, b, "wgsl")
    assert oracle.rel_err(wg, ex) < 1e-5


def test_elementwise_oracles_follow_wgsl_expressions():
    a, b = oracle.make_inputs([(4, 5), (4, 5)], seed=6)
    np.testing.assert_array_equal(oracle.add(a, b, 1.5), a + np.float16(1.5) * b)
    np.testing.assert_array_equal(oracle.relu(a), np.maximum(a, 0))
    s = oracle.sigmoid(a).astype(np.float64)
    assert np.all((s > 0) & (s < 1))
