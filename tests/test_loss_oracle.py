"""Check the CPU oracle's L1 + DSSIM loss against the published SSIM definition (no GPU needed).

The reference computes SSIM with FastCUDASSIM v0.2.1 (training.jl:196-217), which is not
vendored, so the oracle follows Wang et al. 2004 ("Image quality assessment: from error
visibility to structural similarity", IEEE TIP 13(4)): 11-tap Gaussian window with sigma 1.5,
zero padding, C1 = 0.01^2, C2 = 0.03^2, the SSIM map averaged over 3 x h x w. These tests
restate that definition independently with scipy and check the oracle's value against it, and
the oracle's analytic gradient against central differences. They pin the oracle to the published
algorithm; parity with FastCUDASSIM itself stays unpinned.
"""
import numpy as np
import pytest
from scipy import ndimage

from oracle import oracle as O

C1, C2 = 0.01 ** 2, 0.03 ** 2


def _window():
    g = np.exp(-((np.arange(11) - 5.0) ** 2) / (2 * 1.5 ** 2))
    return (g / g.sum()).astype(np.float32).astype(np.float64)


def _blur(plane):
    w = _window()
    out = ndimage.correlate1d(plane, w, axis=0, mode="constant", cval=0.0)
    return ndimage.correlate1d(out, w, axis=1, mode="constant", cval=0.0)


def _ssim_mean(K, I):
    """Mean SSIM over every channel and pixel of two (w, h, 3) images (float64)."""
    total = 0.0
    for c in range(3):
        x = K[:, :, c].astype(np.float64)
        y = I[:, :, c].astype(np.float64)
        mx, my = _blur(x), _blur(y)
        sxx = _blur(x * x) - mx * mx
        syy = _blur(y * y) - my * my
        sxy = _blur(x * y) - mx * my
        S = ((2 * mx * my + C1) * (2 * sxy + C2)) / ((mx * mx + my * my + C1) * (sxx + syy + C2))
        total += S.sum()
    return total / K.size


def _images(w, h, seed, close=False):
    rng = np.random.default_rng(seed)
    K = rng.uniform(0, 1, (w, h, 3)).astype(np.float32)
    if close:
        I = np.clip(K + rng.normal(0, 0.05, K.shape), 0, 1).astype(np.float32)
    else:
        I = rng.uniform(0, 1, (w, h, 3)).astype(np.float32)
    return K, I


@pytest.mark.parametrize("w,h", [(1, 1), (3, 5), (11, 11), (16, 16), (37, 23), (64, 9)])
@pytest.mark.parametrize("close", [False, True])
def test_oracle_loss_matches_published_ssim(w, h, close):
    K, I = _images(w, h, seed=w * 100 + h, close=close)
    (loss, l1, dssim), _ = O.loss(K, I, weight=0.2)
    want_l1 = np.abs(K.astype(np.float64) - I.astype(np.float64)).mean()
    want_dssim = 1.0 - _ssim_mean(K, I)
    assert l1 == pytest.approx(want_l1, rel=1e-12, abs=1e-15)
    assert dssim == pytest.approx(want_dssim, rel=1e-10, abs=1e-12)
    w32 = float(np.float32(0.2))                 # the weight crosses the ABI as a float
    assert loss == pytest.approx((1 - w32) * want_l1 + w32 * want_dssim, rel=1e-10, abs=1e-12)


def test_identical_images_have_zero_dssim():
    K, _ = _images(20, 13, seed=3)
    (loss, l1, dssim), grad = O.loss(K, K.copy(), weight=0.2)
    assert l1 == 0.0
    assert abs(dssim) < 1e-12 and abs(loss) < 1e-12
    # ties take the negative L1 sign (training.jl: ">" comparison)
    l1w = np.float32(0.8) / np.float32(K.size)
    np.testing.assert_allclose(grad, -l1w, rtol=0, atol=1e-9)


@pytest.mark.parametrize("w,h", [(9, 7), (24, 17)])
def test_oracle_dssim_gradient_matches_central_differences(w, h):
    K, I = _images(w, h, seed=w + h, close=True)
    _, grad = O.loss(K, I, weight=1.0)           # weight 1: pure DSSIM, smooth in K
    rng = np.random.default_rng(7)
    flat = K.reshape(-1)
    picks = rng.choice(flat.size, 24, replace=False)
    for i in picks:
        d = np.float32(1e-2)
        Kp, Km = flat.copy(), flat.copy()
        Kp[i] += d
        Km[i] -= d
        hi = float(Kp[i]) - float(flat[i])
        lo = float(flat[i]) - float(Km[i])
        (Lp, _, _), _ = O.loss(Kp.reshape(K.shape), I, weight=1.0)
        (Lm, _, _), _ = O.loss(Km.reshape(K.shape), I, weight=1.0)
        fd = (Lp - Lm) / (hi + lo)
        an = float(grad.reshape(-1)[i])
        scale = max(abs(fd), 1e-3 / flat.size)
        assert abs(an - fd) <= 2e-3 * scale, (i, an, fd)


def test_oracle_l1_gradient_sign_and_size():
    K, I = _images(12, 10, seed=11)
    _, g_mixed = O.loss(K, I, weight=0.2)
    _, g_ssim = O.loss(K, I, weight=1.0)
    _, g_zero = O.loss(K, I, weight=0.0)
    l1w = np.float32(1.0) / np.float32(K.size)
    want = np.where(K > I, l1w, -l1w)
    np.testing.assert_allclose(g_zero, want, rtol=1e-6, atol=0)
    # the gradient is linear in the weight: (1 - w) * L1 part + w * DSSIM part
    np.testing.assert_allclose(g_mixed, 0.8 * g_zero + 0.2 * g_ssim, rtol=1e-5, atol=1e-9)
