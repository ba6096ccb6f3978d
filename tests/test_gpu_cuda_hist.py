"""GPU parity of the build_hist drop-in (yabt_b200.cuda_hist) against the
oracle's restatement of the reference's scatter histogram
(yabt/tree.py:442-452, yabt/_cuda/hist.cu) and the reference's golden
vectors. The reference's own tests (tests/test_cuda_hist.py) accept a relative
error of 1e-5 of the largest bin against torch's float scatter; the same bound
is asserted here, plus bit-exactness against an exact fixed-point restatement
(each channel quantised to rint(x * 2^q) with |x| * 2^q < 2^30, summed in
int64, rounded once to float32), and bit-exactness against the float32
scatter wherever float32 sums are exact (dyadic inputs)."""

import numpy as np
import pytest
import torch

from oracle.grow import scatter_hist

pytestmark = pytest.mark.gpu
B = 256


def exact_fixed(binned, slot, g, h, w, K, Bo=B):
    n, F = binned.shape
    out = np.zeros((3, K, F, Bo), np.float32)
    flat = (slot.astype(np.int64)[:, None] * (F * Bo) + np.arange(F, dtype=np.int64)[None, :] * Bo
            + binned.astype(np.int64)).reshape(-1)
    for c, x in enumerate((g, h, w)):
        x = np.asarray(x, np.float32)
        amax = float(np.abs(x).max()) if n else 0.0
        e = int(np.frexp(np.float32(amax))[1]) if amax > 0 else 0
        q = max(-100, min(30 - e, 100))
        V = np.rint(x.astype(np.float64) * 2.0 ** q).astype(np.int64)
        acc = np.zeros(K * F * Bo, np.int64)
        np.add.at(acc, flat, np.repeat(V, F))
        out[c] = (acc.astype(np.float32) * np.float32(2.0 ** -q)).reshape(K, F, Bo)
    return out


def run(binned, slot, g, h, w, K, F, Bo=B):
    from yabt_b200.cuda_hist import build_hist
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return build_hist(t(binned), t(slot), t(g), t(h), t(w), K, F, Bo).cpu().numpy()


def rel_err(ref, got):
    return float(np.abs(ref.astype(np.float64) - got).max() / max(np.abs(ref).max(), 1e-9))


def _case(seed, n, F, K, Bo=B):
    rng = np.random.default_rng(seed)
    binned = rng.integers(0, Bo, size=(n, F)).astype(np.uint8)
    g = rng.normal(size=n).astype(np.float32)
    h = (rng.random(n) + 0.1).astype(np.float32)
    w = np.ones(n, np.float32)
    slot = np.zeros(n, np.int64) if K == 1 else rng.integers(0, K, size=n).astype(np.int64)
    return binned, slot, g, h, w


@pytest.mark.parametrize("K", [1, 4, 31])
def test_matches_reference_scatter(K):
    """Reference tests/test_cuda_hist.py:26-45 (n=20000, F=24)."""
    n, F = 20000, 24
    binned, slot, g, h, w = _case(0, n, F, K)
    got = run(binned, slot, g, h, w, K, F)
    assert rel_err(scatter_hist(binned, slot, g, h, w, K), got) < 1e-5
    np.testing.assert_array_equal(got, exact_fixed(binned, slot, g, h, w, K))


def test_count_weight_mask():
    """Reference tests/test_cuda_hist.py:48-68: the count channel takes a 0/1
    weight; g and h arrive pre-masked."""
    n, F, K = 8000, 16, 6
    binned, slot, g, h, _ = _case(1, n, F, K)
    w = (np.random.default_rng(2).random(n) > 0.5).astype(np.float32)
    got = run(binned, slot, g * w, h * w, w, K, F)
    ref = scatter_hist(binned, slot, g * w, h * w, w, K)
    assert rel_err(ref, got) < 1e-5
    np.testing.assert_array_equal(got, exact_fixed(binned, slot, g * w, h * w, w, K))
    assert abs(float(got[2].sum()) - float(w.sum()) * F) < 1.0


def test_golden_vectors(golden):
    """The reference's torch scatter histogram recorded on seeded inputs."""
    z = golden("hist")
    w = z["w"]
    n, F = z["binned"].shape
    got = run(z["binned"], z["slot"], z["g"] * w, z["h"] * w, w, 5, F)
    assert rel_err(z["hist"], got) < 1e-5
    np.testing.assert_array_equal(got, exact_fixed(z["binned"], z["slot"], z["g"] * w, z["h"] * w, w, 5))


def test_dyadic_bit_exact_with_float_scatter():
    """Sums of small dyadic values are exact in float32, so the reference's
    float scatter and the fixed-point sums must agree bit for bit."""
    rng = np.random.default_rng(3)
    n, F, K = 30000, 40, 7
    binned = rng.integers(0, B, size=(n, F)).astype(np.uint8)
    g = (rng.integers(-64, 65, size=n) / 16).astype(np.float32)
    h = (rng.integers(1, 17, size=n) / 8).astype(np.float32)
    w = rng.integers(0, 2, size=n).astype(np.float32)
    slot = rng.integers(0, K, size=n).astype(np.int64)
    np.testing.assert_array_equal(run(binned, slot, g, h, w, K, F), scatter_hist(binned, slot, g, h, w, K))


@pytest.mark.parametrize("n,F,K,Bo", [(70000, 1, 3, 256), (5000, 33, 1000, 256), (40000, 200, 2, 256),
                                      (9000, 20, 5, 64), (1, 5, 1, 256)])
def test_shapes(n, F, K, Bo):
    """Ragged feature groups, many empty slots, several items per slot, B < 256."""
    binned, slot, g, h, w = _case(4, n, F, K, Bo)
    got = run(binned, slot, g, h, w, K, F, Bo)
    np.testing.assert_array_equal(got, exact_fixed(binned, slot, g, h, w, K, Bo))
    ref = scatter_hist(binned, slot, g, h, w, K)[..., :Bo]
    assert rel_err(ref, got) < 1e-5


def test_limb_extremes():
    """One hot bin filled by several full items of the largest value: the
    low limb of every item reaches its maximum without overflowing."""
    n, F = 3 * 8192 + 5, 3
    binned = np.full((n, F), 7, np.uint8)
    g = np.full(n, -1.9999999, np.float32)
    h = np.full(n, 1.9999999, np.float32)
    w = np.ones(n, np.float32)
    slot = np.zeros(n, np.int64)
    got = run(binned, slot, g, h, w, 1, F)
    np.testing.assert_array_equal(got, exact_fixed(binned, slot, g, h, w, 1))
    assert got[2, 0, 0, 7] == n
    np.testing.assert_allclose(got[0, 0, :, 7], float(g[0]) * n, rtol=1e-6)


def test_empty_and_deterministic():
    from yabt_b200.cuda_hist import build_hist
    e = torch.zeros(0, 4, dtype=torch.uint8, device="cuda")
    z = torch.zeros(0, device="cuda")
    out = build_hist(e, torch.zeros(0, dtype=torch.int64, device="cuda"), z, z, z, 3, 4, B)
    assert out.shape == (3, 3, 4, B) and not out.any()
    binned, slot, g, h, w = _case(5, 50000, 24, 9)
    a = run(binned, slot, g, h, w, 9, 24)
    b = run(binned, slot, g, h, w, 9, 24)
    np.testing.assert_array_equal(a, b)


def test_bad_input_raises():
    from yabt_b200._lib import YabtError
    binned, slot, g, h, w = _case(6, 1000, 8, 4)
    bad = slot.copy()
    bad[17] = 4
    with pytest.raises(YabtError, match="out of range"):
        run(binned, bad, g, h, w, 4, 8)
    gn = g.copy()
    gn[3] = np.nan
    with pytest.raises(YabtError, match="non-finite"):
        run(binned, slot, gn, h, w, 4, 8)
    with pytest.raises(YabtError, match="out of range"):
        run(binned, slot, g, h, w, 4, 8, 16)      # bins up to 255 with B = 16
    # the context stays usable after the rejected calls
    got = run(binned, slot, g, h, w, 4, 8)
    np.testing.assert_array_equal(got, exact_fixed(binned, slot, g, h, w, 4))
