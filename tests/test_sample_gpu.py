"""Token sampling (msgl_sample) on a B200 against a numpy restatement of the algorithm stated
in include/msgl_kernels.h: greedy rows bit-exact (first index of the maximum, as the reference's
scheduler), sampled rows equal to the restatement fed the same SplitMix64 draws (all but a few
rows; every row within what a 1e-4 shift of the draw or of top-p allows, since the device's expf
and the host's exp may round a cumulative sum to the other side of the draw), and the empirical
distribution of many draws close to the softmax."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
M64 = (1 << 64) - 1


def uniform24(seed, step, row):
    z = (seed ^ ((step * 0x9E3779B97F4A7C15) & M64) ^ ((row * 0xC2B2AE3D27D4EB4F) & M64)) & M64
    z = (z + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    z ^= z >> 31
    return np.float32(z >> 40) * np.float32(1.0 / 16777216.0)


def restate(l, T, k, p, seed, step, row, du=0.0, dp=0.0, f64=False):
    """The stated algorithm on the host; du / dp shift the draw and top-p (for the rounding
    allowance), f64 accumulates the weights in float64."""
    l = np.asarray(l, np.float32)
    V = l.size
    if T <= 0 or k == 1:
        return int(np.argmax(l))
    K = min(k, V) if 1 < k <= 1024 else min(V, 1024)
    order = np.lexsort((np.arange(V), -l.astype(np.float64)))[:K]  # logit desc, id asc
    v = l[order]
    if f64:
        c = np.cumsum(np.exp((v.astype(np.float64) - v[0]) / T))
    else:
        w = np.exp((v - v[0]) * np.float32(np.float32(1.0) / np.float32(T))).astype(np.float32)
        c = np.cumsum(w, dtype=np.float32)
    n = K
    if p + dp < 1:
        cut = (p + dp) * c[K - 1]
        n = 1
        while n < K and c[n - 1] < cut:
            n += 1
    u = min(max(float(uniform24(seed, step, row)) + du, 0.0), 1.0)
    target = u * c[n - 1]
    idx = np.nonzero(c[:n] > target)[0]
    return int(order[int(idx[0]) if idx.size else n - 1])


def allowed(l, T, k, p, seed, step, row, d=1e-4):
    """Tokens the algorithm gives when the draw and top-p move by up to d: a result outside
    this set cannot be explained by fp32 rounding of the weights."""
    return {restate(l, T, k, p, seed, step, row, du, dp, True)
            for du in (-d, 0.0, d) for dp in (-d, 0.0, d)}


def run(logits, T, k, p, seed, step):
    from msgl import ops
    d = lambda a, dt: torch.tensor(a, dtype=dt, device="cuda")
    return ops.sample(d(logits, torch.float32), d(T, torch.float32), d(k, torch.int32),
                      d(p, torch.float32), seed, step).cpu().numpy()


@pytest.mark.parametrize("V", [1000, 151936])
def test_sample_matches_restatement(cuda, V):
    from msgl import ops
    rng = np.random.default_rng(V)
    B = 12
    logits = (rng.standard_normal((B, V)) * 3).astype(np.float32)
    logits[3, 7] = logits[3, 900] = logits[3].max() + 1  # a tie at the top
    logits[5, :] = np.round(logits[5, :])                 # many ties at every value
    T = [0.0, 0.7, 1.0, 1.3, 0.5, 1.0, 0.9, 2.0, 1.0, 0.0, 1.0, 0.8]
    k = [-1, 50, -1, 1000, 2000, 20, 1, 5, 1024, 10, -1, 3]
    p = [1.0, 1.0, 0.9, 0.95, 1.0, 0.8, 0.5, 1.0, 0.99, 0.3, 0.5, 0.7]
    exact = total = 0
    for step in range(6):
        got = run(logits, T, k, p, 1234, step)
        for r in range(B):
            total += 1
            exact += int(got[r] == restate(logits[r], T[r], k[r], p[r], 1234, step, r))
            assert got[r] in allowed(logits[r], T[r], k[r], p[r], 1234, step, r), (step, r)
    assert exact >= total - 3, (exact, total)
    assert ops.device_error() == (0, 0)


def test_greedy_rows_take_the_first_maximum(cuda):
    l = np.zeros((3, 5000), np.float32)
    l[0, [17, 4000]] = 2.0
    l[1, 4999] = -1e-3
    l[1, :4999] = -1.0
    l[2, :] = 5.0
    got = run(l, [0.0, -1.0, 2.0], [-1, 7, 1], [1.0, 0.2, 1.0], 0, 0)
    assert got.tolist() == [17, 4999, 0]


def test_sampled_frequencies_follow_the_softmax(cuda):
    rng = np.random.default_rng(5)
    V, B = 20, 8192
    base = rng.standard_normal(V).astype(np.float32)
    logits = np.tile(base, (B, 1))
    got = run(logits, [0.8] * B, [-1] * B, [1.0] * B, 99, 3)
    q = np.exp((base - base.max()) / 0.8)
    q /= q.sum()
    freq = np.bincount(got, minlength=V) / B
    assert np.abs(freq - q).max() < 0.02
    # top-k 4: nothing outside the four largest logits
    got = run(logits, [0.8] * B, [4] * B, [1.0] * B, 99, 4)
    assert set(got.tolist()) <= set(np.argsort(-base)[:4].tolist())
