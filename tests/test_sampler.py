"""The token sampler's restatement (oracle.sample_token, with the uniform draw
given) against the reference's own sample_token (src/sampler.cpp:11-148, run
from oracle/_ref, which draws from its own randomly seeded mt19937):
identical tokens wherever the configuration leaves one candidate (top_k 1,
with temperature and repetition penalty applied first), every reference token
inside the restatement's kept set otherwise, and the reference's token
frequencies over many draws matching the restatement's probabilities."""
import numpy as np

from oracle.oracle import Reference, sample_token


def ref_sample(L, lg, T, tp, tk, pen, seen):
    seen = np.asarray(seen, np.int32)
    return L.tvref_sample_token(lg, lg.size, T, tp, tk, pen, seen, len(seen))


def test_single_candidate_is_identical():
    L = Reference().L
    rng = np.random.default_rng(0)
    for trial in range(40):
        lg = (rng.standard_normal(1000) * 3).astype(np.float32)
        seen = rng.integers(0, 1000, 30)
        for T, tp, pen in [(0.8, 0.9, 1.1), (1.0, 0.5, 1.3), (0.0, 1.0, 1.0), (2.0, 0.95, 2.0)]:
            assert ref_sample(L, lg, T, tp, 1, pen, seen) == sample_token(lg, T, tp, 1, pen, list(seen),
                                                                          u=rng.random())


def test_reference_tokens_stay_in_the_kept_set():
    L = Reference().L
    rng = np.random.default_rng(1)
    for trial in range(40):
        lg = (rng.standard_normal(2000) * 2).astype(np.float32)
        seen = rng.integers(0, 2000, 50)
        _, cdf = sample_token(lg, 0.8, 0.9, 40, 1.1, list(seen), return_cdf=True)
        kept = set(np.nonzero(cdf > np.concatenate([[0], cdf[:-1]]))[0].tolist())
        assert 1 <= len(kept) <= 40
        assert ref_sample(L, lg, 0.8, 0.9, 40, 1.1, seen) in kept


def test_reference_frequencies_match():
    """Eight candidates, no filtering left active: 20000 reference draws per
    case against the restatement's probabilities (differences of the CDF)."""
    L = Reference().L
    rng = np.random.default_rng(2)
    lg = rng.standard_normal(8).astype(np.float32)
    for T, tk, tp, pen, seen in [(1.0, 0, 1.0, 1.0, []), (0.7, 5, 0.95, 1.5, [1, 3, 3])]:
        _, cdf = sample_token(lg, T, tp, tk, pen, seen, return_cdf=True)
        prob = np.diff(np.concatenate([[0.0], cdf.astype(np.float64)]))
        n = 20000
        counts = np.bincount([ref_sample(L, lg, T, tp, tk, pen, seen) for _ in range(n)], minlength=8)
        assert np.all(np.abs(counts / n - prob) < 5 * np.sqrt(prob * (1 - prob) / n) + 1e-3), (counts / n, prob)
