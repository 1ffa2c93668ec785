"""The device sampler (tvb_sample) against the restatement of the reference's
sample_token (pinned by tests/test_sampler.py) with the same uniform draws:
the same token for every row, except a row whose draw lies within 1e-5 of the
boundary between the restated token and its neighbour in the cumulative
distribution, which may draw that neighbour (the device's expf and tree sums
may move a boundary by a few F32 ulps).  Rows up to 196,608 entries run on one
8-CTA cluster per row (100, 1000 and 128,256 here, the first with CTAs whose
slice is empty); the 200,000-entry rows take the single-CTA kernel, and so does
top-p with top_k 0 or above 1024 (the nucleus searched 1024 keys at a time)."""
import ctypes as C

import numpy as np
import pytest

from oracle.oracle import sample_token

pytestmark = pytest.mark.gpu


def run(lib, torch, logits, cfg, seen, u):
    from ternative_b200._lib import SamplerConfig
    B, V = logits.shape
    max_seen = max(1, max(len(s) for s in seen))
    sd = np.zeros((B, max_seen), np.int32)
    for b, s in enumerate(seen):
        sd[b, :len(s)] = s
    d_lg = torch.from_numpy(logits).cuda()
    d_seen = torch.from_numpy(sd).cuda()
    d_n = torch.tensor([len(s) for s in seen], dtype=torch.int32).cuda()
    d_u = torch.from_numpy(np.asarray(u, np.float32)).cuda()
    d_out = torch.full((B,), -1, dtype=torch.int32).cuda()
    c = SamplerConfig(*cfg)
    st = lib.tvb_sample(d_lg.data_ptr(), B, V, V, C.byref(c), d_seen.data_ptr(), d_n.data_ptr(), max_seen,
                        d_u.data_ptr(), d_out.data_ptr(), None)
    torch.cuda.synchronize()
    return st, d_out.cpu().numpy()


@pytest.mark.parametrize("V", [100, 1000, 128256, 200000])
@pytest.mark.parametrize("cfg", [(0.8, 0.9, 40, 1.1), (1.0, 1.0, 0, 1.0), (0.5, 0.95, 1024, 1.2),
                                 (0.0, 0.5, 1, 1.0), (1.3, 1.0, 7, 1.0)])
def test_device_sampler_matches_restatement(V, cfg):
    import torch
    from ternative_b200 import load
    lib = load()
    rng = np.random.default_rng(V + int(cfg[2]))
    B = 6
    logits = (rng.standard_normal((B, V)) * 2.5).astype(np.float32)
    seen = [rng.integers(0, V, n).tolist() for n in (0, 5, 40, 200, 3, 77)]
    u = rng.random(B).astype(np.float32)
    u[0] = 0.0   # the first index whose running sum is >= 0
    st, got = run(lib, torch, logits, cfg, seen, u)
    assert st == 0, lib.tvb_last_error()
    T, tp, tk, pen = cfg
    for b in range(B):
        tok, cdf = sample_token(logits[b], T, tp, tk, pen, seen[b], u=float(u[b]), return_cdf=True)
        if got[b] == tok:
            continue
        # Every row draws the restated token, except where its draw lies within
        # 1e-5 of the boundary between that token and the device's: the two are
        # neighbours in the cumulative sum (nothing of nonzero probability lies
        # between them) and |u - the running sum at the first of them| <= 1e-5
        # (the device's expf and tree sums move a boundary by a few F32 ulps).
        assert cdf is not None and u[b] > 0, (b, got[b], tok)
        g = int(got[b])
        lo, hi = min(g, tok), max(g, tok)
        neighbours = float(cdf[hi - 1]) == float(cdf[lo])
        near = abs(float(u[b]) - float(cdf[lo])) <= 1e-5
        assert neighbours and near, (b, g, tok, float(u[b]), float(cdf[lo]))


@pytest.mark.parametrize("V", [1000, 128256])
@pytest.mark.parametrize("cfg,scale", [((0.8, 0.9, 0, 1.1), 2.5), ((1.0, 0.95, 5000, 1.0), 2.5),
                                       ((1.0, 0.9, 0, 1.0), 0.05)])
def test_device_sampler_top_p_over_the_whole_vocabulary(V, cfg, scale):
    """top_p with top_k 0 (the nucleus over every token) or above 1024: the
    one-CTA kernel takes the sorted probabilities 1024 at a time; scale 0.05
    makes the distribution nearly flat, so the nucleus holds ~90% of the
    vocabulary (over a hundred rounds at 128,256 entries)."""
    import torch
    from ternative_b200 import load
    lib = load()
    rng = np.random.default_rng(V + int(cfg[2]) + int(100 * scale))
    B = 4
    logits = (rng.standard_normal((B, V)) * scale).astype(np.float32)
    seen = [rng.integers(0, V, n).tolist() for n in (0, 5, 40, 3)]
    u = rng.random(B).astype(np.float32)
    st, got = run(lib, torch, logits, cfg, seen, u)
    assert st == 0, lib.tvb_last_error()
    T, tp, tk, pen = cfg
    for b in range(B):
        tok, cdf = sample_token(logits[b], T, tp, tk, pen, seen[b], u=float(u[b]), return_cdf=True)
        if got[b] == tok:
            continue
        g = int(got[b])
        lo, hi = min(g, tok), max(g, tok)
        neighbours = float(cdf[hi - 1]) == float(cdf[lo])
        near = abs(float(u[b]) - float(cdf[lo])) <= 1e-5
        assert neighbours and near, (b, g, tok, float(u[b]), float(cdf[lo]))
