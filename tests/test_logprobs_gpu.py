"""Log-probabilities of a scored sequence on the device (tvb_score_logprobs)
against the reference's own Model::score_logprobs (model.cpp:1746-1831, run
from oracle/_ref on the same merged weights): every scored token's
log-probability within 2e-3 of the largest |log-probability| (the tolerance
the logits tests use relative to the largest |logit|: the reference runs the
layers as F32 CPU GEMVs and sums the softmax sequentially in F32, here the
tensor-core prefill and a tree sum), the top-k values within it, and the
top-k ids equal wherever neighbouring log-probabilities are clear of it.  Covers a start
position, a prompt longer than one prefill chunk (scored rows in every chunk)
and k = 0."""
import dataclasses

import numpy as np
import pytest

from oracle.oracle import ModelShape, Reference, ReferenceModel

pytestmark = pytest.mark.gpu

RTOL = 2e-3   # of the largest |log-probability|, as the logits tests' 2e-3 of the largest |logit|


def shape_of(cfg):
    return ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads, cfg.num_kv_heads,
                      cfg.intermediate_size, cfg.max_seq_len, cfg.rope_theta, cfg.rms_norm_eps)


@pytest.mark.parametrize("T,start,k,max_prefill", [(40, 0, 5, 256), (90, 30, 8, 256), (150, 0, 4, 64),
                                                   (20, 5, 0, 256)])
def test_score_logprobs_matches_reference(T, start, k, max_prefill):
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    cfg = dataclasses.replace(SHAPES["small"], max_seq_len=256, max_prefill=max_prefill)
    m = Model.load(SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=9))
    tokens = np.random.default_rng(T + start).integers(0, cfg.vocab_size, T).astype(np.int32)
    lp, ids, top = m.backend.score_logprobs(tokens, k, start)
    ref = ReferenceModel(Reference(), shape_of(cfg), m.host_weights())
    rlp, rids, rtop = ref.score_logprobs(tokens, max(k, 1), start)
    n = T - max(1, start)
    assert lp.shape == (n,) and rlp.shape == (n,)
    tol = RTOL * float(np.max(np.abs(rlp)))
    assert np.max(np.abs(lp - rlp)) < tol, (np.max(np.abs(lp - rlp)), tol)
    if k:
        assert np.max(np.abs(top - rtop)) < tol
        for i in range(n):
            for j in range(k):
                gap = min(abs(rtop[i, j] - rtop[i, j - 1]) if j > 0 else 1.0,
                          abs(rtop[i, j] - rtop[i, j + 1]) if j + 1 < k else 1.0)
                if gap > 2 * tol:
                    assert ids[i, j] == rids[i, j], (i, j)
    m.backend.close()
