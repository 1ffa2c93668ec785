"""GPU parity of the batched decode step (tvb_decode_batch): B sequences in
their own KV cache slots, each advanced one token per step with every weight
read once for all rows (tensor-core GEMM with B activation rows, split over
K).  The reference serves one sequence at a time (Model::forward_gpu,
model.cpp:1354-1582; a batch of 8 is 8 sequential runs), so each sequence of
the batch is checked against the single-sequence path -- prefill of its prompt
then decode steps over the same tokens (teacher-forced) -- which the decode
parity tests pin to the oracle: logits within 2e-3 relative, next tokens equal
to the argmax of the batch's own logits, and equal to the single-sequence
argmax wherever its top-2 margin is clear of the tolerance."""
import dataclasses

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 2e-3


def rel_err(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def run_case(cfg_name, lens, steps, int8_layers=()):
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    B = len(lens)
    cfg = dataclasses.replace(SHAPES[cfg_name], max_batch=B, max_seq_len=256, max_prefill=256)
    synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=11)
    rng = np.random.default_rng(sum(lens))
    prompts = [rng.integers(0, cfg.vocab_size, n).astype(np.int32) for n in lens]

    m = Model.load(synth, int8_layers=int8_layers)
    be = m.backend
    be.clear_kv_d()
    toks = []
    for b, p in enumerate(prompts):
        _, am = be.prefill_slot(b, p, want_logits=False)
        toks.append([int(t) for t in p] + [am])
    batch_logits = []
    for _ in range(steps):
        cur = np.array([t[-1] for t in toks], np.int32)
        pos = np.array([len(t) - 1 for t in toks], np.int32)
        lg, nxt = be.decode_batch(cur, pos)
        for b in range(B):
            assert nxt[b] == int(np.argmax(lg[b])), (b, nxt[b])
            toks[b].append(int(nxt[b]))
        batch_logits.append(lg)
    m.backend.close()

    ref = Model.load(SyntheticModel.generate(dataclasses.replace(cfg, max_batch=1), rank=16, alpha=32.0,
                                             seed=11), int8_layers=int8_layers)
    for b in range(B):
        rb = ref.backend
        rb.clear_kv_d()
        n = lens[b]
        _, am = rb.prefill(prompts[b], want_logits=False)
        assert am == toks[b][n], (b, "prefill into a slot differs from prefill into slot 0")
        for i in range(steps):
            lg, _ = rb.decode_step(toks[b][n + i], n + i)
            err = rel_err(batch_logits[i][b], lg)
            assert err < RTOL, (b, i, err)
            top2 = np.sort(lg)[-2:]
            if top2[1] - top2[0] > 10 * RTOL * np.abs(lg).max():
                assert toks[b][n + i + 1] == int(np.argmax(lg)), (b, i)
    ref.backend.close()


def test_batch_decode_three_sequences():
    """Three prompts of different lengths (different positions and KV lengths
    per row), six batched steps."""
    run_case("small", [5, 17, 40], 6)


def test_batch_decode_eight_sequences_int8_layers():
    """Eight sequences (the 8-sequence serving batch) with INT8 per-row layers
    mixed in (their weights widened to F16 for the tensor cores, scales in the
    epilogue)."""
    run_case("small", [3, 8, 12, 20, 31, 33, 64, 100], 4, int8_layers=(1,))


def test_batch_decode_single_row():
    """B = 1 through the batched path equals the single-sequence step."""
    run_case("tiny", [9], 5)


def test_batch_decode_rejects_bad_arguments():
    from ternative_b200 import TvbError
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    cfg = dataclasses.replace(SHAPES["tiny"], max_batch=2)
    m = Model.load(SyntheticModel.generate(cfg, rank=4, alpha=8.0, seed=1))
    with pytest.raises(TvbError, match="B=3"):
        m.backend.decode_batch(np.zeros(3, np.int32), np.zeros(3, np.int32))
    with pytest.raises(TvbError, match="position"):
        m.backend.decode_batch(np.zeros(2, np.int32), np.array([0, cfg.max_seq_len], np.int32))
    with pytest.raises(TvbError, match="slot"):
        m.backend.prefill_slot(2, np.zeros(4, np.int32))
    m.backend.close()
