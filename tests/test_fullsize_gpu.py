"""Full-size parity of the fused decode path on the BitNet-b1.58-2B shape
(hidden 2560, 30 layers, 20/5 heads, FFN 6912, vocab 128256) against the
reference's own Model::forward_prefill (oracle/_ref, src/model.cpp:1139-1234),
teacher-forced over the tokens the device generated:

* all-F16 layers, I2_S + rank-16 LoRA alpha 32 merged on the device (seed 0):
  a 32-token prompt of uniform-random ids, then 128 greedy tokens.  The
  reference's forward_prefill over prompt + generated tokens, on the same
  merged F16 weights, must put its argmax on every generated token, and every
  step's device logits must lie within 2e-3 of the reference's row.
* layers 0-13 F16 and 14-29 per-row INT8: a 1024-token prompt, then 256
  greedy tokens at positions 1024..1279 (past the reference GPU path's
  1024-slot KV cache, so its CPU forward_prefill is the only oracle there).
  The reference runs the INT8 layers on their exact dequantised values (code x
  row scale, F32 weights); its forward_prefill_hidden gives the final-norm
  rows and the tied lm_head of the 256 decoded rows is applied here in F32.

Norm weights.  With every norm weight 1.0 (the measured workload's values)
this random-weight model is ill-conditioned: q and k entries have a standard
deviation of about 34, so q.k/sqrt(128) has one of about 1100 and every
softmax is nearly a hard maximum whose near-ties amplify rounding noise.  The
reference's own F32 forward_prefill and its float64 restatement then already
differ by 4e-2 (relative) in the logits of the 4th token of a 4-token prompt,
so token identity there would test summation order, not correctness.  The
parity models below keep every shape and weight distribution and set the norm
weights to 1/32 (exact in binary), which brings q.k/sqrt(128) to a standard
deviation of about 1.1.  A mismatch reports the reference's top-2 margin.
"""
import numpy as np
import pytest

from oracle.oracle import ModelShape, ReferenceModel

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

RTOL = 2e-3   # GEMV/layer outputs within 2e-3 relative (max |a - b| / max |b| per row)
NORM = 1.0 / 32   # every norm weight (see the module docstring)


def rel_err(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def oracle_shape(cfg):
    return ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                      cfg.num_kv_heads, cfg.intermediate_size, cfg.max_seq_len, cfg.rope_theta,
                      cfg.rms_norm_eps)


def decode_with_logits(m, prompt, n_new):
    """Prefill, then n_new steps through tvb_decode_step (host logits out).
    Returns (tokens prompt + generated, logits [n_new][V] of each generated token)."""
    be = m.backend
    be.clear_kv_d()
    lg, tok = be.prefill(prompt)
    toks = [int(t) for t in prompt] + [int(tok)]
    rows = [lg]
    for _ in range(n_new - 1):
        lg, tok = be.decode_step(toks[-1], len(toks) - 1)
        rows.append(lg)
        toks.append(int(tok))
    return np.asarray(toks, np.int32), np.stack(rows)


def check_rows(dev_logits, ref_logits, toks, first):
    """Row i of both predicts token first + i + 1."""
    bad = []
    worst = 0.0
    for i in range(dev_logits.shape[0]):
        ref = ref_logits[i]
        err = rel_err(dev_logits[i], ref)
        worst = max(worst, err)
        want = int(toks[first + i + 1])
        if int(np.argmax(ref)) != want or err >= RTOL:
            top2 = np.sort(ref)[-2:]
            bad.append(f"t={first + i}: ref argmax {int(np.argmax(ref))} vs device {want}, "
                       f"ref top-2 margin {top2[1] - top2[0]:.3g}, rel err {err:.3g}")
    assert not bad, "\n".join(bad[:10])
    return worst


@pytest.fixture(scope="module")
def synth_2b(cuda):
    from ternative_b200.model import SHAPES, SyntheticModel
    import dataclasses
    cfg = dataclasses.replace(SHAPES["bitnet-2b"], max_seq_len=1536)
    return SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=0, norm_value=NORM)


def test_bitnet2b_greedy_128_matches_reference(synth_2b, reference):
    from ternative_b200.model import Model
    cfg = synth_2b.cfg
    m = Model.load(synth_2b)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, 32).astype(np.int32)
    toks, dev = decode_with_logits(m, prompt, 128)
    # the device-chained greedy loop (no host between steps) gives the same ids
    assert list(m.generate_greedy(prompt, 128)) == list(toks)
    hw = m.host_weights()
    m.backend.close()
    rm = ReferenceModel(reference, oracle_shape(cfg), hw)
    del hw
    ref = rm.forward_prefill(toks[:-1])
    rm.close()
    worst = check_rows(dev, ref[len(prompt) - 1:], toks, len(prompt) - 1)
    print(f"2B F16: 128 greedy tokens identical, worst row rel err {worst:.3g}")


def test_bitnet2b_mixed_int8_past_1024_matches_reference(synth_2b, reference, restated):
    from ternative_b200._lib import TVB_I8_ROW
    from ternative_b200.model import Model
    cfg = synth_2b.cfg
    m = Model.load(synth_2b, int8_layers=range(14, cfg.num_layers))
    assert m.layer_dtype[13] != TVB_I8_ROW and m.layer_dtype[14] == TVB_I8_ROW
    prompt = np.random.default_rng(3).integers(0, cfg.vocab_size, 1024).astype(np.int32)
    toks, dev = decode_with_logits(m, prompt, 256)
    hw = m.host_weights()
    for li in range(14, cfg.num_layers):
        for name, q in hw["layers"][li].items():
            if q.dtype == np.int8:
                s = m.row_scales[li][name].cpu().numpy()
                hw["layers"][li][name] = q.astype(np.float32) * s[:, None]
    m.backend.close()
    rm = ReferenceModel(reference, oracle_shape(cfg), hw)
    hidden = rm.forward_prefill_hidden(toks[:-1])[len(prompt) - 1:]
    rm.close()
    emb = restated.f16_to_f32(hw["tok_embd"])
    del hw
    ref = hidden @ emb.T   # the tied lm_head (model.cpp:1227-1231) on the decoded rows
    del emb
    worst = check_rows(dev, ref, toks, len(prompt) - 1)
    print(f"2B mixed F16/INT8: 256 greedy tokens past 1024 identical, worst row rel err {worst:.3g}")
