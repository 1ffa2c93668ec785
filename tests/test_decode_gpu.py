"""GPU parity of the fused, graph-captured decode/prefill steps against the
oracle on small BitNet-shaped models:

* every decode step's logits vs the numpy restatement's teacher-forced
  forward over the same tokens (2e-3 relative) and vs the reference's own
  Model::forward_prefill (oracle/_ref, when built);
* greedy tokens identical to the argmax of the oracle's teacher-forced logits;
* KV-cache rows identical in layout and within tolerance of the reference's;
* mixed F16 / per-row INT8 layers against the oracle run on the dequantised
  INT8 weights.
"""
import numpy as np
import pytest

from oracle.oracle import ModelShape, ReferenceModel, forward_prefill

pytestmark = pytest.mark.gpu

RTOL = 2e-3


def rel_err(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def oracle_shape(cfg):
    return ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                      cfg.num_kv_heads, cfg.intermediate_size, cfg.max_seq_len, cfg.rope_theta,
                      cfg.rms_norm_eps)


@pytest.fixture(scope="module")
def small_model(cuda):
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    cfg = SHAPES["small"]
    synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=1)
    m = Model.load(synth)
    return cfg, m, m.host_weights()


def test_prefill_and_decode_match_oracle(small_model, restated):
    cfg, m, hw = small_model
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, cfg.vocab_size, 8).astype(np.int32)
    m.backend.clear_kv_d()
    last, am = m.backend.prefill(prompt)
    toks = list(prompt) + [am]
    step_logits = [last]
    for i in range(12):
        lg, am = m.backend.decode_step(toks[-1], len(toks) - 1)
        step_logits.append(lg)
        toks.append(am)
    ref = forward_prefill(oracle_shape(cfg), hw, toks[:-1], restated.f16_to_f32)
    for i, lg in enumerate(step_logits):
        row = len(prompt) - 1 + i
        assert rel_err(lg, ref[row]) < RTOL, (i, rel_err(lg, ref[row]))
        assert int(np.argmax(lg)) == toks[row + 1]


def test_greedy_teacher_forced_vs_reference(small_model, reference):
    cfg, m, hw = small_model
    rng = np.random.default_rng(1)
    prompt = rng.integers(0, cfg.vocab_size, 16).astype(np.int32)
    seq = m.generate_greedy(prompt, 40)
    rm = ReferenceModel(reference, oracle_shape(cfg), hw)
    logits = rm.forward_prefill(seq[:-1])
    for t in range(len(prompt) - 1, len(seq) - 1):
        top2 = np.sort(logits[t])[-2:]
        assert int(np.argmax(logits[t])) == seq[t + 1], \
            f"t={t}: margin {top2[1] - top2[0]:.3g}"
    # KV rows written by the GPU steps vs the reference's CPU KV cache
    for layer in range(cfg.num_layers):
        k_ref, v_ref = rm.kv(layer, len(seq) - 1)
        k_gpu = np.stack([m.backend.download_kv_slot_d(layer, p, k_ref.shape[1])
                          for p in range(0, len(seq) - 1, 7)])
        assert rel_err(k_gpu, k_ref[::7]) < RTOL
    rm.close()


def test_generate_greedy_matches_stepwise(small_model):
    cfg, m, _ = small_model
    prompt = np.arange(5, dtype=np.int32) * 17
    seq = m.generate_greedy(prompt, 10)
    m.backend.clear_kv_d()
    _, am = m.backend.prefill(prompt, want_logits=False)
    toks = list(prompt) + [am]
    for _ in range(9):
        _, am = m.backend.decode_step(toks[-1], len(toks) - 1, want_logits=False)
        toks.append(am)
    assert list(seq) == toks


def test_mixed_int8_layers(cuda, restated):
    from ternative_b200._lib import TVB_I8_ROW
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    cfg = SHAPES["small"]
    synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=2)
    m = Model.load(synth, int8_layers=[1, 2])
    assert m.layer_dtype == [1, TVB_I8_ROW, TVB_I8_ROW]
    hw = m.host_weights()
    # oracle weights: the INT8 codes times their row scales, as F32 -> exact F16 not needed,
    # so feed F32 through a custom f16_to_f32 that passes F32 through.
    for li in (1, 2):
        for name in ["wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"]:
            q = hw["layers"][li][name].astype(np.float32)
            s = m.row_scales[li][name].cpu().numpy()
            hw["layers"][li][name] = (q * s[:, None]).astype(np.float32)

    def to32(w):
        return restated.f16_to_f32(w) if w.dtype == np.uint16 else w

    prompt = np.array([3, 14, 15, 92, 65, 35], np.int32)
    m.backend.clear_kv_d()
    last, am = m.backend.prefill(prompt)
    ref = forward_prefill(oracle_shape(cfg), hw, prompt, to32)
    assert rel_err(last, ref[-1]) < RTOL
    lg, _ = m.backend.decode_step(am, len(prompt))
    ref = forward_prefill(oracle_shape(cfg), hw, list(prompt) + [am], to32)
    assert rel_err(lg, ref[-1]) < RTOL


def test_decode_rejects_out_of_range(small_model):
    from ternative_b200 import TvbError
    cfg, m, _ = small_model
    with pytest.raises(TvbError, match="KV capacity"):
        m.backend.decode_step(1, cfg.max_seq_len)
    with pytest.raises(TvbError, match="vocab"):
        m.backend.decode_step(cfg.vocab_size, 0)
