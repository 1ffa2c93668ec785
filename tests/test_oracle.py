"""CPU tests: the plain-C / numpy restatement (oracle/) against the golden
vectors produced by the reference's own code (tests/golden/make_golden.py),
and -- where the reference build exists -- against the reference directly on
fresh random inputs.  Bit-exact for codes, casts and merges."""
import numpy as np
import pytest

from oracle.oracle import ModelShape, ReferenceModel, forward_prefill


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint16)


def test_f16_truncation_golden(restated, golden):
    out = restated.f32_to_f16(golden["f16_in"])
    assert np.array_equal(out, golden["f16_out"])


def test_f16_expand_all_codes(restated, golden):
    h = np.arange(65536, dtype=np.uint16)
    f = restated.f16_to_f32(h)
    finite = np.isfinite(f)
    # exact round trip for every non-NaN half (truncation of an exact value is the identity)
    rt = restated.f32_to_f16(f[finite])
    assert np.array_equal(rt, h[finite])


def test_i2s_unpack_golden(restated, golden):
    out = restated.i2s_unpack(golden["i2s_raw"], 128 * 6, float(golden["i2s_raw_scale"]))
    assert np.array_equal(bits(out), bits(golden["i2s_raw_out"]))


@pytest.mark.parametrize("ci", range(4))
def test_merge_golden(restated, golden, ci):
    K, N, r, alpha = golden[f"m{ci}_meta"]
    K, N = int(K), int(N)
    f32, f16 = restated.merge(golden[f"m{ci}_i2s"], float(golden[f"m{ci}_scale"]), K, N,
                              golden[f"m{ci}_A"], golden[f"m{ci}_B"], float(alpha))
    assert np.array_equal(bits(f32), bits(golden[f"m{ci}_f32"]))
    assert np.array_equal(f16, golden[f"m{ci}_f16"])
    q, s = restated.quantize_int8_tensor(f16)
    assert np.array_equal(q, golden[f"m{ci}_i8t"])
    assert np.float32(s) == golden[f"m{ci}_i8t_scale"]


def test_merge_zero_codes_carry_delta(restated, golden):
    """Where the ternary code is 0 the merged weight is the LoRA delta alone."""
    K, N, r, alpha = golden["m0_meta"]
    K, N = int(K), int(N)
    f32, _ = restated.merge(golden["m0_i2s"], float(golden["m0_scale"]), K, N, golden["m0_A"],
                            golden["m0_B"], float(alpha))
    base = restated.i2s_unpack(golden["m0_i2s"], K * N, float(golden["m0_scale"])).reshape(N, K)
    zero = base == 0
    assert zero.mean() > 0.2
    delta = (golden["m0_B"].astype(np.float64) @ golden["m0_A"].astype(np.float64)) * (alpha / r)
    np.testing.assert_allclose(f32[zero], delta[zero], rtol=1e-4, atol=1e-12)


def test_gemv_and_rmsnorm_golden(restated, golden):
    y = restated.gemv_f16(golden["gemv_x"], golden["gemv_w16"])
    np.testing.assert_allclose(y, golden["gemv_y"], rtol=2e-5, atol=2e-6)
    n = restated.rms_norm(golden["gemv_x"], golden["rms_w"], 1e-5)
    np.testing.assert_allclose(n, golden["rms_out"], rtol=1e-6, atol=1e-7)


def test_rope_golden(restated, golden):
    q, k = golden["rope_q"], golden["rope_k"]
    S, nh, hd = q.shape
    nkv = k.shape[1]
    for s in range(S):
        qo, ko = restated.rope(q[s].reshape(-1), k[s].reshape(-1), nh, nkv, hd, s, 500000.0)
        np.testing.assert_array_equal(qo.reshape(nh, hd), golden["rope_q_out"][s])
        np.testing.assert_array_equal(ko.reshape(nkv, hd), golden["rope_k_out"][s])


def test_attention_golden(restated, golden):
    q, k, v = golden["rope_q_out"], golden["rope_k_out"], golden["attn_v"]
    S, nh, hd = q.shape
    nkv = k.shape[1]
    for s in range(S):
        out = restated.attention_decode(q[s].reshape(-1), k, v, s + 1, nh, nkv, hd)
        np.testing.assert_allclose(out.reshape(nh, hd), golden["attn_out"][s], rtol=2e-5, atol=2e-6)


def tiny_from_golden(g):
    V, H, L, nh, nkv, I, ms = (int(x) for x in g["tiny_shape"])
    shp = ModelShape(V, H, L, nh, nkv, I, ms)
    w = {"tok_embd": g["tiny_tok_embd"], "output_norm": g["tiny_output_norm"], "layers": []}
    for li in range(L):
        w["layers"].append({k: g[f"tiny_l{li}_{k}"] for k in
                            ["wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "attn_norm",
                             "attn_sub_norm", "ffn_norm", "ffn_sub_norm"]})
    return shp, w


def test_model_forward_prefill_golden(restated, golden):
    shp, w = tiny_from_golden(golden)
    logits = forward_prefill(shp, w, golden["tiny_tokens"], restated.f16_to_f32)
    ref = golden["tiny_logits"]
    err = np.abs(logits - ref).max() / np.abs(ref).max()
    assert err < 1e-4, err
    assert np.array_equal(logits.argmax(-1), ref.argmax(-1))


# ---- restatement vs the reference build on fresh inputs -------------------------
@pytest.mark.parametrize("K,N,r", [(128, 5, 2), (640, 33, 16), (1024, 16, 32)])
def test_merge_matches_reference(restated, reference, K, N, r):
    rng = np.random.default_rng(K + N + r)
    lat = rng.standard_normal((N, K)).astype(np.float32)
    s = float(np.abs(lat).mean())
    codes = (np.round(np.clip(lat / s, -1, 1)) + 1).astype(np.uint8)
    i2s = restated.i2s_pack(codes)
    A = (rng.standard_normal((r, K)) / np.sqrt(K)).astype(np.float32)
    B = (rng.standard_normal((N, r)) * 1e-3).astype(np.float32)
    f32, f16 = restated.merge(i2s, s, K, N, A, B, 2.0 * r)
    assert np.array_equal(bits(f32), bits(reference.merge_f32(i2s, s, K, N, A, B, 2.0 * r)))
    assert np.array_equal(f16, reference.apply_lora_f16(i2s, s, K, N, A, B, 2.0 * r))


def test_i2s_pack_matches_reference_quantizer(restated, reference):
    """tensor_quantize_i2_s (max-abs scale, sign threshold) packs the same bits."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal(128 * 5).astype(np.float32)
    x[rng.random(x.size) < 0.3] = 0.0
    packed, scale = reference.i2s_quantize(x)
    q8 = np.where(np.abs(x) < 1e-6, 1, np.where(x > 0, 2, 0)).astype(np.uint8)
    assert np.array_equal(restated.i2s_pack(q8), packed)
    assert np.array_equal(bits(restated.i2s_unpack(packed, x.size, scale)),
                          bits(reference.i2s_dequant(packed, x.size, scale)))


def test_model_restatement_vs_reference_random(restated, reference):
    rng = np.random.default_rng(11)
    shp = ModelShape(vocab=300, hidden=256, layers=1, heads=2, kv_heads=2, inter=256, max_seq=32)
    Hq = Hk = 256
    dims = {"wq": (Hq, 256), "wk": (Hk, 256), "wv": (Hk, 256), "wo": (256, Hq),
            "w_gate": (256, 256), "w_up": (256, 256), "w_down": (256, 256)}
    lw = {n: restated.f32_to_f16((rng.standard_normal(d) / 16).astype(np.float32))
          for n, d in dims.items()}
    for n in ["attn_norm", "attn_sub_norm", "ffn_norm", "ffn_sub_norm"]:
        lw[n] = np.ones(256, np.float32)
    w = {"tok_embd": restated.f32_to_f16((rng.standard_normal((300, 256)) * 0.02).astype(np.float32)),
         "output_norm": np.ones(256, np.float32), "layers": [lw]}
    toks = rng.integers(0, 300, 7).astype(np.int32)
    rm = ReferenceModel(reference, shp, w)
    ref = rm.forward_prefill(toks)
    rm.close()
    mine = forward_prefill(shp, w, toks, restated.f16_to_f32)
    assert np.abs(mine - ref).max() / np.abs(ref).max() < 1e-4
