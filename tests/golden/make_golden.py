"""Generate tests/golden/golden.npz by running the REFERENCE's own CPU code
(oracle/_ref/libtvref.so, built from the reference sources by oracle/Makefile)
on small seeded inputs.  The reference ships no tests or fixtures, so these
vectors are the pin for the plain-C restatement in oracle/tvoracle.c and for
the numpy model restatement in oracle/oracle.py.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.oracle import ModelShape, Reference, ReferenceModel, build  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden", "golden.npz")


def ternary_codes(rng, N, K):
    lat = rng.standard_normal((N, K)).astype(np.float32)
    s = np.float32(np.abs(lat).mean())
    return (np.round(np.clip(lat / s, -1, 1)) + 1).astype(np.uint8), s


def pack(codes):
    N, K = codes.shape
    c = codes.reshape(N, K // 128, 4, 32).astype(np.uint8)
    return ((c[:, :, 0] << 6) | (c[:, :, 1] << 4) | (c[:, :, 2] << 2) | c[:, :, 3]).reshape(-1)


def main():
    build(reference=True)
    ref = Reference()
    rng = np.random.default_rng(20261201)
    g = {}

    # F32 -> F16 truncation edge values and a random spread (tensor.cpp:33-57)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.0, 65520.0, 1e10, -1e10, np.inf, -np.inf,
                     6.1035156e-05, 6.0e-05, 5.96e-08, 2.98e-08, 2.9e-8, 1e-9, -3.3e-7,
                     0.33333334, -0.9999999, 1.0009766, 1.0009765], np.float32)
    spread = (rng.standard_normal(4096) * 10.0 ** rng.uniform(-9, 5, 4096)).astype(np.float32)
    f16_in = np.concatenate([edge, spread]).astype(np.float32)
    g["f16_in"] = f16_in
    g["f16_out"] = ref.f32_to_f16(f16_in)

    # I2_S unpack incl. the unused code 3 (-> 0), tensor.cpp:1006-1050
    raw = rng.integers(0, 256, 32 * 6, dtype=np.uint8)
    g["i2s_raw"] = raw
    g["i2s_raw_scale"] = np.float32(0.7312)
    g["i2s_raw_out"] = ref.i2s_dequant(raw, 128 * 6, 0.7312)

    # Merges: (K, N, r, alpha) incl. ragged N, rank 1 and rank 64
    cases = [(256, 40, 16, 32.0), (384, 7, 3, 6.0), (128, 9, 1, 2.0), (512, 24, 64, 128.0)]
    for ci, (K, N, r, alpha) in enumerate(cases):
        codes, s = ternary_codes(rng, N, K)
        A = (rng.standard_normal((r, K)) / np.sqrt(K)).astype(np.float32)
        B = (rng.standard_normal((N, r)) * 1e-3).astype(np.float32)
        i2s = pack(codes)
        g[f"m{ci}_i2s"] = i2s
        g[f"m{ci}_scale"] = np.float32(s)
        g[f"m{ci}_A"] = A
        g[f"m{ci}_B"] = B
        g[f"m{ci}_meta"] = np.array([K, N, r, alpha], np.float64)
        g[f"m{ci}_f32"] = ref.merge_f32(i2s, s, K, N, A, B, alpha)
        f16 = ref.apply_lora_f16(i2s, s, K, N, A, B, alpha)
        g[f"m{ci}_f16"] = f16
        q, qs = ref.quantize_int8_tensor(f16)
        g[f"m{ci}_i8t"] = q
        g[f"m{ci}_i8t_scale"] = np.float32(qs)

    # GEMV with F16 weights (tensor_matmul M=1 AVX2 path) and rms_norm
    K, N = 256, 72
    x = rng.standard_normal(K).astype(np.float32)
    w16 = ref.f32_to_f16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    g["gemv_x"], g["gemv_w16"] = x, w16
    g["gemv_y"] = ref.matmul_f16(x[None, :], w16)[0]
    nw = (1.0 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    g["rms_w"] = nw
    g["rms_out"] = ref.rms_norm(x[None, :], nw, 1e-5)[0]

    # Batched RoPE (tensor.cpp:890-940) and causal GQA attention (model.cpp:1071-1137)
    S, nh, nkv, hd = 9, 4, 2, 128
    q = rng.standard_normal((S, nh, hd)).astype(np.float32)
    k = rng.standard_normal((S, nkv, hd)).astype(np.float32)
    v = rng.standard_normal((S, nkv, hd)).astype(np.float32)
    g["rope_q"], g["rope_k"] = q, k
    qr, kr = ref.rope_batched(q, k, nh, nkv, hd, 0, 500000.0)
    g["rope_q_out"], g["rope_k_out"] = qr, kr
    g["attn_v"] = v
    g["attn_out"] = ref.batched_attention(qr, kr, v, S, nh, nkv, hd).reshape(S, nh, hd)

    # Whole tiny model: teacher-forced forward_prefill logits (model.cpp:1139-1234)
    shp = ModelShape(vocab=512, hidden=256, layers=2, heads=2, kv_heads=1, inter=384, max_seq=64)
    weights = {"tok_embd": ref.f32_to_f16((rng.standard_normal((shp.vocab, shp.hidden)) * 0.02)
                                          .astype(np.float32)),
               "output_norm": np.ones(shp.hidden, np.float32), "layers": []}
    Hq, Hk = shp.heads * shp.head_dim, shp.kv_heads * shp.head_dim
    dims = {"wq": (Hq, shp.hidden), "wk": (Hk, shp.hidden), "wv": (Hk, shp.hidden),
            "wo": (shp.hidden, Hq), "w_gate": (shp.inter, shp.hidden),
            "w_up": (shp.inter, shp.hidden), "w_down": (shp.hidden, shp.inter)}
    for li in range(shp.layers):
        lw = {}
        for name, (n_, k_) in dims.items():
            lw[name] = ref.f32_to_f16((rng.standard_normal((n_, k_)) * (1.0 / np.sqrt(k_)))
                                      .astype(np.float32))
            g[f"tiny_l{li}_{name}"] = lw[name]
        for name, n_ in {"attn_norm": shp.hidden, "attn_sub_norm": Hq, "ffn_norm": shp.hidden,
                         "ffn_sub_norm": shp.inter}.items():
            lw[name] = (1.0 + 0.05 * rng.standard_normal(n_)).astype(np.float32)
            g[f"tiny_l{li}_{name}"] = lw[name]
        weights["layers"].append(lw)
    g["tiny_tok_embd"] = weights["tok_embd"]
    g["tiny_output_norm"] = weights["output_norm"]
    g["tiny_shape"] = np.array([shp.vocab, shp.hidden, shp.layers, shp.heads, shp.kv_heads,
                                shp.inter, shp.max_seq], np.int64)
    toks = rng.integers(0, shp.vocab, 12).astype(np.int32)
    g["tiny_tokens"] = toks
    rm = ReferenceModel(ref, shp, weights)
    g["tiny_logits"] = rm.forward_prefill(toks)
    rm.close()

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: {len(g)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
