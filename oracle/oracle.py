"""Test infrastructure only: Python access to the two oracles.

* ``Restated`` -- ``libtvoracle.so``, the plain-C restatement of the reference's
  CPU arithmetic (tvoracle.c), plus numpy restatements of the model-level
  forward (``forward_prefill`` below, following src/model.cpp:1139-1234).
* ``Reference`` -- ``_ref/libtvref.so``, the reference's OWN sources compiled by
  oracle/Makefile behind a C-ABI harness (ref_harness.cpp).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg use
this module, and only as the checker.  The product path never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
RESTATED_SO = os.path.join(HERE, "libtvoracle.so")
REFERENCE_SO = os.path.join(HERE, "_ref", "libtvref.so")
DROPIN_SO = os.path.join(HERE, "_ref", "libtvref_dropin.so")
# Where the reference sources lie (oracle/Makefile's REF); only build() reads it.
REFERENCE_SRC = os.environ.get("TVB_REFERENCE_SRC", "/root/reference")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64 = C.c_int64


def build(reference: bool = True) -> None:
    """Compile the restatement (and, where the reference sources exist, the
    reference harness) with oracle/Makefile."""
    targets = ["libtvoracle.so"]
    if reference and os.path.isdir(REFERENCE_SRC):
        targets += ["ref", "dropin"]
    subprocess.run(["make", "-s", "-C", HERE, f"REF={REFERENCE_SRC}", *targets], check=True)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------------------
# Restated oracle (plain C)
# ---------------------------------------------------------------------------
class Restated:
    def __init__(self, path: str = RESTATED_SO):
        if not os.path.exists(path):
            build(reference=False)
        L = C.CDLL(path)
        L.tvo_f32_to_f16_n.argtypes = [_f32p, _i64, _u16p]
        L.tvo_f16_to_f32_n.argtypes = [_u16p, _i64, _f32p]
        L.tvo_i2s_unpack.argtypes = [_u8p, _i64, C.c_float, _f32p]
        L.tvo_i2s_pack.argtypes = [_u8p, _i64, _u8p]
        L.tvo_merge.argtypes = [_u8p, C.c_float, _i64, _i64, _f32p, _f32p, C.c_int, C.c_float,
                                C.c_void_p, C.c_void_p]
        L.tvo_quantize_int8_tensor.argtypes = [_u16p, _i64, _i8p, C.POINTER(C.c_float)]
        L.tvo_quantize_int8_rows.argtypes = [_u16p, _i64, _i64, _i8p, _f32p]
        L.tvo_gemv_f16.argtypes = [_f32p, _u16p, _i64, _i64, _f32p]
        L.tvo_gemv_int8.argtypes = [_f32p, _i8p, C.c_void_p, C.c_float, _i64, _i64, _f32p]
        L.tvo_rms_norm.argtypes = [_f32p, _i64, _f32p, C.c_float, _f32p]
        L.tvo_rope.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.tvo_rope_table.argtypes = [C.c_int, C.c_int, C.c_float, _f32p, _f32p]
        L.tvo_attention_decode.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int,
                                           C.c_int, _f32p]
        self.L = L

    def f32_to_f16(self, x):
        x = _c(x, np.float32)
        out = np.empty(x.shape, np.uint16)
        self.L.tvo_f32_to_f16_n(x.reshape(-1), x.size, out.reshape(-1))
        return out

    def f16_to_f32(self, h):
        h = _c(h, np.uint16)
        out = np.empty(h.shape, np.float32)
        self.L.tvo_f16_to_f32_n(h.reshape(-1), h.size, out.reshape(-1))
        return out

    def i2s_unpack(self, codes, n, scale):
        out = np.empty(n, np.float32)
        self.L.tvo_i2s_unpack(_c(codes, np.uint8), n, scale, out)
        return out

    def i2s_pack(self, q8):
        q8 = _c(q8, np.uint8).reshape(-1)
        out = np.empty(((q8.size + 127) // 128) * 32, np.uint8)
        self.L.tvo_i2s_pack(q8, q8.size, out)
        return out

    def merge(self, codes, scale, K, N, A, B, alpha):
        """-> (merged F32 [N][K], merged F16 bits [N][K])."""
        A = _c(A, np.float32)
        B = _c(B, np.float32)
        r = A.shape[0]
        f32 = np.empty((N, K), np.float32)
        f16 = np.empty((N, K), np.uint16)
        self.L.tvo_merge(_c(codes, np.uint8), scale, K, N, A, B, r, alpha,
                         f32.ctypes.data, f16.ctypes.data)
        return f32, f16

    def quantize_int8_rows(self, w16):
        w16 = _c(w16, np.uint16)
        N, K = w16.shape
        q = np.empty((N, K), np.int8)
        s = np.empty(N, np.float32)
        self.L.tvo_quantize_int8_rows(w16, N, K, q, s)
        return q, s

    def quantize_int8_tensor(self, w16):
        w16 = _c(w16, np.uint16)
        q = np.empty(w16.shape, np.int8)
        s = C.c_float()
        self.L.tvo_quantize_int8_tensor(w16.reshape(-1), w16.size, q.reshape(-1), C.byref(s))
        return q, s.value

    def gemv_f16(self, x, w16):
        w16 = _c(w16, np.uint16)
        N, K = w16.shape
        y = np.empty(N, np.float32)
        self.L.tvo_gemv_f16(_c(x, np.float32), w16, K, N, y)
        return y

    def gemv_int8(self, x, q, row_scales=None, tensor_scale=1.0):
        q = _c(q, np.int8)
        N, K = q.shape
        y = np.empty(N, np.float32)
        rs = None if row_scales is None else _c(row_scales, np.float32)
        self.L.tvo_gemv_int8(_c(x, np.float32), q, None if rs is None else rs.ctypes.data,
                             tensor_scale, K, N, y)
        return y

    def rms_norm(self, x, w, eps):
        x = _c(x, np.float32)
        out = np.empty_like(x)
        self.L.tvo_rms_norm(x, x.size, _c(w, np.float32), eps, out)
        return out

    def rope(self, q, k, nh, nkv, hd, pos, theta):
        q = _c(q, np.float32).copy()
        k = _c(k, np.float32).copy()
        self.L.tvo_rope(q, k, nh, nkv, hd, pos, theta)
        return q, k

    def rope_table(self, n_pos, hd, theta):
        c = np.empty((n_pos, hd // 2), np.float32)
        s = np.empty((n_pos, hd // 2), np.float32)
        self.L.tvo_rope_table(n_pos, hd, theta, c, s)
        return c, s

    def attention_decode(self, q, kc, vc, kv_len, nh, nkv, hd):
        out = np.empty(nh * hd, np.float32)
        self.L.tvo_attention_decode(_c(q, np.float32), _c(kc, np.float32), _c(vc, np.float32),
                                    kv_len, nh, nkv, hd, out)
        return out


# ---------------------------------------------------------------------------
# Reference harness (the reference's own code)
# ---------------------------------------------------------------------------
class Reference:
    def __init__(self, path: str = REFERENCE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing; build it with `make -C oracle ref`")
        L = C.CDLL(path)
        L.tvref_f32_to_f16.argtypes = [_f32p, _i64, _u16p]
        L.tvref_f16_to_f32.argtypes = [_u16p, _i64, _f32p]
        L.tvref_i2s_quantize.argtypes = [_f32p, _i64, _u8p, C.POINTER(C.c_float)]
        L.tvref_i2s_dequant.argtypes = [_u8p, _i64, C.c_float, _f32p]
        L.tvref_lora_delta.argtypes = [_f32p, _f32p, _i64, _i64, C.c_int, _f32p]
        L.tvref_merge_f32.argtypes = [_u8p, C.c_float, _i64, _i64, _f32p, _f32p, C.c_int,
                                      C.c_float, _f32p]
        L.tvref_apply_lora_f16.argtypes = [_u8p, C.c_float, _i64, _i64, _f32p, _f32p, C.c_int,
                                           C.c_float, _u16p]
        L.tvref_quantize_int8_tensor.argtypes = [_u16p, _i64, _i8p, C.POINTER(C.c_float)]
        L.tvref_matmul_f16.argtypes = [_f32p, _i64, _i64, _u16p, _i64, _f32p]
        L.tvref_rms_norm.argtypes = [_f32p, _i64, _i64, _f32p, C.c_float, _f32p]
        L.tvref_rope_batched.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _i64, C.c_int, C.c_float]
        L.tvref_batched_attention.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _f32p, _f32p,
                                              _f32p, _f32p]
        L.tvref_model_create.restype = C.c_void_p
        L.tvref_model_create.argtypes = [C.c_int] * 7 + [C.c_float, C.c_float]
        L.tvref_model_free.argtypes = [C.c_void_p]
        L.tvref_model_set.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.tvref_model_set_f32.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.tvref_forward_prefill.argtypes = [C.c_void_p, _i32p, C.c_int, _f32p]
        L.tvref_forward_prefill_hidden.argtypes = [C.c_void_p, _i32p, C.c_int, _f32p]
        L.tvref_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, _f32p]
        L.tvref_kv_read.argtypes = [C.c_void_p, C.c_int, C.c_int, _f32p, _f32p]
        L.tvref_kv_set_seq_len.argtypes = [C.c_void_p, C.c_int]
        L.tvref_omp_threads.restype = C.c_int
        L.tvref_omp_threads.argtypes = []
        L.tvref_set_threads.argtypes = [C.c_int]
        L.tvref_cache_save.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_char_p, C.c_float, C.c_int]
        L.tvref_cache_load.argtypes = [C.c_void_p, C.c_char_p]
        L.tvref_model_get.restype = C.c_longlong
        L.tvref_model_get.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        L.tvref_model_lora.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.POINTER(C.c_int)]
        L.tvref_sample_token.argtypes = [_f32p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float, _i32p,
                                         C.c_int]
        L.tvref_score_logprobs.argtypes = [C.c_void_p, _i32p, C.c_int, C.c_int, C.c_int, _f32p, _i32p, _f32p]
        L.tvref_gguf_tensor.restype = C.c_longlong
        L.tvref_gguf_tensor.argtypes = [C.c_char_p, C.c_char_p, C.c_void_p, C.POINTER(C.c_int),
                                        C.POINTER(C.c_int), C.POINTER(C.c_longlong)]
        L.tvref_time_decode.restype = C.c_double
        L.tvref_time_decode.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        self.L = L

        if hasattr(L, "tvref_init_gpu"):   # drop-in build only
            L.tvref_init_gpu.argtypes = [C.c_void_p]
            L.tvref_init_gpu.restype = C.c_int
            L.tvref_sync_kv_to_gpu.argtypes = [C.c_void_p, C.c_int]

    def f32_to_f16(self, x):
        x = _c(x, np.float32)
        out = np.empty(x.shape, np.uint16)
        self.L.tvref_f32_to_f16(x.reshape(-1), x.size, out.reshape(-1))
        return out

    def f16_to_f32(self, h):
        h = _c(h, np.uint16)
        out = np.empty(h.shape, np.float32)
        self.L.tvref_f16_to_f32(h.reshape(-1), h.size, out.reshape(-1))
        return out

    def i2s_quantize(self, x):
        x = _c(x, np.float32).reshape(-1)
        nb = (x.size + 127) // 128
        out = np.empty(nb * 32 + 4, np.uint8)
        s = C.c_float()
        self.L.tvref_i2s_quantize(x, x.size, out, C.byref(s))
        return out[: nb * 32].copy(), s.value

    def i2s_dequant(self, codes, n, scale):
        out = np.empty(n, np.float32)
        self.L.tvref_i2s_dequant(_c(codes, np.uint8), n, scale, out)
        return out

    def lora_delta(self, A, B, K, N):
        A = _c(A, np.float32)
        out = np.empty((N, K), np.float32)
        self.L.tvref_lora_delta(A, _c(B, np.float32), K, N, A.shape[0], out)
        return out

    def merge_f32(self, codes, scale, K, N, A, B, alpha):
        A = _c(A, np.float32)
        out = np.empty((N, K), np.float32)
        self.L.tvref_merge_f32(_c(codes, np.uint8), scale, K, N, A, _c(B, np.float32),
                               A.shape[0], alpha, out)
        return out

    def apply_lora_f16(self, codes, scale, K, N, A, B, alpha):
        A = _c(A, np.float32)
        out = np.empty((N, K), np.uint16)
        self.L.tvref_apply_lora_f16(_c(codes, np.uint8), scale, K, N, A, _c(B, np.float32),
                                    A.shape[0], alpha, out)
        return out

    def quantize_int8_tensor(self, w16):
        w16 = _c(w16, np.uint16)
        q = np.empty(w16.shape, np.int8)
        s = C.c_float()
        self.L.tvref_quantize_int8_tensor(w16.reshape(-1), w16.size, q.reshape(-1), C.byref(s))
        return q, s.value

    def matmul_f16(self, x, w16):
        x = _c(x, np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        w16 = _c(w16, np.uint16)
        N, K = w16.shape
        out = np.empty((x2.shape[0], N), np.float32)
        self.L.tvref_matmul_f16(x2, x2.shape[0], K, w16, N, out)
        return out.reshape(x.shape[:-1] + (N,))

    def rms_norm(self, x, w, eps):
        x = _c(x, np.float32)
        x2 = x.reshape(-1, x.shape[-1])
        out = np.empty_like(x2)
        self.L.tvref_rms_norm(x2, x2.shape[0], x2.shape[1], _c(w, np.float32), eps, out)
        return out.reshape(x.shape)

    def rope_batched(self, q, k, nh, nkv, hd, start_pos, theta):
        q = _c(q, np.float32).copy()
        k = _c(k, np.float32).copy()
        S = q.size // (nh * hd)
        self.L.tvref_rope_batched(q.reshape(-1), k.reshape(-1), S, nh, nkv, hd, start_pos, theta)
        return q, k

    def batched_attention(self, q, kc, vc, S, nh, nkv, hd):
        out = np.empty(S * nh * hd, np.float32)
        self.L.tvref_batched_attention(S, nh, nkv, hd, _c(q, np.float32).reshape(-1),
                                       _c(kc, np.float32).reshape(-1),
                                       _c(vc, np.float32).reshape(-1), out)
        return out


@dataclass
class ModelShape:
    vocab: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    inter: int
    max_seq: int
    rope_theta: float = 500000.0
    eps: float = 1e-5

    @property
    def head_dim(self):
        return self.hidden // self.heads


def PROJ_DIMS(shape: ModelShape) -> dict:
    """(out rows N, in K) of each projection, stored [N][K] (GGUF ne = [K, N])."""
    H, I = shape.hidden, shape.inter
    Hq, Hk = shape.heads * shape.head_dim, shape.kv_heads * shape.head_dim
    return {"wq": (Hq, H), "wk": (Hk, H), "wv": (Hk, H), "wo": (H, Hq), "w_gate": (I, H),
            "w_up": (I, H), "w_down": (H, I)}


class ReferenceModel:
    """A ternative::Model on the reference CPUBackend, filled from merged F16
    weights held in numpy (``weights`` as produced by ternative_b200's synthetic
    model helpers: dict with tok_embd, output_norm and per-layer lists)."""

    LAYER_KEYS = ["attn_norm", "wq", "wk", "wv", "wo", "attn_sub_norm", "ffn_norm",
                  "w_gate", "w_up", "w_down", "ffn_sub_norm"]

    def __init__(self, ref: Reference, shape: ModelShape, weights: dict = None):
        self.ref = ref
        self.shape = shape
        L = ref.L
        self.h = L.tvref_model_create(shape.vocab, shape.hidden, shape.layers, shape.heads,
                                      shape.kv_heads, shape.inter, shape.max_seq,
                                      shape.rope_theta, shape.eps)
        self._keep = []
        if weights is None:   # an empty model (e.g. to load a .tvcache into)
            return

        def put(which, layer, arr):
            arr = np.ascontiguousarray(arr)
            # F16 bits (uint16) are the merged weights; an F32 projection holds the
            # exact dequantised values of a per-row INT8 layer
            setter = L.tvref_model_set_f32 if arr.dtype == np.float32 and which not in (1, 2, 7, 8, 12) \
                else L.tvref_model_set
            rc = setter(self.h, which, layer, arr.ctypes.data)
            if rc != 0:
                raise RuntimeError(f"tvref_model_set({which}, {layer}) -> {rc}")

        put(0, -1, weights["tok_embd"])
        put(1, -1, weights["output_norm"])
        for li in range(shape.layers):
            lw = weights["layers"][li]
            for j, key in enumerate(self.LAYER_KEYS):
                put(2 + j, li, lw[key])

    # ---- the reference's .tvcache (cache.cpp:263-470) ------------------------------
    def cache_save(self, path: str, base_hex: str = "", lora_hex: str = "", alpha: float = 0.0,
                   rank: int = 0):
        """ModelCache::save of this model's tensors."""
        self.ref.L.tvref_cache_save(self.h, path.encode(), base_hex.encode(), lora_hex.encode(), alpha, rank)

    def cache_load(self, path: str) -> bool:
        """ModelCache::try_load into this model."""
        return self.ref.L.tvref_cache_load(self.h, path.encode()) == 1

    def get(self, which: int, layer: int = -1):
        """Raw bytes of a tensor (numbering of tvref_model_set), or None if empty."""
        n = self.ref.L.tvref_model_get(self.h, which, layer, None)
        if n < 0:
            return None
        out = np.empty(n, np.uint8)
        self.ref.L.tvref_model_get(self.h, which, layer, out.ctypes.data)
        return out

    def lora(self):
        a, r = C.c_float(), C.c_int()
        self.ref.L.tvref_model_lora(self.h, C.byref(a), C.byref(r))
        return a.value, r.value

    def score_logprobs(self, tokens, k: int, start: int = 0):
        """Model::score_logprobs: (logprobs [n], top ids [n][k], top logprobs [n][k])."""
        tokens = _c(tokens, np.int32)
        n = max(0, tokens.size - max(1, start))
        lp = np.zeros(max(n, 1), np.float32)
        ids = np.zeros(max(n * k, 1), np.int32)
        top = np.zeros(max(n * k, 1), np.float32)
        got = self.ref.L.tvref_score_logprobs(self.h, tokens, tokens.size, k, start, lp, ids, top)
        return lp[:got], ids[:got * k].reshape(got, k), top[:got * k].reshape(got, k)

    def forward_prefill(self, tokens):
        tokens = _c(tokens, np.int32)
        out = np.empty((tokens.size, self.shape.vocab), np.float32)
        if self.ref.L.tvref_forward_prefill(self.h, tokens, tokens.size, out) != 0:
            raise RuntimeError("forward_prefill failed")
        return out

    def forward_prefill_hidden(self, tokens):
        tokens = _c(tokens, np.int32)
        out = np.empty((tokens.size, self.shape.hidden), np.float32)
        if self.ref.L.tvref_forward_prefill_hidden(self.h, tokens, tokens.size, out) != 0:
            raise RuntimeError("forward_prefill_hidden failed")
        return out

    def forward(self, token, pos, prefill):
        out = np.empty(self.shape.vocab, np.float32)
        self.ref.L.tvref_forward(self.h, int(token), int(pos), int(bool(prefill)), out)
        return out

    def kv(self, layer, n):
        row = self.shape.kv_heads * self.shape.head_dim
        k = np.empty(n * row, np.float32)
        v = np.empty(n * row, np.float32)
        self.ref.L.tvref_kv_read(self.h, layer, n, k, v)
        return k.reshape(n, row), v.reshape(n, row)

    def init_gpu(self) -> int:
        """Drop-in build: the reference's init_gpu_backend on the tvb200 shim."""
        return self.ref.L.tvref_init_gpu(self.h)

    def sync_kv_to_gpu(self, n):
        self.ref.L.tvref_kv_set_seq_len(self.h, n)
        self.ref.L.tvref_sync_kv_to_gpu(self.h, n)

    def time_decode(self, token, pos0, steps):
        return self.ref.L.tvref_time_decode(self.h, int(token), int(pos0), int(steps))

    def close(self):
        if self.h:
            self.ref.L.tvref_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# numpy restatement of the model-level forward (src/model.cpp:1139-1234)
# ---------------------------------------------------------------------------
def _rms(x, w, eps):
    # tensor.cpp:655-685: ss in F32, rms = sqrt(ss/n + eps), out = x * inv * w
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    inv = 1.0 / np.sqrt(ss / x.shape[-1] + eps)
    return (x * inv * w).astype(np.float32)


def forward_prefill(shape: ModelShape, weights: dict, tokens, f16_to_f32, return_hidden=False):
    """Teacher-forced causal forward over ``tokens`` -> logits [S][V] (or the
    final-norm hidden [S][H]).  Same layer order as model.cpp:1139-1234:
    attn_norm, q/k/v, batched NeoX RoPE from position 0, causal GQA attention
    (self-inclusive), attn_sub_norm, wo, residual, ffn_norm, gate/up, relu^2*up,
    ffn_sub_norm, down, residual; final norm and tied lm_head.  Accumulates in
    float64 (a tighter truth than the reference's float32)."""
    S = len(tokens)
    H, nh, nkv, hd = shape.hidden, shape.heads, shape.kv_heads, shape.head_dim
    f = lambda w16: f16_to_f32(w16).astype(np.float64)
    x = f16_to_f32(weights["tok_embd"][np.asarray(tokens)]).astype(np.float64)
    half = hd // 2
    ic = np.arange(half)
    freq = (1.0 / np.power(np.float32(shape.rope_theta),
                           (2 * ic).astype(np.float32) / np.float32(hd))).astype(np.float32)
    ang = (np.arange(S, dtype=np.float32)[:, None] * freq[None, :]).astype(np.float32)
    cos, sin = np.cos(ang.astype(np.float64)), np.sin(ang.astype(np.float64))

    def rope(t, nheads):
        t = t.reshape(S, nheads, hd)
        a, b = t[..., :half], t[..., half:]
        c, s = cos[:, None, :], sin[:, None, :]
        return np.concatenate([a * c - b * s, a * s + b * c], axis=-1)

    mask = np.triu(np.full((S, S), -np.inf), k=1)
    for lw in weights["layers"]:
        xn = _rms(x, lw["attn_norm"], shape.eps)
        q = rope(xn @ f(lw["wq"]).T, nh)
        k = rope(xn @ f(lw["wk"]).T, nkv)
        v = (xn @ f(lw["wv"]).T).reshape(S, nkv, hd)
        g = nh // nkv
        att = np.empty((S, nh, hd))
        for h in range(nh):
            sc = (q[:, h, :] @ k[:, h // g, :].T) / np.sqrt(np.float32(hd)) + mask
            sc = np.exp(sc - sc.max(axis=1, keepdims=True))
            sc /= sc.sum(axis=1, keepdims=True)
            att[:, h, :] = sc @ v[:, h // g, :]
        a = _rms(att.reshape(S, nh * hd), lw["attn_sub_norm"], shape.eps)
        x = x + a @ f(lw["wo"]).T
        xn = _rms(x, lw["ffn_norm"], shape.eps)
        gt = xn @ f(lw["w_gate"]).T
        up = xn @ f(lw["w_up"]).T
        mid = np.maximum(gt, 0.0) ** 2 * up
        mid = _rms(mid, lw["ffn_sub_norm"], shape.eps)
        x = x + mid @ f(lw["w_down"]).T
    xn = _rms(x, weights["output_norm"], shape.eps)
    if return_hidden:
        return xn.astype(np.float32)
    return (xn @ f(weights["tok_embd"]).T).astype(np.float32)


# ---------------------------------------------------------------------------
# sample_token (src/sampler.cpp:11-148) restated with an explicit uniform draw
# ---------------------------------------------------------------------------
def sample_token(logits, temperature=0.8, top_p=0.9, top_k=40, penalty=1.1, seen=(), u=0.5,
                 return_cdf=False):
    """The reference's sampler with the draw `u` given (it draws u from its own
    mt19937, sampler.cpp:120-131).  F32 values, F64 sums, as the reference."""
    lg = np.asarray(logits, np.float32)
    V = lg.size
    p = lg.copy()
    if temperature > 0.0 and temperature != 1.0:                       # :20-25
        p = (p / np.float32(temperature)).astype(np.float32)
    if penalty > 1.0 and len(seen):                                    # :27-37
        done = set()
        for t in seen:
            if 0 <= t < V and t not in done:
                p[t] = np.float32(p[t] / np.float32(penalty))
                done.add(t)
    mx = p.max()                                                       # :39-48
    e = np.exp((p - mx).astype(np.float32)).astype(np.float32)
    s = float(np.sum(e.astype(np.float64)))
    p = (e.astype(np.float64) / s).astype(np.float32)
    order = np.lexsort((np.arange(V), p))[::-1]                         # (p, index) descending
    if 0 < top_k < V:                                                  # :50-72
        keep = np.zeros(V, bool)
        keep[order[:top_k]] = True
        p[~keep] = 0.0
    if 0.0 < top_p < 1.0:                                              # :74-103
        idx = [i for i in np.lexsort((np.arange(V), p))[::-1] if p[i] > 0.0]
        cum = np.float32(0.0)
        nucleus = np.zeros(V, bool)
        for i in idx:
            cum = np.float32(cum + p[i])
            nucleus[i] = True
            if cum >= np.float32(top_p):
                break
        p[~nucleus] = 0.0
    s2 = float(np.sum(p.astype(np.float64)))                           # :105-121
    if s2 <= 0.0:
        return int(np.argmax(lg)) if not return_cdf else (int(np.argmax(lg)), None)
    p = (p.astype(np.float64) / s2).astype(np.float32)
    cdf = np.cumsum(p, dtype=np.float32)                               # :133-147 (sequential)
    hit = np.nonzero(np.float32(u) <= cdf)[0]
    tok = int(hit[0]) if hit.size else V - 1
    return (tok, cdf) if return_cdf else tok


def reference_gguf_tensor(ref, path: str, name: str):
    """gguf_load's view of one tensor: (ggml type, shape, raw bytes), or None."""
    t, nd = C.c_int(), C.c_int()
    shape = (C.c_longlong * 8)()
    n = ref.L.tvref_gguf_tensor(path.encode(), name.encode(), None, C.byref(t), C.byref(nd), shape)
    if n < 0:
        return None
    out = np.empty(n, np.uint8)
    ref.L.tvref_gguf_tensor(path.encode(), name.encode(), out.ctypes.data, C.byref(t), C.byref(nd), shape)
    return t.value, tuple(shape[:nd.value]), out
