"""ctypes binding of libtvb200.so (the C ABI declared in include/tvb200.h).

The library is built in-tree (ternative_b200/libtvb200.so) by
``ternative_b200.build.build()``.  Loading fails loudly when it is missing:
there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# TVB200_LIB selects another build of the library (e.g. a tuning variant).
LIB_PATH = os.environ.get("TVB200_LIB") or os.path.join(HERE, "libtvb200.so")

# tvb_status
TVB_OK = 0
STATUS_NAMES = {
    0: "TVB_OK", 1: "TVB_ERR_INVALID", 2: "TVB_ERR_CUDA", 3: "TVB_ERR_OOM",
    4: "TVB_ERR_UNSUPPORTED", 5: "TVB_ERR_TIMEOUT", 6: "TVB_ERR_COMM", 7: "TVB_ERR_STATE",
}
# tvb_dtype
TVB_F32, TVB_F16, TVB_I8_ROW, TVB_I8_TENSOR = 0, 1, 2, 3


class TvbError(RuntimeError):
    """A failed tvb_* call.  Mirrors the reference's CUDA_CHECK, which throws
    std::runtime_error (cuda/ops_cuda.cu:30-37)."""

    def __init__(self, status: int, func: str, message: str):
        self.status = status
        super().__init__(f"[tvb200] {func}: {STATUS_NAMES.get(status, status)}: {message}")


class MergeDesc(C.Structure):
    _fields_ = [("i2s", C.c_void_p), ("scale", C.c_float), ("K", C.c_int), ("N", C.c_int),
                ("A", C.c_void_p), ("B", C.c_void_p), ("r", C.c_int), ("alpha", C.c_float),
                ("dst", C.c_void_p), ("row_scales", C.c_void_p), ("k0", C.c_int), ("ld", C.c_int)]


class ModelConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("hidden_size", C.c_int), ("num_layers", C.c_int),
                ("num_heads", C.c_int), ("num_kv_heads", C.c_int), ("head_dim", C.c_int),
                ("intermediate_size", C.c_int), ("max_seq_len", C.c_int),
                ("rope_theta", C.c_float), ("rms_norm_eps", C.c_float), ("max_prefill", C.c_int),
                ("max_batch", C.c_int)]


class Buffers(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in
                ["d_x", "d_norm", "d_q", "d_k", "d_v", "d_gate", "d_up", "h_qkv", "h_attn",
                 "h_logit"]]


class Weight(C.Structure):
    _fields_ = [("w", C.c_void_p), ("dtype", C.c_int), ("row_scales", C.c_void_p),
                ("tensor_scale", C.c_float)]


class LayerWeights(C.Structure):
    _fields_ = [("attn_norm", C.c_void_p), ("wq", Weight), ("wk", Weight), ("wv", Weight),
                ("attn_sub_norm", C.c_void_p), ("wo", Weight), ("ffn_norm", C.c_void_p),
                ("w_gate", Weight), ("w_up", Weight), ("ffn_sub_norm", C.c_void_p),
                ("w_down", Weight)]


class CacheKey(C.Structure):
    _fields_ = [("base_size", C.c_uint64), ("base_sha256", C.c_ubyte * 32), ("lora_size", C.c_uint64),
                ("lora_sha256", C.c_ubyte * 32), ("lora_alpha", C.c_float), ("lora_rank", C.c_uint32)]


class CacheTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ggml_type", C.c_int), ("n_dims", C.c_int),
                ("shape", C.c_int64 * 4), ("data", C.c_void_p), ("row_scales", C.c_void_p)]


class SamplerConfig(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int),
                ("repetition_penalty", C.c_float)]


class IpcHandle(C.Structure):
    _fields_ = [("bytes", C.c_ubyte * 64)]


_P = C.c_void_p
_I = C.c_int
_F = C.c_float
_I64 = C.c_int64

# name -> argtypes (all return tvb_status unless listed in _RESTYPES)
_SIGS = {
    "tvb_version": [],
    "tvb_status_string": [_I],
    "tvb_last_error": [],
    "tvb_free_vram_bytes": [C.POINTER(C.c_size_t)],
    "tvb_alloc": [C.c_size_t, C.POINTER(C.c_void_p)],
    "tvb_upload": [_P, _P, C.c_size_t],
    "tvb_download": [_P, _P, C.c_size_t],
    "tvb_release": [_P],
    "tvb_merge_i2s_lora": [_P, _F, _I, _I, _P, _P, _I, _F, _I, _P, _P, _P],
    "tvb_merge_batch": [C.POINTER(MergeDesc), _I, _I, _P],
    "tvb_merge_batch_tc": [C.POINTER(MergeDesc), _I, _I, _P],
    "tvb_i2s_unpack": [_P, _I64, _F, _P, _P],
    "tvb_quantize_int8": [_P, _I, _I, _I, _P, _P, _P],
    "tvb_gemv_f16": [_P, _P, _P, _I, _I, _P],
    "tvb_gemv_int8": [_P, _P, _P, _F, _I, _I, _P],
    "tvb_gemv_int8_rows": [_P, _P, _P, _P, _I, _I, _P],
    "tvb_rms_norm": [_P, _P, _P, _F, _I, _P],
    "tvb_add": [_P, _P, _P, _I, _P],
    "tvb_mul": [_P, _P, _P, _I, _P],
    "tvb_relu2": [_P, _P, _I, _P],
    "tvb_rope_inplace": [_P, _P, _I, _F, _I, _I, _I, _P],
    "tvb_kv_write": [_P, _P, _P, _P, _I, _I, _P],
    "tvb_attention_decode": [_P, _P, _P, _I, _P, _I, _I, _I, _F, _P],
    "tvb_matmul": [_P, _P, _I, _I, C.POINTER(Weight), _I, _P],
    "tvb_attention_decode_noalloc": [_P, _P, _P, _I, _P, _I, _I, _I, _F, _P],
    "tvb_context_create": [C.POINTER(ModelConfig), C.POINTER(C.c_void_p)],
    "tvb_context_destroy": [_P],
    "tvb_context_stream": [_P],
    "tvb_context_buffers": [_P, C.POINTER(Buffers)],
    "tvb_kv_clear": [_P],
    "tvb_kv_capacity": [_P],
    "tvb_kv_layer_ptrs": [_P, _I, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)],
    "tvb_kv_upload_layer": [_P, _I, _I, _P, _P],
    "tvb_kv_download_slot": [_P, _I, _I, _I, _P],
    "tvb_context_sync": [_P],
    "tvb_trace_set": [_P, _I],
    "tvb_tp_recover": [_P],
    "tvb_set_layer": [_P, _I, C.POINTER(LayerWeights)],
    "tvb_set_output": [_P, _P, _P],
    "tvb_decode_step": [_P, _I, _I, _P, _P],
    "tvb_generate_greedy": [_P, _I, _I, _I, _P],
    "tvb_decode_enqueue": [_P, _I, _I, _I],
    "tvb_prefill": [_P, _P, _I, _P, _P],
    "tvb_prefill_slot": [_P, _I, _P, _I, _P, _P],
    "tvb_sample": [_P, _I, _I, _I, _P, _P, _P, _I, _P, _P, _P],
    "tvb_score_logprobs": [_P, _P, _I, _I, _I, _P, _P, _P],
    "tvb_cache_write": [C.c_char_p, _P, _P, _I],
    "tvb_cache_open": [C.c_char_p, _P],
    "tvb_cache_count": [_P],
    "tvb_cache_info": [_P, _P, _P],
    "tvb_cache_entry": [_P, _I, _P, _P],
    "tvb_cache_read": [_P, C.c_char_p, _P, C.c_uint64],
    "tvb_cache_close": [_P],
    "tvb_gguf_open": [C.c_char_p, _P],
    "tvb_gguf_count": [_P],
    "tvb_gguf_tensor": [_P, _I, _P, _P],
    "tvb_gguf_read": [_P, C.c_char_p, _P, C.c_uint64],
    "tvb_gguf_close": [_P],
    "tvb_decode_batch": [_P, _P, _P, _I, _P, _P],
    "tvb_tp_init": [_P, _I, _I, C.POINTER(C.c_void_p)],
    "tvb_tp_set_peers": [_P, C.POINTER(C.c_void_p)],
    "tvb_ipc_export": [_P, C.POINTER(IpcHandle)],
    "tvb_ipc_import": [C.POINTER(IpcHandle), C.POINTER(C.c_void_p)],
    "tvb_ipc_close": [_P],
}
_RESTYPES = {
    "tvb_version": C.c_int,
    "tvb_status_string": C.c_char_p,
    "tvb_last_error": C.c_char_p,
    "tvb_context_stream": C.c_void_p,
    "tvb_kv_capacity": C.c_int,
    "tvb_cache_count": C.c_int,
    "tvb_gguf_count": C.c_int,
}

EXPORTED = tuple(_SIGS)

_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load libtvb200.so once; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is not built; run `python -c 'import ternative_b200.build as b; b.build()'`")
    lib = C.CDLL(path)
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, C.c_int)
    _lib = lib
    return lib


def check(status: int, func: str) -> None:
    if status != TVB_OK:
        msg = load().tvb_last_error()
        raise TvbError(status, func, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    """Call a status-returning tvb_* function and raise TvbError on failure."""
    check(getattr(load(), name)(*args), name)
