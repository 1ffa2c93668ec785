"""Python host mirror of ternative::CUDABackend (include/ternative/ops.h:47-168)
on top of libtvb200's C ABI.

Method names, argument order and meaning follow the reference class so that a
host written against it reads the same; device pointers are plain ints (torch
``data_ptr()`` values or pointers from ``alloc_gpu_mem``).  Errors raise
``TvbError`` (a RuntimeError), as the reference's CUDA_CHECK throws
std::runtime_error.  There is no CPU fallback: every call goes to the CUDA
library, and constructing the backend fails when it is not built.

Beyond the reference's per-op API, the backend exposes the load-time merge
(``apply_lora_i2s``/``merge_batch``, replacing apply_lora in src/model.cpp) and
the fused, graph-captured decode/prefill steps (``decode_step``, ``prefill``,
``generate_greedy``) that replace the layer loop of Model::forward_gpu.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import (TVB_F16, TVB_F32, TVB_I8_ROW, TVB_I8_TENSOR, Buffers, IpcHandle, LayerWeights,
                   MergeDesc, ModelConfig, Weight, call, load)


def _ptr(x) -> Optional[int]:
    """Device/host address of a torch tensor, numpy array or int (None -> NULL)."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)!r}")


@dataclass
class Config:
    """ternative::ModelConfig (include/ternative/model.h:13-25) plus the
    device KV capacity and prefill limit of this backend."""
    vocab_size: int = 128256
    hidden_size: int = 2560
    num_layers: int = 30
    num_heads: int = 20
    num_kv_heads: int = 5
    head_dim: int = 128
    intermediate_size: int = 6912
    max_seq_len: int = 4096
    rope_theta: float = 500000.0
    rms_norm_eps: float = 1e-5
    max_prefill: int = 1024
    max_batch: int = 1      # KV cache slots for batched decode

    def to_c(self) -> ModelConfig:
        return ModelConfig(self.vocab_size, self.hidden_size, self.num_layers, self.num_heads,
                           self.num_kv_heads, self.head_dim, self.intermediate_size,
                           self.max_seq_len, self.rope_theta, self.rms_norm_eps, self.max_prefill,
                           self.max_batch)


@dataclass
class DeviceWeight:
    """One projection as the fused step consumes it (tvb_weight)."""
    ptr: int
    dtype: int = TVB_F16
    row_scales: Optional[int] = None
    tensor_scale: float = 1.0

    def to_c(self) -> Weight:
        return Weight(self.ptr, self.dtype, self.row_scales, self.tensor_scale)


class CUDABackend:
    def __init__(self):
        self.lib = load()
        self.ctx = None
        self.cfg: Optional[Config] = None
        self._bufs: Optional[Buffers] = None

    # ---- memory management (ops.h:80-92) ------------------------------------
    @staticmethod
    def free_vram_bytes() -> int:
        v = C.c_size_t()
        call("tvb_free_vram_bytes", C.byref(v))
        return v.value

    def alloc_gpu_mem(self, nbytes: int) -> int:
        p = C.c_void_p()
        call("tvb_alloc", nbytes, C.byref(p))
        return p.value

    def upload(self, dst: int, src: np.ndarray, nbytes: Optional[int] = None) -> None:
        src = np.ascontiguousarray(src)
        call("tvb_upload", dst, src.ctypes.data, src.nbytes if nbytes is None else nbytes)

    def release_gpu_mem(self, ptr: int) -> None:
        call("tvb_release", ptr)

    # ---- activation pipeline (ops.h:93-123) -----------------------------------
    def init_gpu_activations(self, cfg: Config) -> None:
        if self.ctx is not None:
            return   # idempotent, like the reference
        c = C.c_void_p()
        call("tvb_context_create", C.byref(cfg.to_c()), C.byref(c))
        self.ctx = c.value
        self.cfg = cfg
        self._bufs = Buffers()
        call("tvb_context_buffers", self.ctx, C.byref(self._bufs))

    def has_gpu_activations(self) -> bool:
        return self.ctx is not None

    @property
    def stream(self) -> int:
        return self.lib.tvb_context_stream(self.ctx) if self.ctx else 0

    def d_x(self): return self._bufs.d_x
    def d_norm(self): return self._bufs.d_norm
    def d_q(self): return self._bufs.d_q
    def d_k(self): return self._bufs.d_k
    def d_v(self): return self._bufs.d_v
    def d_gate(self): return self._bufs.d_gate
    def d_up(self): return self._bufs.d_up
    def h_qkv(self): return self._bufs.h_qkv
    def h_attn(self): return self._bufs.h_attn
    def h_logit(self): return self._bufs.h_logit

    def add_d(self, d_out, d_a, d_b, n):
        call("tvb_add", _ptr(d_out), _ptr(d_a), _ptr(d_b), n, self.stream)

    def mul_d(self, d_out, d_a, d_b, n):
        call("tvb_mul", _ptr(d_out), _ptr(d_a), _ptr(d_b), n, self.stream)

    def relu2_d(self, d_out, d_x, n):
        call("tvb_relu2", _ptr(d_out), _ptr(d_x), n, self.stream)

    def rms_norm_d(self, d_out, d_x, d_w, eps, n):
        call("tvb_rms_norm", _ptr(d_out), _ptr(d_x), _ptr(d_w), eps, n, self.stream)

    def gemv_d2d(self, d_out, d_in, d_w_f16, K, N):
        call("tvb_gemv_f16", _ptr(d_out), _ptr(d_in), _ptr(d_w_f16), K, N, self.stream)

    def gemv_d2d_int8(self, d_out, d_in, d_w_int8, scale, K, N):
        call("tvb_gemv_int8", _ptr(d_out), _ptr(d_in), _ptr(d_w_int8), scale, K, N, self.stream)

    def gemv_d2d_int8_rows(self, d_out, d_in, d_w_int8, d_row_scales, K, N):
        call("tvb_gemv_int8_rows", _ptr(d_out), _ptr(d_in), _ptr(d_w_int8), _ptr(d_row_scales),
             K, N, self.stream)

    def upload_pinned(self, d_dst, h_src: np.ndarray, n_floats: int):
        h = np.ascontiguousarray(h_src, np.float32).reshape(-1)
        if h.size < n_floats:
            raise ValueError("upload_pinned: source shorter than n_floats")
        self.sync_d()
        call("tvb_upload", _ptr(d_dst), h.ctypes.data, n_floats * 4)

    def download_pinned(self, d_src, n_floats: int) -> np.ndarray:
        self.sync_d()
        out = np.empty(n_floats, np.float32)
        call("tvb_download", out.ctypes.data, _ptr(d_src), n_floats * 4)
        return out

    def sync_d(self):
        call("tvb_context_sync", self.ctx)

    # ---- RoPE / KV cache / attention (ops.h:127-162) ---------------------------
    def rope_inplace_d(self, d_q, d_k, pos, theta, n_heads, n_kv_heads, head_dim):
        call("tvb_rope_inplace", _ptr(d_q), _ptr(d_k), pos, theta, n_heads, n_kv_heads, head_dim,
             self.stream)

    def kv_layer_ptrs(self, layer):
        k, v = C.c_void_p(), C.c_void_p()
        call("tvb_kv_layer_ptrs", self.ctx, layer, C.byref(k), C.byref(v))
        return k.value, v.value

    def kv_write_d(self, d_k, d_v, layer, pos):
        k, v = self.kv_layer_ptrs(layer)
        Hk = self.cfg.num_kv_heads * self.cfg.head_dim
        call("tvb_kv_write", _ptr(d_k), _ptr(d_v), k, v, pos, Hk, self.stream)

    def attention_d(self, d_q, layer, kv_len, d_out, n_heads, n_kv_heads, head_dim, scale):
        k, v = self.kv_layer_ptrs(layer)
        call("tvb_attention_decode", _ptr(d_q), k, v, kv_len, _ptr(d_out), n_heads, n_kv_heads,
             head_dim, scale, self.stream)

    def clear_kv_d(self):
        if self.ctx:
            call("tvb_kv_clear", self.ctx)

    def has_gpu_kv(self, min_seq: int = 1) -> bool:
        return self.ctx is not None and self.gpu_kv_max_seq() >= min_seq

    def gpu_kv_max_seq(self) -> int:
        return self.lib.tvb_kv_capacity(self.ctx) if self.ctx else 0

    def upload_kv_layer_d(self, layer, n_positions, h_k: np.ndarray, h_v: np.ndarray):
        h_k = np.ascontiguousarray(h_k, np.float32)
        h_v = np.ascontiguousarray(h_v, np.float32)
        call("tvb_kv_upload_layer", self.ctx, layer, n_positions, h_k.ctypes.data, h_v.ctypes.data)

    def download_kv_slot_d(self, layer, pos, n_floats) -> np.ndarray:
        out = np.empty(n_floats, np.float32)
        call("tvb_kv_download_slot", self.ctx, layer, pos, n_floats, out.ctypes.data)
        return out

    # ---- load-time merge (replaces apply_lora, src/model.cpp:205-258) ----------
    def apply_lora_i2s(self, i2s, scale, K, N, lora_a, lora_b, alpha, out_dtype, dst,
                       row_scales=None, stream=None):
        r = 0 if lora_a is None else int(lora_a.shape[0])
        call("tvb_merge_i2s_lora", _ptr(i2s), scale, K, N, _ptr(lora_a), _ptr(lora_b), r, alpha,
             out_dtype, _ptr(dst), _ptr(row_scales), self.stream if stream is None else stream)

    def merge_batch(self, descs: Sequence[MergeDesc], out_dtype: int, stream=None):
        arr = (MergeDesc * len(descs))(*descs)
        call("tvb_merge_batch", arr, len(descs), out_dtype, self.stream if stream is None else stream)

    def merge_batch_tc(self, descs: Sequence[MergeDesc], out_dtype: int, stream=None):
        """merge_batch with the LoRA delta on the tensor cores (F16 within 1 ulp)."""
        arr = (MergeDesc * len(descs))(*descs)
        call("tvb_merge_batch_tc", arr, len(descs), out_dtype, self.stream if stream is None else stream)

    def i2s_unpack(self, i2s, n, scale, out, stream=None):
        call("tvb_i2s_unpack", _ptr(i2s), n, scale, _ptr(out), self.stream if stream is None else stream)

    def quantize_int8(self, w_f16, N, K, per_row, q, scales, stream=None):
        call("tvb_quantize_int8", _ptr(w_f16), N, K, int(per_row), _ptr(q), _ptr(scales),
             self.stream if stream is None else stream)

    # ---- fused step -------------------------------------------------------------
    def set_layer(self, layer: int, *, attn_norm, wq, wk, wv, attn_sub_norm, wo, ffn_norm, w_gate,
                  w_up, ffn_sub_norm, w_down):
        lw = LayerWeights(_ptr(attn_norm), wq.to_c(), wk.to_c(), wv.to_c(), _ptr(attn_sub_norm),
                          wo.to_c(), _ptr(ffn_norm), w_gate.to_c(), w_up.to_c(), _ptr(ffn_sub_norm),
                          w_down.to_c())
        call("tvb_set_layer", self.ctx, layer, C.byref(lw))

    def set_output(self, tok_embd_f16, output_norm):
        call("tvb_set_output", self.ctx, _ptr(tok_embd_f16), _ptr(output_norm))

    # ---- tensor parallelism (one process and context per GPU) -------------------
    def tp_init(self, rank: int, world: int) -> int:
        """Make this context rank `rank` of `world`; returns its exchange buffer."""
        p = C.c_void_p()
        call("tvb_tp_init", self.ctx, rank, world, C.byref(p))
        self.tp_world = world
        return p.value

    def tp_set_peers(self, buffers: Sequence[int]) -> None:
        arr = (C.c_void_p * len(buffers))(*buffers)
        call("tvb_tp_set_peers", self.ctx, arr)

    def tp_recover(self) -> None:
        """After a tensor-parallel step failed on any rank: zero this rank's
        exchange buffer and step counters.  Every rank calls it; no rank may
        start a step before all ranks have returned (a host-side barrier)."""
        call("tvb_tp_recover", self.ctx)

    @staticmethod
    def ipc_export(dev_ptr: int) -> bytes:
        h = IpcHandle()
        call("tvb_ipc_export", dev_ptr, C.byref(h))
        return bytes(h.bytes)

    @staticmethod
    def ipc_import(handle: bytes) -> int:
        h = IpcHandle()
        C.memmove(h.bytes, handle, 64)
        p = C.c_void_p()
        call("tvb_ipc_import", C.byref(h), C.byref(p))
        return p.value

    @staticmethod
    def ipc_close(dev_ptr: int) -> None:
        call("tvb_ipc_close", dev_ptr)

    def n_logits(self) -> int:
        """Logits a step returns: the whole vocabulary, or this rank's slice."""
        return self.cfg.vocab_size // getattr(self, "tp_world", 1)

    def decode_step(self, token: int, pos: int, want_logits: bool = True):
        """Model::forward_gpu: returns (logits [V] float32 or None, argmax).
        Under tensor parallelism the logits are this rank's vocabulary slice."""
        am = C.c_int()
        logits = np.empty(self.n_logits(), np.float32) if want_logits else None
        call("tvb_decode_step", self.ctx, token, pos, None if logits is None else logits.ctypes.data,
             C.byref(am))
        return logits, am.value

    def generate_greedy(self, token: int, pos: int, n_steps: int) -> np.ndarray:
        out = np.empty(n_steps, np.int32)
        call("tvb_generate_greedy", self.ctx, token, pos, n_steps, out.ctypes.data)
        return out

    def decode_enqueue(self, token: int, pos: int, n_steps: int) -> None:
        call("tvb_decode_enqueue", self.ctx, token, pos, n_steps)

    def prefill(self, tokens, want_logits: bool = True):
        """Model::forward_prefill over tokens from position 0: fills the KV cache
        and returns (last-row logits or None, argmax)."""
        t = np.ascontiguousarray(tokens, np.int32)
        am = C.c_int()
        logits = np.empty(self.n_logits(), np.float32) if want_logits else None
        call("tvb_prefill", self.ctx, t.ctypes.data, t.size,
             None if logits is None else logits.ctypes.data, C.byref(am))
        return logits, am.value

    def score_logprobs(self, tokens, k: int = 5, start_pos: int = 0):
        """Model::score_logprobs: (logprob of each scored token [n], top ids [n][k],
        top logprobs [n][k]) for positions max(1, start_pos) .. len(tokens) - 1."""
        t = np.ascontiguousarray(tokens, np.int32)
        n = max(0, t.size - max(1, start_pos))
        lp = np.empty(max(n, 1), np.float32)
        ids = np.empty(max(n * k, 1), np.int32)
        top = np.empty(max(n * k, 1), np.float32)
        call("tvb_score_logprobs", self.ctx, t.ctypes.data, t.size, start_pos, k, lp.ctypes.data,
             ids.ctypes.data, top.ctypes.data)
        return lp[:n], ids[:n * k].reshape(n, k), top[:n * k].reshape(n, k)

    def prefill_slot(self, slot: int, tokens, want_logits: bool = True):
        """prefill() into KV cache slot `slot` (batched decode); slot 0 is the
        single-sequence cache."""
        t = np.ascontiguousarray(tokens, np.int32)
        am = C.c_int()
        logits = np.empty(self.n_logits(), np.float32) if want_logits else None
        call("tvb_prefill_slot", self.ctx, slot, t.ctypes.data, t.size,
             None if logits is None else logits.ctypes.data, C.byref(am))
        return logits, am.value

    def decode_batch(self, tokens, positions, want_logits: bool = True):
        """One greedy step of sequences 0..B-1 (sequence b in KV slot b, token
        tokens[b] at positions[b]).  Returns (logits [B][n_logits] or None,
        next tokens [B])."""
        t = np.ascontiguousarray(tokens, np.int32)
        p = np.ascontiguousarray(positions, np.int32)
        if t.shape != p.shape or t.ndim != 1:
            raise ValueError("tokens and positions must be 1-D of the same length")
        nxt = np.empty(t.size, np.int32)
        logits = np.empty((t.size, self.n_logits()), np.float32) if want_logits else None
        call("tvb_decode_batch", self.ctx, t.ctypes.data, p.ctypes.data, t.size,
             None if logits is None else logits.ctypes.data, nxt.ctypes.data)
        return logits, nxt

    def close(self):
        if self.ctx is not None:
            self.lib.tvb_context_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
