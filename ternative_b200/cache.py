"""The merged-weight cache (.tvcache) on the device path: ModelCache::save and
ModelCache::try_load (src/cache.cpp:263-470, format include/ternative/cache.h:
28-62) through tvb_cache_* (csrc/tvcache.cpp), which stream tensors between
device memory and the file without a host copy of the model.

Tensor names and order follow the reference's collect_tensors (cache.cpp:
210-233): tok_embd, output_norm, then per layer attn_norm, attn_q, attn_k,
attn_v, attn_output, attn_sub_norm, ffn_norm, ffn_gate, ffn_up, ffn_down,
ffn_sub_norm.  Shapes are in ggml order (ne0 first): a projection stored
[out][in] has shape (in, out)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from ._lib import CacheKey, CacheTensor, call, load

GGML_F32, GGML_F16, GGML_I8 = 0, 1, 24

# our projection names -> the reference's tensor names (cache.cpp:218-230)
TENSOR_NAME = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output",
               "w_gate": "ffn_gate", "w_up": "ffn_up", "w_down": "ffn_down"}
LAYER_ORDER = ["attn_norm", "wq", "wk", "wv", "wo", "attn_sub_norm", "ffn_norm", "w_gate", "w_up",
               "w_down", "ffn_sub_norm"]


@dataclass
class Entry:
    """One tensor to write: ``data`` / ``row_scales`` are raw pointers (host or
    device); ``shape`` in ggml order."""
    name: str
    ggml_type: int
    shape: Sequence[int]
    data: int
    row_scales: Optional[int] = None


def make_key(base_sha256: bytes = b"", lora_sha256: bytes = b"", lora_alpha: float = 0.0,
             lora_rank: int = 0) -> CacheKey:
    k = CacheKey()
    for dst, src in ((k.base_sha256, base_sha256), (k.lora_sha256, lora_sha256)):
        for i, b in enumerate(src[:32]):
            dst[i] = b
    k.lora_alpha = lora_alpha
    k.lora_rank = lora_rank
    return k


def write(path: str, key: CacheKey, entries: List[Entry]) -> None:
    """ModelCache::save: write `entries` to `path` (through <path>.tmp)."""
    arr = (CacheTensor * max(1, len(entries)))()
    names = [e.name.encode() for e in entries]   # kept alive across the call
    for i, e in enumerate(entries):
        t = arr[i]
        t.name = names[i]
        t.ggml_type = e.ggml_type
        t.n_dims = len(e.shape)
        for d, v in enumerate(e.shape):
            t.shape[d] = int(v)
        t.data = e.data
        t.row_scales = e.row_scales
    call("tvb_cache_write", path.encode(), C.byref(key), arr, len(entries))


class CacheFile:
    """ModelCache::try_load's view of a file: its key, its tensor table, and
    reads of single tensors into host or device buffers."""

    def __init__(self, path: str):
        self.lib = load()
        self.h = C.c_void_p()
        call("tvb_cache_open", path.encode(), C.byref(self.h))
        self.key = CacheKey()
        v = C.c_int()
        call("tvb_cache_info", self.h, C.byref(self.key), C.byref(v))
        self.version = v.value
        self.entries = {}
        for i in range(self.lib.tvb_cache_count(self.h)):
            t = CacheTensor()
            n = C.c_uint64()
            call("tvb_cache_entry", self.h, i, C.byref(t), C.byref(n))
            self.entries[t.name.decode()] = (t.ggml_type, tuple(t.shape[:t.n_dims]), n.value)

    def read(self, name: str, dst: int, capacity: int) -> None:
        call("tvb_cache_read", self.h, name.encode(), dst, capacity)

    def read_numpy(self, name: str) -> np.ndarray:
        _, _, n = self.entries[name]
        out = np.empty(n, np.uint8)
        self.read(name, out.ctypes.data, n)
        return out

    def close(self):
        if self.h:
            self.lib.tvb_cache_close(self.h)
            self.h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def model_entries(model) -> List[Entry]:
    """The tensors of a device-resident ``model.Model`` in the reference's
    order; per-row INT8 layers as I8 codes + row scales (version-2 file)."""
    from ._lib import TVB_I8_ROW, TVB_I8_TENSOR
    from .model import norm_len, proj_shape
    cfg = model.cfg
    out = [Entry("tok_embd", GGML_F16, (cfg.hidden_size, cfg.vocab_size), model.tok_embd.data_ptr()),
           Entry("output_norm", GGML_F32, (cfg.hidden_size,), model.output_norm.data_ptr())]
    for li in range(cfg.num_layers):
        dt = model.layer_dtype[li]
        if dt == TVB_I8_TENSOR:
            raise ValueError("per-tensor INT8 layers are re-quantised at load (model.cpp:374-410), "
                             "not cached")
        for key in LAYER_ORDER:
            name = f"blk.{li}.{TENSOR_NAME.get(key, key)}"
            if key in TENSOR_NAME:
                N, K = proj_shape(cfg, key)
                w = model.weights[li][key]
                if dt == TVB_I8_ROW:
                    out.append(Entry(name, GGML_I8, (K, N), w.data_ptr(),
                                     model.row_scales[li][key].data_ptr()))
                else:
                    out.append(Entry(name, GGML_F16, (K, N), w.data_ptr()))
            else:
                out.append(Entry(name, GGML_F32, (norm_len(cfg, key),), model.norms[li][key].data_ptr()))
    return out


class GGUFFile:
    """A GGUF v3 file's tensor table (gguf.cpp's parse) and single tensors
    streamed into host or device buffers (tvb_gguf_*), without reading the
    whole file into memory as gguf_load does."""

    def __init__(self, path: str):
        self.lib = load()
        self.h = C.c_void_p()
        call("tvb_gguf_open", path.encode(), C.byref(self.h))
        self.entries = {}
        for i in range(self.lib.tvb_gguf_count(self.h)):
            t = CacheTensor()
            n = C.c_uint64()
            call("tvb_gguf_tensor", self.h, i, C.byref(t), C.byref(n))
            self.entries[t.name.decode()] = (t.ggml_type, tuple(t.shape[:t.n_dims]), n.value)

    def read(self, name: str, dst: int, capacity: int) -> None:
        call("tvb_gguf_read", self.h, name.encode(), dst, capacity)

    def read_numpy(self, name: str) -> np.ndarray:
        _, _, n = self.entries[name]
        out = np.empty(n, np.uint8)
        self.read(name, out.ctypes.data, n)
        return out

    def close(self):
        if self.h:
            self.lib.tvb_gguf_close(self.h)
            self.h = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
