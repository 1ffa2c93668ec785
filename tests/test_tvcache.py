"""The merged-weight cache (.tvcache) against the reference's own writer and
reader (ModelCache::save / try_load, src/cache.cpp:263-470, run from
oracle/_ref): for the same tensors and key our writer produces the reference's
file byte for byte, the reference loads our file, and we read the reference's.
Per-row INT8 (our extension) makes a version-2 file, which the reference
refuses rather than misreads.  Host pointers here (no GPU needed); the device
path is tests/test_tvcache_gpu.py."""
import hashlib
import os

import numpy as np
import pytest

from oracle.oracle import ModelShape, Reference, ReferenceModel
from ternative_b200 import TvbError
from ternative_b200 import cache as tc

SHAPE = ModelShape(300, 256, 2, 2, 1, 512, 64)   # vocab, hidden, layers, heads, kv heads, ffn, max_seq
KEYS = ReferenceModel.LAYER_KEYS


def dims(key):
    H, I = SHAPE.hidden, SHAPE.inter
    Hq, Hk = SHAPE.heads * 128, SHAPE.kv_heads * 128
    return {"attn_norm": (H,), "attn_sub_norm": (Hq,), "ffn_norm": (H,), "ffn_sub_norm": (I,),
            "wq": (H, Hq), "wk": (H, Hk), "wv": (H, Hk), "wo": (Hq, H),
            "w_gate": (H, I), "w_up": (H, I), "w_down": (I, H)}[key]   # ggml order (in, out)


def random_weights(seed):
    rng = np.random.default_rng(seed)

    def f16(shape):   # F16 bit patterns stored [out][in]
        return rng.integers(0, 1 << 16, size=shape[::-1], dtype=np.uint16)

    w = {"tok_embd": f16((SHAPE.hidden, SHAPE.vocab)),
         "output_norm": rng.standard_normal(SHAPE.hidden).astype(np.float32), "layers": []}
    for _ in range(SHAPE.layers):
        lw = {}
        for k in KEYS:
            d = dims(k)
            lw[k] = f16(d) if len(d) == 2 else rng.standard_normal(d[0]).astype(np.float32)
        w["layers"].append(lw)
    return w


def entries(w):
    out = [tc.Entry("tok_embd", tc.GGML_F16, (SHAPE.hidden, SHAPE.vocab), w["tok_embd"].ctypes.data),
           tc.Entry("output_norm", tc.GGML_F32, (SHAPE.hidden,), w["output_norm"].ctypes.data)]
    for li, lw in enumerate(w["layers"]):
        for k in KEYS:
            a = lw[k]
            out.append(tc.Entry(f"blk.{li}.{tc.TENSOR_NAME.get(k, k)}",
                                tc.GGML_F16 if a.dtype == np.uint16 else tc.GGML_F32, dims(k), a.ctypes.data))
    return out


BASE = hashlib.sha256(b"base gguf").digest()
LORA = hashlib.sha256(b"lora gguf").digest()


def test_writer_matches_reference_bytes(tmp_path):
    w = random_weights(1)
    ref = ReferenceModel(Reference(), SHAPE, w)
    ref_path = str(tmp_path / "ref.tvcache")
    ref.cache_save(ref_path, BASE.hex(), LORA.hex(), 32.0, 16)
    ours = str(tmp_path / "ours.tvcache")
    tc.write(ours, tc.make_key(BASE, LORA, 32.0, 16), entries(w))
    a, b = open(ref_path, "rb").read(), open(ours, "rb").read()
    assert len(a) == len(b)
    assert a == b
    assert not os.path.exists(ours + ".tmp")


def test_reference_loads_our_file(tmp_path):
    w = random_weights(2)
    path = str(tmp_path / "ours.tvcache")
    tc.write(path, tc.make_key(BASE, b"", 0.0, 0), entries(w))
    m = ReferenceModel(Reference(), SHAPE)
    assert m.cache_load(path)
    assert np.array_equal(m.get(0), w["tok_embd"].view(np.uint8).ravel())
    assert np.array_equal(m.get(1), w["output_norm"].view(np.uint8))
    for li in range(SHAPE.layers):
        for j, k in enumerate(KEYS):
            assert np.array_equal(m.get(2 + j, li), w["layers"][li][k].view(np.uint8).ravel()), (li, k)
    assert m.lora() == (0.0, 0)


def test_reader_reads_reference_file(tmp_path):
    w = random_weights(3)
    ref = ReferenceModel(Reference(), SHAPE, w)
    path = str(tmp_path / "ref.tvcache")
    ref.cache_save(path, BASE.hex(), LORA.hex(), 64.0, 32)
    with tc.CacheFile(path) as f:
        assert f.version == 1
        assert bytes(f.key.base_sha256) == BASE and bytes(f.key.lora_sha256) == LORA
        assert f.key.lora_alpha == 64.0 and f.key.lora_rank == 32
        assert f.entries["blk.1.ffn_down"] == (tc.GGML_F16, dims("w_down"), 2 * SHAPE.inter * SHAPE.hidden)
        assert np.array_equal(f.read_numpy("tok_embd"), w["tok_embd"].view(np.uint8).ravel())
        for li in range(SHAPE.layers):
            for k in KEYS:
                got = f.read_numpy(f"blk.{li}.{tc.TENSOR_NAME.get(k, k)}")
                assert np.array_equal(got, w["layers"][li][k].view(np.uint8).ravel()), (li, k)


def test_int8_rows_make_a_version2_file(tmp_path):
    rng = np.random.default_rng(4)
    q = rng.integers(-127, 128, size=(40, 256), dtype=np.int8)
    s = rng.random(40).astype(np.float32)
    norm = np.ones(256, np.float32)
    path = str(tmp_path / "i8.tvcache")
    tc.write(path, tc.make_key(), [tc.Entry("blk.0.attn_q", tc.GGML_I8, (256, 40), q.ctypes.data, s.ctypes.data),
                                   tc.Entry("blk.0.attn_norm", tc.GGML_F32, (256,), norm.ctypes.data)])
    with tc.CacheFile(path) as f:
        assert f.version == 2
        assert f.entries["blk.0.attn_q"] == (tc.GGML_I8, (256, 40), 40 * 256)
        assert f.entries["blk.0.attn_q.row_scale"] == (tc.GGML_F32, (40,), 160)
        assert np.array_equal(f.read_numpy("blk.0.attn_q").view(np.int8).reshape(40, 256), q)
        assert np.array_equal(f.read_numpy("blk.0.attn_q.row_scale").view(np.float32), s)
    assert not ReferenceModel(Reference(), SHAPE).cache_load(path)   # refused, not misread


def test_bad_files_are_rejected(tmp_path):
    bad = tmp_path / "bad.tvcache"
    bad.write_bytes(b"NOTCACHE" + bytes(300))
    with pytest.raises(TvbError, match="not a .tvcache"):
        tc.CacheFile(str(bad))
    w = random_weights(5)
    good = str(tmp_path / "good.tvcache")
    tc.write(good, tc.make_key(), entries(w)[:3])
    data = open(good, "rb").read()
    (tmp_path / "short.tvcache").write_bytes(data[:300])
    with pytest.raises(TvbError):
        tc.CacheFile(str(tmp_path / "short.tvcache"))
    with tc.CacheFile(good) as f:
        small = np.empty(8, np.uint8)
        with pytest.raises(TvbError, match="no tensor"):
            f.read("blk.9.attn_q", small.ctypes.data, 8)
        with pytest.raises(TvbError, match="needs"):
            f.read("tok_embd", small.ctypes.data, 8)
