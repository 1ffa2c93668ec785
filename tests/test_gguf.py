"""GGUF ingest (tvb_gguf_*) against the reference's own gguf_load
(src/gguf.cpp, run from oracle/_ref): the same tensor table (types, shapes)
and the same bytes per tensor, sized as the reference's Tensor, for files with
every metadata value type, two alignments, and I2_S / F32 / F16 tensors;
malformed files are rejected.  Host memory here; the device path (straight
into the merge) is tests/test_gguf_gpu.py."""
import numpy as np
import pytest

from oracle.oracle import reference_gguf_tensor
from ternative_b200 import TvbError
from ternative_b200.cache import GGUFFile

from gguf_util import GGML_F16, GGML_F32, GGML_I2_S, i2s_tensor, write_gguf


@pytest.mark.parametrize("alignment", [32, 64])
def test_tensors_match_reference_gguf_load(tmp_path, restated, reference, alignment):
    rng = np.random.default_rng(alignment)
    w, _ = i2s_tensor(restated, 256, 24, 1)
    a = rng.standard_normal((4, 256)).astype(np.float32)
    h = rng.integers(0, 1 << 16, size=(7, 128), dtype=np.uint16)
    tensors = [("blk.0.attn_q.weight", GGML_I2_S, (256, 24), w),
               ("blk.0.attn_q.lora_a", GGML_F32, (256, 4), a.tobytes()),
               ("token_embd.weight", GGML_F16, (128, 7), h.tobytes())]
    path = str(tmp_path / "m.gguf")
    write_gguf(path, tensors, alignment)
    with GGUFFile(path) as g:
        assert set(g.entries) == {t[0] for t in tensors}
        for name, t, shape, data in tensors:
            rt, rshape, rbytes = reference_gguf_tensor(reference, path, name)
            assert g.entries[name] == (rt, rshape, rbytes.size), name
            assert np.array_equal(g.read_numpy(name), rbytes), name
            assert rbytes.tobytes() == data[:rbytes.size]


def test_malformed_files_are_rejected(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(64))
    with pytest.raises(TvbError, match="not a GGUF"):
        GGUFFile(str(bad))
    v2 = tmp_path / "v2.gguf"
    v2.write_bytes(b"GGUF" + (2).to_bytes(4, "little") + bytes(16))
    with pytest.raises(TvbError, match="version"):
        GGUFFile(str(v2))
    cut = tmp_path / "cut.gguf"
    write_gguf(str(cut), [("x", GGML_F32, (8,), np.zeros(8, np.float32).tobytes())])
    data = cut.read_bytes()
    cut.write_bytes(data[:40])
    with pytest.raises(TvbError):
        GGUFFile(str(cut))


def test_file_sizes_that_would_wrap_are_rejected(tmp_path):
    """Sizes from the file are checked before any arithmetic on them can wrap:
    an element count past 64 bits, an alignment past 1 MiB, a tensor offset
    near 2^64 (whose end would wrap back into the file), more than 4 dims."""
    huge = tmp_path / "huge.gguf"
    write_gguf(str(huge), [("x", GGML_F32, (1 << 40, 1 << 40), b"")])
    with pytest.raises(TvbError, match="overflows"):
        GGUFFile(str(huge))
    align = tmp_path / "align.gguf"
    write_gguf(str(align), [("x", GGML_F32, (8,), np.zeros(8, np.float32).tobytes())], alignment=1 << 21)
    with pytest.raises(TvbError, match="alignment"):
        GGUFFile(str(align))
    # a tensor whose offset is 2^64 - 16: its end wraps to a small number
    wrap = tmp_path / "wrap.gguf"
    write_gguf(str(wrap), [("x", GGML_F32, (8,), np.zeros(8, np.float32).tobytes())])
    blob = bytearray(wrap.read_bytes())
    at = blob.rfind(b"\x01\x00\x00\x00\x00\x00\x00\x00x")   # the tensor info: name length 1, "x"
    assert at > 0
    off_at = at + 9 + 4 + 8 + 4                             # name, n_dims, dim 0, type -> offset
    blob[off_at:off_at + 8] = ((1 << 64) - 16).to_bytes(8, "little")
    wrap.write_bytes(bytes(blob))
    with GGUFFile(str(wrap)) as g:
        out = np.empty(32, np.uint8)
        with pytest.raises(TvbError, match="past the file end"):
            g.read("x", out.ctypes.data, out.size)
    five = tmp_path / "five.gguf"
    write_gguf(str(five), [("x", GGML_F32, (2, 1, 1, 1, 2), np.zeros(4, np.float32).tobytes())])
    with pytest.raises(TvbError, match="dimensions"):
        GGUFFile(str(five))
