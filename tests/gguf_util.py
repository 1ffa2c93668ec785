"""A GGUF v3 writer for the ingest tests (the layout gguf.cpp parses:
header, metadata key/values of every value type, tensor infos, the data
section at general.alignment)."""
import struct

import numpy as np

GGML_F32, GGML_F16, GGML_I2_S = 0, 1, 36


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q",
           12: "<d"}
    if t == 8:
        return _s(v.encode())
    if t == 9:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(fmt[t], v)


def write_gguf(path, tensors, alignment=32, extra_kv=()):
    """tensors: list of (name, ggml type, shape (ggml order), raw bytes)."""
    kv = [("general.architecture", 8, "bitnet"), ("general.alignment", 4, alignment),
          ("tokenizer.ggml.tokens", 9, (8, ["a", "bc", "<s>", "été"])),
          ("tokenizer.ggml.scores", 9, (6, [0.5, -1.0, 2.0])), ("bitnet.rope.freq_base", 6, 500000.0),
          ("some.flag", 7, True), ("some.u64", 10, 12345678901), ("some.i32", 5, -7),
          ("nested", 9, (9, [(4, [1, 2]), (8, ["x"])]))] + list(extra_kv)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for k, t, v in kv:
        head += _s(k.encode()) + struct.pack("<I", t) + _value(t, v)
    off, offs = 0, []
    for name, t, shape, data in tensors:
        offs.append(off)
        off += (len(data) + alignment - 1) // alignment * alignment
    for (name, t, shape, data), o in zip(tensors, offs):
        head += _s(name.encode()) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        head += struct.pack("<IQ", t, o)
    pad = (-len(head)) % alignment
    blob = bytearray(head + bytes(pad))
    for (name, t, shape, data), o in zip(tensors, offs):
        blob += bytes(data) + bytes((-len(data)) % alignment)
    with open(path, "wb") as f:
        f.write(bytes(blob))


def i2s_tensor(restated, K, N, seed):
    """An I2_S weight [N][K] (ggml shape (K, N)): codes, then the F32 scale."""
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 3, size=(N, K)).astype(np.uint8)
    scale = np.float32(rng.random() + 0.5)
    return restated.i2s_pack(codes).tobytes() + struct.pack("<f", float(scale)), float(scale)
