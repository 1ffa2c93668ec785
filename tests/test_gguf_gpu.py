"""GGUF ingest on the device path: a base file's I2_S projection and an
adapter file's F32 lora_a / lora_b are streamed by tvb_gguf_read straight
into device buffers (staged through pinned memory, no host copy of the
file), then merged on the device; the merged F32 and F16 weights equal the
oracle's merge of the same tensors bit for bit, as the reference's
load_tensor_from_gguf + apply_lora (src/model.cpp:136-258) compute them from
gguf_load's in-memory file."""
import numpy as np
import pytest

from gguf_util import GGML_F32, GGML_I2_S, write_gguf

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("K,N,r", [(256, 40, 16), (2560, 96, 16), (6912, 24, 64)])
def test_gguf_tensors_stream_into_device_merge(tmp_path, backend, restated, K, N, r):
    import torch
    from ternative_b200 import TVB_F16, TVB_F32
    from ternative_b200.cache import GGUFFile
    rng = np.random.default_rng(K + N + r)
    codes = rng.integers(0, 3, size=(N, K)).astype(np.uint8)
    scale = np.float32(0.75)
    w = restated.i2s_pack(codes).tobytes() + scale.tobytes()
    A = (rng.standard_normal((r, K)) / np.sqrt(K)).astype(np.float32)
    B = (rng.standard_normal((N, r)) * 1e-3).astype(np.float32)
    base, lora = str(tmp_path / "base.gguf"), str(tmp_path / "lora.gguf")
    write_gguf(base, [("blk.0.attn_q.weight", GGML_I2_S, (K, N), w)])
    write_gguf(lora, [("blk.0.attn_q.weight.lora_a", GGML_F32, (K, r), A.tobytes()),
                      ("blk.0.attn_q.weight.lora_b", GGML_F32, (r, N), B.tobytes())], alignment=64)

    def load(g, name):
        _, _, n = g.entries[name]
        buf = torch.empty(n, dtype=torch.uint8, device="cuda")
        g.read(name, buf.data_ptr(), n)
        return buf

    with GGUFFile(base) as gb, GGUFFile(lora) as gl:
        wd = load(gb, "blk.0.attn_q.weight")
        ad = load(gl, "blk.0.attn_q.weight.lora_a").view(torch.float32)
        bd = load(gl, "blk.0.attn_q.weight.lora_b").view(torch.float32)
    torch.cuda.synchronize()
    nc = K * N // 4
    s = float(wd[nc:].cpu().numpy().view(np.float32)[0])
    assert s == scale
    alpha = 2.0 * r
    ref32, ref16 = restated.merge(restated.i2s_pack(codes), s, K, N, A, B, alpha)
    for out, dt in ((TVB_F32, torch.float32), (TVB_F16, torch.float16)):
        dst = torch.empty(N, K, dtype=dt, device="cuda")
        backend.apply_lora_i2s(wd[:nc], s, K, N, ad.view(r, K), bd.view(N, r), alpha, out, dst, None, stream=0)
        torch.cuda.synchronize()
        got = dst.cpu().numpy()
        if out == TVB_F32:
            assert np.array_equal(got.view(np.uint32), ref32.view(np.uint32))
        else:
            assert np.array_equal(got.view(np.uint16), ref16)
