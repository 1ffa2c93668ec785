"""GPU parity of the per-op device API (the CUDABackend surface,
include/ternative/ops.h:102-162) against the oracle restatement.  Floating
point results are held to the path's 2e-3 relative tolerance (element-wise
rtol 2e-3 with an absolute floor of 2e-3 x RMS of the reference output)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 2e-3


def close(got, ref, rtol=RTOL):
    ref = np.asarray(ref, np.float64)
    floor = rtol * max(np.sqrt(np.mean(ref ** 2)), 1e-30)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=floor)


def T(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture(scope="module")
def ctx_backend(backend):
    from ternative_b200 import Config
    backend.init_gpu_activations(Config(vocab_size=4096, hidden_size=512, num_layers=2, num_heads=4,
                                        num_kv_heads=2, head_dim=128, intermediate_size=1024,
                                        max_seq_len=256))
    return backend


GEMV_SHAPES = [(2560, 2560), (640, 2560), (6912, 2560), (2560, 6912), (128256, 2560), (37, 264),
               (3, 8), (1, 2560)]


@pytest.mark.parametrize("N,K", GEMV_SHAPES)
def test_gemv_f16(ctx_backend, restated, N, K):
    import torch
    rng = np.random.default_rng(N + K)
    x = rng.standard_normal(K).astype(np.float32)
    w = restated.f32_to_f16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    ctx_backend.gemv_d2d(y, T(x), T(w), K, N)
    close(host(y), restated.gemv_f16(x, w))


@pytest.mark.parametrize("N,K", [(2560, 2560), (6912, 2560), (2560, 6912), (100, 272)])
def test_gemv_int8(ctx_backend, restated, N, K):
    import torch
    rng = np.random.default_rng(3 * N + K)
    x = rng.standard_normal(K).astype(np.float32)
    w = restated.f32_to_f16((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    qt, st = restated.quantize_int8_tensor(w)
    qr, sr = restated.quantize_int8_rows(w)
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    ctx_backend.gemv_d2d_int8(y, T(x), T(qt), st, K, N)
    close(host(y), restated.gemv_int8(x, qt, None, st))
    ctx_backend.gemv_d2d_int8_rows(y, T(x), T(qr), T(sr), K, N)
    close(host(y), restated.gemv_int8(x, qr, sr))


@pytest.mark.parametrize("n", [2560, 6912, 640, 13])
def test_rms_norm_and_elementwise(ctx_backend, restated, n):
    import torch
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32) * 3
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    ctx_backend.rms_norm_d(out, T(x), T(w), 1e-5, n)
    close(host(out), restated.rms_norm(x, w, 1e-5), rtol=1e-5)
    ctx_backend.add_d(out, T(x), T(b), n)
    assert np.array_equal(host(out), x + b)
    ctx_backend.mul_d(out, T(x), T(b), n)
    assert np.array_equal(host(out), x * b)
    ctx_backend.relu2_d(out, T(x), n)
    r = np.maximum(x, 0)
    assert np.array_equal(host(out), r * r)


@pytest.mark.parametrize("pos", [0, 1, 31, 159, 1023, 4000])
def test_rope(ctx_backend, restated, pos):
    rng = np.random.default_rng(pos)
    nh, nkv, hd = 20, 5, 128
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    rq, rk = restated.rope(q, k, nh, nkv, hd, pos, 500000.0)
    dq, dk = T(q), T(k)
    ctx_backend.rope_inplace_d(dq, dk, pos, 500000.0, nh, nkv, hd)
    # device powf/sincosf vs the host libm: a few ulp on the angle, which grows with pos
    close(host(dq), rq)
    close(host(dk), rk)


@pytest.mark.parametrize("kv_len", [1, 2, 7, 160, 1000])
def test_kv_write_and_attention(ctx_backend, restated, kv_len):
    import torch
    nh, nkv, hd = 4, 2, 128
    rng = np.random.default_rng(kv_len)
    kc = rng.standard_normal((kv_len, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((kv_len, nkv * hd)).astype(np.float32)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    dk = torch.zeros(1024, nkv * hd, dtype=torch.float32, device="cuda")
    dv = torch.zeros(1024, nkv * hd, dtype=torch.float32, device="cuda")
    dk[: kv_len - 1] = T(kc[:-1])
    dv[: kv_len - 1] = T(vc[:-1])
    # the last row goes through kv_write at pos = kv_len - 1
    from ternative_b200._lib import call
    k_last, v_last, dq = T(kc[-1]), T(vc[-1]), T(q)   # keep the device copies alive
    call("tvb_kv_write", k_last.data_ptr(), v_last.data_ptr(), dk.data_ptr(), dv.data_ptr(),
         kv_len - 1, nkv * hd, 0)
    out = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    call("tvb_attention_decode", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv_len,
         out.data_ptr(), nh, nkv, hd, float(1 / np.sqrt(hd)), 0)
    close(host(out), restated.attention_decode(q, kc, vc, kv_len, nh, nkv, hd), rtol=1e-4)


def test_context_kv_roundtrip(ctx_backend):
    rng = np.random.default_rng(1)
    Hk = 2 * 128
    hk = rng.standard_normal((10, Hk)).astype(np.float32)
    hv = rng.standard_normal((10, Hk)).astype(np.float32)
    ctx_backend.upload_kv_layer_d(1, 10, hk, hv)
    assert np.array_equal(ctx_backend.download_kv_slot_d(1, 7, Hk), hk[7])
    assert ctx_backend.has_gpu_kv(256) and not ctx_backend.has_gpu_kv(257)
    ctx_backend.clear_kv_d()
    assert not ctx_backend.download_kv_slot_d(1, 7, Hk).any()


def test_reference_buffers_usable(ctx_backend):
    x = np.arange(512, dtype=np.float32)
    ctx_backend.upload_pinned(ctx_backend.d_x(), x, 512)
    ctx_backend.add_d(ctx_backend.d_norm(), ctx_backend.d_x(), ctx_backend.d_x(), 512)
    assert np.array_equal(ctx_backend.download_pinned(ctx_backend.d_norm(), 512), 2 * x)
