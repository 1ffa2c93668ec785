"""tvb_attention_decode_noalloc: the split-KV decode attention whose scratch
is a static array inside libtvb200, for callers that cannot allocate device
memory when they call (a host that gives its device memory to its own pool at
start-up, or a thread that must not risk the device synchronisation
cudaMalloc/cudaFree can imply).

Checked through the C ABI against tvb_attention_decode on the same inputs,
twice in a row (the shared scratch keeps the previous call's contents), with
the tolerance of the other attention tests, and against the oracle's
restatement of the reference's decode attention (cuda/ops_cuda.cu:205-259).
Kept in its own file, named to be collected last."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-4


def close(got, ref, rtol=RTOL):
    ref = np.asarray(ref, np.float64)
    floor = rtol * max(np.sqrt(np.mean(ref ** 2)), 1e-30)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=floor)


def attention_pair(lib, torch, nh, nkv, kv_len, seed):
    hd = 128
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal(nh * hd).astype(np.float32)).cuda()
    kc = torch.from_numpy(rng.standard_normal((kv_len, nkv * hd)).astype(np.float32)).cuda()
    vc = torch.from_numpy(rng.standard_normal((kv_len, nkv * hd)).astype(np.float32)).cuda()
    ref = torch.empty(nh * hd, dtype=torch.float32, device="cuda")
    got = torch.full((nh * hd,), float("nan"), dtype=torch.float32, device="cuda")
    scale = float(1 / np.sqrt(hd))
    assert lib.tvb_attention_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kv_len,
                                    ref.data_ptr(), nh, nkv, hd, scale, None) == 0
    assert lib.tvb_attention_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kv_len,
                                            got.data_ptr(), nh, nkv, hd, scale, None) == 0, \
        lib.tvb_last_error()
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy(), (q.cpu().numpy(), kc.cpu().numpy(), vc.cpu().numpy())


def test_noalloc_attention_matches_attention_decode(cuda, restated):
    import torch
    from ternative_b200 import load
    lib = load()
    # two calls in a row: a long context (8 splits), then a short one (1 split)
    for nh, nkv, kv_len, seed in ((32, 8, 1000, 1), (20, 5, 37, 2)):
        got, ref, (q, kc, vc) = attention_pair(lib, torch, nh, nkv, kv_len, seed)
        close(got, ref)
        close(got, restated.attention_decode(q, kc, vc, kv_len, nh, nkv, 128))


def test_noalloc_attention_rejects_oversize(cuda):
    from ternative_b200 import load
    lib = load()
    p = C.c_void_p(256)   # never dereferenced: the size check fails first
    assert lib.tvb_attention_decode_noalloc(p, p, p, 16, p, 128, 8, 128, 1.0, None) == 1
    assert b"static scratch limit" in lib.tvb_last_error()
