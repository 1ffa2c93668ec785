"""GPU parity of tvb_merge_batch_tc, the merge whose rank-r LoRA delta runs on
the tensor cores (tcgen05.mma over F16 hi/lo splits of A and B), against the
oracle's bit-exact restatement of apply_lora (src/model.cpp:180-258): F16
outputs within one unit in the last place (the tolerance for merged F16
weights) and nearly always identical; per-row INT8 as the reference's row
quantisation of those F16 rows (codes within one of the exact merge's); outputs
the tensor-core path does not take (F32, ranks above 64) bit-identical through
the exact path."""
import numpy as np
import pytest

from ternative_b200 import TVB_F16, TVB_F32, TVB_I8_ROW, MergeDesc

pytestmark = pytest.mark.gpu

from tests.test_merge_gpu import dev, make_case   # noqa: E402


def f16_key(bits):
    """Order-preserving integer key of F16 bit patterns (adjacent values differ by 1)."""
    b = bits.astype(np.int32)
    return np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), 0x8000 + b)


def run_tc(backend, torch, cases, out=TVB_F16):
    descs, keep = [], []
    for (i2s, s, K, N, A, B, r, alpha, k0, ld) in cases:
        dt = {TVB_F16: torch.float16, TVB_F32: torch.float32, TVB_I8_ROW: torch.int8}[out]
        t = [dev(i2s, torch), dev(A, torch), dev(B, torch), torch.empty(N, K, dtype=dt, device="cuda"),
             torch.empty(N, dtype=torch.float32, device="cuda")]
        keep.append(t)
        descs.append(MergeDesc(t[0].data_ptr(), s, K, N, t[1].data_ptr() if r else None,
                               t[2].data_ptr() if r else None, r, alpha, t[3].data_ptr(),
                               t[4].data_ptr() if out == TVB_I8_ROW else None, k0, ld))
    backend.merge_batch_tc(descs, out, stream=0)
    torch.cuda.synchronize()
    return [(t[3].cpu().numpy(), t[4].cpu().numpy()) for t in keep]


@pytest.mark.parametrize("K,N,r", [(256, 40, 16), (384, 7, 3), (128, 9, 1), (2560, 640, 16),
                                   (6912, 130, 64), (2560, 33, 0), (4096, 257, 32)])
def test_tc_merge_f16_within_one_ulp(backend, restated, K, N, r):
    import torch
    i2s, s, A, B = make_case(restated, K, N, r, 11 * K + N + r)
    alpha = 2.0 * max(r, 1)
    got = run_tc(backend, torch, [(i2s, s, K, N, A, B, r, alpha, 0, 0)])[0][0].view(np.uint16)
    A0 = A if r else np.zeros((1, K), np.float32)
    B0 = B if r else np.zeros((N, 1), np.float32)
    ref = restated.merge(i2s, s, K, N, A0, B0, alpha)[1]
    d = np.abs(f16_key(got) - f16_key(ref))
    assert d.max() <= 1, (int(d.max()), int((d > 0).sum()))
    assert (d == 0).mean() > 0.999


def test_tc_merge_batch_and_column_slices(backend, restated):
    import torch
    K, N, r = 1024, 96, 64
    i2s, s, A, B = make_case(restated, K, N, r, 5)
    full = restated.merge(i2s, s, K, N, A, B, 128.0)[1]
    cases = [(i2s, s, K, N, A, B, r, 128.0, 0, 0)]
    for k0 in (0, 256, 768):   # column slices of 256 (row-parallel shards)
        cases.append((i2s, s, 256, N, A, B, r, 128.0, k0, K))
    outs = run_tc(backend, torch, cases)
    d = np.abs(f16_key(outs[0][0].view(np.uint16)) - f16_key(full))
    assert d.max() <= 1
    for (o, _), k0 in zip(outs[1:], (0, 256, 768)):
        assert np.array_equal(o.view(np.uint16), outs[0][0].view(np.uint16)[:, k0:k0 + 256])


def test_tc_merge_exact_outputs_fall_back(backend, restated):
    import torch
    K, N, r = 512, 24, 128   # rank above 64 -> exact path
    i2s, s, A, B = make_case(restated, K, N, r, 8)
    got = run_tc(backend, torch, [(i2s, s, K, N, A, B, r, 64.0, 0, 0)])[0][0].view(np.uint16)
    assert np.array_equal(got, restated.merge(i2s, s, K, N, A, B, 64.0)[1])


@pytest.mark.parametrize("K,N,r", [(512, 24, 16), (2560, 640, 64), (6912, 130, 32)])
def test_tc_merge_int8_rows(backend, restated, K, N, r):
    """Per-row INT8 through the tensor cores: exactly the reference's row
    quantisation of the tensor-core F16 rows; against the bit-exact merge's
    codes, within one code (and identical scales wherever the row maxima agree)."""
    import torch
    i2s, s, A, B = make_case(restated, K, N, r, 9 + K)
    case = [(i2s, s, K, N, A, B, r, 2.0 * r, 0, 0)]
    q, sc = run_tc(backend, torch, case, out=TVB_I8_ROW)[0]
    f16 = run_tc(backend, torch, case)[0][0].view(np.uint16)
    qr, sr = restated.quantize_int8_rows(f16)
    assert np.array_equal(q, qr)
    assert np.array_equal(sc.view(np.uint32), sr.view(np.uint32))
    qe, se = restated.quantize_int8_rows(restated.merge(i2s, s, K, N, A, B, 2.0 * r)[1])
    assert np.abs(q.astype(np.int32) - qe.astype(np.int32)).max() <= 1
    assert np.abs(sc / se - 1.0).max() <= 2.0 ** -10
    assert (q == qe).mean() > 0.999
