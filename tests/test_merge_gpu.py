"""GPU parity of the load-time merge (tvb_merge_i2s_lora / tvb_merge_batch /
tvb_quantize_int8) against the oracle: bit-exact for the merged F32, the F16
cast and the INT8 codes and scales, as the reference's apply_lora
(src/model.cpp:205-258) and INT8 quantizer (:374-410) compute them."""
import numpy as np
import pytest

from ternative_b200 import TVB_F16, TVB_F32, TVB_I8_ROW, MergeDesc, TvbError

pytestmark = pytest.mark.gpu


def make_case(restated, K, N, r, seed):
    rng = np.random.default_rng(seed)
    lat = rng.standard_normal((N, K)).astype(np.float32)
    s = float(np.abs(lat).mean())
    codes = (np.round(np.clip(lat / s, -1, 1)) + 1).astype(np.uint8)
    i2s = restated.i2s_pack(codes)
    A = (rng.standard_normal((r, K)) / np.sqrt(K)).astype(np.float32) if r else None
    B = (rng.standard_normal((N, r)) * 1e-3).astype(np.float32) if r else None
    return i2s, s, A, B


def dev(x, torch):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).cuda()


def gpu_merge(backend, torch, i2s, s, K, N, A, B, alpha, out):
    dt = {TVB_F32: torch.float32, TVB_F16: torch.float16, TVB_I8_ROW: torch.int8}[out]
    dst = torch.empty(N, K, dtype=dt, device="cuda")
    rs = torch.empty(N, dtype=torch.float32, device="cuda") if out == TVB_I8_ROW else None
    backend.apply_lora_i2s(dev(i2s, torch), s, K, N, dev(A, torch), dev(B, torch), alpha, out, dst, rs,
                           stream=0)
    torch.cuda.synchronize()
    return dst.cpu().numpy(), None if rs is None else rs.cpu().numpy()


CASES = [(256, 40, 16), (384, 7, 3), (128, 9, 1), (2560, 640, 16), (6912, 24, 64), (2560, 33, 0),
         (4096, 17, 32), (14336, 5, 32), (512, 64, 256)]


@pytest.mark.parametrize("K,N,r", CASES)
def test_merge_f32_f16_bit_exact(backend, restated, K, N, r):
    import torch
    i2s, s, A, B = make_case(restated, K, N, r, K * 31 + N + r)
    alpha = 2.0 * r if r else 0.0
    A0 = A if r else np.zeros((1, K), np.float32)
    B0 = B if r else np.zeros((N, 1), np.float32)
    ref32, ref16 = restated.merge(i2s, s, K, N, A0, B0, alpha if r else 1.0)
    g32, _ = gpu_merge(backend, torch, i2s, s, K, N, A, B, alpha, TVB_F32)
    g16, _ = gpu_merge(backend, torch, i2s, s, K, N, A, B, alpha, TVB_F16)
    assert np.array_equal(g32.view(np.uint32), ref32.view(np.uint32))
    assert np.array_equal(g16.view(np.uint16), ref16)


@pytest.mark.parametrize("K,N,r", [(256, 40, 16), (2560, 37, 16), (6912, 16, 64), (14336, 6, 32)])
def test_merge_int8_rows_bit_exact(backend, restated, K, N, r):
    import torch
    i2s, s, A, B = make_case(restated, K, N, r, 7 + K + N)
    _, ref16 = restated.merge(i2s, s, K, N, A, B, 2.0 * r)
    rq, rs = restated.quantize_int8_rows(ref16)
    gq, gs = gpu_merge(backend, torch, i2s, s, K, N, A, B, 2.0 * r, TVB_I8_ROW)
    assert np.array_equal(gq, rq)
    assert np.array_equal(gs.view(np.uint32), rs.view(np.uint32))


def test_merge_golden_vectors(backend, golden):
    """The reference's own outputs (tests/golden) reproduced on the GPU."""
    import torch
    for ci in range(4):
        K, N, r, alpha = golden[f"m{ci}_meta"]
        K, N, r = int(K), int(N), int(r)
        args = (golden[f"m{ci}_i2s"], float(golden[f"m{ci}_scale"]), K, N, golden[f"m{ci}_A"],
                golden[f"m{ci}_B"], float(alpha))
        g32, _ = gpu_merge(backend, torch, *args, TVB_F32)
        g16, _ = gpu_merge(backend, torch, *args, TVB_F16)
        assert np.array_equal(g32.view(np.uint32), golden[f"m{ci}_f32"].view(np.uint32))
        assert np.array_equal(g16.view(np.uint16), golden[f"m{ci}_f16"])
        # per-tensor INT8 (the reference's init_gpu_backend quantizer)
        w16 = torch.from_numpy(g16).cuda()
        q = torch.empty(N, K, dtype=torch.int8, device="cuda")
        sc = torch.empty(1, dtype=torch.float32, device="cuda")
        backend.quantize_int8(w16, N, K, False, q, sc, stream=0)
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), golden[f"m{ci}_i8t"])
        assert np.float32(sc.item()) == golden[f"m{ci}_i8t_scale"]


def test_merge_batch_many_tensors(backend, restated):
    """One launch over tensors of mixed shapes and ranks (sharded-by-tensor merge)."""
    import torch
    shapes = [(256, 40, 16), (384, 7, 3), (512, 24, 8), (2560, 9, 16), (128, 130, 4)] * 3
    descs, keep, refs = [], [], []
    for i, (K, N, r) in enumerate(shapes):
        i2s, s, A, B = make_case(restated, K, N, r, 100 + i)
        t = [dev(i2s, torch), dev(A, torch), dev(B, torch), torch.empty(N, K, dtype=torch.float16,
                                                                         device="cuda")]
        keep.append(t)
        descs.append(MergeDesc(t[0].data_ptr(), s, K, N, t[1].data_ptr(), t[2].data_ptr(), r,
                               2.0 * r, t[3].data_ptr(), None))
        refs.append(restated.merge(i2s, s, K, N, A, B, 2.0 * r)[1])
    backend.merge_batch(descs, TVB_F16, stream=0)
    torch.cuda.synchronize()
    for t, ref in zip(keep, refs):
        assert np.array_equal(t[3].cpu().numpy().view(np.uint16), ref)


def test_i2s_unpack_golden(backend, golden):
    import torch
    raw = dev(golden["i2s_raw"], torch)
    out = torch.empty(128 * 6, dtype=torch.float32, device="cuda")
    backend.i2s_unpack(raw, 128 * 6, float(golden["i2s_raw_scale"]), out, stream=0)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), golden["i2s_raw_out"].view(np.uint32))


def test_quantize_int8_rows_matches_oracle(backend, restated):
    import torch
    rng = np.random.default_rng(5)
    w = restated.f32_to_f16((rng.standard_normal((50, 1024)) * 0.03).astype(np.float32))
    w[3] = 0   # all-zero row -> scale 1/127 (max_abs 0 -> 1)
    rq, rs = restated.quantize_int8_rows(w)
    q = torch.empty(50, 1024, dtype=torch.int8, device="cuda")
    sc = torch.empty(50, dtype=torch.float32, device="cuda")
    backend.quantize_int8(dev(w, torch), 50, 1024, True, q, sc, stream=0)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_merge_rejects_bad_shapes(backend):
    import torch
    dst = torch.empty(4, 100, dtype=torch.float16, device="cuda")
    src = torch.zeros(100, dtype=torch.uint8, device="cuda")
    with pytest.raises(TvbError, match="multiple of 128"):
        backend.apply_lora_i2s(src, 1.0, 100, 4, None, None, 0.0, TVB_F16, dst, stream=0)
    with pytest.raises(TvbError, match="aligned"):
        backend.apply_lora_i2s(src, 1.0, 128, 1, None, None, 0.0, TVB_F16, dst.data_ptr() + 2,
                               stream=0)


def test_merge_tensor_parallel_slices(backend, restated):
    """Shards of one tensor, merged separately (row slices for column-parallel
    projections, column slices for row-parallel ones), are bit-identical to the
    slices of the whole-tensor merge."""
    import torch
    K, N, r = 1024, 96, 16
    i2s, s, A, B = make_case(restated, K, N, r, 777)
    full = restated.merge(i2s, s, K, N, A, B, 2.0 * r)[1]          # [N][K] F16 bits
    ti, tA, tB = dev(i2s, torch), dev(A, torch), dev(B, torch)
    T = 4
    descs, outs = [], []
    for rank in range(T):
        # column-parallel: rows [rank * N/T, ...)
        n0, nn = rank * N // T, N // T
        o = torch.empty(nn, K, dtype=torch.float16, device="cuda")
        descs.append(MergeDesc(ti.data_ptr() + n0 * K // 4, s, K, nn, tA.data_ptr(),
                               tB.data_ptr() + n0 * r * 4, r, 2.0 * r, o.data_ptr(), None, 0, 0))
        outs.append(("rows", n0, nn, o))
        # row-parallel: columns [rank * K/T, ...) of every row
        k0, kk = rank * K // T, K // T
        o = torch.empty(N, kk, dtype=torch.float16, device="cuda")
        descs.append(MergeDesc(ti.data_ptr(), s, kk, N, tA.data_ptr(), tB.data_ptr(), r, 2.0 * r,
                               o.data_ptr(), None, k0, K))
        outs.append(("cols", k0, kk, o))
    backend.merge_batch(descs, TVB_F16, stream=0)
    torch.cuda.synchronize()
    for kind, a0, n, o in outs:
        got = o.cpu().numpy().view(np.uint16)
        ref = full[a0:a0 + n] if kind == "rows" else full[:, a0:a0 + n]
        assert np.array_equal(got, ref), (kind, a0)


def test_merge_rejects_bad_slice(backend):
    import torch
    from ternative_b200 import TvbError
    o = torch.empty(8, 128, dtype=torch.float16, device="cuda")
    src = torch.zeros(8 * 256 // 4 + 4, dtype=torch.uint8, device="cuda")
    d = MergeDesc(src.data_ptr(), 1.0, 128, 8, None, None, 0, 0.0, o.data_ptr(), None, 64, 256)
    with pytest.raises(TvbError, match="column slice"):
        backend.merge_batch([d], TVB_F16, stream=0)
