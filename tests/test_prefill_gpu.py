"""GPU parity of the batched prefill (Model::forward_prefill, model.cpp:1139-1234):

* the tensor-core GEMM behind tvb_matmul for batched rows (CUDABackend::matmul
  with M > 1, ops_cuda.cu:440-491, 600-631) against an F64 product of the same
  F32 activations and F16 / INT8 weights: F32 activations reach the tensor
  cores as F16 hi + lo planes with a power-of-two row scale, so the result
  stays within ~1e-5 of the F32 product whatever the row magnitudes;
* the whole prefill -- tensor-core projections with fused RoPE / KV append /
  residual / relu^2 epilogues, causal GQA attention -- against the numpy
  restatement of forward_prefill (2e-3 relative): prompts spanning several
  128-token tiles, prompts cut into chunks (attention over earlier chunks'
  KV rows), and the KV rows it leaves for the decode steps that follow.
"""
import ctypes as C
import dataclasses

import numpy as np
import pytest

from oracle.oracle import ModelShape, forward_prefill

pytestmark = pytest.mark.gpu

RTOL = 2e-3
GEMM_RTOL = 2e-5


def rel_err(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def oracle_shape(cfg):
    return ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                      cfg.num_kv_heads, cfg.intermediate_size, cfg.max_seq_len, cfg.rope_theta,
                      cfg.rms_norm_eps)


def matmul(lib, torch, x, w, dtype, row_scales=None, tensor_scale=1.0):
    from ternative_b200._lib import Weight
    M, K = x.shape
    N = w.shape[0]
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    wt = Weight(w.data_ptr(), dtype, row_scales.data_ptr() if row_scales is not None else None,
                tensor_scale)
    st = lib.tvb_matmul(y.data_ptr(), x.data_ptr(), M, K, C.byref(wt), N, None)
    assert st == 0, lib.tvb_last_error()
    torch.cuda.synchronize()
    return y.cpu().numpy()


# (1024, 6912, 2560), (512, 6912, 2560), (1024, 4096, 4096) and (900, 8192, 2304)
# take the persistent stream-K kernel (at least 64 k-blocks, fewer output tiles
# than SMs, each cut into at most four pieces finished by their owner); the
# other large ones the data-parallel tile kernel with TMA-stored outputs
# (1002 columns: a row pitch TMA cannot take, per-thread stores)
@pytest.mark.parametrize("M,K,N", [(200, 2560, 640), (37, 512, 1000), (130, 1024, 1002), (8, 6912, 256),
                                   (1024, 6912, 2560), (512, 6912, 2560), (1024, 4096, 4096),
                                   (900, 8192, 2304), (640, 2560, 3840), (1000, 512, 6912),
                                   (300, 1024, 16000), (129, 2560, 10240)])
def test_tensor_core_matmul_f16(cuda, M, K, N):
    import torch
    from ternative_b200 import TVB_F16, load
    lib = load()
    g = torch.Generator().manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=g).cuda()
    w = (torch.randn(N, K, generator=g) * 0.02).half().cuda()
    got = matmul(lib, torch, x, w, TVB_F16)
    ref = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    assert rel_err(got, ref) < GEMM_RTOL, rel_err(got, ref)
    worst = max(rel_err(got[r], ref[r]) for r in range(M))
    assert worst < GEMM_RTOL, worst


def test_tensor_core_matmul_int8_rows_stream_k(cuda):
    """Per-row INT8 weights through the stream-K kernel (the down shape)."""
    import torch
    from ternative_b200 import TVB_I8_ROW, load
    lib = load()
    g = torch.Generator().manual_seed(6)
    M, K, N = 1024, 6912, 2560
    x = torch.randn(M, K, generator=g).cuda()
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).cuda()
    s = (torch.rand(N, generator=g) * 1e-3 + 1e-4).cuda()
    got = matmul(lib, torch, x, q, TVB_I8_ROW, row_scales=s)
    ref = (x.double().cpu().numpy() @ q.double().cpu().numpy().T) * s.double().cpu().numpy()[None, :]
    worst = max(rel_err(got[r], ref[r]) for r in range(M))
    assert worst < GEMM_RTOL, worst


def test_tensor_core_matmul_int8_row_and_tensor(cuda):
    import torch
    from ternative_b200 import TVB_I8_ROW, TVB_I8_TENSOR, load
    lib = load()
    g = torch.Generator().manual_seed(5)
    M, K, N = 150, 2560, 768
    x = torch.randn(M, K, generator=g).cuda()
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).cuda()
    s = (torch.rand(N, generator=g) * 1e-3 + 1e-4).cuda()
    got = matmul(lib, torch, x, q, TVB_I8_ROW, row_scales=s)
    qd = q.double().cpu().numpy()
    ref = (x.double().cpu().numpy() @ qd.T) * s.double().cpu().numpy()[None, :]
    assert rel_err(got, ref) < GEMM_RTOL
    got = matmul(lib, torch, x, q, TVB_I8_TENSOR, tensor_scale=0.0123)
    ref = (x.double().cpu().numpy() @ qd.T) * np.float64(np.float32(0.0123))
    assert rel_err(got, ref) < GEMM_RTOL


def test_tensor_core_matmul_row_magnitudes(cuda):
    """Rows of very different scale (1e-6 .. 1e6, beyond the F16 range): the
    power-of-two row exponent keeps each row's relative accuracy."""
    import torch
    from ternative_b200 import TVB_F16, load
    lib = load()
    g = torch.Generator().manual_seed(9)
    M, K, N = 64, 1024, 512
    scales = torch.logspace(-6, 6, M, dtype=torch.float64)
    x = (torch.randn(M, K, generator=g, dtype=torch.float64) * scales[:, None]).float().cuda()
    w = (torch.randn(N, K, generator=g) * 0.05).half().cuda()
    got = matmul(lib, torch, x, w, TVB_F16)
    ref = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    for r in range(M):
        assert rel_err(got[r], ref[r]) < GEMM_RTOL, r


@pytest.fixture(scope="module")
def small_synth(cuda):
    from ternative_b200.model import SHAPES, SyntheticModel
    cfg = SHAPES["small"]
    return SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=3)


def _load(synth, **cfg_changes):
    from ternative_b200.model import Model
    if cfg_changes:
        synth = dataclasses.replace(synth, cfg=dataclasses.replace(synth.cfg, **cfg_changes))
    m = Model.load(synth)
    return m, m.host_weights()


def test_prefill_2b_dims_stream_k_matches_oracle(restated):
    """The projections of the 2B shape (hidden 2560, 20/5 heads, FFN 6912) at
    640 and 1024 tokens -- every GEMM on the persistent stream-K kernel -- in a
    2-layer model with a 4096-token vocabulary, against the numpy restatement;
    then one decode step over the KV rows the prefill wrote."""
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    cfg = dataclasses.replace(SHAPES["bitnet-2b"], vocab_size=4096, num_layers=2, max_seq_len=1152,
                              max_prefill=1024)
    synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=5, norm_value=1.0 / 32)
    m = Model.load(synth)
    hw = m.host_weights()
    for S in (640, 1024):
        prompt = np.random.default_rng(S).integers(0, cfg.vocab_size, S).astype(np.int32)
        m.backend.clear_kv_d()
        last, am = m.backend.prefill(prompt)
        lg, _ = m.backend.decode_step(am, S)
        # causal: row S - 1 of the S + 1 tokens is the prompt's last row
        ref = forward_prefill(oracle_shape(cfg), hw, list(prompt) + [am], restated.f16_to_f32)
        assert rel_err(last, ref[-2]) < RTOL, (S, rel_err(last, ref[-2]))
        assert am == int(np.argmax(last))
        assert rel_err(lg, ref[-1]) < RTOL, (S, rel_err(lg, ref[-1]))
    m.backend.close()


@pytest.mark.parametrize("S,max_prefill", [(200, 512), (150, 64), (1, 512), (129, 512)])
def test_batched_prefill_matches_oracle(small_synth, restated, S, max_prefill):
    m, hw = _load(small_synth, max_prefill=max_prefill)
    cfg = m.cfg
    rng = np.random.default_rng(S)
    prompt = rng.integers(0, cfg.vocab_size, S).astype(np.int32)
    m.backend.clear_kv_d()
    last, am = m.backend.prefill(prompt)
    ref = forward_prefill(oracle_shape(cfg), hw, prompt, restated.f16_to_f32)
    assert rel_err(last, ref[-1]) < RTOL, rel_err(last, ref[-1])
    assert am == int(np.argmax(last))
    # the decode step that follows reads the KV rows the prefill wrote
    lg, _ = m.backend.decode_step(am, S)
    ref2 = forward_prefill(oracle_shape(cfg), hw, list(prompt) + [am], restated.f16_to_f32)
    assert rel_err(lg, ref2[-1]) < RTOL, rel_err(lg, ref2[-1])
