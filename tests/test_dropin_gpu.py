"""Drop-in check: the reference host's own src/model.cpp, compiled unchanged
with TERNATIVE_USE_CUDA against ternative_b200/shim/ops_tvb200.cpp (instead of
cuda/ops_cuda.cu) into oracle/_ref/libtvref_dropin.so, runs its GPU paths on
libtvb200:

* init_gpu_backend uploads every layer through the shim (alloc/upload);
* forward_prefill's projections go through CUDABackend::matmul on the GPU;
* Model::forward(prefill=false) takes forward_gpu, i.e. the reference's own
  per-op decode loop (rms_norm_d, gemv_d2d, rope_inplace_d, kv_write_d,
  attention_d, add_d, relu2_d, mul_d) on the tvb200 kernels.

Results are compared with the same reference host on its CPU backend."""
import os

import numpy as np
import pytest

from oracle.oracle import DROPIN_SO, ModelShape, Reference, ReferenceModel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dropin(cuda):
    if not os.path.exists(DROPIN_SO):
        pytest.skip("oracle/_ref/libtvref_dropin.so not built")
    return Reference(DROPIN_SO)


def tiny_weights(g):
    V, H, L, nh, nkv, I, ms = (int(x) for x in g["tiny_shape"])
    shp = ModelShape(V, H, L, nh, nkv, I, 64)
    w = {"tok_embd": g["tiny_tok_embd"], "output_norm": g["tiny_output_norm"], "layers": []}
    for li in range(L):
        w["layers"].append({k: g[f"tiny_l{li}_{k}"] for k in
                            ["wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "attn_norm",
                             "attn_sub_norm", "ffn_norm", "ffn_sub_norm"]})
    return shp, w


def test_reference_host_runs_on_tvb200(dropin, reference, golden):
    shp, w = tiny_weights(golden)
    prompt = golden["tiny_tokens"][:8]
    gpu = ReferenceModel(dropin, shp, w)
    assert gpu.init_gpu() == shp.layers          # every layer offloaded as F16
    pre = gpu.forward_prefill(prompt)             # matmul on GPU-resident weights
    cpu = ReferenceModel(reference, shp, w)
    ref_pre = cpu.forward_prefill(prompt)
    assert np.abs(pre - ref_pre).max() / np.abs(ref_pre).max() < 2e-3
    gpu.sync_kv_to_gpu(len(prompt))
    toks = list(prompt) + [int(np.argmax(pre[-1]))]
    for step in range(6):                         # forward_gpu per-op loop
        lg = gpu.forward(toks[-1], len(toks) - 1, False)
        ref = cpu.forward_prefill(np.array(toks, np.int32))[-1]
        err = np.abs(lg - ref).max() / np.abs(ref).max()
        assert err < 2e-3, (step, err)
        toks.append(int(np.argmax(lg)))
    gpu.close()
    cpu.close()
