"""The .tvcache on the device path: the merged weights are written from device
memory (staged through pinned buffers, no host copy of the model), the
reference's own ModelCache::try_load (oracle/_ref) reads the file back to the
same bytes, and tvb_cache_read uploads every tensor into device buffers
bit-identically; per-row INT8 layers round-trip through a version-2 file."""
import dataclasses

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_device_cache_round_trip(tmp_path):
    import torch
    from oracle.oracle import ModelShape, Reference, ReferenceModel
    from ternative_b200 import cache as tc
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    cfg = dataclasses.replace(SHAPES["small"], max_seq_len=128, max_prefill=128)
    m = Model.load(SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=2))
    path = str(tmp_path / "small.tvcache")
    key = tc.make_key(bytes(range(32)), bytes(range(32, 64)), 32.0, 16)
    m.save_cache(path, key)
    ents = tc.model_entries(m)

    # the reference reads it: every tensor equals the device copy
    shape = ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads, cfg.num_kv_heads,
                       cfg.intermediate_size, 64)
    ref = ReferenceModel(Reference(), shape)
    assert ref.cache_load(path)
    assert ref.lora() == (32.0, 16)
    dev = {"tok_embd": m.tok_embd, "output_norm": m.output_norm}
    assert np.array_equal(ref.get(0), dev["tok_embd"].cpu().numpy().view(np.uint8).ravel())
    for li in range(cfg.num_layers):
        for j, k in enumerate(ReferenceModel.LAYER_KEYS):
            t = m.weights[li][k] if k in tc.TENSOR_NAME else m.norms[li][k]
            assert np.array_equal(ref.get(2 + j, li), t.cpu().numpy().view(np.uint8).ravel()), (li, k)

    # our reader uploads into device buffers, bit-identical to the originals
    orig = {"tok_embd": m.tok_embd, "output_norm": m.output_norm}
    for li in range(cfg.num_layers):
        for k in ReferenceModel.LAYER_KEYS:
            orig[f"blk.{li}.{tc.TENSOR_NAME.get(k, k)}"] = m.weights[li][k] if k in tc.TENSOR_NAME else m.norms[li][k]
    with tc.CacheFile(path) as f:
        assert f.version == 1 and len(f.entries) == len(ents)
        for e in ents:
            _, _, n = f.entries[e.name]
            t = orig[e.name]
            got = torch.empty_like(t)
            assert n == t.numel() * t.element_size()
            f.read(e.name, got.data_ptr(), n)
            torch.cuda.synchronize()
            assert torch.equal(got, t), e.name
    m.backend.close()


def test_device_cache_int8_rows(tmp_path):
    import torch
    from ternative_b200 import cache as tc
    from ternative_b200.model import SHAPES, Model, SyntheticModel
    cfg = dataclasses.replace(SHAPES["tiny"], max_seq_len=64, max_prefill=64)
    m = Model.load(SyntheticModel.generate(cfg, rank=4, alpha=8.0, seed=3), int8_layers=(1,))
    path = str(tmp_path / "i8.tvcache")
    m.save_cache(path)
    with tc.CacheFile(path) as f:
        assert f.version == 2
        for k, name in tc.TENSOR_NAME.items():
            codes = m.weights[1][k]
            scales = m.row_scales[1][k]
            got = torch.empty_like(codes)
            f.read(f"blk.1.{name}", got.data_ptr(), codes.numel())
            got_s = torch.empty_like(scales)
            f.read(f"blk.1.{name}.row_scale", got_s.data_ptr(), 4 * scales.numel())
            torch.cuda.synchronize()
            assert torch.equal(got, codes) and torch.equal(got_s, scales), name
            # layer 0 stays F16
            w0 = m.weights[0][k]
            got0 = torch.empty_like(w0)
            f.read(f"blk.0.{name}", got0.data_ptr(), 2 * w0.numel())
            torch.cuda.synchronize()
            assert torch.equal(got0, w0), name
    m.backend.close()
