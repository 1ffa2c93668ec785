"""Model-level host code: seeded synthetic BitNet-shaped weights (I2_S + LoRA),
the load-time merge on the device, and a ``Model`` that drives the fused
decode/prefill steps.

This mirrors the reference's Model (include/ternative/model.h:104-223) for
the quantized-weight path only: ``Model.load`` plays the role of
Model::load + init_gpu_backend (src/model.cpp:264-788) with the LoRA merge and
INT8 cast done by the CUDA merge kernel; ``forward_gpu``, ``forward_prefill``
and ``generate_greedy`` replace the layer loops of src/model.cpp:1139-1582.

Synthetic inputs (no checkpoints are available offline): latent weights
N(0,1) ternarised by absmean (scale = mean|W|, code = round(clip(W/scale,-1,1)))
and packed as I2_S; token embeddings F16 N(0, 0.02); norm weights 1.0; LoRA
A ~ N(0, 1/in) (variance), B ~ N(0, 1e-3) (standard deviation).  All
generated on the device from a seeded torch generator.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from ._lib import TVB_F16, TVB_I8_ROW, TVB_I8_TENSOR, MergeDesc
from .backend import Config, CUDABackend, DeviceWeight

PROJ = ["wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"]
NORMS = ["attn_norm", "attn_sub_norm", "ffn_norm", "ffn_sub_norm"]

# Named shapes of the workloads this path is measured on.
SHAPES = {
    # BitNet-b1.58-2B: hidden 2560, 30 layers, 20/5 heads, FFN 6912, vocab 128256
    "bitnet-2b": Config(128256, 2560, 30, 20, 5, 128, 6912, 4096, 500000.0, 1e-5, 1024),
    # 8B-class (Llama-3-8B shape) for tensor parallelism
    "8b": Config(128256, 4096, 32, 32, 8, 128, 14336, 4096, 500000.0, 1e-5, 1024),
    # small shapes for parity tests against the CPU oracles
    "tiny": Config(1024, 256, 2, 2, 1, 128, 512, 256, 500000.0, 1e-5, 256),
    "small": Config(4096, 512, 3, 4, 2, 128, 1024, 512, 500000.0, 1e-5, 512),
}


def proj_shape(cfg: Config, name: str):
    """(N out rows, K in) of a projection, stored [N][K] (GGUF ne = [K, N])."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    Hq = cfg.num_heads * cfg.head_dim
    Hk = cfg.num_kv_heads * cfg.head_dim
    return {"wq": (Hq, H), "wk": (Hk, H), "wv": (Hk, H), "wo": (H, Hq),
            "w_gate": (I, H), "w_up": (I, H), "w_down": (H, I)}[name]


def norm_len(cfg: Config, name: str) -> int:
    H, I = cfg.hidden_size, cfg.intermediate_size
    Hq = cfg.num_heads * cfg.head_dim
    return {"attn_norm": H, "attn_sub_norm": Hq, "ffn_norm": H, "ffn_sub_norm": I}[name]


def pack_i2s_torch(codes):
    """Ternary codes {0,1,2} [N][K] (uint8, K % 128 == 0) -> I2_S bytes, the
    layout of tensor.cpp:984-1000: per 128-weight block, byte gp holds elements
    gp, gp+32, gp+64, gp+96 in bits [7:6], [5:4], [3:2], [1:0]."""
    N, K = codes.shape
    c = codes.reshape(N, K // 128, 4, 32)
    packed = (c[:, :, 0] << 6) | (c[:, :, 1] << 4) | (c[:, :, 2] << 2) | c[:, :, 3]
    return packed.reshape(-1).contiguous()


@dataclass
class I2STensor:
    i2s: object          # torch.uint8 [N*K/4] on the device
    scale: float
    N: int
    K: int


@dataclass
class SyntheticModel:
    cfg: Config
    rank: int
    alpha: float
    layers: List[Dict[str, I2STensor]]
    lora: List[Dict[str, tuple]]          # name -> (A [r][K], B [N][r]) float32 device tensors
    norms: List[Dict[str, object]]
    tok_embd: object                      # torch.float16 [V][H]
    output_norm: object

    @staticmethod
    def generate(cfg: Config, rank: int = 16, alpha: float = 32.0, seed: int = 0, device="cuda",
                 norm_value: float = 1.0) -> "SyntheticModel":
        import torch
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        layers, lora, norms = [], [], []
        for _ in range(cfg.num_layers):
            lt, ll, ln = {}, {}, {}
            for name in PROJ:
                N, K = proj_shape(cfg, name)
                lat = torch.randn(N, K, generator=g, device=device, dtype=torch.float32)
                scale = lat.abs().mean()
                codes = (torch.round(torch.clamp(lat / scale, -1.0, 1.0)) + 1).to(torch.uint8)
                lt[name] = I2STensor(pack_i2s_torch(codes), float(scale.item()), N, K)
                del lat, codes
                if rank > 0:
                    A = torch.randn(rank, K, generator=g, device=device) * (1.0 / np.sqrt(K))
                    B = torch.randn(N, rank, generator=g, device=device) * 1e-3
                    ll[name] = (A.contiguous(), B.contiguous())
            for name in NORMS:
                ln[name] = torch.full((norm_len(cfg, name),), norm_value, device=device,
                                      dtype=torch.float32)
            layers.append(lt)
            lora.append(ll)
            norms.append(ln)
        tok = (torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g, device=device) * 0.02).half()
        onorm = torch.full((cfg.hidden_size,), norm_value, device=device, dtype=torch.float32)
        return SyntheticModel(cfg, rank, alpha, layers, lora, norms, tok, onorm)

    def merge_descs(self, outputs: List[Dict[str, object]], row_scales=None,
                    layers: Optional[List[int]] = None) -> List[MergeDesc]:
        """One tvb_merge_desc per projection of the selected layers."""
        descs = []
        for li in (range(self.cfg.num_layers) if layers is None else layers):
            for name in PROJ:
                t = self.layers[li][name]
                A, B = self.lora[li].get(name, (None, None))
                rs = None if row_scales is None else row_scales[li][name]
                descs.append(MergeDesc(t.i2s.data_ptr(), t.scale, t.K, t.N,
                                       None if A is None else A.data_ptr(),
                                       None if B is None else B.data_ptr(),
                                       0 if A is None else A.shape[0], self.alpha,
                                       outputs[li][name].data_ptr(),
                                       None if rs is None else rs.data_ptr()))
        return descs


class Model:
    """Merged, device-resident model + fused step driver."""

    def __init__(self, backend: CUDABackend, cfg: Config):
        self.backend = backend
        self.cfg = cfg
        self.weights: List[Dict[str, object]] = []
        self.row_scales: List[Dict[str, object]] = []
        self.tensor_scales: List[Dict[str, float]] = []
        self.layer_dtype: List[int] = []
        self.norms = None
        self.tok_embd = None
        self.output_norm = None

    @staticmethod
    def load(synth: SyntheticModel, int8_layers=(), per_row: bool = True,
             backend: Optional[CUDABackend] = None, exact_merge: bool = False) -> "Model":
        """Merge every projection on the device (F16, or INT8 for the layers in
        ``int8_layers``) and register the result with the fused step.  F16 layers
        take the tensor-core merge (within one F16 unit in the last place of the
        reference's apply_lora, usually identical; INT8 layers quantise those
        F16 rows per row) unless ``exact_merge``, which takes the bit-exact
        CUDA-core merge for both."""
        import torch
        cfg = synth.cfg
        be = backend or CUDABackend()
        be.init_gpu_activations(cfg)
        m = Model(be, cfg)
        int8_layers = set(int8_layers)
        f16_out, i8_out, i8_scales = [], [], []
        for li in range(cfg.num_layers):
            fo, io, so = {}, {}, {}
            for name in PROJ:
                N, K = proj_shape(cfg, name)
                if li in int8_layers and per_row:
                    io[name] = torch.empty(N, K, dtype=torch.int8, device="cuda")
                    so[name] = torch.empty(N, dtype=torch.float32, device="cuda")
                else:
                    fo[name] = torch.empty(N, K, dtype=torch.float16, device="cuda")
            f16_out.append(fo)
            i8_out.append(io)
            i8_scales.append(so)
        f16_layers = [li for li in range(cfg.num_layers) if f16_out[li]]
        if f16_layers:
            merge = be.merge_batch if exact_merge else be.merge_batch_tc
            merge(synth.merge_descs(f16_out, layers=f16_layers), TVB_F16)
        if int8_layers and per_row:
            merge = be.merge_batch if exact_merge else be.merge_batch_tc
            merge(synth.merge_descs(i8_out, i8_scales, layers=sorted(int8_layers)), TVB_I8_ROW)
        m.row_scales = [{} for _ in range(cfg.num_layers)]
        m.tensor_scales = [{} for _ in range(cfg.num_layers)]
        for li in range(cfg.num_layers):
            if li in int8_layers and not per_row:
                # reference semantics: per-tensor INT8 of the F16 merge (model.cpp:374-410)
                q, ts = {}, {}
                for name in PROJ:
                    N, K = proj_shape(cfg, name)
                    q[name] = torch.empty(N, K, dtype=torch.int8, device="cuda")
                    sc = torch.empty(1, dtype=torch.float32, device="cuda")
                    be.quantize_int8(f16_out[li][name], N, K, False, q[name], sc)
                    be.sync_d()
                    ts[name] = float(sc.item())
                m.weights.append(q)
                m.tensor_scales[li] = ts
                m.layer_dtype.append(TVB_I8_TENSOR)
            elif li in int8_layers:
                m.weights.append(i8_out[li])
                m.row_scales[li] = i8_scales[li]
                m.layer_dtype.append(TVB_I8_ROW)
            else:
                m.weights.append(f16_out[li])
                m.layer_dtype.append(TVB_F16)
        be.sync_d()
        m.norms = synth.norms
        m.tok_embd = synth.tok_embd
        m.output_norm = synth.output_norm
        m._register()
        return m

    def device_weight(self, li: int, name: str) -> DeviceWeight:
        dt = self.layer_dtype[li]
        w = self.weights[li][name]
        if dt == TVB_I8_ROW:
            return DeviceWeight(w.data_ptr(), dt, self.row_scales[li][name].data_ptr())
        if dt == TVB_I8_TENSOR:
            return DeviceWeight(w.data_ptr(), dt, None, self.tensor_scales[li][name])
        return DeviceWeight(w.data_ptr(), TVB_F16)

    def _register(self):
        for li in range(self.cfg.num_layers):
            n = self.norms[li]
            self.backend.set_layer(
                li, attn_norm=n["attn_norm"], attn_sub_norm=n["attn_sub_norm"],
                ffn_norm=n["ffn_norm"], ffn_sub_norm=n["ffn_sub_norm"],
                **{name: self.device_weight(li, name) for name in PROJ})
        self.backend.set_output(self.tok_embd, self.output_norm)

    def save_cache(self, path: str, key=None) -> None:
        """ModelCache::save of the merged device weights (no host copy of the
        model; .tvcache format of cache.cpp:263-375)."""
        from . import cache
        cache.write(path, key if key is not None else cache.make_key(), cache.model_entries(self))

    # ---- reference Model API on the fused path ----------------------------------
    def forward_gpu(self, token: int, pos: int):
        return self.backend.decode_step(token, pos)

    def forward_prefill(self, tokens):
        return self.backend.prefill(tokens)

    def generate_greedy(self, prompt, n_new: int) -> np.ndarray:
        """Prefill the prompt, then greedy-decode n_new tokens on the device.
        Returns prompt + generated ids."""
        prompt = np.asarray(prompt, np.int32)
        self.backend.clear_kv_d()
        _, first = self.backend.prefill(prompt, want_logits=False)
        gen = [first]
        if n_new > 1:
            rest = self.backend.generate_greedy(first, len(prompt), n_new - 1)
            gen.extend(int(t) for t in rest)
        return np.concatenate([prompt, np.asarray(gen[:n_new], np.int32)])

    def host_weights(self) -> dict:
        """Merged weights in numpy, in the layout the reference Model holds
        (F16 bits [out][in], norms F32) -- the input to the CPU oracles."""
        out = {"tok_embd": self.tok_embd.cpu().numpy().view(np.uint16),
               "output_norm": self.output_norm.cpu().numpy(), "layers": []}
        for li in range(self.cfg.num_layers):
            lw = {}
            for name in PROJ:
                w = self.weights[li][name]
                lw[name] = w.cpu().numpy().view(np.uint16) if self.layer_dtype[li] == TVB_F16 \
                    else w.cpu().numpy()
            for name in NORMS:
                lw[name] = self.norms[li][name].cpu().numpy()
            out["layers"].append(lw)
        return out
