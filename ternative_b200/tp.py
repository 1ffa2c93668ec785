"""Tensor parallelism of the decode path: one process and one libtvb200 context
per GPU, the plan of which rows and columns each rank owns, and the loader that
merges only this rank's shards.

Split (the Megatron-style plan the path calls for): q/k/v by heads and
gate/up by intermediate rows (column-parallel: each rank computes its own
output rows from the replicated residual), o_proj and down by input columns
(row-parallel: each rank produces partial sums of every output row, exchanged
over NVLink inside the decode-step kernel, together with each rank's partial
sum of squares of the sub-norm input), the tied lm_head by vocabulary rows.
The embedding table stays whole on every rank (the token gather reads one row).
The reference runs on one device; this layout is new and its pieces are pinned
by tests against the single-GPU path.
"""
from __future__ import annotations

import dataclasses
from typing import Callable, List, Sequence

from ._lib import TVB_F16, MergeDesc
from .backend import Config, CUDABackend, DeviceWeight

COLUMN_PARALLEL = ("wq", "wk", "wv", "w_gate", "w_up")   # split by output rows
ROW_PARALLEL = ("wo", "w_down")                          # split by input columns
PROJ = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")


def check_world(cfg: Config, world: int) -> None:
    """Raise ValueError when `cfg` cannot be split over `world` ranks."""
    if world < 1 or world > 8:
        raise ValueError(f"tensor parallelism over {world} ranks (1..8)")
    if cfg.num_heads % world or cfg.num_kv_heads % world:
        raise ValueError(f"{cfg.num_heads} query / {cfg.num_kv_heads} KV heads over {world} ranks")
    if (cfg.intermediate_size // world) % 128 or cfg.intermediate_size % world:
        raise ValueError(f"intermediate {cfg.intermediate_size} over {world} ranks: shards must be "
                         "multiples of 128 (I2_S blocks)")
    if (cfg.num_heads // world * cfg.head_dim) % 128:
        raise ValueError("query shard not a multiple of 128 columns")
    if cfg.vocab_size % world:
        raise ValueError(f"vocabulary {cfg.vocab_size} over {world} ranks")


def shard_config(cfg: Config, world: int) -> Config:
    """The dimensions one rank's context is created with."""
    check_world(cfg, world)
    return dataclasses.replace(cfg, num_heads=cfg.num_heads // world,
                               num_kv_heads=cfg.num_kv_heads // world,
                               intermediate_size=cfg.intermediate_size // world)


def proj_full(cfg: Config, name: str):
    """(N rows, K columns) of the whole projection."""
    H, I = cfg.hidden_size, cfg.intermediate_size
    Hq, Hk = cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
    return {"wq": (Hq, H), "wk": (Hk, H), "wv": (Hk, H), "wo": (H, Hq),
            "w_gate": (I, H), "w_up": (I, H), "w_down": (H, I)}[name]


def proj_slice(cfg: Config, name: str, world: int, rank: int):
    """(row0, rows, col0, cols) of this rank's shard, in whole-tensor coordinates."""
    N, K = proj_full(cfg, name)
    if name in COLUMN_PARALLEL:
        n = N // world
        return rank * n, n, 0, K
    k = K // world
    return 0, N, rank * k, k


def norm_slice(cfg: Config, name: str, world: int, rank: int):
    """(start, length) of this rank's part of a norm weight: the sub-norms act on
    sharded vectors, the input norms on the replicated residual."""
    if name == "attn_sub_norm":
        n = cfg.num_heads * cfg.head_dim // world
        return rank * n, n
    if name == "ffn_sub_norm":
        n = cfg.intermediate_size // world
        return rank * n, n
    return 0, cfg.hidden_size


def vocab_slice(cfg: Config, world: int, rank: int):
    n = cfg.vocab_size // world
    return rank * n, n


def merge_descs(synth, world: int, rank: int, outputs: Sequence[dict]) -> List[MergeDesc]:
    """tvb_merge_desc entries merging only this rank's shards (the load-time merge
    sharded by tensor slice): row slices offset the codes and LoRA B, column
    slices select [k0, k0 + cols) of the whole rows."""
    descs = []
    for li in range(synth.cfg.num_layers):
        for name in PROJ:
            t = synth.layers[li][name]
            A, B = synth.lora[li].get(name, (None, None))
            r = 0 if A is None else A.shape[0]
            r0, rows, k0, cols = proj_slice(synth.cfg, name, world, rank)
            i2s = t.i2s.data_ptr() + r0 * t.K // 4
            bptr = None if B is None else B.data_ptr() + r0 * r * 4
            descs.append(MergeDesc(i2s, t.scale, cols, rows, None if A is None else A.data_ptr(),
                                   bptr, r, synth.alpha, outputs[li][name].data_ptr(), None,
                                   k0, t.K if name in ROW_PARALLEL else 0))
    return descs


class TPModel:
    """One rank's shard of a merged model, registered with the fused step and
    wired to its peers.  `all_gather(obj) -> list` exchanges small host objects
    between the ranks (e.g. torch.distributed.all_gather_object)."""

    def __init__(self, synth, world: int, rank: int, all_gather: Callable[[object], list],
                 backend: CUDABackend = None):
        import torch
        self.world, self.rank = world, rank
        self.cfg = synth.cfg
        self.local = shard_config(synth.cfg, world)
        be = backend or CUDABackend()
        be.init_gpu_activations(self.local)
        self.backend = be
        outs = []
        for li in range(synth.cfg.num_layers):
            o = {}
            for name in PROJ:
                _, rows, _, cols = proj_slice(synth.cfg, name, world, rank)
                o[name] = torch.empty(rows, cols, dtype=torch.float16, device="cuda")
            outs.append(o)
        be.merge_batch(merge_descs(synth, world, rank, outs), TVB_F16)
        be.sync_d()
        self.weights = outs
        self.norms = []
        for li in range(synth.cfg.num_layers):
            n = {}
            for name, w in synth.norms[li].items():
                s0, ln = norm_slice(synth.cfg, name, world, rank)
                n[name] = w[s0:s0 + ln].contiguous()
            self.norms.append(n)
        for li in range(synth.cfg.num_layers):
            n = self.norms[li]
            be.set_layer(li, attn_norm=n["attn_norm"], attn_sub_norm=n["attn_sub_norm"],
                         ffn_norm=n["ffn_norm"], ffn_sub_norm=n["ffn_sub_norm"],
                         **{name: DeviceWeight(outs[li][name].data_ptr(), TVB_F16) for name in PROJ})
        self.tok_embd, self.output_norm = synth.tok_embd, synth.output_norm
        be.set_output(self.tok_embd, self.output_norm)
        # exchange buffers: export ours, import everyone else's
        own = be.tp_init(rank, world)
        handles = all_gather(CUDABackend.ipc_export(own))
        self._imported = []
        bufs = []
        for r, h in enumerate(handles):
            if r == rank:
                bufs.append(own)
            else:
                p = CUDABackend.ipc_import(h)
                self._imported.append(p)
                bufs.append(p)
        be.tp_set_peers(bufs)

    def recover(self, barrier: Callable[[], None]) -> None:
        """Re-align the ranks after a step failed (TVB_ERR_TIMEOUT on some
        rank): every rank zeroes its exchange buffer and counters, then the
        ranks meet at `barrier` before any of them runs another step."""
        self.backend.tp_recover()
        barrier()

    def close(self):
        self.backend.close()
        for p in self._imported:
            CUDABackend.ipc_close(p)
        self._imported = []
