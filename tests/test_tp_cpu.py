"""Host-side logic of the tensor-parallel decode path, on CPU with two gloo ranks:
the shard plan (ternative_b200.tp) applied to a numpy layer, with the
partial rows and sub-norm sums of squares all-reduced across real ranks, must
reproduce the unsharded layer; the vocabulary-sliced argmax must pick the
global argmax; the merge descriptors must address the right code and LoRA
bytes.  The device kernels that do the same over NVLink are checked against
the single-GPU path in test_tp_gpu.py."""
import os
import socket

import numpy as np
import pytest

from ternative_b200.backend import Config
from ternative_b200 import tp

CFG = Config(vocab_size=1024, hidden_size=256, num_layers=1, num_heads=4, num_kv_heads=2,
             head_dim=128, intermediate_size=512, max_seq_len=64)
EPS = 1e-5


def _layer(seed=0):
    rng = np.random.default_rng(seed)
    w = {n: rng.standard_normal(tp.proj_full(CFG, n)).astype(np.float64) * 0.05 for n in tp.PROJ}
    w["attn_sub_norm"] = 1.0 + 0.1 * rng.standard_normal(CFG.num_heads * CFG.head_dim)
    w["ffn_sub_norm"] = 1.0 + 0.1 * rng.standard_normal(CFG.intermediate_size)
    w["ffn_norm"] = 1.0 + 0.1 * rng.standard_normal(CFG.hidden_size)
    w["lm"] = rng.standard_normal((CFG.vocab_size, CFG.hidden_size))
    x = rng.standard_normal(CFG.hidden_size)
    attn = rng.standard_normal(CFG.num_heads * CFG.head_dim)   # per-head outputs (local per rank)
    return w, x, attn


def rms(v, wt):
    return v / np.sqrt(np.mean(v * v) + EPS) * wt


def reference(w, x, attn):
    x1 = x + w["wo"] @ rms(attn, w["attn_sub_norm"])
    xn = rms(x1, w["ffn_norm"])
    h = np.maximum(w["w_gate"] @ xn, 0) ** 2 * (w["w_up"] @ xn)
    x2 = x1 + w["w_down"] @ rms(h, w["ffn_sub_norm"])
    return x1, h, x2, int(np.argmax(w["lm"] @ x2))


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        w, x, attn = _layer()
        # o_proj: columns of wo, this rank's heads of the attention output
        _, _, c0, nc = tp.proj_slice(CFG, "wo", world, rank)
        s0, ns = tp.norm_slice(CFG, "attn_sub_norm", world, rank)
        assert (s0, ns) == (c0, nc)
        a = attn[c0:c0 + nc]
        part = np.concatenate([w["wo"][:, c0:c0 + nc] @ (a * w["attn_sub_norm"][s0:s0 + ns]),
                               [np.sum(a * a)]])
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        tot = t.numpy()
        x1 = x + tot[:-1] / np.sqrt(tot[-1] / (CFG.num_heads * CFG.head_dim) + EPS)
        # gate/up: this rank's intermediate rows from the replicated residual
        r0, nr, _, _ = tp.proj_slice(CFG, "w_gate", world, rank)
        xn = rms(x1, w["ffn_norm"])
        h = np.maximum(w["w_gate"][r0:r0 + nr] @ xn, 0) ** 2 * (w["w_up"][r0:r0 + nr] @ xn)
        # down: columns of w_down = this rank's intermediate rows
        _, _, d0, nd = tp.proj_slice(CFG, "w_down", world, rank)
        assert (d0, nd) == (r0, nr)
        f0, nf = tp.norm_slice(CFG, "ffn_sub_norm", world, rank)
        part = np.concatenate([w["w_down"][:, d0:d0 + nd] @ (h * w["ffn_sub_norm"][f0:f0 + nf]),
                               [np.sum(h * h)]])
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        tot = t.numpy()
        x2 = x1 + tot[:-1] / np.sqrt(tot[-1] / CFG.intermediate_size + EPS)
        # vocabulary-parallel lm_head: local argmax, then the best over ranks
        v0, nv = tp.vocab_slice(CFG, world, rank)
        lg = w["lm"][v0:v0 + nv] @ x2
        best = [None] * world
        dist.all_gather_object(best, (float(lg.max()), v0 + int(lg.argmax())))
        token = max(best, key=lambda b: (b[0], -b[1]))[1]
        hs = [None] * world
        dist.all_gather_object(hs, (r0, h))
        q.put((rank, x1, x2, token, hs))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_tp_plan_matches_unsharded_layer(world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    w, x, attn = _layer()
    x1_ref, h_ref, x2_ref, tok_ref = reference(w, x, attn)
    for rank, x1, x2, token, hs in res:
        np.testing.assert_allclose(x1, x1_ref, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(x2, x2_ref, rtol=1e-10, atol=1e-10)
        assert token == tok_ref
        h = np.zeros_like(h_ref)
        for r0, part in hs:
            h[r0:r0 + len(part)] = part
        np.testing.assert_allclose(h, h_ref, rtol=1e-12, atol=1e-12)


def test_shard_config_and_checks():
    from ternative_b200.model import SHAPES
    c8 = tp.shard_config(SHAPES["8b"], 8)
    assert (c8.num_heads, c8.num_kv_heads, c8.intermediate_size) == (4, 1, 1792)
    assert c8.hidden_size == 4096 and c8.vocab_size == 128256
    with pytest.raises(ValueError):
        tp.shard_config(SHAPES["bitnet-2b"], 2)   # 5 KV heads do not split
    # every column of every projection belongs to exactly one rank
    for name in tp.PROJ:
        N, K = tp.proj_full(SHAPES["8b"], name)
        seen = np.zeros((N, K), np.int8) if N * K < 1 << 26 else None
        cover = 0
        for r in range(4):
            r0, rows, k0, cols = tp.proj_slice(SHAPES["8b"], name, 4, r)
            cover += rows * cols
            assert 0 <= r0 and r0 + rows <= N and 0 <= k0 and k0 + cols <= K
            assert k0 % 128 == 0 and cols % 128 == 0
        assert cover == N * K


def test_merge_descs_address_the_shards():
    class T:
        def __init__(self, base, N, K):
            self.N, self.K, self.scale = N, K, 0.5
            self._b = base

        class _P:
            def __init__(self, v):
                self.v = v

            def data_ptr(self):
                return self.v

        @property
        def i2s(self):
            return T._P(self._b)

    class L:
        def __init__(self, base, shape):
            self.shape = shape
            self._b = base

        def data_ptr(self):
            return self._b

    class Synth:
        cfg = CFG
        alpha = 32.0

    s = Synth()
    s.layers, s.lora = [{}], [{}]
    base = 1 << 20
    for i, n in enumerate(tp.PROJ):
        N, K = tp.proj_full(CFG, n)
        s.layers[0][n] = T(base * (i + 1), N, K)
        s.lora[0][n] = (L(base * (i + 10), (16, K)), L(base * (i + 20), (N, 16)))
    outs = [{n: L(base * (i + 30), None) for i, n in enumerate(tp.PROJ)}]
    d = {n: desc for n, desc in zip(tp.PROJ, tp.merge_descs(s, 2, 1, outs))}
    N, K = tp.proj_full(CFG, "wq")
    assert d["wq"].i2s == base * 1 + (N // 2) * K // 4 and d["wq"].N == N // 2 and d["wq"].K == K
    assert d["wq"].B == base * 20 + (N // 2) * 16 * 4 and d["wq"].k0 == 0 and d["wq"].ld == 0
    N, K = tp.proj_full(CFG, "w_down")
    assert d["w_down"].i2s == base * 7 and d["w_down"].N == N and d["w_down"].K == K // 2
    assert d["w_down"].k0 == K // 2 and d["w_down"].ld == K and d["w_down"].B == base * 26
