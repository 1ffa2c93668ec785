"""Tensor-parallel prefill and decode on 2 (and 4) GPUs against the single-GPU path.

Each rank is a process on its own GPU (spawned), holds its shard of a small
model merged from the same synthetic I2_S + LoRA weights, and runs the batched
prefill (partial rows exchanged through the ranks' IPC-mapped regions) and
greedy decode steps whose row-parallel exchanges go over NVLink inside the
decode-step kernel.  Checked: every rank produces the same tokens; the ranks'
vocabulary slices of the logits, put together, match the single-GPU decode
steps over the same tokens within 2e-3 relative; the tokens are the argmax of
those single-GPU logits.  Skipped on machines with fewer GPUs than ranks."""
import dataclasses
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _child(rank, world, port, cfg, prompt, n_new, q):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        from ternative_b200.model import Model, SyntheticModel
        from ternative_b200.tp import TPModel

        def all_gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=4)
        m = TPModel(synth, world, rank, all_gather)
        be = m.backend
        be.clear_kv_d()
        last, am = be.prefill(prompt)
        toks = [int(t) for t in prompt] + [am]
        logits = [last]
        for _ in range(n_new - 1):
            lg, am = be.decode_step(toks[-1], len(toks) - 1)
            logits.append(lg)
            toks.append(am)
        parts = all_gather(np.stack(logits))
        res = {"rank": rank, "toks": toks}
        if rank == 0:
            res["full"] = np.concatenate(parts, axis=1)
            ref = Model.load(synth)
            ref.backend.clear_kv_d()
            rl, _ = ref.backend.prefill(np.asarray(toks[:len(prompt)], np.int32))
            refs = [rl]
            for t in range(len(prompt), len(toks) - 1):
                lg, _ = ref.backend.decode_step(toks[t], t)
                refs.append(lg)
            res["ref"] = np.stack(refs)
            ref.backend.close()
        dist.barrier()
        m.close()
        q.put(res)
    except Exception as e:   # report, do not hang the parent
        q.put({"rank": rank, "error": repr(e)})
        raise
    finally:
        dist.destroy_process_group()


def _child_batch(rank, world, port, cfg, prompts, steps, q):
    """Batched decode under tensor parallelism: every prompt prefilled into
    its KV slot, then `steps` batched greedy steps; rank 0 checks each
    sequence against the single-GPU single-sequence path (teacher-forced)."""
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        from ternative_b200.model import Model, SyntheticModel
        from ternative_b200.tp import TPModel

        def all_gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=4)
        m = TPModel(synth, world, rank, all_gather)
        be = m.backend
        be.clear_kv_d()
        toks = []
        for b, p in enumerate(prompts):
            _, am = be.prefill_slot(b, p, want_logits=False)
            toks.append([int(t) for t in p] + [am])
        logits = []
        for _ in range(steps):
            cur = np.array([t[-1] for t in toks], np.int32)
            pos = np.array([len(t) - 1 for t in toks], np.int32)
            lg, nxt = be.decode_batch(cur, pos)
            for b in range(len(prompts)):
                toks[b].append(int(nxt[b]))
            logits.append(lg)
        parts = all_gather(np.stack(logits))           # [steps][B][V / world] per rank
        res = {"rank": rank, "toks": toks}
        if rank == 0:
            full = np.concatenate(parts, axis=2)         # [steps][B][V]
            ref = Model.load(SyntheticModel.generate(dataclasses.replace(cfg, max_batch=1), rank=16,
                                                     alpha=32.0, seed=4))
            errs = []
            for b, p in enumerate(prompts):
                ref.backend.clear_kv_d()
                ref.backend.prefill(p, want_logits=False)
                for i in range(steps):
                    lg, _ = ref.backend.decode_step(toks[b][len(p) + i], len(p) + i)
                    errs.append(float(np.abs(full[i][b].astype(np.float64) - lg).max() / np.abs(lg).max()))
                    assert int(np.argmax(full[i][b])) == toks[b][len(p) + i + 1]
            res["errs"] = errs
            ref.backend.close()
        dist.barrier()
        m.close()
        q.put(res)
    except Exception as e:   # report, do not hang the parent
        q.put({"rank": rank, "error": repr(e)})
        raise
    finally:
        dist.destroy_process_group()


def _run(world, cfg, prompt, n_new, child=None, args=None):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=child or _child, args=(r, world, port, cfg) + (args or (prompt, n_new)) + (q,))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=600)
        res[r["rank"]] = r
    for p in procs:
        p.join(timeout=120)
    for r in res.values():
        assert "error" not in r, r["error"]
    for p in procs:
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("world,prompt_len,max_prefill", [(2, 9, 256), (4, 9, 256), (2, 150, 64)])
def test_tp_decode_matches_single_gpu(world, prompt_len, max_prefill):
    """The batched tensor-parallel prefill (one chunk, or three chunks of at
    most 64 rows) followed by tensor-parallel decode steps."""
    from ternative_b200.backend import Config
    # 8 query / 4 KV heads, FFN 2048: shards of whole heads and 128-column blocks at 2 and 4 ranks
    cfg = Config(vocab_size=4096, hidden_size=512, num_layers=3, num_heads=8, num_kv_heads=4,
                 head_dim=128, intermediate_size=2048, max_seq_len=256, max_prefill=max_prefill)
    prompt = np.random.default_rng(world + prompt_len).integers(0, cfg.vocab_size,
                                                                prompt_len).astype(np.int32)
    res = _run(world, cfg, prompt, 12)
    toks = res[0]["toks"]
    for r in range(world):
        assert res[r]["toks"] == toks
    full, ref = res[0]["full"], res[0]["ref"]
    assert full.shape == ref.shape
    for i in range(len(ref)):
        err = float(np.abs(full[i].astype(np.float64) - ref[i]).max() / np.abs(ref[i]).max())
        assert err < RTOL, (i, err)
        assert int(np.argmax(ref[i])) == toks[len(prompt) + i]


def test_tp_batch_decode_matches_single_gpu():
    """Three sequences decoded together on 2 ranks (row-parallel partials of all
    rows exchanged per projection, per-row argmax keys exchanged) against the
    single-GPU single-sequence path."""
    from ternative_b200.backend import Config
    cfg = Config(vocab_size=4096, hidden_size=512, num_layers=3, num_heads=8, num_kv_heads=4,
                 head_dim=128, intermediate_size=2048, max_seq_len=256, max_prefill=256, max_batch=3)
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, cfg.vocab_size, n).astype(np.int32) for n in (6, 19, 44)]
    res = _run(2, cfg, None, None, child=_child_batch, args=(prompts, 5))
    for r in range(2):
        assert res[r]["toks"] == res[0]["toks"]
    assert max(res[0]["errs"]) < RTOL, res[0]["errs"]
