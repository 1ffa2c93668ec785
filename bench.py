"""Benchmark of the quantized-weight hot path on B200.

Headline (one JSON line on rank 0): batch-1 greedy decode tok/s of the
BitNet-b1.58-2B-shaped ternary+LoRA model (I2_S weights, rank-16 LoRA alpha 32,
merged on the device to F16), after a 32-token prompt, seed 0.  A "step" is
one decoded token: all 30 layers + lm_head + argmax on the device.

  value  -- K chained decode steps timed with CUDA events on the context
            stream (weights, KV cache and token ids resident in HBM)
  e2e    -- the same K steps through the reference-facing C ABI
            (tvb_decode_step: host token/pos in, host logits out, synchronous)
  roofline -- the dominant kernel (the streaming F16 GEMV) timed live here on
            the gate-projection shape, rotating over all 30 layers
  cpu_baseline -- the reference's own --no-gpu decode (oracle/_ref, built from
            the reference sources) on this host's cores, on a bounded sample

``--impl reference`` times the reference's CPU decode alone (the reference
has no B200 path; its CPU implementation is the arm the ratio is taken on).

Multi-GPU: the 2B shape has 5 KV heads, so it does not shard by heads; N GPUs
run N independent replicas (weak scaling), value = total tok/s, timed as the
max over ranks.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
# The CPU legs (the reference's OpenMP loops) use every host core: a launcher
# such as torchrun sets OMP_NUM_THREADS=1, which would time them on one core.
HOST_CORES = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
os.environ["OMP_NUM_THREADS"] = str(HOST_CORES)

import numpy as np  # noqa: E402

L2_BYTES = 126 * 1024 * 1024


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 tensor throughput (TFLOP/s) a burst of kernels is compared with."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


class ClockSampler:
    """Samples SM clock and clock-event reasons via NVML (read-only) while running."""

    def __init__(self, cuda_index: int = 0, period: float = 0.02):
        self.period = period
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.h = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(cuda_index).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode() if isinstance(uuid, str) else uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.nv = pynvml
        except Exception as e:   # NVML unavailable: report what we can
            self.err = repr(e)

    def _run(self):
        nv = self.nv
        names = {
            getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8): "hw_slowdown",
            getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40): "hw_thermal_slowdown",
            getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20): "sw_thermal_slowdown",
            getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4): "sw_power_cap",
            getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80): "hw_power_brake_slowdown",
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in names.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self.h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def report(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
def profiled_traffic(kernel: str, layers: int):
    """DRAM bytes (read + write) per launch of `kernel`, from the ncu summary
    committed under profiles/ (`traffic_bytes_per_layer:` and
    `traffic_bytes_fixed:` lines, scaled to `layers`).  None when absent."""
    path = os.path.join(ROOT, "profiles", f"{kernel}.md")
    if not os.path.exists(path):
        return None
    vals = {}
    for line in open(path):
        for key in ("traffic_bytes_per_layer:", "traffic_bytes_fixed:"):
            if line.strip().startswith(key):
                vals[key] = float(line.split(":", 1)[1].strip().split()[0])
    if len(vals) != 2:
        return None
    return vals["traffic_bytes_fixed:"] + layers * vals["traffic_bytes_per_layer:"]


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reference_model_random(shape, seed=0):
    """The reference Model (oracle/_ref) on the 2B shape with random F16
    weights of merged-weight magnitude, generated on the host."""
    from oracle.oracle import PROJ_DIMS, ReferenceModel, Reference
    rng = np.random.default_rng(seed)

    def f16(n, k):
        # sign | exponent in [2^-10, 2^-3) | mantissa: F16 values of the merged weights' range
        b = rng.integers(0, 1 << 15, size=(n, k), dtype=np.uint16)
        return ((b & 0x83FF) | (((b >> 10) % 7 + 5) << 10)).astype(np.uint16)

    w = {"tok_embd": f16(shape.vocab, shape.hidden), "output_norm": np.ones(shape.hidden, np.float32),
         "layers": []}
    for _ in range(shape.layers):
        lw = {n: f16(*d) for n, d in PROJ_DIMS(shape).items()}
        for n, length in (("attn_norm", shape.hidden), ("attn_sub_norm", shape.heads * shape.head_dim),
                          ("ffn_norm", shape.hidden), ("ffn_sub_norm", shape.inter)):
            lw[n] = np.ones(length, np.float32)
        w["layers"].append(lw)
    return ReferenceModel(Reference(), shape, w)


def time_reference_decode(rm, steps: int, pos0: int = 32, budget_s: float = 20.0):
    """Seconds per token of the reference's CPU decode (Model::forward with
    prefill=false, model.cpp:851-1066), on a bounded sample of `steps`."""
    t1 = rm.time_decode(1, pos0, 1)   # warm-up + estimate
    n = max(1, min(steps, int(budget_s / max(t1, 1e-3))))
    t = rm.time_decode(1, pos0 + 1, n)
    return t / n, n


def run_reference(args, world, rank):
    if rank != 0:
        return
    from oracle.oracle import ModelShape
    from ternative_b200.model import SHAPES
    cfg = SHAPES[args.config]
    shape = ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                       cfg.num_kv_heads, cfg.intermediate_size, 512)
    rm = reference_model_random(shape)
    rm.ref.L.tvref_set_threads(HOST_CORES)
    threads = rm.ref.L.tvref_omp_threads()
    for _ in range(max(0, min(args.warmup, 2))):
        rm.time_decode(1, 32, 1)
    sec, n = time_reference_decode(rm, args.steps, pos0=40, budget_s=args.cpu_seconds * 3)
    tps = 1.0 / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16-weights/f32-compute",
        "data": "synthetic", "config": config_block(args, cfg),
        "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": "reference",
                         "sample": f"{n} decode tokens at positions 41..{40 + n} (Model::forward, "
                                   f"prefill=false) of the 2B shape, random F16 weights; the GPU arm "
                                   f"times 128 steps from position 40 (KV reads differ by < 1% of "
                                   f"the bytes per token)"},
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    rm.close()
    print(json.dumps(line), flush=True)


METRIC = "batch-1 decode tok/s (BitNet-2B ternary+LoRA, F16-merged)"


def reference_cpu_baselines(rm, hw, cfg, synth, cores, budget_s):
    """The reference's --no-gpu code beside the other measured rows, on this
    host (oracle/_ref built from the reference sources):
      prefill -- Model::forward_prefill of a 128-token prompt (OpenMP);
      gemv    -- tensor_matmul with one activation row on each sweep shape (OpenMP);
      merge   -- apply_lora (I2_S dequant + rank-64 matmul_lora + F16 cast,
                 single-threaded as in the reference) of one 2560x2560 tensor,
                 scaled to the 210 tensors of the 2B model by weight count."""
    import torch
    from ternative_b200.model import PROJ, proj_shape
    L = rm.ref.L
    out = {}
    toks = np.random.default_rng(5).integers(0, cfg.vocab_size, 128).astype(np.int32)
    t0 = time.perf_counter()
    rm.forward_prefill(toks)
    sec = time.perf_counter() - t0
    out["prefill"] = {"tok_s": 128 / sec, "ms": sec * 1e3, "cores": cores, "kind": "reference",
                      "sample": "Model::forward_prefill of a 128-token prompt (logits of every row), same merged model"}
    gemv = {}
    x = np.random.default_rng(6).standard_normal(cfg.intermediate_size).astype(np.float32)
    for name, w in [("wk", hw["layers"][0]["wk"]), ("wq", hw["layers"][0]["wq"]), ("w_gate", hw["layers"][0]["w_gate"]),
                    ("w_down", hw["layers"][0]["w_down"]), ("lm_head", hw["tok_embd"])]:
        N, K = w.shape
        y = np.empty(N, np.float32)
        xk = np.ascontiguousarray(x[:K]) if K <= x.size else np.random.default_rng(7).standard_normal(K).astype(np.float32)
        w = np.ascontiguousarray(w)
        L.tvref_matmul_f16(xk, 1, K, w, N, y)   # warm
        reps = 0
        t0 = time.perf_counter()
        while reps < 3 or (time.perf_counter() - t0 < 0.5 and reps < 50):
            L.tvref_matmul_f16(xk, 1, K, w, N, y)
            reps += 1
        us = (time.perf_counter() - t0) / reps * 1e6
        gemv[f"{N}x{K}_f16"] = {"us": us, "GB/s": (2 * N * K + 4 * K + 4 * N) / (us * 1e-6) / 1e9}
    out["gemv"] = {"shapes": gemv, "cores": cores, "kind": "reference",
                   "sample": "tensor_matmul (tensor.cpp:375-486, one activation row) on layer 0's merged weights "
                             "and the tied lm_head, host memory"}
    # merge: one q-shaped tensor at rank 64 (alpha 128), the merge microbench's configuration
    t = synth.layers[0]["wq"]
    codes = t.i2s.cpu().numpy()
    Kq, Nq = t.K, t.N
    g = torch.Generator(device="cpu").manual_seed(64)
    A = (torch.randn(64, Kq, generator=g) / np.sqrt(Kq)).numpy()
    B = (torch.randn(Nq, 64, generator=g) * 1e-3).numpy()
    dst = np.empty(Nq * Kq, np.uint16)
    t0 = time.perf_counter()
    L.tvref_apply_lora_f16(codes, np.float32(t.scale), Kq, Nq, A, B, 64, 128.0, dst)
    sec = time.perf_counter() - t0
    n_all = sum(proj_shape(cfg, n)[0] * proj_shape(cfg, n)[1] for n in PROJ) * cfg.num_layers
    total = sec * n_all / (Nq * Kq)
    out["merge"] = {"r64_f16_seconds_all_210": total, "seconds_per_sample": sec, "cores": 1, "kind": "reference",
                    "sample": f"apply_lora of one {Nq}x{Kq} I2_S tensor, rank 64 alpha 128, scaled by weight "
                              f"count to the 210 projections ({n_all / 1e9:.2f} G weights)"}
    return out


def config_block(args, cfg):
    return {"workload": f"{args.config} batch-1 greedy decode after a {args.prompt}-token prompt "
                        "(I2_S + rank-16 LoRA alpha 32 merged to F16; hidden 2560, 30 layers, "
                        "20/5 heads, FFN 6912, vocab 128256)",
            "batch": 1, "prompt": args.prompt, "lora_rank": 16,
            "l2": "weights stream 4.83 GB per step (> 126 MB L2); no flush needed",
            "parallelism": "replicas" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "single"}


# ---------------------------------------------------------------------------
def run_tp_8b(args, world, rank):
    """Batch-1 greedy decode of the 8B-shaped model (hidden 4096, 32 layers,
    32/8 heads, FFN 14336, vocab 128256; I2_S + rank-32 LoRA alpha 64 merged to
    F16), tensor-parallel over all ranks of this job: q/k/v and gate/up split by
    rows, o_proj and down by columns, lm_head by vocabulary rows, partial rows
    exchanged over NVLink inside the decode-step kernel.  A `tp_prompt`-token
    random prompt is prefilled first; the timed region is `steps` chained decode
    steps (CUDA events on the context stream, max over ranks)."""
    import torch
    import torch.distributed as dist
    from ternative_b200.model import SHAPES, SyntheticModel
    from ternative_b200.tp import TPModel, shard_config

    cfg = SHAPES["8b"]
    # KV for the batch-1 run and the batch of 8 sequences (slots 0..7); each
    # sequence needs its prompt plus the warm-up and timed steps
    cfg = dataclasses.replace(cfg, max_seq_len=args.tp_prompt + args.warmup + args.steps + 8,
                              max_batch=TP_BATCH)

    def all_gather(obj):
        if world == 1:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    synth = SyntheticModel.generate(cfg, rank=32, alpha=64.0, seed=0)
    m = TPModel(synth, world, rank, all_gather)
    be = m.backend
    stream = torch.cuda.ExternalStream(be.stream)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, args.tp_prompt).astype(np.int32)
    # the first prefill also builds the decode graphs; the second is timed
    # (CUDA events on the context stream, max over ranks)
    be.clear_kv_d()
    be.prefill(prompt, want_logits=False)
    be.clear_kv_d()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    _, tok = be.prefill(prompt, want_logits=False)
    p1.record(stream)
    p1.synchronize()
    prefill_ms = p0.elapsed_time(p1)
    if world > 1:
        t = torch.tensor([prefill_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_ms = float(t.item())
    pos = len(prompt)
    be.decode_enqueue(tok, pos, args.warmup)
    be.sync_d()
    pos += args.warmup
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    be.decode_enqueue(0, pos, args.steps)   # the device chains its own greedy tokens
    e1.record(stream)
    e1.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # every rank must have decoded the same greedy tokens: 8 more steps, compared
    check = be.generate_greedy(0, pos + args.steps, 8)
    tokens_agree = all(np.array_equal(t, check) for t in all_gather(check))
    local = shard_config(cfg, world)
    n_w = sum(2 * a * b for a, b in [(local.num_heads * 128, 4096), (2 * local.num_kv_heads * 128, 4096),
                                     (4096, local.num_heads * 128), (2 * local.intermediate_size, 4096),
                                     (4096, local.intermediate_size)]) * cfg.num_layers
    n_w += 2 * (cfg.vocab_size // world) * cfg.hidden_size
    kv = cfg.num_layers * 2 * (pos + args.steps // 2) * local.num_kv_heads * 128 * 4
    hbm, kind = peaks()
    per_gpu = (n_w + kv) / (ms / args.steps * 1e-3) / 1e9
    res = {"workload": f"8B-shaped batch-1 greedy decode, tensor-parallel over {world} GPU(s), "
                       f"after a {args.tp_prompt}-token prompt",
           "n_gpus": world, "tokens_agree_all_ranks": bool(tokens_agree),
           "tok_s": args.steps / (ms * 1e-3), "ms_per_token": ms / args.steps,
           "per_gpu_bytes_per_token": n_w + kv, "per_gpu_GB/s": per_gpu, "frac_of_hbm": per_gpu / hbm,
           "peak_kind": kind, "prefill_ms": prefill_ms,
           "prefill_tok_s": args.tp_prompt / (prefill_ms * 1e-3),
           "prefill_path": "batched tensor cores" + (", partial rows exchanged over NVLink" if world > 1 else "")}
    res["batch8"] = tp_batch_decode(args, be, cfg, world, stream, n_w, hbm)
    if world > 1:
        dist.barrier()
    m.close()
    del synth
    torch.cuda.empty_cache()
    return res


TP_BATCH = 8


def tp_parity_check(world, rank, all_gather):
    """Tensor-parallel correctness on this job's ranks: a 3-layer model with 8
    query / 8 KV heads (hidden 1024, FFN 2048, vocabulary 4096; I2_S + rank-16
    LoRA merged to F16, norm weights 1/16 so the attention is not a hard
    maximum) prefills 11 tokens and decodes 10 greedy tokens split over the
    ranks; rank 0 compares the assembled logits with the reference's own
    Model::forward_prefill (oracle/_ref) over the same tokens."""
    from ternative_b200.backend import Config
    from ternative_b200.model import Model, SyntheticModel
    from ternative_b200.tp import TPModel
    cfg = Config(vocab_size=4096, hidden_size=1024, num_layers=3, num_heads=8, num_kv_heads=8,
                 head_dim=128, intermediate_size=2048, max_seq_len=256, max_prefill=256)
    synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=4, norm_value=1.0 / 16)
    m = TPModel(synth, world, rank, all_gather)
    be = m.backend
    prompt = np.random.default_rng(100 + world).integers(0, cfg.vocab_size, 11).astype(np.int32)
    be.clear_kv_d()
    last, am = be.prefill(prompt)
    toks, logits = [int(t) for t in prompt] + [am], [last]
    for _ in range(9):
        lg, am = be.decode_step(toks[-1], len(toks) - 1)
        logits.append(lg)
        toks.append(am)
    parts = all_gather((toks, np.stack(logits)))
    m.close()
    if rank != 0:
        return None
    agree = all(p[0] == toks for p in parts)
    full = np.concatenate([p[1] for p in parts], axis=1)
    from oracle.oracle import ModelShape, Reference, ReferenceModel
    whole = Model.load(synth, exact_merge=True)   # the ranks merge exactly
    rm = ReferenceModel(Reference(), ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                                                cfg.num_kv_heads, cfg.intermediate_size, cfg.max_seq_len,
                                                cfg.rope_theta, cfg.rms_norm_eps), whole.host_weights())
    whole.backend.close()
    ref = rm.forward_prefill(np.asarray(toks[:-1], np.int32))[len(prompt) - 1:]
    rm.close()
    errs = [float(np.abs(full[i].astype(np.float64) - ref[i]).max() / np.abs(ref[i]).max()) for i in range(len(ref))]
    follows = all(int(np.argmax(ref[i])) == toks[len(prompt) + i] for i in range(len(ref)))
    return {"ranks": world, "tokens_agree_all_ranks": bool(agree), "max_rel_err_vs_reference": max(errs),
            "tokens_follow_reference_argmax": bool(follows), "ok": bool(agree and follows and max(errs) < 2e-3),
            "note": "hidden 1024, 8/8 heads, FFN 2048, 3 layers; prefill 11 + 10 greedy steps; "
                    "reference = oracle/_ref forward_prefill, teacher-forced; tolerance 2e-3"}


def tp_batch_decode(args, be, cfg, world, stream, n_w, hbm):
    """Batch of TP_BATCH concurrent sequences on the 8B shape: each prompt
    (tp_prompt random ids) prefilled into its own KV slot, then greedy steps
    that advance all sequences by one token (tvb_decode_batch: one tensor-core
    GEMM per projection over the B rows, every weight read once per step).
    Timed: `steps` host-driven batched steps (each returns the B next tokens to
    the host), CUDA events on the context stream, max over ranks."""
    import torch
    import torch.distributed as dist
    from ternative_b200.tp import shard_config
    B = TP_BATCH
    rng = np.random.default_rng(7)
    be.clear_kv_d()
    cur = np.empty(B, np.int32)
    for b in range(B):
        prompt = rng.integers(0, cfg.vocab_size, args.tp_prompt).astype(np.int32)
        _, cur[b] = be.prefill_slot(b, prompt, want_logits=False)
    pos = np.full(B, args.tp_prompt, np.int32)
    for _ in range(args.warmup):
        _, cur = be.decode_batch(cur, pos, want_logits=False)
        pos += 1
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        _, cur = be.decode_batch(cur, pos, want_logits=False)
        pos += 1
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    local = shard_config(cfg, world)
    kv = B * cfg.num_layers * 2 * (int(pos.mean()) - args.steps // 2) * local.num_kv_heads * 128 * 4
    per_gpu = (n_w + kv) / (ms / args.steps * 1e-3) / 1e9
    return {"sequences": B, "tok_s": B * args.steps / (ms * 1e-3), "ms_per_step": ms / args.steps,
            "per_gpu_GB/s": per_gpu, "frac_of_hbm": per_gpu / hbm,
            "note": f"{B} sequences after {args.tp_prompt}-token prompts; tok_s counts every sequence's "
                    "token; bytes = this rank's weights once per step + the 8 sequences' KV rows"}


def gemv_tp_sweep(be, m, cfg, stream, world, rank, hbm):
    """The GEMV sweep's large shapes split over the job's ranks, one rank per
    GPU: column split on N (gate 6912x2560 and the 128256x2560 lm_head: each
    rank streams N/T rows, no exchange) and row split on K (down 2560x6912:
    each rank streams its K/T columns, then an NCCL all-reduce of the N
    partial outputs).  Each rank's shard is a contiguous copy per layer, so the
    rotation over the layers' copies keeps the weights coming from HBM.  Time
    per GEMV = CUDA events on the backend stream, max over ranks; GB/s = the
    whole matrix's bytes / that time (aggregate over the ranks)."""
    import torch
    import torch.distributed as dist
    from ternative_b200.model import proj_shape

    def timed(run, reps):
        for i in range(3):
            run(i)
        be.sync_d()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(reps):
            run(i)
        e1.record(stream)
        e1.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / reps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    out = {}
    cases = [("w_gate", "column"), ("w_down", "row")]
    for name, split in cases:
        N, K = proj_shape(cfg, name)
        if split == "column":
            n = N // world
            shards = [m.weights[li][name][rank * n:(rank + 1) * n].contiguous() for li in range(cfg.num_layers)]
            x = torch.randn(K, device="cuda")
            y = torch.empty(n, device="cuda")
            us = timed(lambda i: be.gemv_d2d(y, x, shards[i % len(shards)], K, n), 2 * cfg.num_layers)
        else:
            k = K // world
            shards = [m.weights[li][name][:, rank * k:(rank + 1) * k].contiguous()
                      for li in range(cfg.num_layers)]
            x = torch.randn(k, device="cuda")
            y = torch.empty(N, device="cuda")

            def run(i):
                be.gemv_d2d(y, x, shards[i % len(shards)], k, N)
                with torch.cuda.stream(stream):
                    dist.all_reduce(y)
            us = timed(run, 2 * cfg.num_layers)
        gb = (N * K * 2 + 4 * K + 4 * N) / (us * 1e-6) / 1e9
        out[f"{N}x{K}_f16_{split}"] = {"us": us, "GB/s": gb, "per_gpu_frac": gb / world / hbm}
        del shards
    N, K = cfg.vocab_size, cfg.hidden_size
    n = N // world
    head = m.tok_embd[rank * n:(rank + 1) * n]
    x = torch.randn(K, device="cuda")
    y = torch.empty(n, device="cuda")
    us = timed(lambda i: be.gemv_d2d(y, x, head, K, n), 10)
    gb = (N * K * 2 + 4 * K + 4 * N) / (us * 1e-6) / 1e9
    out[f"{N}x{K}_f16_column"] = {"us": us, "GB/s": gb, "per_gpu_frac": gb / world / hbm}
    out["note"] = (f"split over {world} ranks; row split includes the NCCL all-reduce of the {cfg.hidden_size} "
                   "partial outputs; time = max over ranks; GB/s = whole matrix bytes / time")
    return out


def write_gguf_i2s(path, cfg, layers, rank, rng):
    """A GGUF v3 file holding the I2_S projections of `layers` layers (random
    codes, F32 scale after each) and their rank-`rank` F32 lora_a / lora_b,
    data section at the default 32-byte alignment.  Returns its tensor names."""
    import struct
    from ternative_b200.model import PROJ, proj_shape
    tensors = []
    for li in range(layers):
        for n in PROJ:
            N, K = proj_shape(cfg, n)
            codes = rng.integers(0, 256, K * N // 4, dtype=np.uint8).tobytes() + struct.pack("<f", 0.02)
            tensors.append((f"blk.{li}.{n}.weight", 36, (K, N), codes))
            tensors.append((f"blk.{li}.{n}.lora_a", 0, (K, rank),
                            rng.standard_normal(rank * K, dtype=np.float32).tobytes()))
            tensors.append((f"blk.{li}.{n}.lora_b", 0, (rank, N),
                            rng.standard_normal(rank * N, dtype=np.float32).tobytes()))

    def s(b):
        return struct.pack("<Q", len(b)) + b
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), 1) + s(b"general.architecture") \
        + struct.pack("<I", 8) + s(b"bitnet")
    off = 0
    for name, t, shape, data in tensors:
        head += s(name.encode()) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        head += struct.pack("<IQ", t, off)
        off += (len(data) + 31) // 32 * 32
    with open(path, "wb") as f:
        f.write(head + bytes((-len(head)) % 32))
        for _, _, _, data in tensors:
            f.write(data + bytes((-len(data)) % 32))
    return [t[0] for t in tensors]


def serving_rows(be, m, cfg, stream, rng, cpu_seconds):
    """The rows either side of the decode path on the 2B model: the device
    sampler over 8 rows, log-probabilities of a 512-token sequence, the
    merged-weight cache (.tvcache) and GGUF ingest into device memory, each
    beside the reference's own CPU code for the same work where that runs
    here (oracle/_ref: sample_token, gguf_load)."""
    import ctypes as C
    import shutil
    import tempfile
    import torch
    from ternative_b200 import cache as tc
    from ternative_b200 import load
    from ternative_b200._lib import SamplerConfig

    def ev_time(fn, reps):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) / reps

    out = {}
    lib = load()
    # ---- sampler: 8 rows of vocab logits, temperature 0.8, top-p 0.9, top-k 40,
    # repetition penalty 1.1 over 64 seen tokens per row
    B, V, NS = 8, cfg.vocab_size, 64
    with torch.cuda.stream(stream):
        lg = torch.randn(B, V, device="cuda") * 3
        seen = torch.from_numpy(rng.integers(0, V, (B, NS)).astype(np.int32)).cuda()
        n_seen = torch.full((B,), NS, dtype=torch.int32, device="cuda")
        u = torch.rand(B, device="cuda")
        tok = torch.empty(B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    sc = SamplerConfig(0.8, 0.9, 40, 1.1)

    def sample():
        st = lib.tvb_sample(lg.data_ptr(), B, V, V, C.byref(sc), seen.data_ptr(), n_seen.data_ptr(), NS,
                            u.data_ptr(), tok.data_ptr(), be.stream)
        if st != 0:
            raise RuntimeError(f"tvb_sample status {st}")
    us = ev_time(sample, 50) * 1e3
    out["sampler"] = {"workload": f"{B} rows x {V} logits, T 0.8, top-p 0.9, top-k 40, penalty 1.1 "
                                  f"over {NS} seen tokens", "us_per_call": us, "rows_per_s": B / (us * 1e-6),
                      "logit_GB/s": B * V * 4 / (us * 1e-6) / 1e9}
    try:
        from oracle.oracle import Reference
        ref = Reference()
        h_lg = lg.cpu().numpy()
        h_seen = seen.cpu().numpy()
        t0 = time.perf_counter()
        n = 0
        while time.perf_counter() - t0 < min(2.0, cpu_seconds):
            for b in range(B):
                ref.L.tvref_sample_token(h_lg[b], V, 0.8, 0.9, 40, 1.1, h_seen[b], NS)
            n += B
        out["sampler"]["cpu_baseline"] = {
            "us_per_row": (time.perf_counter() - t0) / n * 1e6, "cores": 1, "kind": "reference",
            "sample": f"{n} rows through sample_token (sampler.cpp) on host logits, no D2H copy counted"}
    except Exception as e:
        out["sampler"]["cpu_baseline"] = {"unavailable": repr(e)}

    # ---- log-probabilities: one 512-token sequence, top 5 per position, through
    # the C ABI (H2D tokens, D2H results)
    T = min(512, cfg.max_prefill, cfg.max_seq_len)
    toks = rng.integers(0, V, T).astype(np.int32)
    ms = ev_time(lambda: be.score_logprobs(toks, k=5), 3)
    out["logprobs"] = {"workload": f"{T}-token sequence, top 5 per position", "ms": ms,
                       "scored_tok_s": (T - 1) / (ms * 1e-3)}

    tmp = tempfile.mkdtemp(prefix="tvb_bench_")
    try:
        # ---- .tvcache of the first 4 layers' merged tensors (+ embedding, norm):
        # write from device memory, then read back into device buffers; the file is in
        # the page cache on read
        ents = tc.model_entries(m)
        ents = [e for e in ents if not e.name.startswith("blk.") or int(e.name.split(".")[1]) < 4]
        path = os.path.join(tmp, "m.tvcache")
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        tc.write(path, tc.make_key(), ents)
        wsec = time.perf_counter() - t0
        nbytes = os.path.getsize(path)
        with tc.CacheFile(path) as f:
            bufs = {n: torch.empty(max(1, b), dtype=torch.uint8, device="cuda") for n, (_, _, b) in f.entries.items()}
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for n, (_, _, b) in f.entries.items():
                f.read(n, bufs[n].data_ptr(), b)
            torch.cuda.synchronize()
            rsec = time.perf_counter() - t0
        del bufs
        out["tvcache"] = {"workload": f"{len(ents)} merged tensors (embedding, output norm, layers 0-3), "
                                      f"{nbytes / 1e9:.2f} GB file", "write_GB/s": nbytes / wsec / 1e9,
                          "read_to_device_GB/s": nbytes / rsec / 1e9}
        os.remove(path)

        # ---- GGUF ingest: I2_S + LoRA (rank 16) of all layers into device memory
        gpath = os.path.join(tmp, "m.gguf")
        names = write_gguf_i2s(gpath, cfg, cfg.num_layers, 16, rng)
        gbytes = os.path.getsize(gpath)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with tc.GGUFFile(gpath) as g:
            total = sum(b for _, _, b in g.entries.values())
            pool = torch.empty(total + 256 * len(names), dtype=torch.uint8, device="cuda")
            off = 0
            for n in names:
                b = g.entries[n][2]
                g.read(n, pool.data_ptr() + off, b)
                off += (b + 255) // 256 * 256
            torch.cuda.synchronize()
        gsec = time.perf_counter() - t0
        del pool
        out["gguf_ingest"] = {"workload": f"{len(names)} tensors (I2_S projections of {cfg.num_layers} layers "
                                          f"+ rank-16 F32 LoRA), {gbytes / 1e9:.2f} GB file in the page cache",
                              "seconds": gsec, "GB/s_to_device": total / gsec / 1e9}
        try:
            t0 = time.perf_counter()
            reference_gguf_load = ref.L.tvref_gguf_tensor
            t = C.c_int()
            nd = C.c_int()
            shp = (C.c_longlong * 8)()
            reference_gguf_load(gpath.encode(), names[0].encode(), None, C.byref(t), C.byref(nd), shp)
            out["gguf_ingest"]["cpu_baseline"] = {
                "seconds": time.perf_counter() - t0, "cores": 1, "kind": "reference",
                "sample": "gguf_load (gguf.cpp) of the same file into host memory, before any upload"}
        except Exception as e:
            out["gguf_ingest"]["cpu_baseline"] = {"unavailable": repr(e)}
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return out


def run_ours(args, world, rank, local):
    import torch
    import torch.distributed as dist
    from ternative_b200 import TVB_F16, TVB_I8_ROW, CUDABackend
    from ternative_b200.model import PROJ, SHAPES, Model, SyntheticModel, proj_shape

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    def all_gather(obj):
        if world == 1:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    tp_parity = None
    if world > 1 and args.only is None:
        try:
            tp_parity = tp_parity_check(world, rank, all_gather)
        except Exception as e:   # reported; the same on every rank
            tp_parity = {"ok": False, "error": repr(e)}
    if args.only_tp:
        res = run_tp_8b(args, world, rank)
        if rank == 0:
            print(json.dumps({"tp_8b": res, "tp_parity": tp_parity}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    cfg = SHAPES[args.config]
    if args.only == "batch8":
        # profiling: W + K batched greedy steps of 8 sequences on the 8B shape
        # (--layers of its 32; 64-token prompts), one GPU
        cfg = dataclasses.replace(SHAPES["8b"], num_layers=args.layers or 32, max_batch=TP_BATCH,
                                  max_seq_len=64 + args.warmup + args.steps + 8)
        m = Model.load(SyntheticModel.generate(cfg, rank=32, alpha=64.0, seed=0))
        rng = np.random.default_rng(7)
        cur = np.empty(TP_BATCH, np.int32)
        for b in range(TP_BATCH):
            _, cur[b] = m.backend.prefill_slot(b, rng.integers(0, cfg.vocab_size, 64).astype(np.int32),
                                               want_logits=False)
        pos = np.full(TP_BATCH, 64, np.int32)
        for _ in range(args.warmup + args.steps):
            _, cur = m.backend.decode_batch(cur, pos, want_logits=False)
            pos += 1
        m.backend.sync_d()
        return
    if args.layers:
        # profiling only: the same shapes with fewer layers (smaller device footprint)
        cfg = dataclasses.replace(cfg, num_layers=args.layers)
    if args.only == "sample":
        # profiling: W + K device samplings of 8 rows of vocabulary logits
        # (temperature 0.8, top-p 0.9, top-k 40, penalty 1.1 over 64 seen tokens)
        import ctypes as C
        from ternative_b200 import load
        from ternative_b200._lib import SamplerConfig
        lib = load()
        B, V = 8, cfg.vocab_size
        lg = torch.randn(B, V, device="cuda") * 3
        seen = torch.randint(0, V, (B, 64), dtype=torch.int32, device="cuda")
        n_seen = torch.full((B,), 64, dtype=torch.int32, device="cuda")
        u = torch.rand(B, device="cuda")
        tok = torch.empty(B, dtype=torch.int32, device="cuda")
        sc = SamplerConfig(0.8, 0.9, 40, 1.1)
        for _ in range(args.warmup + args.steps):
            if lib.tvb_sample(lg.data_ptr(), B, V, V, C.byref(sc), seen.data_ptr(), n_seen.data_ptr(), 64,
                              u.data_ptr(), tok.data_ptr(), None) != 0:
                raise RuntimeError(lib.tvb_last_error().decode())
        torch.cuda.synchronize()
        return
    synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=0)
    be = CUDABackend()
    if args.only == "merge":
        # profiling: the F16 merge of layer 0's 7 projections, exact (CUDA-core)
        # and tensor-core delta, W + K times each
        outs = [{n: torch.empty(proj_shape(cfg, n), dtype=torch.float16, device="cuda")
                 for n in PROJ}]
        for _ in range(args.warmup + args.steps):
            be.merge_batch(synth.merge_descs(outs, layers=[0]), TVB_F16, stream=0)
            be.merge_batch_tc(synth.merge_descs(outs, layers=[0]), TVB_F16, stream=0)
        torch.cuda.synchronize()
        return
    m = Model.load(synth, backend=be)
    if args.only == "gemv":
        # profiling: standalone streaming GEMV on the gate shape, rotating layers
        N, K = proj_shape(cfg, "w_gate")
        x = torch.randn(K, device="cuda")
        y = torch.empty(N, device="cuda")
        for i in range(args.warmup + args.steps):
            be.gemv_d2d(y, x, m.weights[i % cfg.num_layers]["w_gate"], K, N)
        be.sync_d()
        return
    if args.only == "prefill":
        # profiling: W + K batched prefills of a --prefill-len random prompt
        ptoks = np.random.default_rng(2).integers(0, cfg.vocab_size, args.prefill_len).astype(np.int32)
        for _ in range(args.warmup + args.steps):
            be.clear_kv_d()
            be.prefill(ptoks, want_logits=False)
        be.sync_d()
        return
    if args.only == "decode":
        # profiling: W + K chained decode steps from position 32 (KV rows zero), nothing else
        be.clear_kv_d()
        be.decode_enqueue(1, 32, args.warmup + args.steps)
        be.sync_d()
        return
    stream = torch.cuda.ExternalStream(be.stream)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, cfg.vocab_size, args.prompt).astype(np.int32)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    # ---- device-timed decode (value) ---------------------------------------------
    be.clear_kv_d()
    _, tok = be.prefill(prompt, want_logits=False)
    pos = len(prompt)
    be.decode_enqueue(tok, pos, args.warmup)
    be.sync_d()
    pos += args.warmup
    st = be.lib  # noqa: F841
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        be.decode_enqueue(tok, pos, args.steps)
        ev1.record(stream)
        ev1.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = world * args.steps / (ms / 1e3)

    # ---- e2e through the C ABI with host buffers ---------------------------------
    be.clear_kv_d()
    _, tok = be.prefill(prompt, want_logits=False)
    pos = len(prompt)
    for _ in range(min(args.warmup, 4)):
        _, tok = be.decode_step(tok, pos)
        pos += 1
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        _, tok = be.decode_step(tok, pos)   # H2D token/pos, D2H logits, synchronous
        pos += 1
    e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": world * args.steps / (e2e_ms / 1e3), "unit": "tok/s",
           "h2d_bytes_per_step": 8, "d2h_bytes_per_step": cfg.vocab_size * 4 + 4 * 76}

    # ---- roofline of the dominant kernel: the decode-step kernel (one launch per
    # token).  Algorithmic bytes per launch: every projection weight (F16), the
    # tied lm_head, the KV rows read by attention and written for this token.
    hbm, peak_kind = peaks()
    pos_mid = args.prompt + args.warmup + args.steps // 2
    Hk = cfg.num_kv_heads * cfg.head_dim
    weight_bytes = sum(2 * proj_shape(cfg, n)[0] * proj_shape(cfg, n)[1] for n in PROJ) \
        * cfg.num_layers + cfg.vocab_size * cfg.hidden_size * 2
    kv_bytes = cfg.num_layers * (2 * pos_mid * Hk * 4 + 2 * Hk * 4)
    step_bytes = weight_bytes + kv_bytes
    achieved = step_bytes / (ms_per_step * 1e-3) / 1e9
    traffic = profiled_traffic("decode_step_kernel", cfg.num_layers)
    roofline = {"bound": "hbm", "kernel": "decode_step_kernel (whole decode step)",
                "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "peak_kind": peak_kind, "bytes_per_launch": step_bytes,
                "us_per_launch": ms_per_step * 1e3, "traffic": traffic}

    # ---- batched prefill (tensor cores): prompt lengths 128 / 512 / 1024 ------------
    # Algorithmic FLOPs per prompt: 2 x (projection weights) per token + causal
    # attention 4 * S^2 * Hq / 2 per layer + the last row's lm_head.  The kernels
    # issue twice the projection MMAs (F16 hi + lo activation planes).
    tpeak, tpeak_kind = tensor_peak()
    n_proj = sum(proj_shape(cfg, n)[0] * proj_shape(cfg, n)[1] for n in PROJ) * cfg.num_layers
    Hq = cfg.num_heads * cfg.head_dim
    prefill = {}
    for S in (128, 512, 1024):
        if S > min(cfg.max_prefill, cfg.max_seq_len):
            continue
        ptoks = rng.integers(0, cfg.vocab_size, S).astype(np.int32)
        for _ in range(2):
            be.clear_kv_d()
            be.prefill(ptoks, want_logits=False)
        best = None
        for _ in range(3):
            be.clear_kv_d()
            be.sync_d()
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(stream)
            be.prefill(ptoks, want_logits=False)
            p1.record(stream)
            p1.synchronize()
            t = p0.elapsed_time(p1)
            best = t if best is None else min(best, t)
        flops = 2.0 * n_proj * S + cfg.num_layers * 4.0 * S * S * Hq / 2 + 2.0 * cfg.vocab_size * cfg.hidden_size
        prefill[str(S)] = {"ms": best, "tok_s": S / (best * 1e-3), "TFLOP/s": flops / (best * 1e-3) / 1e12,
                           "frac": flops / (best * 1e-3) / 1e12 / tpeak}
    prefill["peak_TFLOP/s"] = tpeak
    prefill["peak_kind"] = tpeak_kind
    prefill["note"] = ("one tvb_prefill call (H2D tokens, all layers, last-row lm_head) timed with "
                       "CUDA events, best of 3; KV cleared before each")

    # ---- the stand-alone streaming GEMV (gemv_d2d) on the GEMV-sweep shapes,
    # rotating over every layer's copy so the weights come from HBM ------------
    gemv = {}
    for name in ("wk", "wq", "w_gate", "w_down"):
        N, K = proj_shape(cfg, name)
        x = torch.randn(K, device="cuda")
        y = torch.empty(N, device="cuda")
        ws = [m.weights[li][name] for li in range(cfg.num_layers)]
        for i in range(3):
            be.gemv_d2d(y, x, ws[i], K, N)
        be.sync_d()
        reps = 2 * cfg.num_layers
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for i in range(reps):
            be.gemv_d2d(y, x, ws[i % len(ws)], K, N)
        g1.record(stream)
        g1.synchronize()
        us = g0.elapsed_time(g1) * 1e3 / reps
        gb = (N * K * 2 + 4 * K + 4 * N) / (us * 1e-6) / 1e9
        gemv[f"{N}x{K}_f16"] = {"us": us, "GB/s": gb, "frac": gb / hbm}
        # the same shape with per-row INT8 weights (per-row absmax of the F16 copies)
        q8 = []
        for w in ws:
            q = torch.empty(N, K, dtype=torch.int8, device="cuda")
            sc = torch.empty(N, dtype=torch.float32, device="cuda")
            be.quantize_int8(w, N, K, True, q, sc)
            q8.append((q, sc))
        be.sync_d()
        for i in range(3):
            be.gemv_d2d_int8_rows(y, x, q8[i][0], q8[i][1], K, N)
        be.sync_d()
        g0.record(stream)
        for i in range(reps):
            q, sc = q8[i % len(q8)]
            be.gemv_d2d_int8_rows(y, x, q, sc, K, N)
        g1.record(stream)
        g1.synchronize()
        us = g0.elapsed_time(g1) * 1e3 / reps
        gb = (N * K + 4 * N + 4 * K + 4 * N) / (us * 1e-6) / 1e9
        gemv[f"{N}x{K}_i8row"] = {"us": us, "GB/s": gb, "frac": gb / hbm}
        del q8
    # the tied lm_head (128256 x 2560, 657 MB: beyond L2 on its own)
    N, K = cfg.vocab_size, cfg.hidden_size
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    for _ in range(3):
        be.gemv_d2d(y, x, m.tok_embd, K, N)
    be.sync_d()
    g0.record(stream)
    for _ in range(10):
        be.gemv_d2d(y, x, m.tok_embd, K, N)
    g1.record(stream)
    g1.synchronize()
    us = g0.elapsed_time(g1) * 1e3 / 10
    gb = (N * K * 2 + 4 * K + 4 * N) / (us * 1e-6) / 1e9
    gemv[f"{N}x{K}_f16"] = {"us": us, "GB/s": gb, "frac": gb / hbm}
    gemv["note"] = ("one tvb_gemv_* launch per call (includes the launch), rotating over the 30 layers' "
                    "copies (lm_head: one 657 MB copy); bytes = weights + scales + x + y")
    if world > 1:
        try:   # a failure here is the same on every rank (no rank is left in a collective)
            gemv["tensor_parallel"] = gemv_tp_sweep(be, m, cfg, stream, world, rank, hbm)
        except Exception as e:
            gemv["tensor_parallel"] = {"unavailable": repr(e)}

    # ---- load-time merge: all 210 projections, F16 and per-row INT8 ---------------
    merge = {}
    outs = [{n: torch.empty(proj_shape(cfg, n), dtype=torch.float16, device="cuda") for n in PROJ}
            for _ in range(cfg.num_layers)]
    descs = synth.merge_descs(outs)
    for _ in range(2):
        be.merge_batch(descs, TVB_F16)
    be.sync_d()
    m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    m0.record(stream)
    be.merge_batch(descs, TVB_F16)
    m1.record(stream)
    m1.synchronize()
    ms_f16 = m0.elapsed_time(m1)
    n_w = sum(proj_shape(cfg, n)[0] * proj_shape(cfg, n)[1] for n in PROJ) * cfg.num_layers
    lora_b = sum(4 * 16 * (proj_shape(cfg, n)[0] + proj_shape(cfg, n)[1]) for n in PROJ) * cfg.num_layers
    merge["r16_f16"] = {"ms": ms_f16, "GB/s": (n_w / 4 + lora_b + 2 * n_w) / (ms_f16 * 1e6),
                        "GFLOP/s": 2 * 16 * n_w / (ms_f16 * 1e6)}
    del outs
    outs = [{n: torch.empty(proj_shape(cfg, n), dtype=torch.int8, device="cuda") for n in PROJ}
            for _ in range(cfg.num_layers)]
    scs = [{n: torch.empty(proj_shape(cfg, n)[0], dtype=torch.float32, device="cuda") for n in PROJ}
           for _ in range(cfg.num_layers)]
    descs = synth.merge_descs(outs, scs)
    be.merge_batch(descs, TVB_I8_ROW)
    be.sync_d()
    m0.record(stream)
    be.merge_batch(descs, TVB_I8_ROW)
    m1.record(stream)
    m1.synchronize()
    ms_i8 = m0.elapsed_time(m1)
    merge["r16_i8row"] = {"ms": ms_i8, "GB/s": (n_w / 4 + lora_b + n_w) / (ms_i8 * 1e6)}
    del outs, scs

    # rank-64 LoRA (alpha 128) on the same I2_S codes: the merge microbench's
    # configuration, exact (CUDA cores, bit-identical) and tensor-core (F16
    # within 1 ulp) deltas to F16, exact per-row INT8
    from ternative_b200._lib import MergeDesc
    g64 = torch.Generator(device="cuda")
    g64.manual_seed(64)
    lora64, descs64 = [], []
    outs = [{n: torch.empty(proj_shape(cfg, n), dtype=torch.float16, device="cuda") for n in PROJ}
            for _ in range(cfg.num_layers)]
    for li in range(cfg.num_layers):
        for name in PROJ:
            N, K = proj_shape(cfg, name)
            A = torch.randn(64, K, generator=g64, device="cuda") / np.sqrt(K)
            B = torch.randn(N, 64, generator=g64, device="cuda") * 1e-3
            lora64.append((A, B))
            t = synth.layers[li][name]
            descs64.append(MergeDesc(t.i2s.data_ptr(), t.scale, K, N, A.data_ptr(), B.data_ptr(), 64, 128.0,
                                     outs[li][name].data_ptr(), None, 0, 0))
    lora64_b = sum(4 * 64 * (proj_shape(cfg, n)[0] + proj_shape(cfg, n)[1]) for n in PROJ) * cfg.num_layers
    for key, fn in (("r64_f16_exact", be.merge_batch), ("r64_f16_tc", be.merge_batch_tc)):
        fn(descs64, TVB_F16)
        be.sync_d()
        m0.record(stream)
        fn(descs64, TVB_F16)
        m1.record(stream)
        m1.synchronize()
        ms = m0.elapsed_time(m1)
        merge[key] = {"ms": ms, "GB/s": (n_w / 4 + lora64_b + 2 * n_w) / (ms * 1e6),
                      "frac_of_hbm": (n_w / 4 + lora64_b + 2 * n_w) / (ms * 1e6) / hbm,
                      "GFLOP/s": 2 * 64 * n_w / (ms * 1e6)}
    del outs
    outs = [{n: torch.empty(proj_shape(cfg, n), dtype=torch.int8, device="cuda") for n in PROJ}
            for _ in range(cfg.num_layers)]
    scs = [{n: torch.empty(proj_shape(cfg, n)[0], dtype=torch.float32, device="cuda") for n in PROJ}
           for _ in range(cfg.num_layers)]
    for d, (li, name) in zip(descs64, [(li, n) for li in range(cfg.num_layers) for n in PROJ]):
        d.dst = outs[li][name].data_ptr()
        d.row_scales = scs[li][name].data_ptr()
    for key, fn in (("r64_i8row_exact", be.merge_batch), ("r64_i8row_tc", be.merge_batch_tc)):
        fn(descs64, TVB_I8_ROW)
        be.sync_d()
        m0.record(stream)
        fn(descs64, TVB_I8_ROW)
        m1.record(stream)
        m1.synchronize()
        ms = m0.elapsed_time(m1)
        merge[key] = {"ms": ms, "GB/s": (n_w / 4 + lora64_b + n_w) / (ms * 1e6)}
    merge["note"] = ("all 210 projections of the 2B shape in one call; GB/s = (I2_S codes + LoRA A,B + "
                     "output) / time; exact = CUDA-core delta bit-identical to apply_lora, tc = "
                     "tcgen05 delta (F16 within 1 ulp; INT8: those F16 rows quantised per row)")
    del outs, scs, lora64, descs64

    # ---- mixed offload (layers 0-13 F16, 14-29 per-row INT8): prefill of a
    # 1024-token prompt, then 256 greedy decode steps from position 1024 ------
    mixed = None
    if args.mixed:
        be2 = CUDABackend()
        m2 = Model.load(synth, int8_layers=range(14, cfg.num_layers), backend=be2)
        stream2 = torch.cuda.ExternalStream(be2.stream)
        ptoks = rng.integers(0, cfg.vocab_size, 1024).astype(np.int32)
        for _ in range(2):
            be2.clear_kv_d()
            _, t2 = be2.prefill(ptoks, want_logits=False)
        be2.clear_kv_d()
        be2.sync_d()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record(stream2)
        _, t2 = be2.prefill(ptoks, want_logits=False)
        q1.record(stream2)
        q1.synchronize()
        pms = q0.elapsed_time(q1)
        be2.decode_enqueue(t2, 1024, 4)
        be2.sync_d()
        q0.record(stream2)
        be2.decode_enqueue(0, 1028, 256)
        q1.record(stream2)
        q1.synchronize()
        dms = q0.elapsed_time(q1) / 256
        Hk = cfg.num_kv_heads * cfg.head_dim
        layer_f16 = sum(2 * proj_shape(cfg, n)[0] * proj_shape(cfg, n)[1] for n in PROJ)
        layer_i8 = sum(proj_shape(cfg, n)[0] * (proj_shape(cfg, n)[1] + 4) for n in PROJ)
        dbytes = 14 * layer_f16 + (cfg.num_layers - 14) * layer_i8 + cfg.vocab_size * cfg.hidden_size * 2 \
            + cfg.num_layers * 2 * (1028 + 128) * Hk * 4
        mixed = {"workload": "2B shape, layers 0-13 F16 and 14-29 per-row INT8: 1024-token prefill, then "
                             "256 greedy decode steps from position 1028",
                 "prefill_ms": pms, "prefill_tok_s": 1024 / (pms * 1e-3),
                 "decode_ms_per_token": dms, "decode_tok_s": 1e3 / dms,
                 "decode_bytes_per_token": dbytes, "decode_GB/s": dbytes / (dms * 1e-3) / 1e9,
                 "decode_frac_of_hbm": dbytes / (dms * 1e-3) / 1e9 / hbm}
        be2.close()
        del m2

    # ---- CPU baselines: the reference's own code on this host (rank 0, all host
    # cores for its OpenMP loops; the merge is single-threaded, as the reference's is)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        try:
            from oracle.oracle import ModelShape, Reference, ReferenceModel
            shape = ModelShape(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                               cfg.num_kv_heads, cfg.intermediate_size, 512)
            hw = m.host_weights()
            rm = ReferenceModel(Reference(), shape, hw)
            rm.ref.L.tvref_set_threads(HOST_CORES)
            cores = rm.ref.L.tvref_omp_threads()
            sec, n = time_reference_decode(rm, 64, pos0=40, budget_s=args.cpu_seconds)
            cpu = {"value": 1.0 / sec, "unit": "tok/s", "cores": cores,
                   "kind": "reference",
                   "sample": f"{n} decode tokens (Model::forward, prefill=false) of the same merged "
                             "2B model, oracle/_ref built from the reference sources"}
            cpu_extra = reference_cpu_baselines(rm, hw, cfg, synth, cores, args.cpu_seconds)
            rm.close()
            del hw
            prefill["cpu_baseline"] = cpu_extra["prefill"]
            gemv["cpu_baseline"] = cpu_extra["gemv"]
            merge["cpu_baseline"] = cpu_extra["merge"]
        except Exception as e:
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "reference",
                   "sample": f"unavailable: {e!r}"}

    serving = None
    if world == 1 and not args.no_serving:
        try:
            serving = serving_rows(be, m, cfg, stream, rng, args.cpu_seconds)
        except Exception as e:   # reported, not fatal to the headline line
            serving = {"unavailable": repr(e)}

    tp8 = None
    if not args.no_tp:
        try:
            tp8 = run_tp_8b(args, world, rank)
        except Exception as e:   # reported, not fatal to the headline line
            tp8 = {"unavailable": repr(e)}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16-weights/f32-compute",
            "data": "synthetic", "config": config_block(args, cfg),
            "roofline": roofline, "gemv_standalone": gemv,
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": args.steps,   # one decode_step_kernel launch per token
            "clocks": clk.report(), "merge": merge, "prefill": prefill, "mixed_offload": mixed, "tp_8b": tp8,
            "tp_parity": tp_parity, "serving_rows": serving,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="bitnet-2b")
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-serving", action="store_true")
    ap.add_argument("--only", choices=["decode", "gemv", "merge", "prefill", "sample", "batch8"], default=None,
                    help="profiling: run only W+K launches of one part, print nothing")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling with --only: use this many layers of the shape")
    ap.add_argument("--no-tp", action="store_true",
                    help="skip the tensor-parallel 8B decode measurement")
    ap.add_argument("--tp-prompt", type=int, default=512)
    ap.add_argument("--no-mixed", dest="mixed", action="store_false",
                    help="skip the mixed F16/INT8 prefill + decode measurement")
    ap.add_argument("--prefill-len", type=int, default=1024,
                    help="profiling with --only prefill: prompt length")
    ap.add_argument("--only-tp", action="store_true",
                    help="run only the tensor-parallel 8B decode measurement and print its JSON")
    args = ap.parse_args()
    if args.warmup < 3 and args.only is None:
        ap.error("--warmup must be >= 3")
    if args.layers and args.only is None:
        ap.error("--layers is for profiling runs (--only)")
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
