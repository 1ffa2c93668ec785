"""Phase trace of the fused decode step: where the time of one decoded token goes.

Runs the synthetic model of a named shape (I2_S + rank-16 LoRA merged to F16 on
the device, seed 0) through a prompt and a few decode steps on the trace build
of the library (libtvb200_trace.so, ``make -C ternative_b200/csrc trace``), then
reads the per-(phase, CTA) %globaltimer stamps of the last traced step and
prints, per phase kind averaged over the layers:

  step_us      time from the previous phase's barrier exit to this one's (median CTA)
  inputs_us    phase start -> inputs staged (GEMV activation prologue; attention item)
  stream_us    inputs staged -> weight stream done (median and slowest CTA)
  epi_us       stream done -> epilogue written
  arrive_us    epilogue -> barrier arrival made (__syncthreads + release add)
  prep_us      arrival -> next phase prepared (its first weight chunks requested,
               its constants staged)
  last_arrive  slowest CTA's arrival minus the median CTA's (straggling)
  bar_us       last arrival -> first CTA out of the barrier (barrier latency)
  exit_spread  first -> last CTA out of the barrier
  poll_us      last arrival -> thread 0's poll saw it (median CTA); poll_spread:
               first -> last CTA whose poll saw it
  after_poll   thread 0's poll -> every warp of its CTA past the barrier (the
               other warps still staging / requesting the next phase)

Usage:  python -m ternative_b200.phase_trace [--config bitnet-2b] [--layers N]
        [--prompt 32] [--steps 8] [--json out.json] [--lib path/to/trace/build.so]
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
TRACE_LIB = os.path.join(HERE, "libtvb200_trace.so")
EVENTS = 8
KINDS = ["qkv", "attn", "o_proj", "gate_up", "down"]


def phase_kinds(n_layers):
    return [k for _ in range(n_layers) for k in KINDS] + ["lm_head"]


def summarize(T, kinds):
    """T: [phases][ctas][EVENTS] int64 ns.  Returns {kind: {metric: mean over layers}}."""
    rows = {}
    P = T.shape[0]
    prev_exit = None
    for p in range(P):
        t = T[p].astype(np.int64)
        k = kinds[p]
        r = {}
        exit_ = np.median(t[:, 5]) if p + 1 < P else np.median(t[:, 3] if k != "attn" else t[:, 1])
        if prev_exit is not None:
            r["step_us"] = (exit_ - prev_exit) / 1e3
        prev_exit = exit_
        r["inputs_us"] = np.median(t[:, 1] - t[:, 0]) / 1e3
        r["inputs_max_us"] = np.max(t[:, 1] - t[:, 0]) / 1e3
        done = t[:, 1] if k == "attn" else t[:, 3]
        if k != "attn":
            r["stream_us"] = np.median(t[:, 2] - t[:, 1]) / 1e3
            r["stream_max_us"] = np.max(t[:, 2] - t[:, 1]) / 1e3
            r["epi_us"] = np.median(t[:, 3] - t[:, 2]) / 1e3
        if p + 1 < P:
            r["arrive_us"] = np.median(t[:, 6] - done) / 1e3
            r["prep_us"] = np.median(t[:, 4] - t[:, 6]) / 1e3
            r["last_arrive_us"] = (np.max(t[:, 6]) - np.median(t[:, 6])) / 1e3
            r["bar_us"] = (np.min(t[:, 5]) - np.max(t[:, 6])) / 1e3
            r["exit_spread_us"] = (np.max(t[:, 5]) - np.min(t[:, 5])) / 1e3
            # thread 0's poll saw the last arrival (median CTA) and the wait
            # from there until every warp of the CTA was past the barrier
            r["poll_us"] = (np.median(t[:, 7]) - np.max(t[:, 6])) / 1e3
            r["poll_spread_us"] = (np.max(t[:, 7]) - np.min(t[:, 7])) / 1e3
            r["after_poll_us"] = np.median(t[:, 5] - t[:, 7]) / 1e3
            r["after_poll_max_us"] = np.max(t[:, 5] - t[:, 7]) / 1e3
        rows.setdefault(k, []).append(r)
    out = {}
    for k, lst in rows.items():
        keys = sorted({key for r in lst for key in r})
        out[k] = {key: float(np.mean([r[key] for r in lst if key in r])) for key in keys}
        out[k]["phases"] = len(lst)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--config", default="bitnet-2b")
    ap.add_argument("--layers", type=int, default=0, help="use this many layers of the shape")
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--steps", type=int, default=8, help="decode steps before the traced one")
    ap.add_argument("--json", default=None, help="also write the summary here")
    ap.add_argument("--lib", default=TRACE_LIB, help="a trace build of the library")
    ap.add_argument("--norm", type=float, default=1.0, help="every norm weight of the synthetic model")
    ap.add_argument("--int8", action="store_true", help="every layer per-row INT8 instead of F16")
    args = ap.parse_args(argv)

    from . import _lib
    if not os.path.exists(args.lib):
        sys.exit(f"{args.lib} is not built: make -C ternative_b200/csrc trace")
    _lib.load(args.lib)   # before anything else loads the product build
    import torch
    from .model import SHAPES, Model, SyntheticModel

    cfg = SHAPES[args.config]
    if args.layers:
        cfg = dataclasses.replace(cfg, num_layers=args.layers)
    synth = SyntheticModel.generate(cfg, rank=16, alpha=32.0, seed=0, norm_value=args.norm)
    m = Model.load(synth, int8_layers=range(cfg.num_layers) if args.int8 else ())
    be = m.backend
    G = torch.cuda.get_device_properties(0).multi_processor_count
    n_phases = len(KINDS) * cfg.num_layers + 1
    buf = torch.zeros(n_phases * G * EVENTS, dtype=torch.int64, device="cuda")
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, args.prompt).astype(np.int32)
    be.clear_kv_d()
    _, tok = be.prefill(prompt, want_logits=False)
    pos = len(prompt)
    be.decode_enqueue(tok, pos, args.steps)
    be.sync_d()
    pos += args.steps
    # one untraced step timed with CUDA events, then the traced one
    stream = torch.cuda.ExternalStream(be.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    be.decode_enqueue(0, pos, 1)
    e1.record(stream)
    e1.synchronize()
    step_us = e0.elapsed_time(e1) * 1e3
    _lib.call("tvb_trace_set", buf.data_ptr(), n_phases)
    be.decode_enqueue(0, pos + 1, 1)
    be.sync_d()
    _lib.call("tvb_trace_set", None, 0)
    T = buf.view(n_phases, G, EVENTS).cpu().numpy()
    t0 = T[0, :, 0].min()
    t_end = T[-1, :, 3].max()
    diffs = np.diff(np.unique(T[T > 0]))
    summary = {
        "config": args.config, "layers": cfg.num_layers, "ctas": G, "kv_len": int(pos + 2),
        "step_us_cuda_events": step_us, "traced_span_us": float(t_end - t0) / 1e3,
        "timer_resolution_ns": int(diffs[diffs > 0].min()) if diffs.size else None,
        "kinds": summarize(T, phase_kinds(cfg.num_layers)),
    }
    hdr = ["phases", "step_us", "inputs_us", "inputs_max_us", "stream_us", "stream_max_us", "epi_us",
           "arrive_us", "prep_us", "last_arrive_us", "bar_us", "exit_spread_us", "poll_us", "poll_spread_us",
           "after_poll_us", "after_poll_max_us"]
    print(f"{args.config}{' INT8' if args.int8 else ''}, {cfg.num_layers} layers, {G} CTAs, kv_len {pos + 2}: "
          f"step {step_us:.1f} us "
          f"(CUDA events), traced span {summary['traced_span_us']:.1f} us, timer resolution "
          f"{summary['timer_resolution_ns']} ns")
    print("kind    " + " ".join(f"{h.replace('_us', ''):>11}" for h in hdr))
    for k in KINDS + ["lm_head"]:
        r = summary["kinds"][k]
        print(f"{k:<8}" + " ".join(f"{r.get(h, float('nan')):>11.2f}" for h in hdr))
    if args.json:
        with open(args.json, "w") as f:
            json.dump(summary, f, indent=1)
    be.close()


if __name__ == "__main__":
    main()
