"""Benchmark of the B200 Qwen3-TTS token loop (codec frames/s, RTF).

One step = one request through the public API: content ids -> device text
prep -> talker prefill -> every 80 ms frame (CodePredictor pass + talker
decode step + on-device sampling) -> codes back on the host. Default workload
is BASELINE.json configs[1] (0.6B-shaped, 64 random ids, 240 frames, Qwen-default
sampling, Philox seed 0, batch 1) on random-init weights (oracle/synth.py).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): independent request replicas, no
collective on the data path; value = all ranks' frames / max-over-ranks time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    # BASELINE.json configs[1]
    "0.6b-sampled": dict(shape="0.6b", n_ids=64, frames=240, do_sample=True, top_k=50,
                         top_p=1.0, temperature=0.9, penalty=1.05, sub_sample=True, sub_top_k=50,
                         sub_temperature=0.9, rng="philox"),
    # north-star target (0.6B greedy 240 frames); prompt as BASELINE configs[0] (32 ids)
    "0.6b-greedy": dict(shape="0.6b", n_ids=32, frames=240, do_sample=False, top_k=50, top_p=1.0,
                        temperature=0.9, penalty=1.0, sub_sample=False, sub_top_k=50,
                        sub_temperature=0.9, rng="lcg"),
    # BASELINE.json configs[2]
    "1.7b-greedy": dict(shape="1.7b", n_ids=128, frames=240, do_sample=False, top_k=50, top_p=1.0,
                        temperature=0.9, penalty=1.0, sub_sample=False, sub_top_k=50,
                        sub_temperature=0.9, rng="lcg"),
    # streaming text, 8-id pushes to 256 ids, generation starts
    # after 1 id (text_lookahead 1), 6-frame code chunks up to 480 frames
    "0.6b-stream": dict(shape="0.6b", n_ids=256, stream=True, push=8, chunk=6, frames=480,
                        do_sample=True, top_k=50, top_p=1.0, temperature=0.9, penalty=1.05,
                        sub_sample=True, sub_top_k=50, sub_temperature=0.9, rng="philox"),
    # batched serving, 16 concurrent requests per GPU,
    # prompt lengths uniform in [16, 256], config-1 sampling, seed = request index
    "1.7b-batch16": dict(shape="1.7b", n_ids=(16, 256), batch=16, frames=240, do_sample=True,
                         top_k=50, top_p=1.0, temperature=0.9, penalty=1.05, sub_sample=True,
                         sub_top_k=50, sub_temperature=0.9, rng="philox"),
    # codec decoder (speech tokenizer, HipCodecInitial): 240 frames of random codes
    # decoded to 24 kHz audio per step; the talker shape is irrelevant (tiny)
    "codec-decode": dict(shape="tiny", codec=True, frames=240),
}
FRAME_SECONDS = 0.08


def options(pkg, c, seed):
    return pkg.GenerateOptions(decode_audio=False, max_frames=c["frames"], do_sample=c["do_sample"],
                               top_k=c["top_k"], top_p=c["top_p"], temperature=c["temperature"],
                               repetition_penalty=c["penalty"], subtalker_dosample=c["sub_sample"],
                               subtalker_top_k=c["sub_top_k"],
                               subtalker_temperature=c["sub_temperature"], seed=seed, rng=c["rng"])


def model_dir(shape: str) -> Path:
    base = Path(os.environ.get("QTTS_BENCH_MODELS", "/tmp/qtts_bench_models"))
    return base / shape


def frame_bytes(shape_name: str, P: int, frames: int, batch: int = 1) -> float:
    """Algorithmic HBM bytes of one average (batch) frame: every weight read
    once per pass (talker step once, CodePredictor layers + head once per group
    pass) for the whole batch, plus each sequence's talker KV cache read
    (positions 0..pos) and append, all bf16."""
    from oracle import synth

    s = synth.SHAPES[shape_name]
    q_out, kv_out = s.q_heads * s.head_dim, s.kv_heads * s.head_dim

    def layer(h, inter):
        return 2 * ((q_out + 2 * kv_out) * h + h * q_out + 2 * inter * h + h * inter)

    talker = s.layers * layer(s.hidden, s.intermediate) + 2 * s.vocab * s.hidden
    kv_per_pos = 2 * s.layers * 2 * kv_out  # K and V, bf16
    avg_pos = P + (frames - 1) / 2.0 + 1
    talker += kv_per_pos * (avg_pos + 1) * batch
    cp_pass = s.cp_layers * layer(s.cp_hidden, s.cp_intermediate) + 2 * s.cp_vocab * s.cp_hidden
    if s.cp_hidden != s.hidden:
        cp_pass += 2 * s.cp_hidden * s.hidden
    return talker + (s.num_code_groups - 1) * cp_pass


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        loaded = [x for x in sm if x > 0.5 * (mx or 1)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, json.JSONDecodeError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# committed ncu summaries holding a `dram_bytes_per_launch:` line, per trace kind
TRAFFIC_FILES = {"attn+o+resid": "attention_decode_0p6b.txt", "gemv+swiglu": "gateup_gemv_0p6b.txt",
                 "gemv+resid": "down_gemv_0p6b.txt",
                 "cp head+select": "cp_head_select_0p6b.txt"}


def trace_bytes(kind, N, K):
    """Weight bytes one launch of a traced kernel streams (bf16 [N, K]; SwiGLU
    reads gate and up rows); the attention kernels' KV reads are left out."""
    if kind == "attn":
        return 0
    return N * K * 2 * (2 if kind == "gemv+swiglu" else 1)


def traced_frame_kernels(eng, ids, opts):
    """Per kernel kind of one traced frame of the live graph: launches, chain
    time per launch (own wait -> next kernel's wait), in-kernel time (own
    wait -> last exit), share of the frame, bytes and GB/s. Sorted by share."""
    import dataclasses
    eng.step_trace_enable(True)
    try:
        eng.generate_codes_from_ids(ids, dataclasses.replace(opts, max_frames=10))
        rows = eng.step_trace()
    finally:
        eng.step_trace_enable(False)
    rows = [r for r in rows if r["wait_ns"] >= 0 and r["exit_ns"] >= 0]
    if len(rows) < 2:
        return None
    span = rows[-1]["exit_ns"] - rows[0]["wait_ns"]
    agg = {}
    for i, r in enumerate(rows):
        chain = (rows[i + 1]["wait_ns"] if i + 1 < len(rows) else r["exit_ns"]) - r["wait_ns"]
        a = agg.setdefault(r["name"], [0, 0, 0])
        a[0] += 1
        a[1] += chain
        a[2] += r["exit_ns"] - r["wait_ns"]
    out = []
    for name, (n, chain, ink) in agg.items():
        kind, N, K = name.rsplit(" ", 2)[0], int(name.split("N=")[1].split()[0]), int(name.split("K=")[1])
        b = trace_bytes(kind, N, K)
        out.append({"kernel": name, "kind": kind, "launches": n, "chain_us": chain / n / 1e3,
                    "in_kernel_us": ink / n / 1e3, "share": chain / span, "bytes_per_launch": b,
                    "chain_gbs": b / (chain / n * 1e-9) / 1e9 if b else None})
    out.sort(key=lambda x: -x["share"])
    return out


def committed_traffic(name="gateup_gemv_0p6b.txt"):
    """DRAM bytes per launch of a kernel from its committed ncu summary
    (`dram_bytes_per_launch:` line), or None."""
    p = ROOT / "profiles" / name
    if not name or not p.is_file():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def cpu_reference_run(c, mdir, ids, n_frames, steps, warmup, seed=0):
    """The CPU oracle (PyTorch-CPU fp32 restatement of the reference loop) on a
    bounded sample: prefill + n_frames frames per step. Returns frames/s."""
    import torch

    from oracle import qtts_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    m = O.OracleModel(mdir, 512)
    t_cfg = O.SamplingConfig(c["do_sample"], c["top_k"], c["top_p"], c["temperature"])
    s_cfg = O.SamplingConfig(c["sub_sample"], c["sub_top_k"], 1.0, c["sub_temperature"])
    pre, tr, pad = m.prepare(list(ids))
    times, frames = [], 0
    with torch.inference_mode():
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            codes, _, _ = m.rollout(pre, tr, pad, n_frames, t_cfg, s_cfg, c["penalty"], seed,
                                    c["rng"])
            dt = time.perf_counter() - t0
            if i >= warmup:
                times.append(dt)
                frames += len(codes) // 16
    total = sum(times)
    return frames / total, frames, total, torch.get_num_threads(), pre.shape[0]


def reduce_over_ranks(maxed, summed, world, device):
    """Whole-job figures from per-rank ones: times as the max over ranks (the
    slowest replica bounds the job), counts as the sum. World 1 returns them
    unchanged; otherwise every rank of the initialised process group calls it."""
    if world <= 1:
        return list(maxed), list(summed)
    import torch
    import torch.distributed as dist

    t = torch.tensor(maxed, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    f = torch.tensor(summed, dtype=torch.float64, device=device)
    dist.all_reduce(f, op=dist.ReduceOp.SUM)
    return t.tolist(), f.tolist()


def codec_flops_per_frame(T: int) -> float:
    """Algorithmic FLOPs (2 per multiply-add) of decoding one frame in a
    T-frame window: every convolution / projection of the decoder at its
    sample rate, plus the causal attention of the pre-transformer."""
    from oracle import codec as K

    f = 2.0 * K.PROJECTED * 2 * K.CODEBOOK_DIM                      # RVQ projections
    f += 2.0 * K.PRE_CONV_OUT * K.PROJECTED * 3                      # pre_conv
    f += 2 * 2.0 * K.HIDDEN * K.PRE_CONV_OUT                         # input/output proj
    qo = K.HEADS * K.HEAD_DIM
    per_layer = 2.0 * (3 * qo * K.HIDDEN + K.HIDDEN * qo + 2 * K.INTER * K.HIDDEN
                       + K.HIDDEN * K.INTER)
    per_layer += 2 * 2.0 * K.HEADS * K.HEAD_DIM * (T + 1) / 2       # scores + values
    f += K.LAYERS * per_layer
    L = 1
    for _ in range(2):                                               # upsample + ConvNeXt
        L *= 2
        f += L * 2.0 * (K.UP_CH * K.UP_CH + K.UP_CH * 7 + 2 * K.CONVNEXT_INTER * K.UP_CH)
    f += L * 2.0 * K.DECODER_INIT * K.PRE_CONV_OUT * 7               # decoder.0
    for cin, cout, st in K.BLOCKS:
        L *= st
        f += L * 2.0 * cout * cin * 2                                # transposed conv (2 taps)
        f += 3 * L * 2.0 * (cout * cout * 7 + cout * cout)           # residual units
    f += L * 2.0 * 96 * 7                                            # final conv
    return f


def codec_main(args, c):
    """bench.py --config codec-decode: the codec decoder (codes -> waveform)."""
    from oracle import codec as K
    from oracle import synth

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    T = c["frames"]
    metric = "codec_decode_frames_per_s"
    workload = {"workload": f"codec-decode: {T} frames of random codes (16 codebooks) -> "
                            f"{T * K.SAMPLES_PER_FRAME} samples at 24 kHz per step, "
                            "seeded synthetic fp32 speech-tokenizer weights",
                "frames_per_step": T, "parallelism": f"replicas{max(world, args.gpus)}",
                "l2": "no flush: weights 456 MB and per-step activations > 1 GB (> 126 MB L2)"}
    mdir = model_dir("tiny_codec")
    codes = np.random.default_rng(rank).integers(0, K.CODEBOOK_SIZE, (T, K.GROUPS)).astype(np.int32)
    flops = codec_flops_per_frame(T) * T

    def cpu_run(n_frames, steps, warmup):
        import torch

        torch.set_num_threads(os.cpu_count() or 1)
        o = K.CodecOracle(K.generate(0))
        sample = codes[:n_frames].reshape(-1)
        times = []
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            o.decode(sample)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
        return n_frames * steps / sum(times), torch.get_num_threads()

    if args.impl == "reference":
        if rank != 0:
            return
        n = max(1, min(args.cpu_frames, T))
        fps, cores = cpu_run(n, args.steps, args.warmup)
        sample = f"{n} frames per step (of {T}), {args.steps} timed steps"
        print(json.dumps({
            "metric": metric, "value": fps, "unit": "frames/s", "impl": "reference", "n_gpus": 0,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * n / fps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload,
            "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "reference's Rust/ROCm codec cannot run here (no cargo, no AMD GPU); timed "
                    "arm is the repo's PyTorch-CPU fp32 restatement (oracle/codec.py)"}))
        return

    import torch
    import torch.distributed as dist

    import __graft_entry__

    pkg = __graft_entry__.load_package()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    if rank == 0:
        synth.write_model(mdir, "tiny", 0)
        K.write_codec(mdir, 0)
    if world > 1:
        dist.barrier()
    eng = pkg.HipTtsEngine.load_with_options(mdir, pkg.EngineOptions(local, 512))
    flat = codes.reshape(-1)
    for _ in range(args.warmup):
        eng.decode_codes(flat)
    dev_ms, wall, launches = 0.0, 0.0, 0
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            wav = eng.decode_codes(flat)
            wall += time.perf_counter() - t0
            ms, n = eng.last_decode_timing()
            dev_ms += ms
            launches += n
    torch.cuda.synchronize()
    (dev_ms_max, wall_max), (frames_all, launches_all) = reduce_over_ranks(
        [dev_ms, wall], [float(T * args.steps), float(launches)], world, torch.device("cuda", local))
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    clocks = clk.summary()
    # streaming: 6-frame chunks of the same codes, with carried decoder state
    # against the reference's re-decode of 25 left-context frames per chunk
    chunk, ctx = 6, 25
    cs = eng.open_codec_stream(T)
    carried_ms = windowed_ms = 0.0
    for s0 in range(0, T, chunk):
        cs.decode(codes[s0:s0 + chunk].reshape(-1))
        carried_ms += eng.last_decode_timing()[0]
        a = max(0, s0 - ctx)
        eng.decode_codes(codes[a:s0 + chunk].reshape(-1))
        windowed_ms += eng.last_decode_timing()[0]
    cs.close()
    peaks, peak_kind = measured_peaks()
    # each fp32 product is three bf16 tensor-core products (hi*hi, hi*lo, lo*hi),
    # so the ceiling of this method is a third of the bf16 tensor peak
    peak = peaks["bf16_tflops"] / 3.0
    achieved = flops * args.steps / (dev_ms / 1000.0) / 1e12
    line = {
        "metric": metric, "value": frames_all / (dev_ms_max / 1000.0), "unit": "frames/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random codes and fp32 codec weights)",
        "audio_seconds_per_s": frames_all * FRAME_SECONDS / (dev_ms_max / 1000.0),
        "config": workload,
        "e2e": {"value": frames_all / wall_max, "unit": "frames/s",
                "h2d_bytes_per_step": int(flat.nbytes), "d2h_bytes_per_step": int(wav.nbytes)},
        "gpu_launches": int(launches_all),
        "roofline": {"bound": "tensor", "kernel": "whole decode (k_codec_conv_tc carries >97 % "
                                                   "of the FLOPs)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "peak_kind": f"{peak_kind} bf16 tensor peak / 3 (fp32 products as three "
                                  "bf16 MMA products); achieved counts the fp32 algorithm's FLOPs",
                     "flops_per_step": flops, "traffic": None},
        "streaming": {"chunk_frames": chunk, "frames": T,
                      "carried_state_ms_per_chunk": carried_ms / ((T + chunk - 1) // chunk),
                      "redecode_ms_per_chunk": windowed_ms / ((T + chunk - 1) // chunk),
                      "redecode_context_frames": ctx,
                      "note": "device time per 6-frame audio chunk: qtts_codec_stream_decode "
                              "(carried state) vs qtts_decode_codes of the chunk plus up to 25 "
                              "context frames (the reference's next_audio_chunk)"},
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        n = max(1, min(args.cpu_frames, T))
        fps, cores = cpu_run(n, 2, 1)
        line["cpu_baseline"] = {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
                                "sample": f"{n} frames per step, 2 timed steps"}
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="0.6b-sampled", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-frames", type=int, default=6, help="frames per CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--frames", type=int, default=0, help="override frames per request (profiling)")
    args = ap.parse_args()
    c = dict(CONFIGS[args.config])
    if args.frames:
        c["frames"] = args.frames
    if c.get("codec"):
        return codec_main(args, c)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    metric = "codec_frames_per_s"
    batch = c.get("batch", 1)
    workload = {"workload": f"{args.config}: {c['shape']}-shaped talker+CodePredictor, "
                            f"{c['n_ids']} random text ids, {c['frames']} frames, "
                            f"batch {batch} per GPU",
                "shape": c["shape"], "frames_per_request": c["frames"], "text_ids": c["n_ids"],
                "sampling": "top_k=50 T=0.9 penalty=1.05, subtalker top_k=50 T=0.9"
                if c["do_sample"] else "greedy", "rng": c["rng"],
                "l2": "no flush: each frame streams ~3.3 GB of weights (> 126 MB L2)",
                "parallelism": f"replicas{max(world, args.gpus)}"}

    from oracle import synth

    mdir = model_dir(c["shape"])
    vocab = synth.SHAPES[c["shape"]].text_vocab - 1000
    rng0 = np.random.default_rng(0)
    if batch > 1:
        lo, hi = c["n_ids"]
        reqs = [rng0.integers(0, vocab, int(rng0.integers(lo, hi + 1))).astype(np.uint32)
                for _ in range(batch)]
        ids = reqs[0]
    else:
        reqs = None
        ids = rng0.integers(0, vocab, c["n_ids"]).astype(np.uint32)

    if args.impl == "reference":
        if rank != 0:
            return
        synth.write_model(mdir, c["shape"], 0)
        fps, frames, total, cores, P = cpu_reference_run(c, mdir, ids, args.cpu_frames,
                                                         args.steps, args.warmup)
        sample = (f"prefill P={P} + {args.cpu_frames} frames per step (of {c['frames']}), "
                  f"{args.steps} timed steps")
        # what this arm actually timed: a bounded sample of the workload
        workload = dict(workload, frames_timed_per_step=args.cpu_frames, prefill_included=True,
                        workload=workload["workload"] + f" (CPU sample: prefill + "
                                                        f"{args.cpu_frames} of the frames)")
        line = {"metric": metric, "value": fps, "unit": "frames/s", "impl": "reference",
                "n_gpus": 0, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1000 * total / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "rtf": 1.0 / (fps * FRAME_SECONDS), "config": workload,
                "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
                                 "sample": sample},
                "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0},
                "note": "reference's Rust/ROCm path cannot run here (no cargo, no AMD GPU); "
                        "timed arm is the repo's PyTorch-CPU fp32 restatement (oracle/)"}
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist

    import __graft_entry__

    pkg = __graft_entry__.load_package()
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    if rank == 0:
        synth.write_model(mdir, c["shape"], 0)
    if world > 1:
        dist.barrier()

    eng = pkg.HipTtsEngine.load_with_options(mdir, pkg.EngineOptions(local, 512))
    opts = options(pkg, c, seed=rank)
    if reqs is not None:
        bopts = [options(pkg, c, seed=b) for b in range(batch)]

    stream_stats = []

    def run_stream():
        """One streamed request: text pushed 8 ids at a time whenever the
        stream asks for more, codes pulled in 6-frame chunks. Records the time
        to the first chunk and the steady-state RTF after it (host wall clock,
        everything through the public API)."""
        ts = eng.start_text_stream_polling(
            opts, pkg.TextStreamOptions(min_start_tokens=1, min_resume_tokens=1))
        pos, frames, first, t_first = 0, 0, None, None
        t0 = time.perf_counter()
        ts.push_ids(ids[pos:pos + c["push"]])
        pos += c["push"]
        while True:
            r = ts.next_codes_chunk(c["chunk"])
            if isinstance(r, pkg.NeedMoreText):
                if pos < len(ids):
                    ts.push_ids(ids[pos:pos + c["push"]])
                    pos += c["push"]
                else:
                    ts.finish_text()
                continue
            if isinstance(r, pkg.Finished) or r is None:
                break
            frames += r.frames
            if first is None:
                t_first, first = time.perf_counter(), r.frames
        t_end = time.perf_counter()
        out = ts.finish_codes()
        ts.close()
        stream_stats.append({"ttfc_ms": 1e3 * (t_first - t0),
                             "steady_rtf": (t_end - t_first) / max(1, (frames - first)) / FRAME_SECONDS,
                             "frames": frames, "wall_s": t_end - t0})
        return out

    def run_step():
        if c.get("stream"):
            return run_stream()
        if reqs is None:
            return eng.generate_codes_from_ids(ids, opts)
        outs = eng.generate_codes_batch_from_ids(reqs, bopts)
        return type(outs[0])(sum((o.codes for o in outs), []), sum(o.frames for o in outs),
                             all(o.ended_by_eos for o in outs))

    for _ in range(args.warmup):
        run_step()

    dev_ms, wall_s, frames, launches, last = 0.0, 0.0, 0, 0, None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            out = run_step()
            wall_s += time.perf_counter() - t0
            tm = eng.last_timings()
            if c.get("stream"):
                # a stream interleaves host polling with device bursts: its
                # time is the wall clock of the whole stream
                tm = dict(tm, prefill_ms=0.0, frames_ms=1e3 * (time.perf_counter() - t0),
                          frames=out.frames)
            dev_ms += tm["prefill_ms"] + tm["frames_ms"]
            frames += out.frames
            launches += tm["kernels"]
            last = (out, tm)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    (dev_ms_max, wall_max), (frames_all, launches_all) = reduce_over_ranks(
        [dev_ms, wall_s], [frames, launches], world, "cuda")
    frames_all, launches_all = int(frames_all), int(launches_all)

    # secondary: the talker gate|up GEMV (+ RMSNorm prologue, SwiGLU epilogue)
    # in a chain of its own launches
    ms_k, bytes_k = eng.profile_projection(0, 280)
    peaks, peak_kind = measured_peaks()
    achieved = bytes_k / (ms_k * 1e-3) / 1e9
    P = 9 + (int(np.mean([r.size for r in reqs])) if reqs is not None else c["n_ids"])
    out, tm = last
    # one batch frame reads every weight once for all `batch` sequences, plus each one's KV
    fb = frame_bytes(c["shape"], P, c["frames"], batch)
    frame_ms = tm["frames_ms"] / max(1, tm["frames"]) * batch
    frame_gbs = fb / (frame_ms * 1e-3) / 1e9

    line_extra = {}
    if batch > 1:
        # batched serving: the batch frame (all tcgen05 projections at M=batch,
        # attention and selection) against HBM, weights read once per batch frame
        roofline = {"bound": "hbm", "kernel": f"batch frame (tcgen05 projections at M={batch}, "
                                              f"attention, selection)",
                    "achieved": frame_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                    "frac": frame_gbs / peaks["hbm_gbs"], "peak_kind": peak_kind,
                    "bytes_per_launch": fb, "ms_per_launch": frame_ms, "traffic": None}
    else:
        gateup = {"bound": "hbm",
                  "kernel": "k_gemv1<4,2> talker gate|up + SwiGLU (1024->2x3072), RMSNorm prologue",
                  "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                  "frac": achieved / peaks["hbm_gbs"], "peak_kind": peak_kind,
                  "bytes_per_launch": bytes_k, "ms_per_launch": ms_k,
                  "timing": "CUDA events around 280 back-to-back launches on the engine stream",
                  "traffic": committed_traffic()}
        roofline = gateup
    if batch == 1 and not c.get("stream"):
        frame_kernels = traced_frame_kernels(eng, ids, opts)
        if frame_kernels:
            top = frame_kernels[0]
            gbs = top["bytes_per_launch"] / (top["chain_us"] * 1e-6) / 1e9
            line_extra["roofline_gateup"] = roofline
            roofline = {"bound": "hbm", "kernel": top["kernel"],
                        "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": gbs / peaks["hbm_gbs"], "peak_kind": peak_kind,
                        "bytes_per_launch": top["bytes_per_launch"],
                        "ms_per_launch": top["chain_us"] * 1e-3,
                        "in_kernel_ms_per_launch": top["in_kernel_us"] * 1e-3,
                        "share_of_frame": top["share"],
                        "timing": "live frame graph, %globaltimer step trace of one frame: per "
                                  "launch, this kernel's first CTA past its dependency wait to the "
                                  "next kernel's (the chain time it holds); in-kernel = to its "
                                  "last CTA's exit",
                        "traffic": committed_traffic(TRAFFIC_FILES.get(top["kind"], ""))}
            line_extra["frame_kernels"] = frame_kernels
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    value = frames_all / (dev_ms_max / 1000.0)
    e2e = frames_all / wall_max
    line = {
        "metric": metric, "value": value, "unit": "frames/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) bf16 weights, seed 0; random text ids)",
        "rtf": (dev_ms_max / 1000.0) / (frames_all / world / batch * FRAME_SECONDS),
        "frames_per_step": frames_all / world / args.steps,
        "config": workload,
        "e2e": {"value": e2e, "unit": "frames/s",
                "rtf": wall_max / (frames_all / world / batch * FRAME_SECONDS),
                "h2d_bytes_per_step": int(sum(r.nbytes for r in reqs) if reqs else ids.nbytes),
                "d2h_bytes_per_step": int(out.frames * 16 * 4 + 64)},
        "gpu_launches": launches_all,
        "roofline": roofline,
        "frame_roofline": {"bytes_per_frame": fb, "ms_per_frame": frame_ms,
                           "achieved": frame_gbs, "unit": "GB/s",
                           "frac": frame_gbs / peaks["hbm_gbs"], "peak_kind": peak_kind,
                           "frac_of_8tbs": frame_gbs / 8000.0},
        "clocks": clk.summary(),
        "prefill_ms": tm["prefill_ms"],
    }
    line.update(line_extra)
    if stream_stats:
        st_last = stream_stats[-len(stream_stats) // 2:] if len(stream_stats) > 1 else stream_stats
        line["streaming"] = {
            "ttfc_ms": statistics.median(x["ttfc_ms"] for x in stream_stats[args.warmup:] or stream_stats),
            "steady_rtf": statistics.median(x["steady_rtf"] for x in stream_stats[args.warmup:] or stream_stats),
            "frames_per_stream": stream_stats[-1]["frames"],
            "note": "host wall clock through the polling text-stream API; chunks of 6 frames"}
    if world == 1 and not args.no_cpu_baseline:
        fps, cf, total, cores, _ = cpu_reference_run(c, mdir, ids, args.cpu_frames, 1, 0)
        line["cpu_baseline"] = {"value": fps, "unit": "frames/s", "cores": cores, "kind": "port",
                                "sample": f"prefill P={P} + {args.cpu_frames} frames of "
                                          f"{c['frames']}, 1 run; frames/s = frames / (prefill + "
                                          f"frame time)"}
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
