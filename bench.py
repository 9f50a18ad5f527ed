#!/usr/bin/env python
"""Benchmark of the ragged continuous-batching ASR path (one JSON line on rank 0).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU)

Workload (per GPU): 512 synthetic 16 kHz clips, durations
lognormal(median 7 s, sigma 0.6) clipped to 1-35 s, Qwen3-ASR-0.6B architecture with
seeded random-init bf16 weights, max_num_seqs = 32, exactly 64 greedy tokens per
request (EOS ignored), CUDA-graph decode on. A step transcribes one slice of
``--clips-per-step`` clips through ``AsrEngine.transcribe``; K steps cover the 512.

* ``value``    audio-s/s with each clip's mel features already resident in HBM
               (device-timed with CUDA events, max over ranks, all ranks summed);
* ``e2e``      the same through the public API from host waveforms: waveform copies,
               GPU log-mel frontend and token read-back inside the timing;
* ``roofline`` the paged decode attention kernel (stream-K split with fused merge) on config 1
               (B = 32, ctx ~ U[64, 1024], 4096-block pool), timed live here with CUDA
               events around a graph of back-to-back launches over rotating KV sets that
               together exceed L2; bytes = algorithmic KV/q/out;
* ``cpu_baseline`` the CPU fp32 restatement of the upstream model (oracle/model.py)
               transcribing a bounded sample of the same workload on the host cores.

Multi-GPU: independent engine replicas (weak scaling), no collective on the data
path; torch.distributed (NCCL) is used only for barriers and the max-over-ranks
timing. ``--impl reference`` times the CPU restatement of the reference's path on
rank 0 with all host threads (other ranks exit 0). ``--impl reference-engine`` runs
the reference's own GPU engine (``qwen_asr_vllm.AsrEngine``, installed under
baseline/_ref) on the same workload for a like-for-like e2e comparison.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "audio-sec/sec at conc 32/GPU, 1–8 B200; decode-attn HBM GB/s vs 8 TB/s"
UNIT = "audio-s/s"
L2_BYTES = 126 * 2**20


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference", "reference-engine"], default="ours")
    p.add_argument("--clips", type=int, default=512)
    p.add_argument("--clips-per-step", type=int, default=128)
    p.add_argument("--concurrency", type=int, default=32)
    p.add_argument("--decode-tokens", type=int, default=64)
    p.add_argument("--decode-steps", type=int, default=4,
                   help="decode steps per CUDA-graph call (EngineConfig.decode_steps)")
    p.add_argument("--preset", default="0.6b")
    p.add_argument("--cpu-sample-clips", type=int, default=2)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--roofline-only", action="store_true",
                   help="only the config-1 paged decode op (e.g. for an ncu capture)")
    return p.parse_args()


# ------------------------------------------------------------------ plumbing


def dist_env():
    from voiceagent_b200.replicas import rank_env

    return rank_env()


def Dist():
    """The replicas' process group (NCCL; one rank per GPU)."""
    from voiceagent_b200.replicas import ReplicaGroup

    return ReplicaGroup("nccl")


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 200 ms during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus: list[int]):
        self.gpus = gpus
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.seek(0)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.file.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        os.unlink(self.file.name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        busy = [s for s in sm if s > 0.5 * max(sm)]
        return {"sm_mhz": float(np.median(busy)), "sm_max_mhz": float(max(smax)),
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peaks() -> dict:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def ncu_traffic() -> int | None:
    """Per-launch DRAM bytes of the decode op from the committed ncu summary."""
    path = REPO / "profiles" / "paged_decode_config1.md"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return int(line.split(":")[1].strip())
    return None


# ------------------------------------------------------------------ roofline


def decode_roofline(torch, device) -> dict:
    """Config 1 paged decode kernel, timed live (voiceagent_b200.microbench.decode_config1:
    CUDA events around a graph of back-to-back launches over rotating KV sets > L2)."""
    from voiceagent_b200.microbench import decode_config1

    with torch.cuda.device(device):
        r = decode_config1()
        chain = decode_config1(pdl=True)
    return {"ms": r["us"] / 1000.0, "algo_bytes": r["algo_bytes"], "sum_ctx": r["sum_ctx"],
            "l2": r["timing"], "pdl_chain_ms": chain["us"] / 1000.0}


# ----------------------------------------------------------------- workloads


def build_features(clips, frontend, torch, device=None):
    feats = []
    for c in clips:
        f = frontend(c)
        if device is not None:
            f.mel = f.mel.to(device, non_blocking=True)
        feats.append(f)
    return feats


def cpu_oracle_rate(clips, preset: str, decode_tokens: int, threads: int) -> dict:
    """Transcribe ``clips`` with the fp32 CPU restatement of the upstream model."""
    import torch

    from oracle import model as M
    from voiceagent_b200.audio.frontend import AudioFrontend
    from voiceagent_b200.checkpoint import PRESETS
    from voiceagent_b200.prompt import PromptBuilder

    torch.set_num_threads(threads)
    cfg = PRESETS[preset]
    thinker = M.OracleThinker(cfg, M.init_weights(cfg, seed=0))
    frontend = AudioFrontend(None)
    builder = PromptBuilder()
    audio_s, total_s = 0.0, 0.0
    for clip in clips:
        t0 = time.perf_counter()
        feats = frontend(clip)
        layout = builder.build(feats.num_audio_tokens, language="English")
        thinker.transcribe(feats.mel.float(), layout.token_ids, decode_tokens)
        total_s += time.perf_counter() - t0
        audio_s += feats.audio_seconds
    return {"value": audio_s / total_s, "audio_s": audio_s, "seconds": total_s}


# ----------------------------------------------------------------------- arms


def run_reference_arm(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from voiceagent_b200.workload import config3_clips

    threads = os.cpu_count() or 1
    clips = config3_clips(args.clips, seed=0)
    order = list(range(args.warmup + args.steps))
    for i in order[:args.warmup]:
        cpu_oracle_rate([clips[i]], args.preset, args.decode_tokens, threads)
    timed = cpu_oracle_rate([clips[args.warmup + i] for i in range(args.steps)], args.preset,
                            args.decode_tokens, threads)
    value = timed["value"]
    sample = (f"{args.steps} clips ({timed['audio_s']:.1f} s of audio) of the config-3 workload, one "
              f"per step, {args.decode_tokens} greedy tokens each, fp32 CPU restatement of the "
              "upstream Qwen3-ASR thinker (oracle/model.py), mel frontend included")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * timed["seconds"] / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config3 sample on host cores", "preset": args.preset,
                   "decode_tokens": args.decode_tokens},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


class _TemplateTokenizer:
    """Stands in for the checkpoint tokenizer, which does not exist offline.

    The reference engine only asks its tokenizer to encode the chat template (once per
    context/language pair), for the EOS id, and to decode output text. This returns the
    same template ids as ``voiceagent_b200.prompt`` (pinned by the reference's
    tests/test_prompt.py) so both engines see prompts of identical length; text output
    is empty. Everything after the prompt -- frontend, scheduler, model, flash-attn,
    Triton store, CUDA graphs -- is the reference's own, unmodified code.
    """

    eos_token_id = 151645

    @classmethod
    def from_pretrained(cls, *args, **kwargs):
        return cls()

    def encode(self, text: str) -> list[int]:
        from voiceagent_b200.prompt import PromptBuilder

        head, sep, tail = text.partition("<|im_start|>assistant\n")
        if not sep or "<|im_start|>system\n<|im_end|>" not in head:
            raise ValueError("template tokenizer: only the empty-context ASR template is known")
        language = tail[len("language "):].replace("<asr_text>", "") if tail else None
        return PromptBuilder().template(None, language or None)[0]

    def decode(self, ids, skip_special_tokens: bool = True) -> str:
        return ""


def run_reference_engine(args) -> None:
    """The reference's own GPU engine (``qwen_asr_vllm.AsrEngine`` from baseline/_ref) on
    the config-3 workload, for comparison with our e2e number: same seeded random
    weights (written as a safetensors checkpoint), clips, concurrency and sampling."""
    ref = Path(__file__).resolve().parent / "baseline" / "_ref"
    if not (ref / "qwen_asr_vllm").is_dir():
        print(json.dumps({"impl": "reference-engine", "unavailable":
                          "baseline/_ref is not installed (pip install --target baseline/_ref)"}))
        return
    sys.path.insert(0, str(ref))
    import torch

    import qwen_asr_vllm.prompt as ref_prompt
    from qwen_asr_vllm import AsrEngine as RefEngine
    from qwen_asr_vllm.engine.request import SamplingParams as RefSampling

    from voiceagent_b200.checkpoint import write_checkpoint
    from voiceagent_b200.workload import config3_clips, lognormal_durations

    ref_prompt.AutoTokenizer = _TemplateTokenizer
    dist = Dist()
    rank, world, local = dist.rank, dist.world, dist.local
    torch.cuda.set_device(local)
    ckpt = write_checkpoint(Path(tempfile.mkdtemp(prefix="b200asr_ref_")) / "ckpt", args.preset,
                            seed=0, weights=True)
    engine = RefEngine(model=str(ckpt), max_num_seqs=args.concurrency, max_model_len=4096,
                       max_num_batched_tokens=8192, max_audio_batch_size=args.concurrency,
                       num_kvcache_blocks=1024, device=f"cuda:{local}")
    sampling = RefSampling(max_new_tokens=args.decode_tokens, ignore_eos=True)
    clips = config3_clips(args.clips, seed=rank)
    durations = lognormal_durations(args.clips, seed=rank)
    n_slices = max(1, args.clips // args.clips_per_step)
    slices = [list(range(i * args.clips_per_step, (i + 1) * args.clips_per_step))
              for i in range(n_slices)]

    def run(i):
        return engine.transcribe([clips[j] for j in slices[i % n_slices]], language="en",
                                 sampling=sampling)

    for i in range(args.warmup):
        run(i)
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    outs = [run(i) for i in range(args.steps)]
    torch.cuda.synchronize()
    sec = time.perf_counter() - t0
    dist.barrier()
    toks = sum(len(o.output_token_ids) for batch in outs for o in batch)
    audio = float(sum(durations[j] for i in range(args.steps) for j in slices[i % n_slices]))
    sec_max = dist.max(sec)
    value = dist.sum(audio) / sec_max
    if rank == 0:
        print(json.dumps({
            "impl": "reference-engine", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1000.0 * sec_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "dtype": "bf16",
            "data": "synthetic (seeded noise + sines; random-init weights, seed 0)",
            "config": {"workload": f"{'config3' if args.preset == '0.6b' else 'config4'} "
                                   f"(Qwen3-ASR-{args.preset.upper()}) through "
                                   "qwen_asr_vllm.AsrEngine.transcribe (flash-attn + Triton, "
                                   "CUDA-graph decode), wall clock, max over ranks",
                       "preset": args.preset, "clips_per_step": args.clips_per_step,
                       "concurrency": args.concurrency, "output_tokens": toks},
        }), flush=True)
    dist.close()


def run_ours(args) -> None:
    import torch

    from voiceagent_b200 import kernels as kx
    from voiceagent_b200.checkpoint import write_checkpoint
    from voiceagent_b200.engine.engine import AsrEngine
    from voiceagent_b200.engine.request import SamplingParams
    from voiceagent_b200.profiling import TRANSFERS
    from voiceagent_b200.workload import config3_clips, lognormal_durations

    dist = Dist()
    rank, world, local = dist.rank, dist.world, dist.local
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    ckpt = write_checkpoint(Path(tempfile.mkdtemp(prefix="b200asr_")) / "ckpt", args.preset,
                            weights=False)
    engine = AsrEngine(str(ckpt), weights="random", seed=0, device=f"cuda:{local}",
                       max_num_seqs=args.concurrency, max_model_len=4096,
                       max_num_batched_tokens=8192, max_audio_batch_size=args.concurrency,
                       num_kvcache_blocks=1024, decode_steps=args.decode_steps)
    sampling = SamplingParams(max_new_tokens=args.decode_tokens, ignore_eos=True)

    clips = config3_clips(args.clips, seed=rank)
    durations = lognormal_durations(args.clips, seed=rank)
    n_steps_total = max(1, args.clips // args.clips_per_step)
    slices = [list(range(i * args.clips_per_step, (i + 1) * args.clips_per_step))
              for i in range(n_steps_total)]

    def step_slice(i):
        return slices[i % len(slices)]

    # Mel features on the host once (for the HBM-resident run), then moved to the GPU.
    from voiceagent_b200.audio.frontend import AudioFrontend

    host_feats = build_features(clips, AudioFrontend(str(ckpt)), torch)
    dev_feats = []
    for f in host_feats:
        g = type(f)(mel=f.mel.to(device=device, dtype=torch.bfloat16), mel_frames=f.mel_frames,
                    num_audio_tokens=f.num_audio_tokens, audio_seconds=f.audio_seconds)
        dev_feats.append(g)
    torch.cuda.synchronize()

    def run_features(i):
        return engine.transcribe([dev_feats[j] for j in step_slice(i)], language="en",
                                 sampling=sampling, features=True)

    def run_waveforms(i):
        return engine.transcribe([clips[j] for j in step_slice(i)], language="en",
                                 sampling=sampling)

    for i in range(args.warmup):
        run_features(i)
    torch.cuda.synchronize()

    clocks = ClockSampler(list(range(world)) if rank == 0 else [local])
    if rank == 0:
        clocks.start()
    stream = torch.cuda.current_stream()

    def timed(fn, profile_range: bool = False):
        dist.barrier()
        torch.cuda.synchronize()
        if profile_range:  # lets `ncu --profile-from-start off` capture exactly this region
            torch.cuda.cudart().cudaProfilerStart()
        launches0 = kx.LAUNCHES["count"]
        xfer0 = dict(TRANSFERS)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        outs = [fn(i) for i in range(args.steps)]
        e.record(stream)
        torch.cuda.synchronize()
        if profile_range:
            torch.cuda.cudart().cudaProfilerStop()
        dist.barrier()
        ms = s.elapsed_time(e)
        audio = sum(o.audio_seconds for batch in outs for o in batch)
        toks = sum(o.num_output_tokens for batch in outs for o in batch)
        return (ms, audio, toks, kx.LAUNCHES["count"] - launches0,
                {k: TRANSFERS[k] - xfer0[k] for k in TRANSFERS})

    ms, audio, toks, launches, _ = timed(run_features, profile_range=True)
    assert toks == sum(len(step_slice(i)) for i in range(args.steps)) * args.decode_tokens
    ms_max = dist.max(ms)
    audio_all = dist.sum(audio)
    value = audio_all / (ms_max / 1000.0)

    e2e = None
    if not args.no_e2e:
        ms_e, audio_e, _, _, xfer = timed(run_waveforms)
        ms_e_max = dist.max(ms_e)
        e2e = {"value": dist.sum(audio_e) / (ms_e_max / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": int(xfer["h2d"] / args.steps),
               "d2h_bytes_per_step": int(xfer["d2h"] / args.steps),
               "ms_per_step": ms_e_max / args.steps,
               "note": "AsrEngine.transcribe from host float32 waveforms: waveform copies "
                       "(one pinned copy per encode batch), GPU log-mel, token read-back "
                       "inside the timing"}
    clock_info = clocks.stop() if rank == 0 else None

    roof = decode_roofline(torch, device)
    peaks = measured_peaks()
    achieved = roof["algo_bytes"] / (roof["ms"] / 1000.0) / 1e9
    traffic = ncu_traffic()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = max(1, min(os.cpu_count() or 1, 32))
        res = cpu_oracle_rate(clips[:args.cpu_sample_clips], args.preset, args.decode_tokens,
                              threads)
        cpu = {"value": res["value"], "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"first {args.cpu_sample_clips} clips of the config-3 workload "
                         f"({res['audio_s']:.1f} s of audio), {args.decode_tokens} greedy tokens "
                         "each, fp32 CPU restatement of the upstream thinker (oracle/model.py), "
                         "mel frontend included"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded noise + sines; random-init weights, seed 0)",
            "config": {
                "workload": f"{'config3' if args.preset == '0.6b' else 'config4'}: "
                            f"Qwen3-ASR-{args.preset.upper()} bf16 random-init, "
                            f"max_num_seqs={args.concurrency}, "
                            f"{args.clips} clips/GPU lognormal(7 s, 0.6) in [1, 35] s, "
                            f"{args.decode_tokens} greedy tokens, CUDA-graph decode",
                "preset": args.preset,
                "clips_per_step": args.clips_per_step, "concurrency": args.concurrency,
                "audio_seconds_per_gpu": float(sum(durations[j] for i in range(args.steps)
                                                   for j in step_slice(i))),
                "parallelism": f"dp{world} (independent replicas)",
                "l2": "inputs larger than L2 (the decoder's weights, 1.2 GB for 0.6B and "
                      "3.4 GB for 1.7B, stream through every decode step)",
                "timing": "CUDA events on the engine stream, max over ranks",
            },
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                         "kernel": "paged_decode_kernel (stream-K, fused merge), config 1",
                         "duration_us": roof["ms"] * 1000.0,
                         "algorithmic_bytes": roof["algo_bytes"], "timing": roof["l2"],
                         "peak_source": f"{peaks['source']} hbm_gbs (MEASURED_PEAKS.json)",
                         # supplementary: the same launches chained with programmatic
                         # dependent launch, as the engine runs them (each launch's
                         # metadata reads and first ring overlap the previous one)
                         "pdl_chain": {
                             "duration_us": roof["pdl_chain_ms"] * 1000.0,
                             "achieved": roof["algo_bytes"] / (roof["pdl_chain_ms"] / 1000.0) / 1e9,
                             "frac": roof["algo_bytes"] / (roof["pdl_chain_ms"] / 1000.0) / 1e9
                             / peaks["hbm_gbs"]}},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if engine.model_runner.graph_runner is not None:
        engine.model_runner.graph_runner.release()
    dist.close()


def run_roofline_only() -> None:
    import torch

    roof = decode_roofline(torch, torch.device("cuda", 0))
    peaks = measured_peaks()
    achieved = roof["algo_bytes"] / (roof["ms"] / 1000.0) / 1e9
    print(json.dumps({"kernel": "paged_decode config 1", "duration_us": roof["ms"] * 1000.0,
                      "algorithmic_bytes": roof["algo_bytes"], "achieved_gbs": achieved,
                      "frac_of_measured_hbm": achieved / peaks["hbm_gbs"]}), flush=True)


def main():
    args = parse_args()
    if args.roofline_only:
        run_roofline_only()
    elif args.impl == "reference":
        run_reference_arm(args)
    elif args.impl == "reference-engine":
        run_reference_engine(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
