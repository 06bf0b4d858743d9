"""Benchmark: decoded tokens/s of the batched Qwen3 decoder step on B200.

Workload: Q8_0 weights (int8 uniform in [-127, 127], f16
scales |N(0, 0.002)|) with bf16 activations, the full Qwen3 backbone shape
(28 layers, hidden 1024, 16/8 heads, FFN 3072, vocab 151936), a queue of 256
requests with prompt lengths log-uniform over 300-8000 and geometric stop steps
(mean 600, cap 4096), decoded 32 at a time by the on-GPU continuous-batching
engine (finished slots refilled on the device, prompts prefilled in 2048-row
chunks inside decode steps).

One bench "step" = one window of `--window` device steps of that engine with
the queue and weights resident in HBM, requests admitted in the workload's
seeded (unsorted) order so that the timed windows see the steady-state mix of
context lengths; `value` = tokens emitted in the K timed
windows / their CUDA-event time (max over ranks), summed over ranks. `e2e` =
the same queue through the public host-buffer entry point (`fmd_generate`:
pinned host arena -> device, run to completion, tokens -> host), wall clock.
The working set (0.63 GB weights + ~10 GB KV) is far larger than L2, so no L2
flush is needed between steps.

`--impl reference` times the CPU restatement of the reference decoder
(oracle/, a PyTorch fp32 port of qwen3.rs; the Rust/candle original cannot be
built here) on a bounded decode sample of the same workload.

Multi-GPU (torchrun): one process per GPU, each with its own seeded config-3
queue (request-level data parallelism, no collective on the hot path);
`scaling` is "weak".
"""

from __future__ import annotations

import argparse
import json
import math
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

import __graft_entry__  # noqa: E402

METRIC = "decoded tokens/s per GPU (Q8_0, bf16) and % of HBM roofline; audio s/s"
UNIT = "tokens/s"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
TRAFFIC_FILE = ROOT / "profiles" / "attn_decode_config3.md"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--window", type=int, default=128, help="device steps per bench step")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--requests", type=int, default=0,
                    help="requests per GPU (configs 2, 3) or in total (config 5); 0: the workload's own")
    ap.add_argument("--batch", type=int, default=0, help="0: the workload's batch (8, 32 or 64)")
    ap.add_argument("--e2e-requests", type=int, default=256,
                    help="the e2e leg runs the first N requests of the shard (the whole shard of configs 2, 3)")
    ap.add_argument("--chunk", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--max-new", type=int, default=4096,
                    help="cap on max_new_tokens per request (bounds the KV pool for profiling runs)")
    ap.add_argument("--workload", choices=["2", "3", "4", "5", "encoder"], default="3",
                    help="3: the headline queue (BASELINE config 3); 2: config 2 (dense bf16, batch 8, forced end "
                         "of turn); 5: config 5 (Q8_0, batch 64 per GPU, one 2048-request queue over the GPUs); "
                         "4: config 4 (chunked prefill of 8 x 16k prompts mixed with 24 decoding sequences), a "
                         "separate report; encoder: the Whisper encoder + adaptor over 30 s mel chunks "
                         "(MossModel::encode_audio), a separate report")
    ap.add_argument("--chunks", type=int, default=64, help="mel chunks per step of --workload encoder")
    ap.add_argument("--precision", default="int8_bf16", help="precision of the --workload 4 report")
    return ap.parse_args()


# ---- distributed plumbing ----------------------------------------------------------
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def reduce(self, value: float, op: str) -> float:
        if not self.pg:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64, device=f"cuda:{self.local}")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX if op == "max" else self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# ---- clocks -----------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None, "samples": len(sm), "reasons": sorted(reasons)}


def load_peaks() -> tuple[float, str]:
    try:
        return float(json.loads(PEAKS_FILE.read_text())["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def traffic_per_kv_token() -> float | None:
    """DRAM bytes per key position of one decode-attention launch, from the
    committed ncu summary (line `traffic_bytes_per_kv_token: X`)."""
    try:
        for ln in TRAFFIC_FILE.read_text().splitlines():
            if ln.strip().startswith("traffic_bytes_per_kv_token:"):
                return float(ln.split(":", 1)[1])
    except OSError:
        pass
    return None


# ---- model + workload ---------------------------------------------------------------------
# Request-queue workloads (3, 5): precision, requests per
# GPU (weak scaling) or in total (strong), the prior mean generation length
# the partitioner may use (the workload's configured mean, never the drawn
# stop steps, which a server cannot know), and the description.
WORKLOADS = {
    "2": dict(precision="bf16", requests=64, per_gpu=True, mean_new=384,
              desc="BASELINE config 2: dense bf16 decoder, batch 8, prompts log-uniform 1.2k-5k, forced end of "
                   "turn at a step drawn uniformly from 256-512 (queue of 8-request rounds), bf16 KV cache"),
    "3": dict(precision="int8_bf16", requests=256, per_gpu=True, mean_new=600,
              desc="BASELINE config 3: Q8_0 decoder + lm_head, bf16 activations, batch 32 continuous batching over "
                   "a 256-request queue (prompts log-uniform 300-8000, geometric stops mean 600 cap 4096), on-GPU "
                   "refill, 2048-row prefill chunks"),
    "5": dict(precision="int8_bf16", requests=2048, per_gpu=False, mean_new=800,
              desc="BASELINE config 5: Q8_0 + bf16, batch 64 per GPU, one 2048-request queue (prompts log-uniform "
                   "300-16k, geometric stops mean 800 cap 4096) length-balanced over the GPUs"),
}


def build_model_and_queue(args, rank: int, world: int = 1):
    """Model and this rank's request queue. Configs 2 and 3 scale weakly:
    every GPU serves the same `args.requests`-request queue as a one-GPU run
    (the same lengths, budgets and stops; prompt rows seeded per rank), so a
    GPU's work does not change with N and the timed windows of every rank see
    the same mix of context lengths. Config 5 is one queue split over the
    GPUs (strong scaling): every rank derives the same LPT partition
    (fmd_b200.dp) from prompt lengths, budgets and the workload's prior mean
    generation length, never the drawn stop steps, and builds prompt
    embeddings for its own shard only."""
    pkg = __graft_entry__.load_package()
    import importlib

    syn = importlib.import_module("fmd_b200.synthetic")
    dp = importlib.import_module("fmd_b200.dp")
    spec = WORKLOADS[args.workload]
    cfg = pkg.TextConfig(num_hidden_layers=args.layers)
    q8 = spec["precision"].startswith("int8")
    w = syn.make_weights(cfg, seed=args.seed, prequantized=q8)
    n_req = args.requests or spec["requests"]
    glob = syn.workload(int(args.workload), cfg, w["embed"], seed=args.seed, n_requests=n_req, with_arena=False)
    glob.max_new = np.minimum(glob.max_new, args.max_new)
    if spec["per_gpu"]:
        wl = glob
    else:
        prior = np.full(len(glob.prompt_lens), spec["mean_new"])
        part = dp.partition(glob.prompt_lens, glob.max_new, world, expected_new=prior)
        wl = glob.subset(part.shard(rank))
    wl.arena = syn.build_prompt_arena(cfg, w["embed"], wl.prompt_lens, args.seed + 7 * 3 + 1000 * rank,
                                      out_bf16=True)
    return pkg, cfg, w, wl


CPU_LENS = [412, 797, 1190, 1500]  # BASELINE config 1's prompts


def cpu_sample(cfg, w, seconds: float = 15.0, steps: int | None = None, warmup: int = 0):
    """The reference's CPU decode path on the host cores: precision f32 (the
    only CPU precision, precision.rs:60-68), the four config-1 prompts decoded
    together as `Engine::generate_batch` does (left-padded batch, shared
    positions plus the padding mask, engine.rs:476-538, qwen3.rs:499-511),
    restated by the oracle. Weights given as Q8_0 are dequantised to their
    exact f32 values. KV caches are pre-filled with seeded values at the
    padded length (prefill not timed); each step is one batched decode of 4
    tokens."""
    import torch

    from oracle import q8_0
    from oracle import qwen3_ref as ref

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    if "q8" in w:  # the f32 values of the Q8_0 projections
        layers = []
        for lw, qw in zip(w["layers"], w["q8"]["layers"]):
            d = dict(lw)
            for k in ("q", "k", "v", "o", "gate", "up", "down"):
                d[k] = q8_0.dequantize(*qw[k])
            layers.append(d)
        w = dict(w, layers=layers, lm_head=q8_0.dequantize(*q8_0.quantize(w["embed"])))
    tmax = max(CPU_LENS)
    model = ref.Qwen3Ref(ref.TextConfig(**cfg.oracle_kwargs()), w, "f32", max_len=tmax + 128)
    rng = torch.Generator().manual_seed(7)
    caches = model.new_caches(len(CPU_LENS), tmax + 96)
    pads = [tmax - n for n in CPU_LENS]
    for c in caches:
        c.k[:, :, :tmax] = torch.randn(c.k[:, :, :tmax].shape, generator=rng)
        c.v[:, :, :tmax] = torch.randn(c.v[:, :, :tmax].shape, generator=rng)
        c.len = tmax
    tok = [int(t) for t in np.random.default_rng(3).integers(0, cfg.vocab_size, len(CPU_LENS))]

    def one_step():
        lg = model.decode_step_padded(tok, caches, pads)
        tok[:] = ref.argmax_rows(lg)

    for _ in range(warmup):
        one_step()
    t0 = time.perf_counter()
    done = 0
    while True:
        one_step()
        done += 1
        el = time.perf_counter() - t0
        if (steps is not None and done >= steps) or (steps is None and (el >= seconds or done >= 64)):
            break
    el = time.perf_counter() - t0
    n = len(CPU_LENS)
    return {"value": n * done / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{done} batched greedy decode steps of the 4 BASELINE config-1 prompts (lengths {CPU_LENS}, "
                      f"left-padded to {tmax} as engine.rs:476-491 does, KV caches pre-filled with seeded values, "
                      f"prefill not timed), {cfg.num_hidden_layers}-layer model in f32 (the reference's CPU precision, "
                      f"precision.rs:60-68; Q8_0 weights dequantised to f32), oracle restatement of qwen3.rs / "
                      f"engine.rs on torch with {threads} threads",
            "seconds": el}


def workload_config(args, cfg, n_requests: int, world: int) -> dict:
    """The `config` object both arms report."""
    spec = WORKLOADS[args.workload]
    if spec["per_gpu"]:
        scale = f"every GPU serves the one-GPU {n_requests}-request queue (prompt rows seeded per GPU)"
        part = "none (weak scaling: the same queue per GPU)"
    else:
        scale = f"LPT request shards of one {spec['requests'] if not args.requests else args.requests}-request queue"
        part = (f"greedy LPT on prompt length + budget + the workload's prior mean generation length "
                f"({spec['mean_new']} tokens); drawn stop steps are not read")
    return {"workload": spec["desc"], "precision": spec["precision"],
            "requests_per_gpu": n_requests, "batch": args.batch, "prefill_chunk": args.chunk,
            "arrival": "seeded workload order for the timed windows; e2e through Engine.generate "
                       "(length-sorted queue, engine.rs:385)",
            "layers": cfg.num_hidden_layers, "step": f"{args.window} device steps",
            "l2": "working set >> L2 (no flush needed)",
            "partition": part,
            "parallelism": f"dp{world} ({scale}, no collective)"}


def run_reference(args):
    """`--impl reference`: the reference's CPU path (restated) on a bounded
    sample; rank 0 alone, the other ranks exit at once."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    pkg = __graft_entry__.load_package()
    import importlib

    syn = importlib.import_module("fmd_b200.synthetic")
    cfg = pkg.TextConfig(num_hidden_layers=args.layers)
    w = syn.make_weights(cfg, seed=args.seed, prequantized=WORKLOADS[args.workload]["precision"].startswith("int8"))
    res = cpu_sample(cfg, w, steps=max(args.steps, 1), warmup=max(args.warmup, 0))
    args.batch = args.batch or {"2": 8, "3": 32, "5": 64}[args.workload]
    args.chunk = args.chunk or 2048
    n_req = args.requests or WORKLOADS[args.workload]["requests"]
    line = {"metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 * res["seconds"] / max(args.steps, 1),
            "higher_is_better": True, "scaling": "weak" if WORKLOADS[args.workload]["per_gpu"] else "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": dict(workload_config(args, cfg, n_req, args.gpus),
                           sample="batched decode steps of the 4 config-1 prompts (see cpu_baseline.sample)"),
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_config4(args):
    """BASELINE config 4 on one GPU: 24 sequences decode while 8 prompts of
    16,384 rows are prefilled in 2,048-row chunks inside the same steps. The
    24 decoders' prompts are prefilled first (untimed); the timed windows are
    the steps that prefill the long prompts. Reports prefill rows/s, decoded
    tokens/s and the tensor-core work rate of the prefill rows (projection
    GEMMs + causal attention) against the measured bf16 peak."""
    import importlib

    pkg = __graft_entry__.load_package()
    syn = importlib.import_module("fmd_b200.synthetic")
    cfg = pkg.TextConfig(num_hidden_layers=args.layers)
    prec = args.precision
    w = syn.make_weights(cfg, seed=args.seed, prequantized=prec.startswith("int8"))
    wl = syn.workload(4, cfg, w["embed"], seed=args.seed, out_bf16=True)
    n_dec = wl.meta["n_decoders"]
    dec = pkg.Qwen3Decoder(cfg, prec, device=0)
    dec.load_weights(w)
    dec.reserve(max_slots=32, max_tokens=int(np.sum(wl.prompt_lens + wl.max_new + 64)), max_rows=32 + 2048)
    eng = pkg.Engine(dec)
    eng.load(wl.prompt_lens, wl.max_new, wl.forced_stop, wl.arena, sort_by_length=False)
    eng.start(32, 2048)
    dec_rows = int(np.sum(wl.prompt_lens[:n_dec]))
    long_len = int(wl.prompt_lens[-1])
    def advance(prev):
        # the engine reports FMD_ETIMEDOUT after 4 polls without progress
        # (over consecutive calls), so a stalled queue ends the run
        return eng.step(16)

    st = advance(None)
    while st.prefill_tokens < dec_rows + 2048:  # decoders running, long prefill under way (warm-up)
        st = advance(st)
    clocks = ClockSampler(0)
    clocks.start()
    t_ms = p_rows = d_tok = steps = mixed = 0
    attn_pos = 0.0
    p0 = st.prefill_tokens
    while st.prefill_tokens < dec_rows + 8 * long_len:
        before = st.prefill_tokens
        st = advance(st)
        t_ms += st.window_device_ms
        d_tok += st.window_tokens
        steps += st.window_steps
        mixed += st.window_mixed_steps
        # causal attention work of the long-prompt rows prefilled in this window:
        # a row at offset o of its prompt attends to o + 1 keys
        for o in range(before - dec_rows, st.prefill_tokens - dec_rows):
            attn_pos += (o % long_len) + 1
    clk = clocks.stop()
    p_rows = st.prefill_tokens - p0
    lin_params = cfg.n_params(with_head=False)  # the projections, lm_head excluded
    per_pos = 4 * cfg.num_attention_heads * cfg.head_dim * cfg.num_hidden_layers
    flops = 2.0 * lin_params * p_rows + per_pos * attn_pos
    secs = t_ms / 1000.0
    peaks = json.loads(PEAKS_FILE.read_text()) if PEAKS_FILE.exists() else {}
    peak = float(peaks.get("bf16_tflops_sustained", 1381.0))
    line = {"metric": "config 4: prefill rows/s and decoded tokens/s of mixed steps", "workload":
            "BASELINE config 4: 8 x 16,384-row prompts prefilled in 2,048-row chunks while 24 sequences "
            "(contexts log-uniform 1k-8k) decode, batch 32", "precision": prec, "layers": cfg.num_hidden_layers,
            "timed_steps": int(steps), "mixed_steps": int(mixed), "ms_per_step": t_ms / max(steps, 1),
            "prefill_rows_per_s": p_rows / secs, "decode_tokens_per_s": d_tok / secs,
            "prefill_tflops_per_s": flops / secs / 1e12,
            "prefill_tensor_frac": flops / secs / 1e12 / peak, "peak_tflops": peak,
            "peak_kind": "measured sustained bf16 (cuBLAS)",
            "note": "time of whole steps (the 24 decode rows included) against the prefill rows' FLOPs",
            "clocks": clk}
    print(json.dumps(line), flush=True)
    dec.close()


def run_encoder(args):
    """The audio tower (Whisper-Medium encoder, 24 layers, + VQ adaptor) over
    `--chunks` 30 s log-mel chunks per step, as `MossModel::encode_audio` runs
    them (encoder batches of 16 chunks, model/mod.rs:20-23): 8 audios, each
    with full 375-token chunks and a 125-token final chunk. `value` = chunks/s
    with the mel resident on the device (CUDA events around each call's device
    work); `e2e` = the same through the host API, wall-clock (f32 mel in host
    memory, the embeddings copied back to the host). The CPU baseline runs the f32 oracle on one chunk."""
    import torch

    pkg = __graft_entry__.load_package()
    from oracle.whisper_ref import AudioConfig as RefConfig
    from oracle.whisper_ref import WhisperRef, random_audio_weights

    cfg = pkg.AudioConfig()
    w = random_audio_weights(RefConfig(**cfg.oracle_kwargs()), args.seed)
    n = args.chunks
    per_audio = max(1, n // 8)
    tokens = [cfg.tokens_per_chunk if (i + 1) % per_audio else 125 for i in range(n)]
    mapping = [min(i // per_audio, 7) for i in range(n)]
    n_audios = max(mapping) + 1
    mel = np.random.default_rng(args.seed + 1).standard_normal((n, cfg.num_mel_bins, cfg.mel_frames),
                                                               dtype=np.float32)
    prec = "bf16" if args.precision == "int8_bf16" else args.precision
    enc = pkg.AudioEncoder(cfg, w, prec, device=0, max_batch=16)
    mel_dev = torch.from_numpy(mel).cuda()
    out, off = enc.encode_audio_device(mel_dev, tokens, mapping, n_audios)
    for _ in range(args.warmup):
        enc.encode_audio_device(mel_dev, tokens, mapping, n_audios, out=out)
    clocks = ClockSampler(0)
    clocks.start()
    dev_ms, kernels = [], 0
    for _ in range(args.steps):
        enc.encode_audio_device(mel_dev, tokens, mapping, n_audios, out=out)
        ms, k = enc.last_timing()
        dev_ms.append(ms)
        kernels += k
    clk = clocks.stop()
    e2e_s = []
    for _ in range(max(2, args.steps // 2)):
        t0 = time.perf_counter()
        emb, _ = enc.encode_audio_device(mel, tokens, mapping, n_audios)  # host mel in
        host = emb.cpu()  # embeddings out (activation dtype)
        e2e_s.append(time.perf_counter() - t0)
    # the whole audio path from host waveforms: chunk planning, GPU log-mel, encoder + adaptor
    fcfg = pkg.FeatureConfig()
    rng = np.random.default_rng(args.seed + 2)
    secs = [30.0 * per_audio - 20.0] * n_audios  # per_audio chunks, the last one 10 s long
    waves = [(0.1 * rng.standard_normal(int(16_000 * s))).astype(np.float32) for s in secs]
    fe = pkg.MelFrontend(fcfg)
    feats = pkg.extract_features(waves, fcfg, fe, cfg.audio_merge_size)
    torch.cuda.synchronize()
    wav_s, mel_ms = [], []
    for _ in range(max(2, args.steps // 2)):
        t0 = time.perf_counter()
        feats = pkg.extract_features(waves, fcfg, fe, cfg.audio_merge_size)
        t1 = time.perf_counter()
        emb, _ = enc.encode_audio_device(feats.mel, feats.chunk_token_lengths, feats.chunk_mapping, n_audios)
        host_w = emb.cpu()
        wav_s.append(time.perf_counter() - t0)
        mel_ms.append((t1 - t0) * 1000.0)
    fe.close()
    mean_ms = float(np.mean(dev_ms))
    flops = pkg.audio.encoder_flops(cfg, n)
    peaks = json.loads(PEAKS_FILE.read_text()) if PEAKS_FILE.exists() else {}
    peak = float(peaks.get("bf16_tflops_sustained", 1381.0))
    achieved = flops / (mean_ms / 1000.0) / 1e12
    cpu = None
    if not args.no_cpu:
        ref = WhisperRef(RefConfig(**cfg.oracle_kwargs()), w)
        torch.set_num_threads(os.cpu_count() or 1)
        t0 = time.perf_counter()
        ref.encode_audio(mel[:1], tokens[:1], [0], 1)
        cpu_s = time.perf_counter() - t0
        cpu = {"value": 1.0 / cpu_s, "unit": "chunks/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": "one 30 s chunk through the f32 oracle (24 encoder layers + adaptor), torch on the "
                         "host cores"}
    e2e_mean = float(np.mean(e2e_s))
    line = {"metric": "audio encoder chunks/s (Whisper-Medium encoder + VQ adaptor, 30 s chunks)",
            "value": n / (mean_ms / 1000.0), "unit": "chunks/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": mean_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": prec, "data": "synthetic (seeded N(0,1) mel, random-init weights)",
            "audio_seconds_per_s": 30.0 * n / (mean_ms / 1000.0),
            "config": {"workload": f"encode_audio over {n} chunks of 30 s (8 audios, final chunk of each 125 "
                                   "tokens), encoder batch 16, 24 layers d_model 1024 heads 16 ffn 4096, "
                                   "adaptor 4096->1024->1024", "chunks": n, "encoder_batch": 16,
                       "l2": "working set >> L2 (no flush needed)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None,
                         "note": "whole encode_audio call (all kernels) against the measured sustained bf16 "
                                 "peak; FLOPs = conv + 24 x (projections + attention) + adaptor"},
            "e2e": {"value": n / e2e_mean, "unit": "chunks/s", "h2d_bytes_per_step": int(mel.nbytes),
                    "d2h_bytes_per_step": int(host.numel() * host.element_size())},
            "e2e_from_waveforms": {"value": feats.n_chunks / float(np.mean(wav_s)), "unit": "chunks/s",
                                   "chunks": feats.n_chunks, "extract_features_ms": float(np.mean(mel_ms)),
                                   "h2d_bytes_per_step": int(sum(w.nbytes for w in waves)),
                                   "d2h_bytes_per_step": int(host_w.numel() * host_w.element_size()),
                                   "note": "host waveforms in (chunk planning + zero-padded windows on the host, "
                                           "log-mel on the GPU), embeddings out; wall clock"},
            "gpu_launches": int(kernels), "cpu_baseline": cpu, "clocks": clk}
    print(json.dumps(line), flush=True)
    enc.close()


def main():
    args = parse_args()
    if args.workload == "encoder":
        run_encoder(args)
        return
    if args.workload == "4":
        run_config4(args)
        return
    if args.impl == "reference":
        run_reference(args)  # host cores only: no process group
        return
    dist = Dist()

    pkg, cfg, w, wl = build_model_and_queue(args, dist.rank, dist.world)
    args.batch = args.batch or wl.max_batch
    args.chunk = args.chunk or wl.prefill_chunk
    dec = pkg.Qwen3Decoder(cfg, wl.precision, device=dist.local)
    dec.load_weights(w)
    top = np.sort(wl.prompt_lens)[-args.batch:]
    pool_tokens = int(np.sum(top + int(np.max(wl.max_new)) + 64))
    dec.reserve(max_slots=args.batch, max_tokens=pool_tokens, max_rows=args.batch + args.chunk)
    eng = pkg.Engine(dec)
    forced = wl.forced_stop
    # requests arrive in the workload's seeded order (no length sort): the
    # continuous-batching steady state of a serving queue, so the timed
    # windows see the workload's mix of context lengths
    eng.load(wl.prompt_lens, wl.max_new, forced, wl.arena, sort_by_length=False)
    eng.start(args.batch, args.chunk)

    # warm-up windows (untimed), then K timed windows
    for _ in range(args.warmup):
        eng.step(args.window)
    dist.barrier()
    clocks = ClockSampler(dist.local)
    clocks.start()
    wins = []
    for _ in range(args.steps):
        st = eng.step(args.window)
        wins.append(st)
        if st.window_steps == 0:
            break
    clk = clocks.stop()
    dist.barrier()
    tokens = sum(s.window_tokens for s in wins)
    dev_ms = sum(s.window_device_ms for s in wins)
    steps_run = sum(s.window_steps for s in wins)
    mixed_run = sum(s.window_mixed_steps for s in wins)
    tot_tokens = dist.reduce(float(tokens), "sum")
    max_ms = dist.reduce(dev_ms, "max")
    value = tot_tokens / (max_ms / 1000.0) if max_ms > 0 else 0.0

    # dominant kernel: decode attention (CUDA events around the middle layer's
    # launch in the last step of every timed window)
    peak, peak_kind = load_peaks()
    samples = [(s.attn_kv_tokens, s.attn_decode_ms, s.attn_rows) for s in wins if s.attn_decode_ms > 0]
    kv_per_launch = statistics.mean(x[0] for x in samples) if samples else 0.0
    ms_per_launch = statistics.mean(x[1] for x in samples) if samples else 0.0
    rows = statistics.mean(x[2] for x in samples) if samples else 0.0
    kvh, hd, hq = cfg.num_key_value_heads, cfg.head_dim, cfg.num_attention_heads
    alg_bytes = kv_per_launch * kvh * hd * 2 * 2 + rows * hq * hd * 2 * 2
    achieved = alg_bytes / (ms_per_launch / 1000.0) / 1e9 if ms_per_launch > 0 else 0.0
    tpk = traffic_per_kv_token()
    # the lm_head launch of each window's last step: its weights (Q8_0: 34
    # bytes per 32 values) and the sampled rows in
    lm_ms = [s.lm_head_ms for s in wins if s.lm_head_ms > 0]
    lm_ms = statistics.mean(lm_ms) if lm_ms else 0.0
    lm_bytes = cfg.vocab_size * cfg.hidden_size * (34 / 32 if wl.precision.startswith("int8") else 2) \
        + rows * cfg.hidden_size * 2
    lm_gbs = lm_bytes / (lm_ms / 1000.0) / 1e9 if lm_ms > 0 else 0.0

    # whole-step HBM roofline at the measured mean context
    w_bytes = cfg.n_params() * (34 / 32 if wl.precision.startswith("int8") else 2)
    mean_kv = kv_per_launch
    step_bytes = w_bytes + mean_kv * cfg.kv_bytes_per_token() + rows * cfg.kv_bytes_per_token()
    step_ms = dev_ms / max(steps_run, 1)

    e2e = None
    if not args.no_e2e:
        import torch

        # configs 2 and 3: the whole shard; config 5: its first --e2e-requests
        # requests (the whole 2048-request queue on one GPU runs for minutes)
        sub = wl if WORKLOADS[args.workload]["per_gpu"] else wl.subset(np.arange(min(args.e2e_requests,
                                                                                       len(wl.prompt_lens))))
        if sub is not wl:
            rows = int(np.sum(sub.prompt_lens))
            sub.arena = wl.arena[:rows]  # the shard's first requests sit first in its arena
        arena_pinned = torch.from_numpy(sub.arena).pin_memory()
        arena_np = arena_pinned.numpy()
        eng2 = pkg.Engine(dec)
        dist.barrier()
        t0 = time.perf_counter()
        out, st2 = eng2.generate(sub.prompt_lens, sub.max_new, sub.forced_stop, arena_np, max_batch=args.batch,
                                 prefill_chunk=args.chunk)
        el = time.perf_counter() - t0
        gen = sum(len(o.tokens) for o in out)
        tot = dist.reduce(float(gen), "sum")
        el_max = dist.reduce(el, "max")
        h2d = sub.arena.nbytes + 24 * len(sub.prompt_lens)
        d2h = 4 * len(sub.prompt_lens) * int(np.max(sub.max_new)) + 8 * len(sub.prompt_lens)
        # audio transcribed: each prompt's N(0,1) span stands for audio at the
        # reference's 12.5 audio tokens per second (16 kHz / (hop 160 x encoder
        # stride 2 x merge 4), config.rs:210-223)
        audio_s = dist.reduce(float(sum(round(0.75 * int(n)) for n in sub.prompt_lens)) / 12.5, "sum")
        e2e = {"value": tot / el_max, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "step": f"whole queue ({len(sub.prompt_lens)} requests per GPU) through fmd_generate (pinned host "
                       f"arena in, tokens out)",
               "seconds": el_max, "tokens": int(tot),
               "audio_seconds_per_s": audio_s / el_max,
               "audio_seconds_note": "decoder only: audio-span rows of the queue's prompts / 12.5 tokens per s, "
                                     "over the whole-queue wall time; the audio tower's own rate is "
                                     "bench.py --workload encoder"}

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = cpu_sample(cfg, w)
        cpu.pop("seconds", None)

    if dist.rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world, "steps": len(wins),
            "warmup": args.warmup, "ms_per_step": max_ms / max(len(wins), 1), "higher_is_better": True,
            "scaling": "weak" if WORKLOADS[args.workload]["per_gpu"] else "strong", "vs_baseline": None,
            "dtype": {"bf16": "bf16 activations, bf16 weights", "int8_bf16": "bf16 activations, Q8_0 weights"}[
                wl.precision], "data": "synthetic",
            "config": dict(workload_config(args, cfg, len(wl.prompt_lens), dist.world),
                           device_steps_timed=int(steps_run)),
            "roofline": {"bound": "hbm", "kernel": "k_attn_decode (split-KV GQA decode attention)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": (tpk * kv_per_launch) if tpk else None, "peak_kind": peak_kind,
                         "alg_bytes_per_launch": alg_bytes, "ms_per_launch": ms_per_launch},
            "lm_head": {"kernel": "k_lm_head_tc (tcgen05, Q8_0)" if wl.precision.startswith("int8") and
                        os.environ.get("FMD_LM_HEAD_TC") == "1" and args.batch <= 64 else "k_lm_head (mma.sync)",
                        "ms_per_launch": lm_ms, "alg_bytes_per_launch": lm_bytes, "achieved_gbs": lm_gbs,
                        "frac": lm_gbs / peak if peak else None},
            "step_roofline": {"bytes_per_step": step_bytes, "ms_per_step": step_ms,
                              "achieved_gbs": step_bytes / (step_ms / 1000.0) / 1e9 if step_ms > 0 else 0.0,
                              "frac": (step_bytes / (step_ms / 1000.0) / 1e9) / peak if step_ms > 0 else 0.0,
                              "mean_decode_rows": rows, "mean_kv_positions": mean_kv},
            "clocks": clk,
            "e2e": e2e,
            "cpu_baseline": cpu,
            # kernel nodes of the two captured step graphs (counted by the library) x their replays
            "gpu_launches": int(mixed_run * wins[-1].graph_kernels_mixed
                                + (steps_run - mixed_run) * wins[-1].graph_kernels_decode),
            "kernels_per_step": {"decode_only": wins[-1].graph_kernels_decode,
                                 "with_prefill": wins[-1].graph_kernels_mixed},
            "mixed_steps_timed": int(mixed_run),
            "tokens_timed": int(tot_tokens),
        }
        print(json.dumps(line), flush=True)
    dec.close()
    dist.close()


if __name__ == "__main__":
    main()
