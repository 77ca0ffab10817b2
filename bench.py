#!/usr/bin/env python
"""Forward + loss throughput of the rustane transformer on B200.

Workload (default): 600m-A (1536d / 4096h / 20L / 12 heads x 128, vocab 8192,
tied head), seq 512, global batch 64 sequences of uniform random tokens,
sharded by sequence over the GPUs (no communication; total work fixed:
strong scaling). Weights ~N(0, 0.02) generated on the device, RMSNorm gains 1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Rank 0 prints one JSON line. Phases (ours):
  1. timed region (value): K forwards from device-resident tokens through
     cb_forward_loss_async (CUDA graph), CUDA events on the bridge's stream,
     barrier + synchronize on both sides, max over ranks;
  2. profiled pass: the same K forwards with CUDA events around every kernel
     (per-kernel durations for the roofline);
  3. e2e pass: K calls of the public host API cb_forward_loss with pinned host
     tokens/targets (H2D copy + forward + D2H loss inside the timed region);
  4. CPU baseline (rank 0, N = 1): the CPU oracle on a bounded sample.
--impl reference times the reference's forward math on the host cores (the CPU
restatement under oracle/; the Rust reference cannot be built here).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "forward tokens/sec (ms/forward, seq512) at 1/2/4/8 B200; % of fp16 TC peak"
GEMM_CLASSES = ("gemm_qkv_rope", "gemm_o", "gemm_w13_swiglu", "gemm_w2", "gemm_lmhead_ce")
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per GEMM launch, averaged
# over the 81 GEMM launches of one forward, from one ncu capture of this bench's own
# workload (profiles/gemm_tc_600m-A_b64_dram.md), keyed by (config, sequences per GPU).
GEMM_TRAFFIC_PER_LAUNCH = {("600m-A", 64): 520.96e6}
GEMM_TRAFFIC_SOURCE = "profiles/gemm_tc_600m-A_b64_dram.md"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--config", default="600m-A")
    p.add_argument("--global-batch", type=int, default=None,
                   help="sequences per step for the whole job (default 64; 16 for 32B)")
    p.add_argument("--tp", action="store_true",
                   help="tensor parallelism over all ranks (Megatron split; the exchange is "
                        "set by CB_TP_REDUCE, sequence-parallel fp16 by default) instead of "
                        "sequence sharding")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--cpu-budget-s", type=float, default=12.0,
                   help="CPU-baseline sample budget (seconds of oracle work)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--decode-batch", type=int, default=64,
                   help="sequences decoded together (--workload decode)")
    p.add_argument("--attn-shape", default=None,
                   help="batch,heads,seq for --workload attention (default: the config's "
                        "heads and seq at --global-batch sequences)")
    p.add_argument("--workload", choices=("forward", "train", "decode", "validate", "rstk-load",
                                          "attention"),
                   default="forward",
                   help="forward: the headline forward+loss step; train: one training step "
                        "(forward + backward into fp32 gradients); validate: the evaluation "
                        "loop over an HBM-resident uint16 token file (val_loss + val_bpb); "
                        "rstk-load: RSTK checkpoint file -> fp16 device weights (1 GPU); "
                        "decode: single-token steps with a KV cache after a prefill (1 GPU); "
                        "attention: the causal attention kernel alone (cb_attention_f16, 1 GPU)")
    return p.parse_args()


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during a region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.6)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def host_threads() -> int:
    """Every core this process may run on (torchrun's OMP_NUM_THREADS=1 is ignored
    on purpose: the CPU legs use the whole host)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_oracle_sample(cfg, seed, tok, tgt, budget_s):
    """Time the CPU oracle on whole sequences until budget_s is spent."""
    from oracle import oracle
    oracle.set_threads(host_threads())
    model = oracle.OracleModel(cfg, seed=seed, scheme=oracle.SCHEME_NORMAL, sigma=0.02)
    threads = oracle.max_threads()
    n_done, elapsed, losses = 0, 0.0, []
    n_avail = tok.size // cfg.seq
    while n_done < n_avail and (n_done == 0 or elapsed < budget_s):
        s = slice(n_done * cfg.seq, (n_done + 1) * cfg.seq)
        t0 = time.perf_counter()
        loss, _, _ = model.forward(tok[s], tgt[s])
        elapsed += time.perf_counter() - t0
        losses.append(loss)
        n_done += 1
    torch_s = torch_cpu_seconds(model, tok[:n_done * cfg.seq], tgt[:n_done * cfg.seq])
    return dict(seqs=n_done, seconds=elapsed, threads=threads, losses=losses,
                torch_seconds=torch_s)


def torch_cpu_seconds(model, tok, tgt):
    """Seconds for torch's own CPU kernels (float32, fused causal attention; the
    optional second CPU figure) to run the same sequences one call each, as the
    reference's forward takes one sequence per call, after one untimed call. An
    optional figure: a failure comes back as its message, not as an exception."""
    try:
        return _torch_cpu_seconds(model, tok, tgt)
    except Exception as e:  # noqa: BLE001
        return f"torch CPU forward failed: {type(e).__name__}: {e}"


def _torch_cpu_seconds(model, tok, tgt):
    import torch
    from oracle import torch_ref
    torch.set_num_threads(host_threads())
    seq = model.cfg.seq
    with torch.inference_mode():
        torch_ref.forward(model, tok[:seq], tgt[:seq], dtype=torch.float32,
                          fused_attention=True)
        t0 = time.perf_counter()
        for i in range(tok.size // seq):
            s = slice(i * seq, (i + 1) * seq)
            torch_ref.forward(model, tok[s], tgt[s], dtype=torch.float32, fused_attention=True)
        return time.perf_counter() - t0


def cpu_oracle_extrapolated(cfg, seed, tok, tgt):
    """For models too deep to push a whole sequence through the CPU oracle inside the
    bench's time box: time one sequence through 1-layer and 2-layer variants of the
    same width (weights from the same generator), the faster of two passes each after
    an untimed one, and extrapolate linearly in depth, t(L) = t(1) + (L - 1) * (t(2) - t(1)). The
    embedding, final norm, head and CE are in t(1) once; every layer costs the same."""
    from oracle import oracle
    oracle.set_threads(host_threads())
    s = slice(0, cfg.seq)
    models = {nl: oracle.OracleModel(cfg.replace(nlayers=nl), seed=seed,
                                     scheme=oracle.SCHEME_NORMAL, sigma=0.02) for nl in (1, 2)}
    for m in models.values():
        m.forward(tok[s], tgt[s])
    t = {nl: float("inf") for nl in models}
    for _ in range(2):  # the faster of two passes: the difference of two times is noisy
        for nl, m in models.items():
            t0 = time.perf_counter()
            m.forward(tok[s], tgt[s])
            t[nl] = min(t[nl], time.perf_counter() - t0)
    tt = {}
    for nl, m in models.items():
        runs = [torch_cpu_seconds(m, tok[s], tgt[s]) for _ in range(2)]
        failed = [x for x in runs if isinstance(x, str)]
        tt[nl] = failed[0] if failed else min(runs)
    del models

    def depth(t):
        return t[1] + (cfg.nlayers - 1) * max(t[2] - t[1], 0.0)

    bad = [x for x in tt.values() if isinstance(x, str)]
    return dict(seqs=1, seconds=depth(t), threads=oracle.max_threads(), t1=t[1], t2=t[2],
                torch_seconds=bad[0] if bad else depth(tt))


def torch_cpu_figure(cfg, r, extrapolated):
    import torch
    if isinstance(r["torch_seconds"], str):
        return {"unavailable": r["torch_seconds"]}
    return {"value": r["seqs"] * cfg.seq / r["torch_seconds"], "unit": "tokens/s",
            "threads": torch.get_num_threads(),
            "sample": ("same sequences, torch float32 on the host cores (fused causal "
                       "attention), one sequence per call"
                       + (", extrapolated in depth like the oracle" if extrapolated else ""))}


def cpu_model_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    """Reference arm: the reference's forward math on the host CPU cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from rustane_b200.model import CONFIGS
    from rustane_b200.sharding import global_tokens
    from oracle import oracle
    cfg = CONFIGS[args.config]
    tok, tgt = global_tokens(cfg.vocab, cfg.seq, 1, args.seed)
    oracle.set_threads(host_threads())
    model = oracle.OracleModel(cfg, seed=args.seed, scheme=oracle.SCHEME_NORMAL, sigma=0.02)
    threads = oracle.max_threads()
    for _ in range(args.warmup):
        model.forward(tok, tgt)
    t0 = time.perf_counter()
    loss = None
    for _ in range(args.steps):
        loss, _, _ = model.forward(tok, tgt)
    dt = time.perf_counter() - t0
    value = args.steps * cfg.seq / dt
    sample = (f"one {cfg.seq}-token sequence of the {args.config} forward+loss per step "
              f"(fp32 CPU restatement of the reference math, {threads} threads, "
              f"{cpu_model_name()})")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} forward+loss, seq {cfg.seq}", "seq_len": cfg.seq,
                   "global_batch": args.global_batch, "sample_per_step": 1},
        "loss": loss,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_io_workload(args):
    """The evaluation-path rows on one GPU (host wall clock around synchronous
    public calls, i.e. end to end): `validate` times cb_eval_windows over a
    synthetic uint16 token file (uniform ids, 0-byte special tokens) resident in
    HBM; `rstk-load` times cb_load_rstk of a synthetic N(0, 0.02) checkpoint
    (page-cache warm, as after a save) and, beside it, the f32 host-array upload."""
    import tempfile

    import torch
    from rustane_b200 import (CB_INIT_NORMAL, CompiledKernels, DeviceTokens, LayerWeights,
                              ModelWeights, TokenBytes)
    from rustane_b200.checkpoint import save_checkpoint
    from rustane_b200.model import CONFIGS

    if args.gpus != 1:
        raise SystemExit("--workload validate / rstk-load run on one GPU")
    torch.cuda.set_device(0)
    torch.zeros(1, device="cuda")  # the CUDA context exists before any timed call
    cfg = CONFIGS[args.config]
    rng = np.random.default_rng(args.seed)
    tmp = Path(tempfile.mkdtemp(prefix="rustane_bench_"))
    clocks = ClockSampler(0)
    if args.workload == "validate":
        batch = args.global_batch
        n_tok = 64 << 20  # 128 MB token file (larger than L2)
        path = tmp / "val.bin"
        path.write_bytes(rng.integers(0, cfg.vocab, n_tok, dtype=np.uint16).tobytes())
        table = rng.integers(1, 9, cfg.vocab).astype(np.int32)
        table[:4] = 0
        tb = TokenBytes(table)
        t0 = time.perf_counter()
        data = DeviceTokens.open(path, 0)
        t_open = time.perf_counter() - t0
        k = CompiledKernels(cfg, 0, batch)
        k.init_weights(args.seed, CB_INIT_NORMAL, 0.02)
        windows = batch * args.steps
        k.eval_windows(data, tb, 0, batch * args.warmup)
        clocks.start()
        t0 = time.perf_counter()
        tot = k.eval_windows(data, tb, 0, windows)
        dt = time.perf_counter() - t0
        clk = clocks.stop()
        line = {
            "metric": "validation tokens/s (cb_eval_windows: windows gathered from an "
                      "HBM-resident uint16 token file, val_loss and val_bpb sums on device)",
            "value": tot["tokens"] / dt, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "dtype": "fp16", "data": "synthetic uniform token ids",
            "config": {"workload": f"{args.config} validate, {batch} windows of seq "
                                   f"{cfg.seq} per forward, {windows} windows",
                       "token_file_tokens": n_tok,
                       "token_file_load_gbs": n_tok * 2 / t_open / 1e9},
            "val_loss": tot["loss_sum"] / tot["tokens"],
            "val_bpb": tot["nats"] / (np.log(2) * tot["bytes"]), "clocks": clk,
        }
        data.close()
    else:
        d, h = cfg.dim, cfg.hidden
        qd, kvd = cfg.heads * cfg.hd, cfg.kv_heads * cfg.hd

        def f(*shape):
            return (rng.standard_normal(shape, dtype=np.float32) * 0.02)

        layers = [LayerWeights(wq=f(d, qd), wk=f(d, kvd), wv=f(d, kvd), wo=f(qd, d),
                               w1=f(d, h), w3=f(d, h), w2=f(d, h), gamma1=np.ones(d, np.float32),
                               gamma2=np.ones(d, np.float32)) for _ in range(cfg.nlayers)]
        w = ModelWeights.from_arrays(f(cfg.vocab, d), layers, np.ones(d, np.float32))
        path = save_checkpoint(cfg, w, 1, tmp)
        nbytes = path.stat().st_size
        k = CompiledKernels(cfg, 0, 1)
        for _ in range(args.warmup):
            k.load_checkpoint(path)
        clocks.start()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            k.load_checkpoint(path)
        dt = (time.perf_counter() - t0) / args.steps
        clk = clocks.stop()
        t0 = time.perf_counter()
        k.load_weights(w)
        dt_host = time.perf_counter() - t0
        line = {
            "metric": "RSTK checkpoint load GB/s (cb_load_rstk: f32 file -> fp16 device "
                      "weights, pinned double-buffered streaming)",
            "value": nbytes / dt / 1e9, "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "dtype": "f32->fp16", "data": "synthetic N(0, 0.02) checkpoint, page cache warm",
            "config": {"workload": f"{args.config} RSTK checkpoint", "file_bytes": nbytes,
                       "host_array_upload_gbs": nbytes / dt_host / 1e9},
            "clocks": clk,
        }
    k.close()
    import shutil
    shutil.rmtree(tmp, ignore_errors=True)
    print(json.dumps(line), flush=True)


def run_decode_workload(args):
    """Decode throughput: `--decode-batch` sequences prefilled with seq/2 random tokens,
    then --steps single-token steps through the public cb_decode_step (host tokens in,
    greedy next tokens and full logits out every step), timed with CUDA events on the
    context's stream. Roofline: HBM bytes a step must read (every weight once plus the
    KV cache up to the current position) over the measured time."""
    import torch
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
    from rustane_b200.model import CONFIGS

    if args.gpus != 1:
        raise SystemExit("--workload decode runs on one GPU")
    torch.cuda.set_device(0)
    cfg = CONFIGS[args.config]
    B = args.decode_batch
    plen = cfg.seq // 2
    if args.warmup + 2 * args.steps > cfg.seq - plen:
        raise SystemExit("warmup + 2 x steps must fit in the second half of the sequence window")
    rng = np.random.default_rng(args.seed)
    k = CompiledKernels(cfg, 0, B)
    k.init_weights(args.seed, CB_INIT_NORMAL, 0.02)
    k.prefill(rng.integers(0, cfg.vocab, (B, plen)).astype(np.uint32))
    cur = np.zeros(B, np.uint32)
    for _ in range(args.warmup):
        _, cur = k.decode_step(cur)
    stream = torch.cuda.ExternalStream(k.stream())
    pos0 = k.decode_position()
    clocks = ClockSampler(0)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        _, cur = k.decode_step(cur)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    # the same steps returning only the greedy tokens (the logits stay on the device)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        _, cur = k.decode_step(cur, logits=False)
    e1.record(stream)
    torch.cuda.synchronize()
    ms_tokens = e0.elapsed_time(e1) / args.steps
    weight_bytes = 2.0 * (cfg.linear_params() + cfg.vocab * cfg.dim)
    mean_keys = pos0 + (args.steps + 1) / 2.0
    kv_bytes = 2.0 * 2 * cfg.nlayers * B * cfg.kv_heads * 128 * mean_keys
    gbs = (weight_bytes + kv_bytes) / (ms / 1e3) / 1e9
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("hbm_gbs", 6450.0))
    line = {
        "metric": "decode tokens/sec (single-token steps with a KV cache)",
        "value": B / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "fp16", "data": "synthetic (random prompt tokens, N(0,0.02) weights)",
        "config": {"workload": f"{args.config} decode, {B} sequences, positions "
                               f"{pos0}..{pos0 + args.steps - 1} of {cfg.seq}",
                   "batch": B, "prompt_len": plen},
        "roofline": {"kernel": "whole decode step", "bound": "hbm", "achieved": round(gbs, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
                     "peak_source": f"hbm_gbs ({peak_kind})",
                     "bytes_per_step": weight_bytes + kv_bytes, "traffic": None},
        "e2e": {"value": B / (ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 4 * B,
                "d2h_bytes_per_step": 4 * B * (cfg.vocab + 1)},
        "tokens_only": {"ms_per_step": ms_tokens, "value": B / (ms_tokens / 1e3),
                        "d2h_bytes_per_step": 4 * B,
                        "note": "the same steps returning only the greedy next tokens "
                                "(positions after the timed ones)"},
        "clocks": clk,
    }
    k.close()
    print(json.dumps(line), flush=True)


def run_attention_workload(args):
    """The causal attention kernel alone through the public cb_attention_f16: K launches
    on device-resident q, k, v ([batch, heads, seq, 128] fp16, N(0, 1)), the L2 flushed
    (a 256 MB write) before each launch, CUDA events around each launch on the launching
    stream, the median reported. Throughput counts the causal FLOPs only,
    4 * 128 * seq * (seq + 1) / 2 per (batch, head); peak = the measured burst bf16 GEMM
    rate (the kernel runs alone). torch's fused SDPA (a library kernel) is timed the same
    way on the same tensors for comparison."""
    import ctypes as C
    import torch
    from rustane_b200 import bridge as B
    from rustane_b200.model import CONFIGS

    if args.gpus != 1:
        raise SystemExit("--workload attention runs on one GPU")
    torch.cuda.set_device(0)
    if args.attn_shape:
        batch, heads, seq = (int(x) for x in args.attn_shape.split(","))
    else:
        cfg = CONFIGS[args.config]
        batch, heads, seq = args.global_batch, cfg.heads, cfg.seq
    lib = B.load_library()
    g = torch.Generator(device="cuda").manual_seed(args.seed)
    q, k, v = (torch.randn(batch, heads, seq, 128, device="cuda", generator=g).half()
               for _ in range(3))
    out = torch.empty(batch * seq, heads * 128, device="cuda", dtype=torch.float16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    flops = 4.0 * batch * heads * 128 * seq * (seq + 1) / 2

    def ours():
        rc = lib.cb_attention_f16(C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()),
                                  C.c_void_p(v.data_ptr()), C.c_void_p(out.data_ptr()),
                                  batch, heads, seq, C.c_void_p(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"cb_attention_f16 returned {rc}")

    def sdpa():
        torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)

    def timed(fn, n):
        ts = []
        for _ in range(n):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    for _ in range(args.warmup):
        ours()
    torch.cuda.synchronize()
    clocks = ClockSampler(0)
    clocks.start()
    ms = timed(ours, args.steps)
    clk = clocks.stop()
    for _ in range(args.warmup):
        sdpa()
    ms_sdpa = timed(sdpa, args.steps)
    ref = torch.nn.functional.scaled_dot_product_attention(q[:1], k[:1], v[:1], is_causal=True)
    got = out[:seq].view(seq, heads, 128).permute(1, 0, 2)
    err = float((got.float() - ref[0].float()).abs().max())
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    tf = flops / (ms / 1e3) / 1e12
    line = {
        "metric": "causal attention TFLOP/s (cb_attention_f16, head dim 128)",
        "value": tf, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "dtype": "fp16", "data": "synthetic (N(0,1) q, k, v)",
        "config": {"workload": f"attention batch {batch} x heads {heads} x seq {seq} x 128",
                   "batch": batch, "heads": heads, "seq_len": seq,
                   "l2": "flushed (256 MB write) before every launch"},
        "roofline": {"kernel": "attn_fwd_tc_kernel", "bound": "tensor", "achieved": round(tf, 1),
                     "peak": peak, "unit": "TFLOP/s", "frac": round(tf / peak, 4),
                     "peak_source": f"bf16_tflops burst ({peak_kind})",
                     "flops_per_launch": flops, "traffic": None},
        "torch_sdpa": {"ms": ms_sdpa, "tflops": round(flops / (ms_sdpa / 1e3) / 1e12, 1)},
        "max_abs_err_vs_torch_sdpa_seq0": err,
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


def run_train_workload(args):
    """Training step throughput (forward + backward, gradients accumulated on the
    device), sequence-sharded over the GPUs like the forward (data parallel: each rank
    trains on its share of the batch; the gradient all-reduce of a data-parallel
    optimizer step is not part of this step). The timed region is K graph replays of
    cb_forward_backward with host tokens (H2D + step + D2H of the loss each step), CUDA
    events on the context's stream, max over ranks."""
    import torch
    import torch.distributed as dist
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels
    from rustane_b200.model import CONFIGS
    from rustane_b200.sharding import global_tokens, rank_shard, reduce_max, shard_sequences

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    cfg = CONFIGS[args.config]
    per = shard_sequences(args.global_batch, world)
    all_tok, all_tgt = global_tokens(cfg.vocab, cfg.seq, args.global_batch, args.seed)
    tok, tgt = rank_shard(all_tok, all_tgt, cfg.seq, rank, per)
    tok = np.ascontiguousarray(tok)
    tgt = np.ascontiguousarray(tgt)
    kern = CompiledKernels(cfg, local, per)
    kern.init_weights(args.seed, CB_INIT_NORMAL, 0.02)
    kern.enable_training()
    stream = torch.cuda.ExternalStream(kern.stream())
    for _ in range(args.warmup):
        loss = kern.forward_backward(tok, tgt)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local) if rank == 0 else None
    if clocks:
        clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        loss = kern.forward_backward(tok, tgt)
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = reduce_max(e0.elapsed_time(e1), device="cuda") / args.steps
    clk = clocks.stop() if clocks else None
    tokens = args.global_batch * cfg.seq
    flops = cfg.train_flops_per_token() * tokens
    peaks, peak_kind = load_peaks()
    peak_tf = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    tf = flops / (ms / 1e3) / 1e12 / world
    if rank == 0:
        line = {
            "metric": "training tokens/sec (forward + backward into fp32 gradients, seq512)",
            "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16", "data": "synthetic (uniform random tokens, N(0,0.02) weights)",
            "config": {"workload": f"{args.config} training step, global batch "
                                   f"{args.global_batch} x seq {cfg.seq}",
                       "global_batch": args.global_batch, "seq_len": cfg.seq,
                       "parallelism": f"dp{world} (sequence sharding; no gradient all-reduce)",
                       "l2": "no flush: every step moves tens of GB, far above the 126 MB L2"},
            "loss": loss,
            "tflops_per_gpu": round(tf, 1),
            "roofline": {"kernel": "whole training step (GEMMs, attention, row kernels)",
                         "bound": "tensor", "achieved": round(tf, 2), "peak": peak_tf,
                         "unit": "TFLOP/s", "frac": round(tf / peak_tf, 4),
                         "peak_source": f"bf16_tflops_sustained ({peak_kind})",
                         "flops_per_token": cfg.train_flops_per_token(), "traffic": None},
            "e2e": {"value": tokens / (ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(tok.nbytes + tgt.nbytes) * world,
                    "d2h_bytes_per_step": 4 * world,
                    "note": "the timed calls are the public host API (cb_forward_backward)"},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    kern.close()
    if world > 1:
        dist.destroy_process_group()


def tp_exchange_label() -> str:
    """How the tensor-parallel ranks combine the O and down projections (CB_TP_REDUCE)."""
    mode = os.environ.get("CB_TP_REDUCE", "sp16")
    if mode == "allreduce":
        return "fp32 NCCL all-reduce after the O and down projections"
    width = "fp32" if mode == "sp32" else "fp16"
    return (f"sequence parallel: {width} NCCL reduce-scatter of the O and down partial sums, "
            "residual + RMSNorm on each rank's token rows, fp16 all-gather of the normalised rows")


def main():
    args = parse_args()
    if args.global_batch is None:
        args.global_batch = 16 if args.config == "32B" else 64
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "train":
        run_train_workload(args)
        return
    if args.workload == "decode":
        run_decode_workload(args)
        return
    if args.workload == "attention":
        run_attention_workload(args)
        return
    if args.workload != "forward":
        run_io_workload(args)
        return

    import torch
    import torch.distributed as dist
    from rustane_b200 import CB_INIT_NORMAL, CompiledKernels, nccl_unique_id
    from rustane_b200.model import CONFIGS
    from rustane_b200.sharding import (global_tokens, rank_shard, reduce_max, reduce_mean,
                                       shard_sequences)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))

    cfg = CONFIGS[args.config]
    all_tok, all_tgt = global_tokens(cfg.vocab, cfg.seq, args.global_batch, args.seed)
    if args.tp and world > 1:
        # every rank runs the whole batch on its slice of the model
        per = args.global_batch
        nid = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        kern = CompiledKernels(cfg, local, per, tp_rank=rank, tp_world=world, nccl_id=nid[0])
        tok_np, tgt_np = all_tok, all_tgt
    else:
        per = shard_sequences(args.global_batch, world)
        kern = CompiledKernels(cfg, local, per)
        tok_np, tgt_np = rank_shard(all_tok, all_tgt, cfg.seq, rank, per)
    kern.init_weights(args.seed, CB_INIT_NORMAL, 0.02)
    d_tok = torch.from_numpy(tok_np.view(np.int32)).cuda()
    d_tgt = torch.from_numpy(tgt_np.view(np.int32)).cuda()
    d_loss = torch.zeros(1, dtype=torch.float32, device="cuda")
    sptr = kern.stream()
    stream = torch.cuda.ExternalStream(sptr)

    def step():
        kern.forward_loss_async(d_tok.data_ptr(), d_tgt.data_ptr(), per, 0.0, d_loss.data_ptr(),
                                0, sptr)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        return reduce_max(x, device="cuda")

    def mean_over_ranks(x: float) -> float:
        return reduce_mean(x, device="cuda")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    kern.check_device_error()

    # ---- 1. timed region (CUDA graph replays, device-resident inputs)
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    kern.check_device_error()
    ms_total = max_over_ranks(e0.elapsed_time(e1))
    loss = mean_over_ranks(float(d_loss.item()))
    ms_step = ms_total / args.steps
    tokens_total = args.global_batch * cfg.seq * args.steps
    value = tokens_total / (ms_total / 1e3)

    # ---- 2. profiled pass: CUDA events around every kernel
    kern.set_profiling(True)
    kern.reset_kernel_times()
    barrier()
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    times = kern.kernel_times()
    kern.set_profiling(False)
    barrier()

    # ---- 3. e2e through the public host API (pinned host buffers)
    e2e = None
    if not args.no_e2e:
        h_tok = torch.from_numpy(tok_np.view(np.int32)).pin_memory()
        h_tgt = torch.from_numpy(tgt_np.view(np.int32)).pin_memory()
        tok_view = h_tok.numpy().view(np.uint32)
        tgt_view = h_tgt.numpy().view(np.uint32)
        kern.forward_loss(tok_view, tgt_view)  # warm the path
        barrier()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            kern.forward_loss(tok_view, tgt_view)
        f1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(f0.elapsed_time(f1))
        e2e = {"value": tokens_total / (e2e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(tok_view.nbytes + tgt_view.nbytes) * world,
               "d2h_bytes_per_step": 4 * world, "ms_per_step": e2e_ms / args.steps,
               "note": ("every TP rank copies the whole batch" if args.tp and world > 1
                        else "each rank copies its own sequences")}

    # ---- roofline of the dominant kernel (the tcgen05 GEMM, all its launches)
    peaks, peak_kind = load_peaks()
    g_launch = sum(times[c]["launches"] for c in GEMM_CLASSES if c in times)
    g_ms = sum(times[c]["total_ms"] for c in GEMM_CLASSES if c in times)
    g_flops = sum(times[c]["flops"] for c in GEMM_CLASSES if c in times)
    all_ms = sum(v["total_ms"] for v in times.values())
    peak_tf = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    achieved = g_flops / (g_ms / 1e3) / 1e12 if g_ms > 0 else 0.0
    roofline = {
        "kernel": "gemm_tn (tcgen05, all 5 fused-epilogue GEMMs, 81 launches per forward)",
        "bound": "tensor", "achieved": round(achieved, 2), "peak": peak_tf, "unit": "TFLOP/s",
        "frac": round(achieved / peak_tf, 4), "peak_source": f"bf16_tflops_sustained ({peak_kind})",
        "flops_per_launch": g_flops / max(g_launch, 1),
        "ms_per_launch": g_ms / max(g_launch, 1),
        "share_of_step": round(g_ms / all_ms, 4) if all_ms > 0 else None,
        "traffic": None if args.tp else GEMM_TRAFFIC_PER_LAUNCH.get((args.config, per)),
        "traffic_unit": "bytes per launch",
        "traffic_source": GEMM_TRAFFIC_SOURCE,
    }
    flops_fwd = cfg.forward_flops_per_token() * args.global_batch * cfg.seq
    kernels = {k: {"launches": v["launches"], "ms": round(v["total_ms"], 3),
                   "share": round(v["total_ms"] / all_ms, 4) if all_ms else None,
                   "tflops": round(v["flops"] / (v["total_ms"] / 1e3) / 1e12, 1)
                   if v["flops"] and v["total_ms"] else None,
                   "gbs": round(v["bytes"] / (v["total_ms"] / 1e3) / 1e9, 1)
                   if v["total_ms"] else None}
               for k, v in times.items()}

    # ---- 4. CPU baseline on the host cores (rank 0 at N = 1)
    cpu = None
    cpu_leg = rank == 0 and world == 1 and not args.no_cpu_baseline
    if cpu_leg and cfg.dim > 2048:
        try:
            r = cpu_oracle_extrapolated(cfg, args.seed, tok_np, tgt_np)
        except (MemoryError, RuntimeError) as e:
            r = None
            cpu = {"unavailable": f"CPU oracle failed: {type(e).__name__}: {e}"}
    if cpu_leg and cfg.dim > 2048 and r is not None:
        cpu = {"value": cfg.seq / r["seconds"], "unit": "tokens/s", "cores": r["threads"],
               "kind": "port",
               "sample": (f"extrapolated: one {cfg.seq}-token sequence through 1- and 2-layer "
                          f"variants of {args.config} ({r['t1']:.2f} s, {r['t2']:.2f} s), "
                          f"linear in depth to {cfg.nlayers} layers; fp32 CPU oracle, "
                          f"{r['threads']} threads, {cpu_model_name()}"),
               "torch_cpu": torch_cpu_figure(cfg, r, extrapolated=True)}
    elif cpu_leg and cfg.dim <= 2048:
        r = cpu_oracle_sample(cfg, args.seed, tok_np, tgt_np, args.cpu_budget_s)
        cpu_val = r["seqs"] * cfg.seq / r["seconds"]
        gpu_seq_losses = kern.forward_loss(tok_np[:r["seqs"] * cfg.seq],
                                           tgt_np[:r["seqs"] * cfg.seq])
        cpu = {"value": cpu_val, "unit": "tokens/s", "cores": r["threads"], "kind": "port",
               "sample": (f"{r['seqs']} x {cfg.seq}-token sequences of the bench workload "
                          f"(same weights and tokens), fp32 CPU oracle, {r['threads']} threads, "
                          f"{cpu_model_name()}"),
               "parity": {"loss_cpu": float(np.mean(r["losses"])), "loss_gpu": gpu_seq_losses,
                          "rel": abs(gpu_seq_losses - float(np.mean(r["losses"])))
                          / float(np.mean(r["losses"]))},
               "torch_cpu": torch_cpu_figure(cfg, r, extrapolated=False)}

    # GPU over CPU, end to end (host copies included), against both CPU figures: the
    # oracle (the reference arm's code) and torch's float32 CPU kernels, the faster one
    speedup = None
    if cpu and "value" in cpu and e2e:
        speedup = {"e2e_vs_cpu_oracle": round(e2e["value"] / cpu["value"], 1)}
        tc = cpu.get("torch_cpu") or {}
        if "value" in tc:
            speedup["e2e_vs_torch_cpu"] = round(e2e["value"] / tc["value"], 1)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic (uniform random tokens, N(0,0.02) weights generated on device)",
            "config": {
                "workload": (f"{args.config} forward+loss ({cfg.dim}d/{cfg.hidden}h/"
                             f"{cfg.nlayers}L/{cfg.heads}x128, vocab {cfg.vocab}, tied head), "
                             f"seq {cfg.seq}, global batch {args.global_batch}"),
                "global_batch": args.global_batch, "seq_len": cfg.seq,
                "parallelism": (f"tp{world} (Megatron column/row split; {tp_exchange_label()})"
                                if args.tp and world > 1 else
                                f"dp{world} (sequence sharding, no communication)"),
                "per_gpu_batch": per,
                "l2": "no flush: every step reads >1.1 GB of weights and >1 GB of "
                      "activations, well above the 126 MB L2",
            },
            "loss": loss,
            "tflops": flops_fwd / (ms_step / 1e3) / 1e12,
            "frac_of_peak_forward": round(flops_fwd / (ms_step / 1e3) / 1e12 / peak_tf, 4),
            "roofline": roofline,
            "kernels": kernels,
            "cpu_baseline": cpu,
            "speedup_over_cpu": speedup,
            "e2e": e2e,
            "gpu_launches": int(sum(v["launches"] for k, v in times.items()
                                    if not k.startswith("nccl"))),
            "clocks": clk,
            "ms_per_step_profiled": all_ms / args.steps,
        }
        print(json.dumps(line), flush=True)

    kern.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
