#!/usr/bin/env python
# SPDX-License-Identifier: MIT
"""Benchmark of the quantized matmul hot path on B200.

Headline metric: Q4_K GEMV HBM GB/s. Workload = BASELINE
config 1 (Q4_K x Q8_K matvec, K=1024, N=3072) over a pool of G distinct
weight matrices per GPU (default 320 -> 566 MB, > 4x the 126 MB L2, so
every step streams weights from HBM; no flush needed). One step = quantize
the G activation rows to Q8_K (one launch) + the G matvecs (one grouped
persistent launch). GB/s counts algorithmic bytes per matvec: weights
1,769,472 + Q8_K activation 1,168 + fp32 output 12,288 = 1,782,928.

  value  -- device-resident inputs, CUDA-event time of K steps (max over ranks);
            activations and outputs are double-buffered, so step i + 1's
            quantization (its own stream) overlaps step i's matvec launch
  e2e    -- the same work through the C-ABI with HOST buffers: per step the
            activations are copied from pinned host memory and the outputs
            read back, inside the timed region (copies on their own streams,
            overlapping the neighbouring steps' compute)
  roofline -- the grouped matvec kernel alone: algorithmic bytes / its mean
            launch time (events around each launch on its stream) vs the
            measured HBM copy bandwidth in MEASURED_PEAKS.json
  cpu_baseline -- the reference's own SIMD row dot (oracle/_ref, compiled
            from its sources) over all host cores on a bounded sample

Multi-GPU (torchrun, one process per GPU): every rank streams its own pool
(weak scaling, no data-path collective); NCCL only carries the barrier and
the max-over-ranks of the elapsed time.

--impl reference runs the reference's CPU implementation of the path
(oracle/_ref/libqhref.so: simd_q4k_row_dot_q8k with rows split over all host
threads) on the same workload/metric; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "qwen.haiku_b200")
sys.path.insert(0, ROOT)

METRIC = "Q4_K GEMV HBM GB/s (% of 8 TB/s); decode tok/s at batch 1 and 64/GPU"
K_IN, N_OUT = 1024, 3072
Q4K_TYPE = 12  # GGUF type id of Q4_K
W_BYTES = N_OUT * (K_IN // 256) * 144          # 1,769,472
X_BYTES = (K_IN // 256) * 292                   # Q8_K activation (reference block size)
O_BYTES = N_OUT * 4
ALGO_BYTES = W_BYTES + X_BYTES + O_BYTES        # 1,782,928 per matvec
SETTLE_STEPS = 400                              # untimed steps before the GEMV timed region
KEV_EVERY = 8                                   # matvec launches bracketed by kernel-time events
NOMINAL_HBM_GBS = 8000.0


def load_pkg():
    name = "qwen_haiku_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.proc = None
        self.path = os.path.join("/tmp", f"qh_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or (self.uuid and parts[0] != self.uuid):
                continue
            try:
                sm.append(float(parts[1].split()[0]))
                smax.append(float(parts[2].split()[0]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU side: the reference's own SIMD dot over all host cores
# ---------------------------------------------------------------------------
def numpy_q4k_blocks(n_blocks: int, seed: int):
    """Seeded Q4_K super-blocks without this library (for the reference arm):
    uniform random bytes with fp16 d and dmin drawn from U[1e-3, 1e-2]."""
    import numpy as np
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (n_blocks, 144), dtype=np.uint8)
    b[:, 0:4] = rng.uniform(1e-3, 1e-2, (n_blocks, 2)).astype(np.float16).view(np.uint8).reshape(n_blocks, 4)
    return b.reshape(-1)


def cpu_reference_run(qh, n_mats: int, passes_budget_s: float, max_passes: int = None):
    """Returns (GB/s, cores, sample description, kind, per-pass seconds list).
    qh None: the inputs are generated with numpy (the reference arm maps no
    library of this repository)."""
    import numpy as np
    from oracle.oracle import Oracle, Ref, to_q8k_blocks
    cores = len(os.sched_getaffinity(0))
    if qh is not None:
        h = qh.host
        base = [h.synth_blocks(Q4K_TYPE, N_OUT * 4, 0xC0FFEE + i) for i in range(min(n_mats, 8))]
        x = h.synth_normal(K_IN, 0xACE)
    else:
        base = [numpy_q4k_blocks(N_OUT * 4, 0xC0FFEE + i) for i in range(min(n_mats, 8))]
        x = np.random.default_rng(0xACE).standard_normal(K_IN).astype(np.float32)
    pool = [base[i % len(base)].copy() for i in range(n_mats)]  # distinct addresses
    if Ref.available():
        ref = Ref()
        qs, d, bs = ref.quantize_q8k(x.reshape(1, K_IN))
        xq = to_q8k_blocks(qs[0], d[0], bs[0])
        out = np.empty(N_OUT, np.float32)

        def one_pass():
            ref.matvec_pool_mt(Q4K_TYPE, pool, N_OUT, K_IN, xq, cores, out)
        kind = "reference"
        label = ref.label
    else:
        orc = Oracle()
        qs, d, bs = orc.quantize_q8k(x.reshape(1, K_IN))

        def one_pass():
            for w in pool:
                orc.matvec_preq(Q4K_TYPE, w, N_OUT, K_IN, qs[0], d[0], bs[0])
        kind, label, cores = "port", "oracle restatement (1 thread)", 1
    times = []
    t_total = 0.0
    while True:
        t0 = time.perf_counter()
        one_pass()
        dt = time.perf_counter() - t0
        times.append(dt)
        t_total += dt
        if max_passes is not None and len(times) >= max_passes:
            break
        if max_passes is None and t_total >= passes_budget_s:
            break
    per_pass = statistics.median(times)
    gbs = n_mats * ALGO_BYTES / per_pass / 1e9
    sample = (f"{n_mats} config-1 Q4_K matvecs ({n_mats * W_BYTES / 1e6:.0f} MB weights) per pass, "
              f"{len(times)} passes; {label}, rows split over {cores} threads")
    return gbs, cores, sample, kind, times


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    n_mats = 64  # inputs from numpy: the reference arm maps only oracle/_ref (and liboracle)
    gbs, cores, sample, kind, times = cpu_reference_run(None, n_mats, 0.0, max_passes=args.warmup + args.steps)
    timed = times[args.warmup:] if len(times) > args.warmup else times
    per = statistics.median(timed)
    value = n_mats * ALGO_BYTES / per / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8+fp32", "data": "synthetic",
        "config": {"workload": f"Q4_K GEMV K={K_IN} N={N_OUT} (BASELINE config 1), reference CPU SIMD path",
                   "k": K_IN, "n": N_OUT, "pool_matrices": n_mats},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# decode of the synthetic Qwen3.5-0.8B-shaped model (configs 4 and 5)
# ---------------------------------------------------------------------------
MODEL_SEED = 0xC0F16


class _DevInts:
    """A device int32 vector seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i4", "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": None}


def decode_step_bytes(cfg, B: int, weight_bytes: int, n_prompt: int, n_new: int) -> float:
    """Algorithmic HBM bytes of one decode step, averaged over the decode
    positions: every weight once (the tied Q6_K LM head included; the
    embedding row gather is negligible), the Gated DeltaNet state read and
    written, the conv ring read and written, the fp16 KV cache rows read up
    to the position plus the new row written."""
    n_attn = sum(1 for l in range(cfg.n_layers) if (l + 1) % cfg.full_attn_interval == 0)
    n_gdn = cfg.n_layers - n_attn
    kdim = cfg.gdn_heads * cfg.gdn_head_dim
    state = n_gdn * cfg.gdn_heads * cfg.gdn_head_dim * cfg.gdn_head_dim * 4
    ring = n_gdn * cfg.conv_kernel * 3 * kdim * 4
    avg_rows = n_prompt + (n_new - 1) / 2.0 + 1
    kv = n_attn * avg_rows * 2 * cfg.n_kv_heads * cfg.head_dim * 2
    return weight_bytes + B * (2 * state + 2 * ring + kv)


# ---------------------------------------------------------------------------
# data-parallel plumbing (one process per GPU; also exercised on CPU/gloo)
# ---------------------------------------------------------------------------
def max_over_ranks(dp, values):
    """Element-wise max of a list of floats over all ranks (the job's time is
    its slowest rank's), through the library's NCCL communicator (qh_dp)."""
    return list(values) if dp is None else dp.max(list(values))


# ---------------------------------------------------------------------------
# prefill GEMMs (config 3) on the tensor cores
# ---------------------------------------------------------------------------
GEMM_CONFIGS = {"3a": (512, 1024, 3584, 12), "3b": (2048, 3584, 1024, 14)}  # M, K, N, GGUF type


def tensor_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured bf16 dense (burst)"
    except Exception:
        return 1590.0, "fallback bf16 dense"


def run_gemm(qh, torch, steps: int, warmup: int):
    """Config 3: device-resident tiled weights and activations, qh_gemm
    timed with CUDA events; e2e through qh_matmul_gemm (GGUF weights on the
    device, fp32 activations from pinned host memory, outputs read back).
    Ops count 2*M*N*K (int8 multiply-adds of the expanded operands)."""
    import ctypes as C
    h, L = qh.host, qh.lib()
    peak, peak_kind = tensor_peak()
    out = {}
    for name, (m, k, n, gt) in GEMM_CONFIGS.items():
        w = h.to_device(h.synth_blocks(gt, n * (k // 256), 0x3A00 + gt))
        x_host = torch.from_numpy(h.synth_normal(m * k, 0x3B00 + m).reshape(m, k)).pin_memory()
        x = x_host.to("cuda")
        wt = h.gemm_pack(gt, w, k, n)
        we = h.gemm_expand(gt, wt, k, n)
        xq = h.quantize_q8kt(x, k, m)
        o = torch.empty((m, n), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()  # packed weights complete: they may stream in early (QH_GEMM_WEIGHTS_READY)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # tiled weights (expanded per launch on the CUDA cores) and expanded
        # weights (the MMA operands stored once, QH_GEMM_EXPANDED)
        mode_ms = {}
        for mode, wbuf, flags in (("tiled", wt, 1), ("expanded", we, 3)):
            for _ in range(warmup):
                h.gemm(gt, [(wbuf, n, o, n)], k, xq, m, split=False, flags=flags)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(steps):
                h.gemm(gt, [(wbuf, n, o, n)], k, xq, m, split=False, flags=flags)
            e1.record()
            torch.cuda.synchronize()
            mode_ms[mode] = e0.elapsed_time(e1) / steps
        best_mode = min(mode_ms, key=mode_ms.get)
        ms = mode_ms[best_mode]
        # end to end: host activations in, outputs out, GGUF weights packed per call
        need = int(L.qh_matmul_gemm_workspace_bytes(gt, k, n, m))
        work = torch.empty(need, dtype=torch.uint8, device="cuda")
        o_host = torch.empty((m, n), dtype=torch.float32).pin_memory()
        sh = C.c_void_p(torch.cuda.current_stream().cuda_stream)

        def e2e_once():
            qh.check(L.qh_memcpy_h2d(C.c_void_p(x.data_ptr()), C.c_void_p(x_host.data_ptr()), m * k * 4, sh), "h2d")
            qh.check(L.qh_matmul_gemm(gt, C.c_void_p(w.data_ptr()), k, n, C.c_void_p(x.data_ptr()), m,
                                      C.c_void_p(o.data_ptr()), C.c_void_p(work.data_ptr()), need, sh), "matmul_gemm")
            qh.check(L.qh_memcpy_d2h(C.c_void_p(o_host.data_ptr()), C.c_void_p(o.data_ptr()), m * n * 4, sh), "d2h")
        for _ in range(2):
            e2e_once()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            e2e_once()
        e1.record()
        torch.cuda.synchronize()
        ms_e2e = e0.elapsed_time(e1) / steps
        ops = 2.0 * m * n * k
        tops = ops / (ms / 1e3) / 1e12
        out[name] = {"workload": f"M={m} K={k} N={n} {'Q4_K' if gt == 12 else 'Q6_K'} x Q8_K -> fp32",
                     "ms": round(ms, 4), "weights": best_mode,
                     "ms_by_weights": {kk: round(v, 4) for kk, v in mode_ms.items()},
                     "tops": round(tops, 2), "tokens_per_s": round(m / (ms / 1e3), 1),
                     "weight_gbs": round(w.numel() / (ms / 1e3) / 1e9, 1),
                     "e2e": {"ms": round(ms_e2e, 4), "tokens_per_s": round(m / (ms_e2e / 1e3), 1),
                             "h2d_bytes": m * k * 4, "d2h_bytes": m * n * 4},
                     "roofline": {"bound": "tensor", "achieved": round(tops, 2), "peak": peak, "unit": "TOP/s",
                                  "frac": round(tops / peak, 4), "peak_source": peak_kind + "; int8 MMA nominal is 2x bf16"}}
        del w, x, wt, we, xq, o, work
    torch.cuda.empty_cache()
    return out


def run_decode(qh, torch, dist, dp, world: int, rank: int, B: int, n_prompt: int, n_new: int,
               profile_step: bool = False):
    """Greedy decode of B sequences per GPU: n_prompt teacher-forced steps,
    then n_new steps timed with CUDA events on the model's stream; the
    sampled tokens are gathered over NCCL after every step when world > 1.
    Returns a dict for the JSON line (rank 0 fills it)."""
    import numpy as np
    h = qh.host
    cfg = h.slm_config(n_prompt + n_new)
    blob = h.Blob(cfg, MODEL_SEED)  # identical weights on every rank (replicated)
    slm = h.Slm(cfg, blob, B)
    import ctypes as C
    wb, sb = C.c_int64(), C.c_int64()
    qh.check(qh.lib().qh_slm_memory(slm.handle, C.byref(wb), C.byref(sb)), "qh_slm_memory")
    rng = np.random.default_rng(0xD3C0 + 7919 * rank + B)
    prompts = rng.integers(0, cfg.vocab, (B, n_prompt)).astype(np.int32)
    stream = torch.cuda.ExternalStream(slm.stream)
    nxt = torch.as_tensor(_DevInts(slm.device_next, B), device="cuda")
    gathered = torch.empty(world * B, dtype=torch.int32, device="cuda")

    def gather():  # the step's sampled tokens of every rank, on the model's stream (qh_dp_gather_tokens)
        if dp is not None:
            dp.gather(slm.device_next, B, gathered.data_ptr(), slm.stream)

    # warm-up: the first steps run directly, then the step is captured; a
    # short prefill allocates the prompt-chunk buffers and tiled weights
    slm.prefill(prompts[:, :min(n_prompt, 9)])
    for _ in range(3):
        slm.advance(1)
        gather()
    slm.reset()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    t0 = time.perf_counter()
    ev[0].record(stream)
    slm.prefill(prompts)  # prompt in chunks: tensor-core projections, per-chunk recurrence/attention
    ev[1].record(stream)
    for _ in range(n_new):
        slm.advance(1)
        gather()
    ev[2].record(stream)
    picks = slm.picks(n_prompt - 1, n_new)  # synchronizes
    wall = time.perf_counter() - t0
    if profile_step and rank == 0:
        # one more decode step between cudaProfilerStart/Stop, outside the
        # timed region, for `ncu --profile-from-start off` launch lists
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        slm.advance(1)
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
    torch.cuda.synchronize()
    prefill_ms, decode_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    prefill_ms, decode_ms, wall = max_over_ranks(dp, [prefill_ms, decode_ms, wall])
    # consistency: the gathered picks of the last step are this rank's picks
    if world > 1:
        mine = gathered.view(world, B)[rank].cpu().numpy()
        if not np.array_equal(mine, picks[:, -1]):
            raise SystemExit("token gather disagrees with the rank's own picks")
    slm.close()
    # the same prompts through the reference's batched prefill path
    # (LLM_USE_FORWARD_BATCH: chunked DeltaNet algebra, QH_PREFILL_CHUNKED)
    ch = h.Slm(cfg, blob, B)
    ch.prefill(prompts[:, :min(n_prompt, 9)], mode=qh.PREFILL_CHUNKED)
    ch.reset()
    cstream = torch.cuda.ExternalStream(ch.stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    cev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    cev[0].record(cstream)
    ch.prefill(prompts)
    cev[1].record(cstream)
    torch.cuda.synchronize()
    chunked_ms = max_over_ranks(dp, [cev[0].elapsed_time(cev[1])])[0]
    ch.close()
    step_bytes = decode_step_bytes(cfg, B, wb.value, n_prompt, n_new)
    step_ms = decode_ms / n_new
    out = {
        "workload": f"{B} sequence(s)/GPU, {n_prompt}-token prompt, {n_new} greedy tokens",
        "tok_s": round(world * B * n_new / (decode_ms / 1e3), 1),
        "ms_per_step": round(step_ms, 4),
        "prefill_tok_s": round(world * B * (n_prompt - 1) / (prefill_ms / 1e3), 1),
        "prefill_chunked_tok_s": round(world * B * (n_prompt - 1) / (chunked_ms / 1e3), 1),
        "e2e_tok_s": round(world * B * (n_prompt - 1 + n_new) / wall, 1),
        "hbm_bytes_per_step": int(step_bytes), "weight_bytes": wb.value,
        "hbm_gbs": round(step_bytes / (step_ms / 1e3) / 1e9, 1),
        "picks_checksum": int(np.bitwise_xor.reduce(picks.ravel() * np.int64(2654435761) % (1 << 31))),
    }
    del blob
    return out, cfg, prompts, picks


def run_sampled(qh, torch, B: int, n_prompt: int, n_new: int):
    """Sampled generation (qh_slm_generate_sampled, the reference's default
    sampler chain: T 0.7, top-k 40, top-p 0.9, min-p 0.05, repetition
    penalty 1.25 over 64 tokens) of B sequences: decode tok/s from the time
    of an n_new-token call minus a 1-token call (the prompt part of both)."""
    import numpy as np
    h = qh.host
    cfg = h.slm_config(n_prompt + n_new + 1)
    blob = h.Blob(cfg, MODEL_SEED)
    slm = h.Slm(cfg, blob, B)
    rng = np.random.default_rng(0x5A3 + B)
    prompts = rng.integers(0, cfg.vocab, (B, n_prompt)).astype(np.int32)
    seeds = np.arange(1, B + 1, dtype=np.uint64)
    sp = h.sampler_defaults()
    slm.generate_sampled(prompts, 4, sp, seeds)  # warm-up: captures the sampled step
    times = {}
    for n in (1, n_new):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = slm.generate_sampled(prompts, n, sp, seeds)
        times[n] = time.perf_counter() - t0
    slm.close()
    dt = times[n_new] - times[1]
    return {"workload": f"{B} sequence(s)/GPU, {n_prompt}-token prompt, {n_new} sampled tokens",
            "sampler": "T 0.7, top-k 40, top-p 0.9, min-p 0.05, repetition penalty 1.25 / 64",
            "tok_s": round(B * (n_new - 1) / dt, 1), "ms_per_step": round(dt / (n_new - 1) * 1e3, 4),
            "tokens_checksum": int(sum(int(np.sum(o.astype(np.int64) * 2654435761 % (1 << 31))) for o in out) % (1 << 31))}


def cpu_decode_baseline(qh, n_steps: int = 4):
    """The reference's own slm_forward_step + sample_argmax (oracle/_ref,
    single-threaded on Linux, as the reference runs it) on the full-size
    model: a bounded sample of n_steps steps from position 0 -- once on one
    core, and as independent sequences on every host core at once (one
    context and thread per core, shared weights: the reference's way to use
    more cores for more sequences). tok/s."""
    from concurrent.futures import ThreadPoolExecutor

    from oracle.oracle import Ref, RefModel
    if not Ref.available():
        return None
    h = qh.host
    cfg = h.slm_config(64)
    blob = h.Blob(cfg, MODEL_SEED)
    ref = Ref()
    tensors = blob.tensors()

    def run(rm, first):
        tok = first
        for pos in range(1, n_steps + 1):
            tok = rm.step(tok, pos)

    rm = RefModel(ref, cfg, tensors)
    rm.step(1, 0)
    t0 = time.perf_counter()
    run(rm, 2)
    one = n_steps / (time.perf_counter() - t0)
    rm.close()
    cores = min(len(os.sched_getaffinity(0)), 64)  # bounded host memory: ~85 MB of caches per context
    models = [RefModel(ref, cfg, tensors) for _ in range(cores)]
    for i, m in enumerate(models):
        m.step(1 + i, 0)
    t0 = time.perf_counter()
    with ThreadPoolExecutor(cores) as ex:  # the foreign calls release the GIL
        list(ex.map(lambda a: run(*a), [(m, 2 + i) for i, m in enumerate(models)]))
    agg = cores * n_steps / (time.perf_counter() - t0)
    for m in models:
        m.close()
    return {"value": round(agg, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
            "one_core_tok_s": round(one, 3),
            "sample": f"{n_steps} decode steps of the full-size model per sequence, {cores} sequences on "
                      f"{cores} host threads at once (slm_forward_step, single-threaded per context); "
                      f"one_core_tok_s: one sequence alone"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import ctypes as C

    import numpy as np
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    qh = load_pkg()
    h = qh.host
    L = qh.lib()
    qh.check(L.qh_set_device(local), "qh_set_device")
    # the library's own communicator (qh_dp, NCCL): token gathers and
    # max-over-ranks timing; torch.distributed only carries its id and the
    # barriers
    dp = h.DataParallel.from_torch(dist, timeout_ms=120000) if world > 1 else None
    G = args.pool
    stream = torch.cuda.current_stream()
    sh = C.c_void_p(stream.cuda_stream)

    # weights: 16 distinct generated matrices replicated over G distinct
    # device regions (distinct addresses defeat L2 reuse; content may repeat)
    n_distinct = min(G, 16)
    host_w = [h.synth_blocks(qh.Q4_K, N_OUT * 4, 0x5EED0000 + 1000 * rank + i) for i in range(n_distinct)]
    wdev = torch.empty((G, W_BYTES), dtype=torch.uint8, device="cuda")
    for g in range(G):
        wdev[g].copy_(torch.from_numpy(host_w[g % n_distinct]), non_blocking=False)
    x_host = h.synth_normal(G * K_IN, 0xABC + rank).reshape(G, K_IN)
    # Two of everything the step touches (activations fp32 and Q8_K, outputs,
    # host staging), so step i + 1's quantization -- and in the end-to-end
    # run its host->device copy -- overlaps step i's matvecs on other streams.
    x_pin = torch.from_numpy(x_host).pin_memory()
    xbytes = int(L.qh_q8k_bytes(K_IN, G))
    x_dev = [x_pin.to("cuda") for _ in range(2)]
    xq = [torch.empty(xbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    out = [torch.empty((G, N_OUT), dtype=torch.float32, device="cuda") for _ in range(2)]
    out_pin = [torch.empty((G, N_OUT), dtype=torch.float32).pin_memory() for _ in range(2)]
    plans = [h.MatvecPlan(qh.Q4_K, [(wdev[g], xq[b], out[b][g], K_IN, N_OUT, G, g) for g in range(G)], 1)
             for b in range(2)]
    plan = plans[0]
    info = plan.info()
    s_q = torch.cuda.Stream()      # quantization of the next step
    s_in = torch.cuda.Stream()     # host -> device copies
    s_out = torch.cuda.Stream()    # device -> host copies

    def quantize(b, st):
        qh.check(L.qh_quantize_q8k(C.c_void_p(x_dev[b].data_ptr()), K_IN, G, C.c_void_p(xq[b].data_ptr()),
                                   C.c_void_p(st.cuda_stream)), "qh_quantize_q8k")

    # parity spot check of the benchmarked path (not timed)
    quantize(0, stream)
    plan.run(sh)
    torch.cuda.synchronize()
    from oracle.oracle import Oracle
    orc = Oracle()
    for g in (0, G - 1):
        want = orc.matmul(qh.Q4_K, host_w[g % n_distinct], N_OUT, K_IN, x_host[g:g + 1])
        if not np.array_equal(out[0][g].cpu().numpy().view(np.uint32), want.view(np.uint32).ravel()):
            raise SystemExit(f"bench parity check failed for matrix {g}")

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_time(v: float) -> float:
        return max_over_ranks(dp, [v])[0]

    def pipelined_steps(n, e2e, kev=None):
        """n steps: step i = (e2e: copy activations in) + quantize into buffer
        i % 2 + the grouped matvecs (+ e2e: copy the outputs out). Quantize /
        copy-in of step i + 1 run on side streams while step i's matvecs run;
        events order every reuse of a buffer."""
        q_done = [torch.cuda.Event() for _ in range(n)]
        g_done = [torch.cuda.Event() for _ in range(n)]
        o_done = [torch.cuda.Event() for _ in range(n)]

        def prepare(i):
            b = i % 2
            if i >= 2:  # buffer b was last read by step i - 2's matvecs
                s_q.wait_event(g_done[i - 2])
            if e2e:
                s_in.wait_stream(s_q)
                with torch.cuda.stream(s_in):
                    qh.check(L.qh_memcpy_h2d(C.c_void_p(x_dev[b].data_ptr()), C.c_void_p(x_pin.data_ptr()),
                                             x_pin.numel() * 4, C.c_void_p(s_in.cuda_stream)), "h2d")
                s_q.wait_stream(s_in)
            quantize(b, s_q)
            q_done[i].record(s_q)

        prepare(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                prepare(i + 1)
            stream.wait_event(q_done[i])
            if e2e and i >= 2:  # outputs of step i - 2 copied out before they are overwritten
                stream.wait_event(o_done[i - 2])
            timed = kev is not None and i % KEV_EVERY == 0
            if timed:
                kev[i // KEV_EVERY][0].record(stream)
            plans[b].run(sh)
            if timed:
                kev[i // KEV_EVERY][1].record(stream)
            g_done[i].record(stream)
            if e2e:
                s_out.wait_event(g_done[i])
                qh.check(L.qh_memcpy_d2h(C.c_void_p(out_pin[b].data_ptr()), C.c_void_p(out[b].data_ptr()),
                                         out[b].numel() * 4, C.c_void_p(s_out.cuda_stream)), "d2h")
                o_done[i].record(s_out)
        if e2e:
            stream.wait_stream(s_out)
        stream.wait_stream(s_q)

    # ---- device-resident timing ----
    pipelined_steps(args.warmup, False)
    # settle: untimed steps until the GPU runs warm (a timed region that
    # starts from the idle set-up phase measured ~4 % low; the end-to-end run,
    # which follows, was unaffected)
    pipelined_steps(SETTLE_STEPS, False)
    torch.cuda.synchronize()
    uuid = ""
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)
    clocks.start()
    time.sleep(0.3)
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the matvec launch is bracketed by events on every KEV_EVERY-th step only:
    # an event between two launches ends programmatic launch overlap (the
    # matvec then cannot stream its weights while the quantizer finishes), so
    # bracketing every step would slow the pipeline being measured
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range((args.steps + KEV_EVERY - 1) // KEV_EVERY)]
    ev0.record(stream)
    pipelined_steps(args.steps, False, kev)
    ev1.record(stream)
    barrier()
    elapsed_ms = max_time(ev0.elapsed_time(ev1))
    kern_ms = [a.elapsed_time(b) for a, b in kev]
    # ---- end to end through the C-ABI with host buffers ----
    pipelined_steps(2, True)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    pipelined_steps(args.steps, True)
    e1.record(stream)
    barrier()
    e2e_ms = max_time(e0.elapsed_time(e1))
    # the host copies alone, every rank at once: the end-to-end bound when
    # many GPUs share the host's PCIe and memory (slowest rank)
    def copy_ms(dst, src, st, n=20):
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        c0.record(st)
        for _ in range(n):
            dst.copy_(src, non_blocking=True)
        c1.record(st)
        barrier()
        return max_time(c0.elapsed_time(c1)) / n
    with torch.cuda.stream(s_out):
        d2h_ms = copy_ms(out_pin[0], out[0], s_out)
    with torch.cuda.stream(s_in):
        h2d_ms = copy_ms(x_dev[0], x_pin, s_in)
    clk = clocks.stop()
    qh.check(L.qh_check_device_error(None), "device error word")
    if not np.array_equal(out_pin[(args.steps - 1) % 2][G - 1].numpy().view(np.uint32),
                          out[0][G - 1].cpu().numpy().view(np.uint32)):
        raise SystemExit("end-to-end outputs differ from the device-resident run")

    total_bytes = world * G * args.steps * ALGO_BYTES
    value = total_bytes / (elapsed_ms / 1e3) / 1e9
    e2e_value = total_bytes / (e2e_ms / 1e3) / 1e9
    kern_mean_ms = statistics.mean(kern_ms)
    achieved = G * ALGO_BYTES / (kern_mean_ms / 1e3) / 1e9
    peak, peak_kind = peaks()

    for pl in plans:
        pl.close()
    del wdev
    torch.cuda.empty_cache()

    # ---- decode of the synthetic model (configs 4 and 5) ----
    gemm = None
    if not args.no_gemm and world == 1:
        gemm = run_gemm(qh, torch, 20, 3)

    decode = None
    if not args.no_decode:
        dclk = ClockSampler(uuid)
        dclk.start()
        decode = {}
        for B, n_prompt in ((1, 64), (args.decode_batch, args.decode_prompt)):
            if args.decode_only_batch and B != args.decode_only_batch:
                continue
            decode[f"batch{B}"], _, _, _ = run_decode(qh, torch, dist, dp, world, rank, B, n_prompt, args.decode_new,
                                                      args.profile_step)
        if args.sampled:
            for B, n_prompt in ((1, 64), (args.decode_batch, args.decode_prompt)):
                if args.decode_only_batch and B != args.decode_only_batch:
                    continue
                decode[f"sampled_batch{B}"] = run_sampled(qh, torch, B, n_prompt, args.decode_new)
        runs = [v for key, v in decode.items() if key.startswith("batch")]
        decode.update({"clocks": dclk.stop(),
                  "data": "synthetic Qwen3.5-0.8B-shaped weights (Q4_K mix), seeded random prompts",
                  "roofline_peak_gbs": peak, "parallelism": f"dp{world}, replicated weights, "
                  "sampled tokens all-gathered each step by qh_dp_gather_tokens (NCCL)"})
        for d in runs:
            d["hbm_frac"] = round(d["hbm_gbs"] / peak, 4)

    if world > 1:
        dist.barrier()
    if dp is not None:
        dp.close()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        gbs, cores, sample, kind, _ = cpu_reference_run(qh, 64, args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample}

    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemv_q4k_traffic.json")
    if os.path.exists(tpath):
        try:
            with open(tpath) as f:
                t = json.load(f)
            # bytes per matvec measured by ncu, scaled to this launch's G matvecs
            traffic = round(t["dram_bytes_per_matvec"] * G)
        except Exception:
            traffic = None

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8+fp32", "data": "synthetic",
        "config": {"workload": f"Q4_K GEMV K={K_IN} N={N_OUT} (BASELINE config 1) x {G} distinct matrices per GPU per step",
                   "k": K_IN, "n": N_OUT, "pool_matrices_per_gpu": G,
                   "pool_bytes_per_gpu": G * W_BYTES, "l2": "inputs larger than L2 (566 MB pool > 126 MB), no flush",
                   "settle_steps": SETTLE_STEPS,
                   "parallelism": f"dp{world} (independent matrices per GPU)",
                   "tiling": info},
        "pct_of_nominal_8tbs": round(value / (NOMINAL_HBM_GBS * world) * 100, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "kernel": "qh::gemv_kernel<Q4_K,1> (grouped)", "launch_ms": round(kern_mean_ms, 5),
                     "launch_samples": f"every {KEV_EVERY}th of the timed steps ({len(kern_ms)} launches)",
                     "algorithmic_bytes_per_launch": G * ALGO_BYTES, "traffic": traffic},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": G * K_IN * 4, "d2h_bytes_per_step": G * N_OUT * 4,
                "ms_per_step": round(e2e_ms / args.steps, 4),
                "host_copy_gbs": {"d2h": round(G * N_OUT * 4 / (d2h_ms / 1e3) / 1e9, 1),
                                  "h2d": round(G * K_IN * 4 / (h2d_ms / 1e3) / 1e9, 1),
                                  "note": "one step's output / input copies alone on every rank at once, "
                                          "pinned host buffers (slowest rank): the end-to-end limiter at many GPUs"}},
        "gpu_launches": 2 * args.steps,
        "pipelining": "two activation/output buffers: quantize (and e2e copy-in) of step i+1 and copy-out of step i-1 overlap step i's matvecs",
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if gemm is not None:
        line["gemm"] = gemm
    if decode is not None:
        if world == 1 and not args.no_cpu_baseline:
            decode["cpu_baseline"] = cpu_decode_baseline(qh)
        line["decode"] = decode
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--pool", type=int, default=320)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the model decode measurement")
    ap.add_argument("--no-gemm", action="store_true", help="skip the prefill GEMM measurement")
    ap.add_argument("--decode-batch", type=int, default=64, help="sequences per GPU of the batched decode")
    ap.add_argument("--decode-new", type=int, default=256, help="greedy tokens per decode run")
    ap.add_argument("--decode-prompt", type=int, default=512, help="prompt tokens of the batched decode")
    ap.add_argument("--decode-only-batch", type=int, default=0, help="run only the decode of this batch size")
    ap.add_argument("--sampled", action="store_true",
                    help="also time sampled generation (the reference's default sampler chain)")
    ap.add_argument("--profile-step", action="store_true",
                    help="after the timed decode, run one more step between cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
