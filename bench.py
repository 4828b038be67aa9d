"""Benchmark of the Decision Transformer attention path on B200.

One "step" is one fused prefill pass (dt_attn_prefill) over the attention-op
workload of 4096 samples x 192 tokens (64 timesteps x 3), 8 query / 2 KV
heads, head_dim 32, bf16, RoPE positions 0..191, causal + per-sample left
padding U{0..96} tokens.  Inputs are seeded synthetic Q/K/V ~ N(0,1) * 0.5
(no dataset exists for this op; the shapes and value ranges follow the
workload definition).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 the script runs under torchrun (one rank per GPU); every rank
processes its own full batch (weak scaling, no data-path collective) and the
reported time is the maximum over ranks.  ``--impl reference`` times the
CPU oracle (the reference algorithm restated in float32 PyTorch) on the
host cores.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

WORKLOAD = dict(batch=4096, seq_len=192, timesteps=64, q_heads=8, kv_heads=2, head_dim=32, max_pad=96)
METRIC = "DT attention prefill tokens/s (4096 x 192 tokens, 8/2 heads, head_dim 32, causal + left padding)"
UNIT = "tokens/s"


def _peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _algorithmic_bytes(B, S, Hq, Hkv, D) -> int:
    # Read Q, K, V and write O once, bf16 (masks and scores are never stored).
    return 2 * B * S * D * (Hq + 2 * Hkv + Hq)


def _profiled_traffic_per_launch(B: int):
    """DRAM bytes per launch from the committed ncu summary, scaled to B samples."""
    f = REPO / "profiles" / "prefill_short_b1024_s192.txt"
    if not f.exists():
        return None
    meas_b, dram = None, None
    for line in f.read_text().splitlines():
        if line.startswith("batch:"):
            meas_b = int(line.split(":", 1)[1])
        if line.startswith("dram_bytes_per_launch:"):
            dram = float(line.split(":", 1)[1])
    if meas_b and dram:
        return dram * B / meas_b
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, device_index: int, period_s: float = 0.001):
        self.idx, self.period = device_index, period_s
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self.ok = False
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def _dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
        pg = dist
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return rank, world, local, pg


def _make_inputs(B, S, Hq, Hkv, D, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    q = (torch.randn(B, S, Hq, D, device=device, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, S, Hkv, D, device=device, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, S, Hkv, D, device=device, generator=g) * 0.5).to(torch.bfloat16)
    pad = torch.randint(0, WORKLOAD["max_pad"] + 1, (B,), device=device, generator=g, dtype=torch.int32)
    return q, k, v, pad


def cpu_oracle_rate(budget_s: float = 12.0, sample_b: int = 256, threads: int | None = None):
    """Tokens/s of the CPU oracle (reference algorithm in float32 PyTorch) on a bounded sample."""
    from oracle import attention_prefill_ref, mask_from_pad_len, precompute_freqs_cis

    if threads:
        torch.set_num_threads(threads)
    W = WORKLOAD
    B, S, Hq, Hkv, D = sample_b, W["seq_len"], W["q_heads"], W["kv_heads"], W["head_dim"]
    g = torch.Generator().manual_seed(1)
    q = (torch.randn(B, S, Hq, D, generator=g) * 0.5).bfloat16().float()
    k = (torch.randn(B, S, Hkv, D, generator=g) * 0.5).bfloat16().float()
    v = (torch.randn(B, S, Hkv, D, generator=g) * 0.5).bfloat16().float()
    pad = torch.randint(0, W["max_pad"] + 1, (B,), generator=g)
    mask = mask_from_pad_len(pad, S)
    cos, sin = precompute_freqs_cis(D, S)
    attention_prefill_ref(q[:8], k[:8], v[:8], cos, sin, mask[:8])  # warm-up
    t0 = time.perf_counter()
    reps = 0
    while True:
        attention_prefill_ref(q, k, v, cos, sin, mask)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s or reps >= 64:
            break
    tokens = reps * B * S
    return tokens / el, {"cores": torch.get_num_threads(),
                         "sample": f"{reps} x B={B} of {W['batch']} samples, S={S}, fp32 oracle, {el:.1f} s"}


def run_reference(args):
    rank, world, local, pg = _dist_setup(args.gpus)
    if rank != 0:
        if pg:
            pg.destroy_process_group()
        return
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        cpu_oracle_rate(budget_s=0.5, sample_b=64, threads=threads)
    rates, samples = [], []
    for _ in range(args.steps):
        r, info = cpu_oracle_rate(budget_s=2.0, sample_b=128, threads=threads)
        rates.append(r)
        samples.append(info["sample"])
    value = statistics.median(rates)
    W = WORKLOAD
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": W["batch"] * W["seq_len"] / value * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "attention-op prefill, B=4096 S=192 Hq=8 Hkv=2 D=32, left pad U{0..96}",
                   "note": "CPU oracle (reference algorithm in float32 PyTorch), bounded sample per step"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": samples[0] if samples else ""},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)
    if pg:
        pg.destroy_process_group()


def run_ours(args):
    from rl_for_mario_b200 import _lib
    from rl_for_mario_b200.dt_model import rope_tables
    from rl_for_mario_b200.kernels import attn_prefill, attn_prefill_host, device_status

    rank, world, local, pg = _dist_setup(args.gpus)
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (there is no CPU path)")
    _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    W = WORKLOAD
    B, S, Hq, Hkv, D = W["batch"], W["seq_len"], W["q_heads"], W["kv_heads"], W["head_dim"]
    q, k, v, pad = _make_inputs(B, S, Hq, Hkv, D, seed=1234 + rank, device=dev)
    cos, sin = (t.to(dev) for t in rope_tables(D, S, 1e4))
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if pg:
            pg.barrier()

    for _ in range(max(args.warmup, 3)):
        attn_prefill(q, k, v, cos, sin, pad, out=out)
    torch.cuda.synchronize()
    if device_status() != 0:
        raise SystemExit("device status error during warm-up")

    # ---- device-timed region: inputs resident in HBM (1.0 GB/step > 126 MB L2).
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches = 0
    with ClockSampler(dev.index) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            attn_prefill(q, k, v, cos, sin, pad, out=out)
            launches += 1
        ev1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    ms_max = ms
    if pg:
        t = torch.tensor([ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms_max = float(t.item())
    tokens_per_rank = B * S
    value = tokens_per_rank * world / (ms_max * 1e-3)

    # ---- end to end through the public API with pinned host buffers.
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hpad = pad.cpu().pin_memory()
    ho = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    dq, dk, dv, dpad = (torch.empty_like(t) for t in (q, k, v, pad))
    e2e_steps = max(3, min(args.steps, 10))

    def e2e_step():
        # the host-buffer entry point: uploads, kernel and download pipelined over chunks of samples
        attn_prefill_host(hq, hk, hv, cos, sin, hpad, ho, (dq, dk, dv, dpad, out), chunks=8)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if pg:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hpad))
    d2h = ho.numel() * ho.element_size()
    if device_status() != 0:
        raise SystemExit("device status error in the timed region")

    peaks = _peaks()
    byts = _algorithmic_bytes(B, S, Hq, Hkv, D)
    achieved = byts / (ms * 1e-3) / 1e9
    traffic = _profiled_traffic_per_launch(B)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": f"attention-op prefill, B={B} S=192 Hq=8 Hkv=2 D=32 per GPU, left pad U{{0..96}}",
                   "parallelism": f"dp{world} (independent batches, no data-path collective)",
                   "l2": "inputs larger than L2 (1.0 GB per step vs 126 MB)",
                   "kernel": "dt_prefill_short_kernel (tcgen05 + TMA, persistent)"},
        "clocks": clk.summary(),
        "e2e": {"value": tokens_per_rank * world / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                     "algorithmic_bytes_per_launch": byts, "peak_source": peaks["source"]},
    }
    if not args.no_decode:
        cpu = world == 1 and not args.no_cpu_baseline
        if world == 1:
            line["dt_forward_cfg1"] = bench_dt_cfg1(dev, cpu=cpu)
            line["decode"] = bench_decode_cfg3(dev, peaks, cpu=cpu)
            line["prefill_long"] = bench_prefill_cfg4(dev, peaks, cpu=cpu)
            line["prefill_long"]["rmsnorm_qkv_kernel"] = bench_rmsnorm_qkv_cfg4(dev, peaks)
            line["prefill_long"]["rmsnorm_swiglu_kernel"] = bench_rmsnorm_swiglu_cfg4(dev, peaks)
            line["prefill_long"]["encoder_conv1_kernel"] = bench_conv1_cfg4(dev, peaks)
            line["prefill_long"]["encoder_conv23_kernels"] = bench_conv23_cfg4(dev, peaks)
            line["prefill_long"]["residual_gemms"] = bench_gemm_residual_cfg4(dev, peaks)
            line["nes_env"] = bench_nes_env(dev, peaks, cpu=cpu)
            line["nes_env"]["policy_loop"] = bench_nes_policy(dev)
        line["rollout"] = bench_rollout_cfg5(dev, world, rank, pg, cpu=cpu)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, info = cpu_oracle_rate(budget_s=12.0, sample_b=256, threads=len(os.sched_getaffinity(0)))
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": info["cores"], "kind": "port",
                                "sample": info["sample"]}
    if rank == 0:
        emit(line)
    if pg:
        pg.destroy_process_group()


# ----------------------------------------------------------------------------- CPU baselines (oracle port)
# The reference's CPU path restated by the oracle (float32 PyTorch, pinned to
# the reference's own outputs by the golden tests), timed on the host cores on a
# bounded slice of each workload.  Reported next to the GPU numbers, not targets.

def _cpu_threads() -> int:
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    return n


def _oracle_cfg(cfg) -> dict:
    return {k: getattr(cfg, k) for k in ("state_shape", "act_dim", "max_ep_len", "context_len", "hidden_size",
                                         "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                                         "intermediate_size", "rms_norm_eps", "rope_theta")}


def _cpu_sd(model) -> dict:
    return {k: v.detach().float().cpu() for k, v in model.state_dict().items()}


def cpu_dt_forward(model, B: int, T: int, pad_max: int, budget_s: float = 6.0, seed: int = 0):
    """Tokens/s of the oracle's full DT forward (fp32, CPU) on B samples of T timesteps."""
    from oracle.dt_ref import dt_forward_ref
    from oracle.seeded import dt_synthetic_inputs

    threads = _cpu_threads()
    cfgd = _oracle_cfg(model.config)
    sd = _cpu_sd(model)
    inp = dt_synthetic_inputs("bench_cpu", seed, B, T, cfgd["state_shape"], cfgd["act_dim"], pad_max)
    reps, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while True:
            dt_forward_ref(sd, cfgd, inp["states"], inp["actions"], inp["rtg"], inp["timesteps"], inp.get("mask"))
            reps += 1
            el = time.perf_counter() - t0
            if el >= budget_s:
                break
    return {"value": reps * B * 3 * T / el, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{reps} forward(s) of B={B} x {3 * T} tokens, fp32 oracle, {el:.1f} s"}


def cpu_cached_steps(model, B: int, prefix: int, steps: int, tokens_per_step: int = 3, seed: int = 0):
    """Env-steps/s of the oracle's cached decode (the reference's cat-based cache,
    fp32, CPU): a prefix of hidden states prefilled (not timed), then `steps`
    cached steps of `tokens_per_step` hidden tokens through every layer, final
    norm and action head."""
    from oracle.attention_ref import precompute_freqs_cis, rmsnorm_ref
    from oracle.dt_ref import block_ref

    threads = _cpu_threads()
    cfgd = _oracle_cfg(model.config)
    sd = _cpu_sd(model)
    H, L = cfgd["hidden_size"], cfgd["num_hidden_layers"]
    cos, sin = precompute_freqs_cis(H // cfgd["num_attention_heads"], prefix + tokens_per_step * steps + 1,
                                    cfgd["rope_theta"])
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        h = torch.randn(B, prefix, H, generator=g)
        past = [None] * L
        for i in range(L):
            h, past[i] = block_ref(sd, cfgd, i, h, cos[:prefix], sin[:prefix], None, True, None)
        pos = prefix
        t0 = time.perf_counter()
        for _ in range(steps):
            h = torch.randn(B, tokens_per_step, H, generator=g)
            c, s_ = cos[pos:pos + tokens_per_step], sin[pos:pos + tokens_per_step]
            for i in range(L):
                h, past[i] = block_ref(sd, cfgd, i, h, c, s_, past[i], True, None)
            st = rmsnorm_ref(h[:, -1], sd["model.norm.weight"], cfgd["rms_norm_eps"])
            (st @ sd["action_head.weight"].t()).argmax(-1)
            pos += tokens_per_step
        el = time.perf_counter() - t0
    return {"value": B * steps / el, "unit": "env-steps/s", "cores": threads, "kind": "port",
            "sample": f"B={B} envs x {steps} cached steps of {tokens_per_step} tokens after a {prefix}-token prefix, "
                      f"fp32 oracle (cat-based cache), {el:.1f} s"}


def cpu_rollout(model, B: int, steps: int, seed: int = 0):
    """Env-steps/s of a cached rollout on the oracle (fp32, CPU): per step the CNN
    on the uint8 frames, the (a, R, s) embeddings, every layer with the cat-based
    cache, final norm and action head, from an empty cache."""
    from oracle.attention_ref import precompute_freqs_cis, rmsnorm_ref
    from oracle.dt_ref import block_ref, embed_tokens_ref

    threads = _cpu_threads()
    cfgd = _oracle_cfg(model.config)
    sd = _cpu_sd(model)
    L = cfgd["num_hidden_layers"]
    cos, sin = precompute_freqs_cis(cfgd["hidden_size"] // cfgd["num_attention_heads"], 3 * steps + 3,
                                    cfgd["rope_theta"])
    g = torch.Generator().manual_seed(seed)
    past = [None] * L
    pos = 0
    with torch.no_grad():
        t0 = time.perf_counter()
        for t in range(steps):
            fr = torch.randint(0, 256, (B, 1) + tuple(cfgd["state_shape"]), generator=g, dtype=torch.uint8)
            act = torch.randint(0, cfgd["act_dim"], (B, 1), generator=g)
            rtg = torch.rand(B, 1, generator=g) * 3000
            ts = torch.full((B, 1), t, dtype=torch.long)
            h = embed_tokens_ref(sd, cfgd, fr, act, rtg, ts)  # 3 tokens per env, as a cached step appends
            c, s_ = cos[pos:pos + 3], sin[pos:pos + 3]
            for i in range(L):
                h, past[i] = block_ref(sd, cfgd, i, h, c, s_, past[i], True, None)
            st = rmsnorm_ref(h[:, -1], sd["model.norm.weight"], cfgd["rms_norm_eps"])
            (st @ sd["action_head.weight"].t()).argmax(-1)
            pos += 3
        el = time.perf_counter() - t0
    return {"value": B * steps / el, "unit": "env-steps/s", "cores": threads, "kind": "port",
            "sample": f"B={B} envs x {steps} steps from an empty cache (CNN + embeddings + {L} layers), "
                      f"fp32 oracle, {el:.1f} s"}


# ----------------------------------------------------------------------------- decode workloads
DECODE_CFG = dict(envs=16384, prefix=189, steps=21, hidden=256, layers=4, q_heads=8, kv_heads=2, head_dim=32)
ROLLOUT_CFG = dict(envs_per_gpu=8192, steps=64, hidden=256, layers=4, q_heads=8, kv_heads=2, context_len=64)


def _decode_kernel_bytes(B, L, Sn, Hq, Hkv, D):
    """Algorithmic bytes of one dt_attn_decode launch: read the L cached K/V rows,
    read q / k_new / v_new, write o and the appended K/V rows (bf16)."""
    return 2 * (2 * B * Hkv * L * D + B * Sn * (2 * Hq + 4 * Hkv) * D)


def bench_decode_cfg3(dev, peaks, cpu: bool = False, envs=None):
    """16,384 environments, cache prefilled with 189 tokens, 21 cached steps of 3 tokens
    (``envs``: another environment count, for profiling a smaller case)."""
    from rl_for_mario_b200 import kernels
    from rl_for_mario_b200.cache import PagedKVCache
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT

    C = DECODE_CFG
    torch.manual_seed(2)
    cfg = DTConfig(hidden_size=C["hidden"], num_hidden_layers=C["layers"], num_attention_heads=C["q_heads"],
                   num_key_value_heads=C["kv_heads"], context_len=(C["prefix"] + 3 * C["steps"]) // 3, dropout=0.0)
    model = MarioDT(cfg).to(dev, torch.bfloat16).eval()
    B, H = envs or C["envs"], C["hidden"]
    max_len = C["prefix"] + 3 * C["steps"]
    cache = PagedKVCache(C["layers"], B, C["kv_heads"], C["head_dim"], max_len, page_size=64, dtype=torch.bfloat16,
                         device=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    steps_h = torch.randn(C["steps"], B, 3, H, device=dev, generator=g).to(torch.bfloat16)
    bb = model.model

    def prefill():
        cache.reset()
        with torch.no_grad():
            hp = torch.randn(B, C["prefix"], H, device=dev, generator=g).to(torch.bfloat16)
            bb.run_layers(hp, None, cache, use_cache=True, flat=True)
            del hp

    def run_steps():
        acts = None
        with torch.no_grad():
            for t in range(C["steps"]):
                h, _ = bb.run_layers(steps_h[t], None, cache, use_cache=True, flat=True)
                acts = model.action_head(h[:, 1]).argmax(-1)  # state token of (R, s, a)
        return acts

    prefill()
    run_steps()  # warm-up
    times = []
    for _ in range(2):
        prefill()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run_steps()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = min(times)
    # The decode kernel alone at the mid-point length (no advance: same slots rewritten).
    lay = cache[0]
    L_mid = C["prefix"] + 3 * (C["steps"] // 2)
    saved = lay.length
    lay.seq_lens.fill_(L_mid)
    lay.length = L_mid
    q = torch.randn(B, 3, C["q_heads"], C["head_dim"], device=dev, generator=g).to(torch.bfloat16)
    kn = torch.randn(B, 3, C["kv_heads"], C["head_dim"], device=dev, generator=g).to(torch.bfloat16)
    cos, sin = bb.freqs_cos[L_mid:L_mid + 3], bb.freqs_sin[L_mid:L_mid + 3]
    out = torch.empty_like(q)
    for _ in range(3):
        kernels.attn_decode(q, kn, kn, lay, cos, sin, out=out)
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 20
    k0.record()
    for _ in range(n):
        kernels.attn_decode(q, kn, kn, lay, cos, sin, out=out)
    k1.record()
    torch.cuda.synchronize()
    kms = k0.elapsed_time(k1) / n
    lay.seq_lens.fill_(saved)
    lay.length = saved
    kb = _decode_kernel_bytes(B, L_mid, 3, C["q_heads"], C["kv_heads"], C["head_dim"])
    ach = kb / (kms * 1e-3) / 1e9
    res = {
        "metric": "rollout decode env-steps/s (cached, 3 tokens per step)", "unit": "env-steps/s",
        "value": B * C["steps"] / (ms * 1e-3), "ms_total": ms,
        "config": {"workload": "16384 envs, 189-token prefix, 21 steps x 3 tokens -> 252, 4 layers, hidden 256, "
                               "8/2 heads, head_dim 32, bf16, hidden inputs N(0,1), argmax of the 7-way head"},
        "kernel_roofline": {"kernel": "dt_decode_kernel", "bound": "hbm", "kv_len": L_mid + 3, "ms": kms,
                            "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": ach / peaks["hbm_gbs"],
                            "algorithmic_bytes_per_launch": kb},
    }
    del cache, steps_h
    torch.cuda.empty_cache()
    if cpu:
        res["cpu_baseline"] = cpu_cached_steps(model, B=512, prefix=C["prefix"], steps=C["steps"])
    del model
    return res


CFG1 = dict(batch=4, timesteps=64, hidden=256, layers=4, q_heads=8, kv_heads=2, pad_max_timesteps=32)


def bench_dt_cfg1(dev, cpu: bool = False):
    """The repo-default DT forward at its own batch (4 x 64 timesteps = 768 tokens,
    hidden 256, 4 layers, 8/2 heads, left padding U{0..32} timesteps): the fp32
    model on the fp32 kernels, the bf16 model with fused blocks, and the oracle's
    fp32 forward on the host cores.  A latency-bound workload (one small batch)."""
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT
    from oracle.seeded import dt_synthetic_inputs

    C = CFG1
    B, T = C["batch"], C["timesteps"]
    torch.manual_seed(0)
    cfg = DTConfig(hidden_size=C["hidden"], num_hidden_layers=C["layers"], num_attention_heads=C["q_heads"],
                   num_key_value_heads=C["kv_heads"], context_len=T, dropout=0.0)
    base = MarioDT(cfg).eval()
    inp = {k: v.to(dev) for k, v in dt_synthetic_inputs("bench_cfg1", 0, B, T, cfg.state_shape, cfg.act_dim,
                                                           C["pad_max_timesteps"]).items()}
    res = {"metric": "DT forward tokens/s (4 x 64 timesteps = 768 tokens, hidden 256, 4 layers, 8/2 heads)",
           "unit": "tokens/s", "config": {"workload": "repo-default DT, batch 4 x 64 timesteps, left pad "
                                                      "U{0..32} timesteps, synthetic inputs, random-init weights"}}
    allow = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    try:
        for name, dtype, fused in (("fp32", torch.float32, False), ("bf16_fused", torch.bfloat16, True)):
            m = MarioDT(cfg).eval()
            m.load_state_dict(base.state_dict())
            m = m.to(dev, dtype)
            if fused:
                m.fuse_norms()

            def fwd():
                with torch.no_grad():
                    return m(inp["states"], inp["actions"], inp["rtg"], inp["timesteps"],
                             attention_mask=inp["mask"]).action_logits

            for _ in range(3):
                fwd()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = 10
            e0.record()
            for _ in range(n):
                fwd()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / n
            res[name] = {"value": B * 3 * T / (ms * 1e-3), "ms": ms}
            del m
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = allow
    res["value"] = res["bf16_fused"]["value"]
    if cpu:
        res["cpu_baseline"] = cpu_dt_forward(base, B=B, T=T, pad_max=C["pad_max_timesteps"], budget_s=6.0)
    return res


PREFILL_LONG_CFG = dict(batch=1024, timesteps=256, hidden=768, layers=12, q_heads=12, kv_heads=4, head_dim=64,
                        ffn=2048, pad_max_timesteps=128)


def _attended_pairs(S: int, pads) -> int:
    """(query, key) pairs the masks allow, summed over samples: a valid row q >= pad
    sees keys pad..q, a fully padded row q < pad sees keys 0..q."""
    tot = 0
    for p in pads:
        p = int(p)
        tot += p * (p + 1) // 2 + (S - p) * (S - p + 1) // 2
    return tot


def bench_prefill_cfg4(dev, peaks, batch=None, model=True, cpu: bool = False):
    """Larger DT prefill: B=1024, 256 timesteps (768 tokens), hidden 768, 12 layers, 12/4 heads, head_dim 64.

    (a) the attention op alone at that shape, with Q / K rotated upstream as in
    the model path (the fused RMSNorm + QKV + RoPE epilogue), timed per launch
    against the tensor-core roofline; (b) the full DT forward (CNN state
    encoder, embeddings, 12 blocks with fused RMSNorm + QKV + RoPE, final norm,
    action head) in tokens/s."""
    from rl_for_mario_b200.kernels import attn_prefill, device_status
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT, rope_tables

    C = PREFILL_LONG_CFG
    B, T = batch or C["batch"], C["timesteps"]
    S, Hq, Hkv, D = 3 * T, C["q_heads"], C["kv_heads"], C["head_dim"]
    g = torch.Generator(device=dev).manual_seed(4)
    # (a) attention op
    q = (torch.randn(B, S, Hq, D, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, S, Hkv, D, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, S, Hkv, D, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    pad_t = torch.randint(0, C["pad_max_timesteps"] + 1, (B,), device=dev, generator=g, dtype=torch.int32)
    pad = (3 * pad_t).to(torch.int32)
    cos, sin = (t.to(dev) for t in rope_tables(D, S, 1e4))
    out = torch.empty_like(q)
    for _ in range(3):
        attn_prefill(q, k, v, cos, sin, pad, out=out, apply_rope=False)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 10
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        e0.record()
        for _ in range(n):
            attn_prefill(q, k, v, cos, sin, pad, out=out, apply_rope=False)
        e1.record()
        torch.cuda.synchronize()
    if device_status() != 0:
        raise SystemExit("device status error in the long-prefill benchmark")
    kms = e0.elapsed_time(e1) / n
    flops = 4 * Hq * D * _attended_pairs(S, pad.cpu().tolist())
    tflops = flops / (kms * 1e-3) / 1e12
    byts = _algorithmic_bytes(B, S, Hq, Hkv, D)
    del q, k, v, out
    torch.cuda.empty_cache()
    # The binding resource: the larger of the FLOP time at the GEMM peak and the
    # byte time at the HBM peak (per launch); frac = that lower bound / the time.
    t_flop = flops / (peaks["bf16_tflops"] * 1e12)
    t_byte = byts / (peaks["hbm_gbs"] * 1e9)
    # One exponential per attended score on the MUFU unit, 16 per clock per SM
    # (measured 15.99 on this part), at the SM clock the timed region ran at.
    exps = Hq * _attended_pairs(S, pad.cpu().tolist())
    props = torch.cuda.get_device_properties(dev)
    sm_hz = (clk.summary().get("sm_mhz") or 1965) * 1e6
    t_exp = exps / (16 * props.multi_processor_count * sm_hz)
    bound = max((t_flop, "tensor"), (t_byte, "hbm"), (t_exp, "mufu (exp2)"))[1]
    kernel_res = {"kernel": "dt_prefill_long_kernel", "inputs": "q / k rotated upstream", "batch": B, "ms": kms,
                  "tokens_per_s": B * S / (kms * 1e-3),
                  "roofline": {"bound": bound, "lower_bound_ms": max(t_flop, t_byte, t_exp) * 1e3,
                               "frac": max(t_flop, t_byte, t_exp) / (kms * 1e-3),
                               "exp_lower_bound_ms": t_exp * 1e3, "exps_per_launch": exps,
                               "exp_frac": t_exp / (kms * 1e-3),
                               "achieved_tflops": tflops, "peak_tflops": peaks["bf16_tflops"],
                               "tensor_frac": tflops / peaks["bf16_tflops"], "flops_per_launch": flops,
                               "achieved_gbs": byts / (kms * 1e-3) / 1e9, "peak_gbs": peaks["hbm_gbs"],
                               "hbm_frac": byts / (kms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                               "algorithmic_bytes_per_launch": byts, "peak_source": peaks["source"]}}
    if not model:
        return {"attention_kernel": kernel_res}

    # (a') the drop-in module on the normalised layer input, as inside the
    # reference's block: q | k | v + RoPE in one GEMM, the attention kernel on
    # pre-rotated q / k, o_proj; against the same module with the projections
    # on cuBLAS and the RoPE inside the attention kernel.
    from rl_for_mario_b200.attention import FastDTAttention

    class _Cfg:
        hidden_size, num_attention_heads, num_key_value_heads = C["hidden"], Hq, Hkv
        dropout, flash_attn = 0.0, True

    att = FastDTAttention(_Cfg()).to(dev, torch.bfloat16).eval()
    xin = torch.randn(B, S, C["hidden"], device=dev, generator=g).to(torch.bfloat16)
    mask_tok = (torch.arange(S, device=dev)[None, :] >= pad[:, None].long()).to(torch.bfloat16)
    dropin = {}
    for name, rounding in (("one_gemm_qkv_rope", "fp32"), ("cublas_projections_rope_in_kernel", "reference")):
        # "reference" RoPE rounding keeps the separate projections + in-kernel RoPE path
        att.rope_rounding = rounding
        with torch.no_grad():
            for _ in range(2):
                att(xin, (cos, sin), attention_mask=mask_tok)
            torch.cuda.synchronize()
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            d0.record()
            for _ in range(3):
                att(xin, (cos, sin), attention_mask=mask_tok)
            d1.record()
            torch.cuda.synchronize()
        dropin[name] = {"ms": d0.elapsed_time(d1) / 3}
    dropin["note"] = ("FastDTAttention.forward on [1024, 768, 768] bf16 input with the padding mask "
                      "(projections, RoPE, attention, o_proj)")
    kernel_res["dropin_module_layer"] = dropin
    del att, xin
    torch.cuda.empty_cache()

    # (b) full model forward
    torch.manual_seed(4)
    cfg = DTConfig(hidden_size=C["hidden"], num_hidden_layers=C["layers"], num_attention_heads=Hq,
                   num_key_value_heads=Hkv, context_len=T, intermediate_size=C["ffn"], dropout=0.0)
    model = MarioDT(cfg).to(dev, torch.bfloat16).eval().fuse_norms()
    states = torch.randint(0, 256, (B, T) + tuple(cfg.state_shape), device=dev, generator=g, dtype=torch.uint8)
    actions = torch.randint(0, cfg.act_dim, (B, T), device=dev, generator=g)
    rtg = torch.rand(B, T, device=dev, generator=g) * 3000.0
    start = torch.randint(0, cfg.max_ep_len - T, (B, 1), device=dev, generator=g)
    ts = start + torch.arange(T, device=dev)
    mask = (torch.arange(T, device=dev)[None, :] >= pad_t[:, None].long()).to(torch.bfloat16)

    def forward():
        with torch.no_grad():
            h, _ = model.model(states, actions, rtg, ts, mask)
            return model.action_head(h[:, -1, 1]).argmax(-1)

    forward()
    torch.cuda.synchronize()
    times = []
    for _ in range(2):
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record()
        forward()
        f1.record()
        torch.cuda.synchronize()
        times.append(f0.elapsed_time(f1))
    fms = min(times)
    # Whole-forward FLOPs: per token and layer the q|k|v, o_proj, gate|up and down GEMMs
    # (2 H ((Hq + 2 Hkv) D + Hq D + 3 F)), the attention (the kernel's count per layer), and
    # the state encoder per frame (8x8/4, 4x4/2, 3x3 convolutions and the Linear).
    H, F, L = C["hidden"], C["ffn"], C["layers"]
    lin_tok = 2 * H * ((Hq + 2 * Hkv) * D + Hq * D + 3 * F)
    enc_frame = 2 * (32 * 4 * 64 * 400 + 64 * 32 * 16 * 81 + 64 * 64 * 9 * 49 + 3136 * H)
    fwd_flops = L * (B * S * lin_tok + flops) + B * T * enc_frame
    ftf = fwd_flops / (fms * 1e-3) / 1e12
    res = {
        "metric": "DT prefill tokens/s (full forward, 1024 x 768 tokens, hidden 768, 12 layers)", "unit": "tokens/s",
        "value": B * S / (fms * 1e-3), "ms": fms,
        "config": {"workload": "1024 x 256 timesteps (768 tokens), hidden 768, 12 layers, 12/4 heads, head_dim 64, "
                               "FFN 2048, bf16, fused blocks (RMSNorm+QKV+RoPE, attention, o_proj+residual, "
                               "RMSNorm+gate/up+SwiGLU, down+residual), synthetic uint8 frames, left pad "
                               "U{0..128} timesteps, random-init weights"},
        # a seconds-long sequence of kernels: the sustained GEMM peak is the denominator
        "roofline": {"bound": "tensor", "achieved": ftf, "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": ftf / peaks["bf16_tflops_sustained"], "flops_per_forward": fwd_flops,
                     "peak_source": peaks["source"] + " (sustained)"},
        "attention_kernel": kernel_res,
    }
    del states
    torch.cuda.empty_cache()
    if cpu:
        res["cpu_baseline"] = cpu_dt_forward(model, B=8, T=T, pad_max=C["pad_max_timesteps"], budget_s=1.0)
    del model
    return res


def bench_rmsnorm_qkv_cfg4(dev, peaks, batch=None):
    """The fused RMSNorm + Q/K/V projection + RoPE kernel at a cfg4 layer's shape:
    M = batch x 768 tokens, K = hidden 768, N = (12 + 2 x 4) x 64 = 1280."""
    from rl_for_mario_b200.dt_model import rope_tables
    from rl_for_mario_b200.kernels import device_status, fold_norm_weight, rmsnorm_qkv

    C = PREFILL_LONG_CFG
    B, S, H = batch or C["batch"], 3 * C["timesteps"], C["hidden"]
    Hq, Hkv, D = C["q_heads"], C["kv_heads"], C["head_dim"]
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(B, S, H, device=dev, generator=g).to(torch.bfloat16)
    wq, wk, wv = (torch.randn(h * D, H, device=dev, generator=g) / H ** 0.5 for h in (Hq, Hkv, Hkv))
    wf = fold_norm_weight(wq, wk, wv, torch.ones(H, device=dev), torch.bfloat16)
    cos, sin = (t.to(dev) for t in rope_tables(D, S, 1e4))
    rope = (cos, sin, (Hq + Hkv) * D, D)
    out = torch.empty(B, S, (Hq + 2 * Hkv) * D, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        rmsnorm_qkv(x, wf, 1e-5, out=out, rope=rope)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 10
    e0.record()
    for _ in range(n):
        rmsnorm_qkv(x, wf, 1e-5, out=out, rope=rope)
    e1.record()
    torch.cuda.synchronize()
    if device_status() != 0:
        raise SystemExit("device status error in the RMSNorm + QKV benchmark")
    ms = e0.elapsed_time(e1) / n
    M, N = B * S, (Hq + 2 * Hkv) * D
    flops = 2 * M * H * N
    tf = flops / (ms * 1e-3) / 1e12
    return {"kernel": "dt_rmsnorm_qkv_persist_kernel", "shape": {"M": M, "K": H, "N": N}, "ms": ms,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "flops_per_launch": flops,
                         "peak_source": peaks["source"]}}


def bench_rmsnorm_swiglu_cfg4(dev, peaks, batch=None):
    """The fused post-attention RMSNorm + gate/up + SwiGLU kernel at a cfg4 layer's
    shape: M = batch x 768 tokens, K = hidden 768, FFN width 2048 (4096 GEMM columns)."""
    from rl_for_mario_b200.kernels import device_status, fold_swiglu_weight, rmsnorm_swiglu

    C = PREFILL_LONG_CFG
    B, S, H, F = batch or C["batch"], 3 * C["timesteps"], C["hidden"], C["ffn"]
    g = torch.Generator(device=dev).manual_seed(6)
    x = torch.randn(B, S, H, device=dev, generator=g).to(torch.bfloat16)
    wg, wu = (torch.randn(F, H, device=dev, generator=g) / H ** 0.5 for _ in range(2))
    wf = fold_swiglu_weight(wg, wu, torch.ones(H, device=dev), torch.bfloat16)
    out = torch.empty(B, S, F, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        rmsnorm_swiglu(x, wf, 1e-5, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 10
    e0.record()
    for _ in range(n):
        rmsnorm_swiglu(x, wf, 1e-5, out=out)
    e1.record()
    torch.cuda.synchronize()
    if device_status() != 0:
        raise SystemExit("device status error in the RMSNorm + SwiGLU benchmark")
    ms = e0.elapsed_time(e1) / n
    M = B * S
    flops = 2 * M * H * 2 * F
    tf = flops / (ms * 1e-3) / 1e12
    return {"kernel": "dt_rmsnorm_qkv_persist_kernel (SwiGLU epilogue)", "shape": {"M": M, "K": H, "N": 2 * F},
            "ms": ms,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": tf / peaks["bf16_tflops"], "flops_per_launch": flops,
                         "peak_source": peaks["source"]}}


def bench_gemm_residual_cfg4(dev, peaks, batch=None):
    """The block's residual GEMMs at a cfg4 layer's shape (M = batch x 768 tokens):
    o_proj (K = 768, N = 768) and down_proj (K = FFN 2048, N = 768), each y += x W^T
    in place on dt_gemm_residual, with cuBLAS's addmm_ on the same operands timed
    beside it."""
    from rl_for_mario_b200.kernels import device_status, gemm_residual

    C = PREFILL_LONG_CFG
    B, S, H = batch or C["batch"], 3 * C["timesteps"], C["hidden"]
    M = B * S
    g = torch.Generator(device=dev).manual_seed(6)
    res = {}
    R = ROLLOUT_CFG
    shapes = (("o_proj", M, C["q_heads"] * C["head_dim"], H), ("down_proj", M, C["ffn"], H),
              # one rollout step of 8,192 environments x 3 tokens, hidden 256, FFN 704
              ("rollout_o_proj", R["envs_per_gpu"] * 3, R["hidden"], R["hidden"]),
              ("rollout_down_proj", R["envs_per_gpu"] * 3, 704, R["hidden"]))
    for name, M, K, H in shapes:
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(H, K, device=dev, generator=g) / K ** 0.5).to(torch.bfloat16)
        y = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
        out = {}
        for impl, fn in (("ours", lambda: gemm_residual(x, w, y)), ("cublas_addmm", lambda: y.addmm_(x, w.t()))):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = 10
            e0.record()
            for _ in range(n):
                fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / n
            tf = 2 * M * K * H / (ms * 1e-3) / 1e12
            out[impl] = {"ms": ms, "tflops": tf, "frac": tf / peaks["bf16_tflops"]}
        if device_status() != 0:
            raise SystemExit("device status error in the residual-GEMM benchmark")
        res[name] = {"kernel": "dt_rmsnorm_qkv_persist_kernel (resid mode)", "M": M, "K": K, "N": H, **out,
                     "roofline": {"bound": "tensor", "achieved": out["ours"]["tflops"], "peak": peaks["bf16_tflops"],
                                  "unit": "TFLOP/s", "frac": out["ours"]["frac"], "peak_source": peaks["source"]}}
        del x, w, y
    torch.cuda.empty_cache()
    return res


def bench_conv1_cfg4(dev, peaks, batch=None):
    """The state encoder's first layer at cfg4's shape: batch x 256 frame stacks of
    4 x 84 x 84 uint8 -> relu(conv 8x8/4 + bias) with the /255 test, one kernel
    (dt_frames_conv1) plus its early-exit frame-max pre-pass."""
    from rl_for_mario_b200.kernels import device_status, frames_conv1

    C = PREFILL_LONG_CFG
    n = (batch or C["batch"]) * C["timesteps"]
    g = torch.Generator(device=dev).manual_seed(7)
    fr = torch.randint(0, 256, (n, 4, 84, 84), device=dev, generator=g, dtype=torch.uint8)
    w = (torch.randn(32, 4, 8, 8, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(32, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    for _ in range(3):
        out, _ = frames_conv1(fr, w, b)
    del out
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record()
    for _ in range(reps):
        out, _ = frames_conv1(fr, w, b)
    e1.record()
    torch.cuda.synchronize()
    if device_status() != 0:
        raise SystemExit("device status error in the first-layer benchmark")
    ms = e0.elapsed_time(e1) / reps
    byts = fr.numel() + out.numel() * 2  # uint8 frames in, bf16 activations out
    flops = 2 * n * 400 * 32 * 256
    gbs = byts / (ms * 1e-3) / 1e9
    del fr, out
    torch.cuda.empty_cache()
    return {"kernel": "frames_conv1_kernel", "frames": n, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_launch": byts,
                         "peak_source": peaks["source"]}}


# Shared-memory operand bytes the fused layer-2/3 kernel's MMAs read per frame:
# conv2 2 x 8 MMAs of 128 x 128 x 16 (4 KB of A + 4 KB of B each), conv3 3 x 4 of
# 128 x 192 x 16 (4 KB + 6 KB); the tensor core reads them at up to 128 bytes
# per clock per SM.
CONV23_OPERAND_BYTES_PER_FRAME = 16 * (4096 + 4096) + 12 * (4096 + 6144)


def conv23_bound(n_frames: int, ms: float, sm_mhz: float, n_sms: int) -> dict:
    """The fused layer-2/3 kernel's binding resource, the shared-memory operand
    path: its floor (operand bytes at 128 B per clock per SM, at the given SM
    clock) and the fraction of it that `ms` reaches."""
    floor_s = n_frames * CONV23_OPERAND_BYTES_PER_FRAME / (128.0 * n_sms * sm_mhz * 1e6)
    return {"bound": "shared-memory operand reads", "operand_bytes_per_frame": CONV23_OPERAND_BYTES_PER_FRAME,
            "lower_bound_ms": floor_s * 1e3, "frac": floor_s / (ms * 1e-3), "sm_mhz": sm_mhz}


def bench_conv23_cfg4(dev, peaks, batch=None):
    """The state encoder's second and third layers at cfg4's shape (batch x 256
    frames of the first layer's 32 x 20 x 20 output): dt_encoder_conv23 (one
    fused tcgen05 kernel; ms with layer 2's output stored, ms_without_y2 as the
    model runs it) against cuDNN's fused convolution + bias + ReLU, one call
    per layer, on the same channels-last bf16 tensors."""
    from rl_for_mario_b200.kernels import device_status, encoder_conv23

    C = PREFILL_LONG_CFG
    n = (batch or C["batch"]) * C["timesteps"]
    g = torch.Generator(device=dev).manual_seed(8)
    cl = torch.channels_last
    x1 = torch.relu(torch.randn(n, 32, 20, 20, device=dev, generator=g)).to(torch.bfloat16).contiguous(memory_format=cl)
    w2 = (torch.randn(64, 32, 4, 4, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    b2 = (torch.randn(64, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    w3 = (torch.randn(64, 64, 3, 3, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    b3 = (torch.randn(64, device=dev, generator=g) * 0.1).to(torch.bfloat16)
    w2c, w3c = w2.contiguous(memory_format=cl), w3.contiguous(memory_format=cl)

    def ours():
        return encoder_conv23(x1, w2, b2, w3, b3)

    def ours_no_y2():  # the model's use: conv2's output stays in shared memory
        return encoder_conv23(x1, w2, b2, w3, b3, keep_y2=False)

    def cudnn():
        y2 = torch.cudnn_convolution_relu(x1, w2c, b2, (2, 2), (0, 0), (1, 1), 1)
        return y2, torch.cudnn_convolution_relu(y2, w3c, b3, (1, 1), (0, 0), (1, 1), 1)

    res, mhz = {}, None
    for name, fn in (("ours", ours), ("ours_no_y2", ours_no_y2), ("cudnn", cudnn)):
        for _ in range(3):
            out = fn()
        del out
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        with ClockSampler(dev.index if dev.index is not None else 0) as clk:
            e0.record()
            for _ in range(reps):
                out = fn()
            e1.record()
            torch.cuda.synchronize()
        if name == "ours_no_y2":
            mhz = clk.summary().get("sm_mhz")
        del out
        res[name] = e0.elapsed_time(e1) / reps
    if device_status() != 0:
        raise SystemExit("device status error in the encoder-conv benchmark")
    flops = 2 * n * (81 * 64 * 512 + 49 * 64 * 576)
    byts = n * (32 * 400 + 2 * 64 * 81 + 64 * 49) * 2  # x1 in, y2 out and in again, y3 out
    ms = res["ours"]
    gbs = byts / (ms * 1e-3) / 1e9
    del x1
    torch.cuda.empty_cache()
    n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    return {"kernel": "encoder_conv23_kernel (conv2 + conv3 fused)", "frames": n, "ms": ms,
            "ms_without_y2": res["ours_no_y2"], "cudnn_ms": res["cudnn"],
            "roofline_operands": conv23_bound(n, res["ours_no_y2"], mhz or 1965.0, n_sms),
            "tflops": flops / (ms * 1e-3) / 1e12,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_launch": byts,
                         "peak_source": peaks["source"]}}



NES_ENV_CFG = {"envs": 65536, "frame_skip": 4, "frame_stack": 4,
               "cartridge": "nes_roms.demo_rom(): synthetic 32 KB NROM (the SMB ROM is not shipped)"}


def _nes_cpu_baseline(seconds: float = 8.0) -> dict:
    """The C oracle (one host thread) on a bounded sample: 8 environments,
    4-frame steps after the boot sequence, until `seconds` have passed."""
    from oracle.nes import OracleEnv
    from rl_for_mario_b200.nes_roms import demo_rom

    env = OracleEnv(8, *demo_rom())
    env.reset()
    rng = np.random.default_rng(0)
    t0, steps = time.perf_counter(), 0
    while time.perf_counter() - t0 < seconds:
        env.step(rng.integers(0, 7, 8))
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": 8 * steps / dt, "unit": "env_steps/s", "cores": 1, "kind": "port",
            "sample": f"oracle/nes_oracle.c, 8 environments x {steps} steps of 4 frames after the boot sequence"}


def bench_nes_env(dev, peaks, envs=None, cpu: bool = True) -> dict:
    """Mario environment step (scope row f4) on the batched NES kernels:
    GpuMarioVecEnv.step_device at 65,536 environments, 4 frames per step (the
    last one rendered), the 84 x 84 observation into the 4-frame stack, and the
    reward / done / auto-reset bookkeeping, all on the device.  Inputs: random
    SIMPLE_MOVEMENT actions resident on the device.  e2e: the reference-facing
    step(actions) with numpy actions in and numpy rewards / dones / infos out."""
    from rl_for_mario_b200.kernels import device_status
    from rl_for_mario_b200.nes import GpuMarioVecEnv
    from rl_for_mario_b200.nes_roms import demo_rom

    n = envs or NES_ENV_CFG["envs"]
    env = GpuMarioVecEnv(n, rom=demo_rom(), device=dev)
    t0 = time.perf_counter()
    env.reset()
    torch.cuda.synchronize(dev)
    boot_s = time.perf_counter() - t0
    g = torch.Generator(device=dev).manual_seed(5)
    acts = [torch.randint(0, 7, (n,), device=dev, generator=g) for _ in range(8)]

    def timed(fn, reps):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i)
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    steps = 10
    ms = timed(lambda i: env.step_device(acts[i % 8]), steps)
    b = env._batch
    frames_ms = timed(lambda i: b.run_frames_all(4), 5)
    frame1_ms = timed(lambda i: b.run_frames_all(1), 5)
    obs_out = torch.empty(n, 84, 84, dtype=torch.uint8, device=dev)
    obs_ms = timed(lambda i: b.obs_device(obs_out), 10)
    acts_np = [a.cpu().numpy() for a in acts]
    e2e_ms = timed(lambda i: env.step(acts_np[i % 8]), steps)
    if device_status() != 0:
        raise SystemExit("device status error in the NES benchmark")
    fb_bytes = n * 240 * 256
    obs_bytes = fb_bytes + n * 84 * 84  # read every framebuffer, write the observation
    gbs = obs_bytes / (obs_ms * 1e-3) / 1e9
    out = {"metric": "env_steps_per_s", "value": n / (ms * 1e-3), "unit": "env_steps/s", "ms_per_step": ms,
           "config": {"workload": f"Mario environment step, {n} environments, frame skip 4, frame stack 4",
                      **NES_ENV_CFG, "envs": n},
           "data": "synthetic cartridge, random actions",
           "kernels_ms": {"nes_frames_kernel x4 frames (last rendered)": frames_ms,
                          "nes_frames_kernel x1 rendered frame": frame1_ms,
                          "nes_observe_kernel": obs_ms},
           "env_frames_per_s": 4 * n / (frames_ms * 1e-3),
           "boot_s": boot_s,
           "e2e": {"value": n / (e2e_ms * 1e-3), "unit": "env_steps/s",
                   "h2d_bytes_per_step": n * 8, "d2h_bytes_per_step": n * (4 + 1 + 4 + 4 + 1)},
           "roofline_observe": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_launch": obs_bytes,
                                "peak_source": peaks["source"]}}
    del env
    torch.cuda.empty_cache()
    if cpu:
        out["cpu_baseline"] = _nes_cpu_baseline()
    return out



def bench_nes_policy(dev, envs: int = 8192, steps: int = 16) -> dict:
    """The closed loop of row f4 feeding the decode: the repo-default DT (bf16,
    fused blocks, CUDA-graph rollout) reads the NES environments' stacked
    frames and its actions step the emulators (nes.run_policy), 8,192
    environments (the rollout's per-GPU count) on the synthetic cartridge, for
    `steps` steps after the boot sequence; no host round trip inside a step."""
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT
    from rl_for_mario_b200.kernels import device_status
    from rl_for_mario_b200.nes import GpuMarioVecEnv, run_policy
    from rl_for_mario_b200.nes_roms import demo_rom
    from rl_for_mario_b200.rollout import DTRollout

    C = ROLLOUT_CFG
    cfg = DTConfig(hidden_size=C["hidden"], num_hidden_layers=C["layers"], num_attention_heads=C["q_heads"],
                   num_key_value_heads=C["kv_heads"], context_len=C["context_len"], dropout=0.0)
    model = MarioDT(cfg).to(dev, torch.bfloat16).eval().fuse_norms()
    env = GpuMarioVecEnv(envs, rom=demo_rom(), device=dev)
    ro = DTRollout(model, num_envs=envs, max_steps=steps, page_size=64, device=dev, graphs=True)
    obs0 = env.reset().clone()
    run_policy(env, ro, steps, start_obs=obs0)      # eager episode (initialises the kernels)
    run_policy(env, ro, steps, start_obs=obs0)      # captures the step graphs
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    acts, _, _ = run_policy(env, ro, steps, start_obs=obs0)
    e1.record()
    torch.cuda.synchronize(dev)
    if device_status() != 0:
        raise SystemExit("device status error in the NES policy benchmark")
    ms = e0.elapsed_time(e1) / steps
    out = {"metric": "env_steps_per_s (policy + environment)", "value": envs / (ms * 1e-3), "unit": "env_steps/s",
           "ms_per_step": ms, "envs": envs, "steps": steps,
           "config": "repo-default DT bf16 (fused blocks, graph-replayed cached rollout) + 4 NES frames per step, "
                     "synthetic cartridge; the episode's reset is outside the timed steps",
           "distinct_actions": len(set(acts.flatten().tolist()))}
    del env, ro, model
    torch.cuda.empty_cache()
    return out

def bench_nes_reference(envs=None) -> dict:
    """The reference's own NESBatchGpu (its kernels, built from its sources)
    at the same size: per step, set_buttons_batch (host buttons), run_frames_all(4),
    get_obs_batch and get_ram_batch (host copies), as GpuMarioVecEnv.step calls
    them; and run_frames_all(4) alone.  Wall clock (its calls synchronise)."""
    from oracle.nes import RefNESBatch
    from rl_for_mario_b200.nes_roms import demo_rom

    n = envs or NES_ENV_CFG["envs"]
    prg, chr_rom, mir = demo_rom()
    ref = RefNESBatch(n)
    ref.load_rom(prg, chr_rom)
    ref.reset_all(mir)
    ref.set_buttons_batch(np.zeros(n, np.uint8))
    t0 = time.perf_counter()
    ref.run_frames_all(286)  # the boot sequence's frame count
    boot_s = time.perf_counter() - t0
    rng = np.random.default_rng(5)
    bits = np.array([0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40], np.uint8)

    def step():
        ref.set_buttons_batch(bits[rng.integers(0, 7, n)])
        ref.run_frames_all(4)
        ref.get_obs_batch()
        ref.get_ram_batch()

    for _ in range(2):
        step()
    t0, k = time.perf_counter(), 5
    for _ in range(k):
        step()
    step_s = (time.perf_counter() - t0) / k
    t0 = time.perf_counter()
    for _ in range(k):
        ref.run_frames_all(4)
    frames_s = (time.perf_counter() - t0) / k
    return {"impl": "reference", "metric": "env_steps_per_s", "value": n / step_s, "unit": "env_steps/s",
            "ms_per_step": step_s * 1e3, "run_frames_all_4_ms": frames_s * 1e3,
            "env_frames_per_s": 4 * n / frames_s, "boot_286_frames_s": boot_s,
            "config": {"workload": f"Mario environment step, {n} environments, frame skip 4", **NES_ENV_CFG,
                       "envs": n}}


def bench_rollout_cfg5(dev, world, rank, pg, cpu: bool = False):
    """8,192 environments per GPU, 64 cached steps, CNN on synthetic frames, all-gather of logits.

    Each step draws the environments' uint8 frames on the device from the seed
    (written straight into the rollout's frame buffer, as a GPU environment
    would), runs the policy step (one CUDA graph per step index after the
    first two episodes) and all-gathers the logits.  Reported: device time of
    the 64-step episode (max over ranks) and the host time to enqueue it."""
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT
    from rl_for_mario_b200.rollout import DTRollout

    C = ROLLOUT_CFG
    torch.manual_seed(4)  # identical replicated weights on every rank
    cfg = DTConfig(hidden_size=C["hidden"], num_hidden_layers=C["layers"], num_attention_heads=C["q_heads"],
                   num_key_value_heads=C["kv_heads"], context_len=C["context_len"], dropout=0.0)
    model = MarioDT(cfg).to(dev, torch.bfloat16).eval().fuse_norms()  # fused blocks
    b = C["envs_per_gpu"]
    B = b * world
    ro = DTRollout(model, num_envs=B, max_steps=C["steps"], page_size=64, device=dev, graphs=True)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    first = torch.empty((b, 4, 84, 84), dtype=torch.uint8, device=dev)
    rtg = torch.rand(C["steps"], b, device=dev, generator=g) * 3000
    ts0 = torch.randint(0, 4000 - C["steps"], (b,), device=dev, generator=g)

    def run():
        ro.reset()
        a = None
        for t in range(C["steps"]):
            fb = ro.frame_buffer if ro.frame_buffer is not None else first
            # the environments' observation of step t: uniform bytes, drawn as 32-bit words
            fb.view(torch.int32).random_(-2 ** 31, 2 ** 31 - 1, generator=g)
            a, _ = ro.step(fb, rtg[t], ts0 + t)
        return a

    run()  # eager episode (initialises kernels and libraries)
    run()  # captures one graph per step index
    run()  # warm replay
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    e0.record()
    run()
    e1.record()
    host_ms = (time.perf_counter() - h0) * 1e3
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if pg:
        t = torch.tensor([ms, host_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms, host_ms = float(t[0].item()), float(t[1].item())
    # The environments' share: the 64 frame draws alone.
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fb = ro.frame_buffer
    f0.record()
    for _ in range(C["steps"]):
        fb.view(torch.int32).random_(-2 ** 31, 2 ** 31 - 1, generator=g)
    f1.record()
    torch.cuda.synchronize()
    frames_ms = f0.elapsed_time(f1)
    res = {"metric": "sharded rollout env-steps/s (CNN + 4 layers + cached attention + all-gather)",
           "unit": "env-steps/s", "value": B * C["steps"] / (ms * 1e-3), "ms_total": ms, "gpu_ms": ms,
           "host_enqueue_ms": host_ms, "frame_draw_ms": frames_ms, "n_gpus": world, "scaling": "weak",
           "config": {"workload": f"{b} envs per GPU ({B} total), 64 steps, window 192, repo-default DT bf16 "
                                  "(fused blocks), all_gather of [B/N, 7] logits per step",
                      "frames": "uint8 U[0,255] drawn on the device from the seed every step (inside the timed "
                                "region), written into the rollout's frame buffer",
                      "step": "one CUDA graph replay per step (embeddings, encoder, 4 layers with cache append "
                              "and attention, action head) + all-gather + argmax"}}
    del ro, first
    torch.cuda.empty_cache()
    if cpu:
        res["cpu_baseline"] = cpu_rollout(model, B=64, steps=C["steps"])
    del model
    return res


_JSON_OUT = None


def emit(line: dict) -> None:
    """Writes the result line to the process's real stdout (library banners go to stderr)."""
    out = _JSON_OUT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _JSON_OUT
    # Keep stdout for the one JSON line: anything a library prints on fd 1
    # (e.g. a collective library's version banner) is sent to stderr instead.
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode / rollout sub-benchmarks")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the batch (profiling of small cases only; the bench line is B=4096)")
    ap.add_argument("--only", choices=["decode", "prefill_long", "rmsnorm_qkv", "rmsnorm_swiglu", "conv1", "conv23",
                                       "rollout", "gemm_residual", "nes"],
                    default=None,
                    help="run one sub-benchmark alone and print its JSON (profiling)")
    ap.add_argument("--long-batch", type=int, default=None,
                    help="with --only prefill_long: batch of the attention-kernel case, model forward skipped")
    ap.add_argument("--with-model", action="store_true",
                    help="with --only prefill_long --long-batch: run the model forward at that batch too")
    args = ap.parse_args()
    if args.only:
        if not torch.cuda.is_available():
            raise SystemExit("bench.py needs a CUDA device (there is no CPU path)")
        from rl_for_mario_b200 import _lib
        _lib.load()
        dev = torch.device("cuda", 0)
        if args.only == "decode":
            emit({"only": "decode", **bench_decode_cfg3(dev, _peaks(), envs=args.batch)})
        elif args.only == "rmsnorm_qkv":
            emit({"only": "rmsnorm_qkv", **bench_rmsnorm_qkv_cfg4(dev, _peaks(), batch=args.long_batch)})
        elif args.only == "conv1":
            emit({"only": "conv1", **bench_conv1_cfg4(dev, _peaks(), batch=args.long_batch)})
        elif args.only == "conv23":
            emit({"only": "conv23", **bench_conv23_cfg4(dev, _peaks(), batch=args.long_batch)})
        elif args.only == "gemm_residual":
            emit({"only": "gemm_residual", **bench_gemm_residual_cfg4(dev, _peaks(), batch=args.long_batch)})
        elif args.only == "rollout":
            emit({"only": "rollout", **bench_rollout_cfg5(dev, 1, 0, None)})
        elif args.only == "nes":
            if args.impl == "reference":
                emit(bench_nes_reference(envs=args.batch))
            else:
                line = bench_nes_env(dev, _peaks(), envs=args.batch, cpu=not args.no_cpu_baseline)
                line["policy_loop"] = bench_nes_policy(dev)
                emit({"only": "nes", **line})
        elif args.only == "rmsnorm_swiglu":
            emit({"only": "rmsnorm_swiglu", **bench_rmsnorm_swiglu_cfg4(dev, _peaks(), batch=args.long_batch)})
        else:
            emit({"only": "prefill_long", **bench_prefill_cfg4(dev, _peaks(), batch=args.long_batch,
                                                                model=args.long_batch is None or args.with_model)})
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.batch:
        WORKLOAD["batch"] = args.batch
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
