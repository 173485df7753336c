"""Benchmark of the B200 attention path for tinylama (one JSON line on rank 0).

Default workload (the batched multi-sequence decode): 256 independent sequences per GPU with
context lengths drawn uniformly from [256, 4096] (seeded), Llama-2-7B-style attention (32 q
heads, 32 kv heads, head_dim 128), one query token each, f32 KV cache.  A step is one decode
step for every sequence: RoPE q/k at position L, append k/v at L, attention over L+1
positions (src/forward.nim:314-317, batched).  The KV read per step (about 18 GB) is far
larger than L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode_batched|decode_batched_bf16|decode_tiny|prefill|splitkv]

N > 1 runs under torchrun, one process per GPU; sequences are sharded by batch (each rank its
own 256 sequences, weak scaling) and timed as the max over ranks.  The `splitkv` workload
splits one 131072-token context along the sequence axis across ranks and merges the (m, l, o)
partials with NCCL.  `--impl reference` times the CPU oracle (a C restatement of the reference's
attention; the reference itself is Nim and cannot be built here) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode attn tok/s"
FALLBACK_HBM = 6650.0
FALLBACK_TFLOPS = 1590.0


# ---------------------------------------------------------------------------------- helpers
def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "src": "measured"}
    return {"hbm_gbs": FALLBACK_HBM, "bf16_tflops": FALLBACK_TFLOPS,
            "bf16_tflops_sustained": 1400.0, "src": "fallback"}


def traffic_from_profiles(kernel_key: str, algorithmic_bytes: int = 0):
    """DRAM bytes per launch from the committed ncu summaries: the captured figure, or the
    captured ratio to the algorithmic bytes times this launch's algorithmic bytes."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    d = json.load(open(p)).get(kernel_key)
    if d is None:
        return None
    if d.get("dram_bytes_per_launch") is not None:
        return d["dram_bytes_per_launch"]
    r = d.get("ratio_to_algorithmic")
    return None if r is None or not algorithmic_bytes else int(r * algorithmic_bytes)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

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
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a moment to start: begin the timed region once it is sampling
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
        except (OSError, FileNotFoundError):
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
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, backend="nccl"):
        import torch
        import datetime
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import torch.distributed as dist
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            import torch
            self.pg.barrier(device_ids=[self.local])

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def seq_lens(seed: int, n: int, lo: int = 256, hi: int = 4096) -> np.ndarray:
    return np.random.default_rng(seed).integers(lo, hi + 1, size=n).astype(np.int32)


# ------------------------------------------------------------------- decode (batched) arm
class DecodeBatched:
    """256 sequences, L ~ U[256, 4096], f32 (or bf16) KV; 32/32 heads of head_dim 128 (Llama-2-7B
    style) by default, or the TinyLlama GQA shape 32/4 heads of head_dim 64."""

    def __init__(self, kvd: int, rank: int, B=256, Hq=32, Hkv=32, D=128, base=10000.0):
        import torch
        from tinylama_b200 import _lib
        self.torch, self._lib = torch, _lib
        self.kvd, self.B, self.Hq, self.Hkv, self.D, self.base = kvd, B, Hq, Hkv, D, base
        self.lens = seq_lens(1000 + rank, B)
        self.maxLen = int(self.lens.max()) + 1
        h = C.c_void_p()
        _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, base, self.maxLen, B, kvd,
                                           torch.cuda.current_device()))
        self.h = h
        # a real (non-null) stream: every torch op, library call and event below uses it
        self.stream = torch.cuda.Stream()
        torch.cuda.set_stream(self.stream)
        g = torch.Generator(device="cuda").manual_seed(77 + rank)
        for b in range(B):  # seeded N(0,1) K/V for positions [0, L_b)
            L = int(self.lens[b])
            k = torch.randn(L, Hkv * D, device="cuda", generator=g)
            v = torch.randn(L, Hkv * D, device="cuda", generator=g)
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                                            L, C.c_void_p(self.stream.cuda_stream)))
        self.q = torch.randn(B, Hq * D, device="cuda", generator=g)
        self.k = torch.randn(B, Hkv * D, device="cuda", generator=g)
        self.v = torch.randn(B, Hkv * D, device="cuda", generator=g)
        self.out = torch.empty(B, Hq * D, device="cuda")
        self.pos_host = np.ascontiguousarray(self.lens)  # new token at position L
        self.pos = torch.from_numpy(self.pos_host).cuda()
        torch.cuda.synchronize()
        _lib.check(_lib.lib.tl_check_device(h, None))

    def ptr(self, t):
        return C.c_void_p(t.data_ptr())

    def step(self):
        _l = self._lib
        _l.check(_l.lib.tl_decode_step(self.h, 0, 0, self.B, self.ptr(self.pos),
                                       self.pos_host.ctypes.data_as(C.c_void_p), self.ptr(self.q),
                                       self.ptr(self.k), self.ptr(self.v), self.ptr(self.out),
                                       C.c_void_p(self.stream.cuda_stream)))

    def attention_only(self):
        _l = self._lib
        _l.check(_l.lib.tl_decode_attention(self.h, 0, 0, self.B, self.ptr(self.pos),
                                            self.pos_host.ctypes.data_as(C.c_void_p), self.ptr(self.q),
                                            self.ptr(self.out), C.c_void_p(self.stream.cuda_stream)))

    launches_per_step = 2  # rope_append + decode

    def kv_bytes(self) -> int:
        es = 4 if self.kvd == 0 else 2
        return int(np.sum(self.lens.astype(np.int64) + 1)) * self.Hkv * self.D * 2 * es

    def algorithmic_bytes_attention(self) -> int:
        # K and V rows read once + q read + ctx written (f32)
        return self.kv_bytes() + 2 * self.B * self.Hq * self.D * 4

    def flops(self) -> int:
        return int(np.sum(self.lens.astype(np.int64) + 1)) * self.Hq * self.D * 4

    def e2e(self, steps: int, warmup: int, dist: "Dist"):
        """tl_decode_batch_host with pinned host buffers: H2D of q, k, v, positions and D2H of
        the context inside every step."""
        torch, _l = self.torch, self._lib
        hq = torch.randn(self.B, self.Hq * self.D).pin_memory()
        hk = torch.randn(self.B, self.Hkv * self.D).pin_memory()
        hv = torch.randn(self.B, self.Hkv * self.D).pin_memory()
        hout = torch.empty(self.B, self.Hq * self.D).pin_memory()
        hpos = torch.from_numpy(self.pos_host.copy()).pin_memory()
        p = lambda t: C.c_void_p(t.data_ptr())

        def call():
            _l.check(_l.lib.tl_decode_batch_host(self.h, 0, 0, self.B, p(hpos), p(hq), p(hk), p(hv), p(hout)))

        for _ in range(warmup):
            call()
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            call()
        dt = (time.perf_counter() - t0) / steps
        dt = dist.max(dt)
        h2d = hq.numel() * 4 + hk.numel() * 4 + hv.numel() * 4 + hpos.numel() * 4
        d2h = hout.numel() * 4 + 4
        return dt, h2d, d2h

    def close(self):
        self._lib.lib.tl_attn_destroy(self.h)


def time_steps(fn, steps, warmup, stream, dist) -> float:
    """Device time per call (ms) with CUDA events on the launching stream, max over ranks."""
    import torch
    for _ in range(warmup):
        fn()
    dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = e0.elapsed_time(e1) / steps
    return dist.max(ms)


# --------------------------------------------------------------------------- CPU baseline
def cpu_decode_sample(lens, Hq, Hkv, D, base, budget_s: float, threads: int, seed: int = 5):
    """Time the oracle's decode step (RoPE + store + attentionCached on the reference's f32
    dim-major cache [nHeadKv*headDim, maxLen]) on a bounded sample of the sequences, `threads`
    host threads in parallel (ctypes releases the GIL).  Inputs are generated before the timed
    region.  Returns (sequences/s, sample description)."""
    from oracle import oracle as ora
    maxLen = int(np.max(lens)) + 1
    rng = np.random.default_rng(seed)
    bufs = []
    for _ in range(threads):
        kc = rng.standard_normal((Hkv * D, maxLen), dtype=np.float32)
        vc = rng.standard_normal((Hkv * D, maxLen), dtype=np.float32)
        bufs.append((kc, vc))
    q = rng.standard_normal((Hq * D, 1), dtype=np.float32)
    k = rng.standard_normal((Hkv * D, 1), dtype=np.float32)
    v = rng.standard_normal((Hkv * D, 1), dtype=np.float32)
    ora.lib()
    # calibrate on one sequence, then size the sample to the budget
    t0 = time.perf_counter()
    ora.decode_step(q, k, v, bufs[0][0], bufs[0][1], int(lens[0]), Hq, Hkv, D, D, base)
    t1 = time.perf_counter() - t0
    n = int(max(threads, min(len(lens), budget_s / max(t1, 1e-6) * threads)))
    n = (n // threads) * threads if n >= threads else n
    order = [i % len(lens) for i in range(1, n + 1)]

    def worker(t):
        kc, vc = bufs[t]
        for i in range(t, len(order), threads):
            ora.decode_step(q, k, v, kc, vc, int(lens[order[i]]), Hq, Hkv, D, D, base)

    ths = [threading.Thread(target=worker, args=(t,)) for t in range(threads)]
    t0 = time.perf_counter()
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    wall = time.perf_counter() - t0
    return len(order) / wall, (f"{len(order)} of {len(lens)} sequences per measurement "
                               f"(oracle decode step, f32, reference layout, {threads} thread(s))")


# ------------------------------------------------------------------------------ workloads
def decode_config(n: int, B: int, lens, Hq: int, Hkv: int, D: int, kvd: int) -> dict:
    """The workload's config dict; the reference arm reports the same one."""
    gqa = Hkv != Hq
    kv_gb = float(np.sum(np.asarray(lens, np.int64) + 1)) * Hkv * D * 2 * (4 if kvd == 0 else 2) / 1e9
    return {"workload": "batched multi-sequence decode (TinyLlama GQA attention)" if gqa else
                        "batched multi-sequence decode (Llama-2-7B-style attention)",
            "seqs_per_gpu": B, "global_batch": B * n, "ctx_len": "U[256,4096] seeded",
            "mean_ctx": float(np.mean(lens)), "n_head": Hq, "n_head_kv": Hkv,
            "head_dim": D, "kv_dtype": "f32" if kvd == 0 else "bf16",
            "parallelism": f"batch-sharded x{n} (no collective)",
            "l2": f"no flush: {kv_gb:.1f} GB of KV read per step >> 126 MB L2"}


def run_decode_batched(args, dist, kvd: int, shape=(32, 32, 128), with_subs=True):
    import torch
    pk = peaks()
    Hq, Hkv, D = shape
    gqa = Hkv != Hq
    w = DecodeBatched(kvd, dist.rank, B=args.seqs, Hq=Hq, Hkv=Hkv, D=D)
    sampler = ClockSampler(dist.local)
    sampler.start()
    ms = time_steps(w.step, args.steps, args.warmup, w.stream, dist)
    clocks = sampler.stop()
    ms_attn = time_steps(w.attention_only, args.steps, args.warmup, w.stream, dist)
    n = dist.world
    value = n * w.B / (ms / 1e3)
    achieved = w.algorithmic_bytes_attention() / (ms_attn / 1e3) / 1e9
    # end to end through the host-buffer call (the headline line only)
    e2e_dt, h2d, d2h = w.e2e(max(3, args.steps // 4), 2, dist) if with_subs else (ms / 1e3, 0, 0)
    e2e_value = n * w.B / e2e_dt
    traffic = traffic_from_profiles(("decode_kernel_f32" if kvd == 0 else "decode_kernel_bf16") + ("_gqa" if gqa else ""),
                                    w.algorithmic_bytes_attention())
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": n, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32" if kvd == 0 else "bf16-kv/f32-math", "data": "synthetic",
        "config": decode_config(n, w.B, w.lens, Hq, Hkv, D, kvd),
        "hbm_gbs_step": round(w.kv_bytes() / (ms / 1e3) / 1e9, 1),
        "clocks": clocks,
        "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "api": "tl_decode_batch_host (pinned host buffers)"},
        "gpu_launches": w.launches_per_step * args.steps,
        "roofline": {"kernel": "decode_mma_kernel" if (gqa or kvd == 1) else "decode_kernel", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "peak_src": pk["src"], "traffic": traffic,
                     "algorithmic_bytes_per_launch": w.algorithmic_bytes_attention(),
                     "launch_ms": round(ms_attn, 4)},
    }
    if n == 1 and dist.rank == 0 and not args.no_cpu_baseline and with_subs:
        rate, sample = cpu_decode_sample(w.lens, w.Hq, w.Hkv, w.D, w.base, args.cpu_budget, 1)
        res["cpu_baseline"] = {"value": round(rate, 3), "unit": "tok/s", "cores": 1, "kind": "port",
                               "sample": sample + "; Malebolgia on/off identical (attention has no "
                                                  "Malebolgia path, src/forward.nim:51-74)"}
    w.close()
    if with_subs and not args.no_subs:
        res["north_star"] = north_star_subs(args, dist)
    return res


def north_star_subs(args, dist) -> dict:
    """Every other measurement the target names, in one flat dict of numbers (kept short so
    that it survives in a log tail).  Decode: attention-kernel GB/s and fraction of the HBM
    peak (256 sequences per GPU, L ~ U[256, 4096]).  Prefill: TFLOP/s and fraction of the burst
    bf16 peak, attention kernel alone ("core") and the whole step (RoPE + cache write +
    attention), 8 sequences sharded over the GPUs.  Split-KV: one 131072-token context per
    sequence (B = 4, 32/8/128, bf16) split over the N GPUs, microseconds per step and the
    fraction of the HBM peak each GPU sustains (strong scaling: the work is fixed).  TinyLlama
    batch-1 decode step (RoPE + append + attention, K/V from HBM) and the whole TinyLlama model
    decode step on the GPU, in microseconds."""
    pk = peaks()
    out = {"n_gpus": dist.world}

    def guarded(name, fn):
        # a sub-measurement that fails is recorded as such; the headline line still prints
        try:
            fn()
        except Exception as e:  # noqa: BLE001
            out[f"{name}_error"] = repr(e)[:160]

    def decode_subs():
        for tag, kvd, shape in (("gqa_f32", 0, (32, 4, 64)), ("gqa_bf16", 1, (32, 4, 64)),
                                ("llama2_bf16", 1, (32, 32, 128))):
            r = run_decode_batched(args, dist, kvd, shape, with_subs=False)
            out[f"{tag}_gbs"] = r["roofline"]["achieved"]
            out[f"{tag}_frac"] = r["roofline"]["frac"]
            if tag == "llama2_bf16":
                out[f"{tag}_tok_s"] = r["value"]

    def prefill_subs():
        pre = run_prefill(args, dist)
        for key, d in pre["by_seq_len"].items():
            k = key.replace(" after ", "_after_").replace(" cached", "")
            out[f"prefill_{k}_core_tflops"] = d["attention_core"]["tflops"]
            out[f"prefill_{k}_core_frac"] = d["attention_core"]["frac_of_bf16_peak"]
            out[f"prefill_{k}_step_frac"] = d["frac_of_bf16_peak"]

    def splitkv_subs():
        sk = run_splitkv(args, dist, L=args.ctx_len)
        out["splitkv_131072_us"] = round(sk["ms_per_step"] * 1e3, 1)
        out["splitkv_131072_local_shard_us"] = round(sk["local_shard_ms"] * 1e3, 1)
        out["splitkv_131072_frac_per_gpu"] = sk["roofline"]["frac"]

    def tiny_subs():
        tiny = run_decode_tiny(args, dist)
        for L, d in tiny["by_ctx_len"].items():
            out[f"tinyllama_b1_us_L{L}"] = d["hbm_rotating_64"]["us_per_step"]

    def model_subs():
        md = run_model_decode(args, dist)
        out["model_decode_us"] = md["us_per_decode_step"]
        out["model_decode_frac"] = md["frac_of_hbm_peak"]

    guarded("decode", decode_subs)
    if not args.no_prefill:
        guarded("prefill", prefill_subs)
    guarded("splitkv", splitkv_subs)
    guarded("tinyllama_b1", tiny_subs)
    guarded("model_decode", model_subs)
    out["peaks"] = f"HBM {pk['hbm_gbs']} GB/s, bf16 {pk['bf16_tflops']} TF/s ({pk['src']})"
    return out


# -------------------------------------------------------------------- prefill (tcgen05)
def kernel_device_ms(fn, reps: int = 3) -> dict:
    """Average device time (ms) per call of each kernel launched by fn(), from CUPTI activity
    records (torch.profiler), after the timed region; keys are the kernels' names."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    out = {}
    for e in prof.key_averages():
        t = getattr(e, "device_time_total", None)
        if t is None:
            t = getattr(e, "cuda_time_total", 0.0)
        if t and e.count:
            out[e.key] = out.get(e.key, 0.0) + t / 1e3 / reps
    return out


def prefill_point(S: int, steps: int, warmup: int, dist, B=8, Hq=32, Hkv=8, D=64, kvd=1, start=0):
    """Causal prefill of B sequences of S tokens, sharded over the ranks (B/N each): RoPE + bf16
    cache write + attention (tl_prefill_step).  With start > 0 the S tokens continue a cached
    prefix of `start` positions (tl_prefill_step_at: token t at start + t attends positions
    0..start+t).  Returns the step time (ms, max over ranks), the device times of the attention
    kernel and of the RoPE/cache-write prologue (ms, max over ranks), and the whole job's flops."""
    import torch
    from tinylama_b200 import _lib
    n = dist.world
    Bl = max(1, B // n)
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, 10000.0, start + S, Bl, kvd,
                                       torch.cuda.current_device()))
    try:
        stream = torch.cuda.Stream()
        torch.cuda.set_stream(stream)
        g = torch.Generator(device="cuda").manual_seed(S * 16 + dist.rank)
        p = lambda t: C.c_void_p(t.data_ptr())
        sp = C.c_void_p(stream.cuda_stream)
        for b in range(Bl if start > 0 else 0):  # the cached prefix (seeded N(0,1) K/V)
            kp = torch.randn(start, Hkv * D, device="cuda", generator=g)
            vp = torch.randn(start, Hkv * D, device="cuda", generator=g)
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, p(kp), p(vp), start, sp))
            del kp, vp
        pos0_host = np.full(Bl, start, np.int32)
        pos0 = torch.from_numpy(pos0_host).cuda()
        q = torch.randn(Bl, S, Hq * D, device="cuda", generator=g)
        k = torch.randn(Bl, S, Hkv * D, device="cuda", generator=g)
        v = torch.randn(Bl, S, Hkv * D, device="cuda", generator=g)
        out = torch.empty_like(q)

        def step():
            if start > 0:
                _lib.check(_lib.lib.tl_prefill_step_at(h, 0, 0, Bl, S, p(pos0), pos0_host.ctypes.data_as(C.c_void_p),
                                                       p(q), p(k), p(v), p(out), sp))
            else:
                _lib.check(_lib.lib.tl_prefill_step(h, 0, 0, Bl, S, p(q), p(k), p(v), p(out), sp))

        ms = time_steps(step, steps, warmup, stream, dist)
        _lib.check(_lib.lib.tl_check_device(h, C.c_void_p(stream.cuda_stream)))
        kt = kernel_device_ms(step)
        core = sum(t for name, t in kt.items() if "prefill_tc_kernel" in name or "prefill_f32_kernel" in name)
        pro = sum(t for name, t in kt.items() if "rope_append" in name)
        # 4*D flops per (query, key) pair; query t attends start + t + 1 keys
        flops = Bl * n * Hq * 2 * D * (S * (S + 1) + 2 * S * start)
        return ms, dist.max(core), dist.max(pro), flops
    finally:
        _lib.lib.tl_attn_destroy(h)


def run_prefill(args, dist):
    sizes = [int(x) for x in args.prefill_sizes.split(",")]
    pk = peaks()
    res = {}
    points = [(0, S) for S in sizes]
    for spec in filter(None, args.prefill_continue.split(",")):
        start, S = (int(x) for x in spec.split(":"))
        points.append((start, S))
    for start, S in points:
        ms, core_ms, pro_ms, flops = prefill_point(S, max(5, args.steps // 2), args.warmup, dist, start=start)
        tf = flops / (ms / 1e3) / 1e12
        tf_core = flops / (core_ms / 1e3) / 1e12 if core_ms > 0 else None
        peak = pk["bf16_tflops"] * dist.world  # whole job: N GPUs
        sus = (pk["bf16_tflops_sustained"] or pk["bf16_tflops"]) * dist.world
        steps = max(5, args.steps // 2)
        res[str(S) if start == 0 else f"{S} after {start} cached"] = {"ms_per_step": round(ms, 4), "tflops": round(tf, 1),
                       "frac_of_bf16_peak": round(tf / peak, 4),
                       "frac_of_bf16_sustained": round(tf / sus, 4), "flops": flops,
                       "timed_ms_total": round(ms * steps, 1),
                       "attention_core": {"ms": round(core_ms, 4),
                                          "tflops": None if tf_core is None else round(tf_core, 1),
                                          "frac_of_bf16_peak": None if tf_core is None else
                                          round(tf_core / peak, 4),
                                          "frac_of_bf16_sustained": None if tf_core is None else
                                          round(tf_core / sus, 4)},
                       "prologue_ms": round(pro_ms, 4)}
    return {"workload": "causal prefill, 8 sequences (sharded over the GPUs), 32 q / 8 kv heads, head_dim 64, "
                        "bf16 KV (tcgen05); step = RoPE + cache write + attention (end to end on the device); "
                        "attention_core = the attention kernel alone (CUPTI device time); \"S after P cached\" = "
                        "S new tokens continuing a cached prefix of P positions (tl_prefill_step_at)",
            "n_gpus": dist.world, "by_seq_len": res, "peak_tflops_per_gpu": pk["bf16_tflops"],
            "sustained_tflops_per_gpu": pk["bf16_tflops_sustained"], "peak_src": pk["src"],
            "peak_note": "frac_of_bf16_peak uses the burst figure, frac_of_bf16_sustained the figure under the "
                         "power cap; a timed region of a few hundred ms (timed_ms_total) runs at the sustained one"}


# ------------------------------------------------------- the whole model on the GPU (tl_model.h)
def synthetic_q2k(rng, rows: int, cols: int) -> np.ndarray:
    """Q2_K blocks of random content with the format's layout: 16 scale bytes, 64 bytes of 2-bit
    weights, f16 d and dmin (positive, of the size N(0, 0.02) weights quantise to)."""
    nb = rows * (cols // 256)
    blk = rng.integers(0, 256, size=(nb, 84), dtype=np.uint8)
    dd = (rng.random((nb, 2), dtype=np.float32) * np.float32(0.004) + np.float32(0.001)).astype(np.float16)
    blk[:, 80:84] = dd.view(np.uint8).reshape(nb, 4)
    return blk


def run_model_decode(args, dist, n_prompt=8, n_new=129):
    """TinyLlama-1.1B shapes (22 layers, dim 2048, 32/4 heads, ffn 5632, vocab 32000), Q2_K
    matrices including the output, f32 embedding and norms, random synthetic weights: greedy
    decode at batch 1 through tl_model_generate.  Each decode step is one CUDA graph replay
    (embedding, per layer rmsnorm+qkv, RoPE+append+attention, wo+residual, rmsnorm+gate/up+silu,
    down+residual, then rmsnorm+output and argmax); the device time of the n_new-1 steps comes
    from CUDA events around them.  Bytes per step: every weight once (Q2_K 84 B per 256)."""
    import torch
    from tinylama_b200 import _lib
    nL, E, H, KV, F, V, D = 22, 2048, 32, 4, 5632, 32000, 64
    rng = np.random.default_rng(2026)

    class Cfg(C.Structure):
        _fields_ = [("nVocab", C.c_int), ("nEmb", C.c_int), ("nLayer", C.c_int), ("nFfn", C.c_int),
                    ("nHead", C.c_int), ("nHeadKv", C.c_int), ("ropeDim", C.c_int),
                    ("ropeFreqBase", C.c_float), ("rmsEps", C.c_float), ("maxLen", C.c_int)]

    h = C.c_void_p()
    _lib.check(_lib.lib.tl_model_create(C.byref(h), C.byref(Cfg(V, E, nL, F, H, KV, D, 10000.0, 1e-5, n_prompt + n_new)),
                                        torch.cuda.current_device()))
    try:
        q2k_bytes = 0

        def put(name, typ, arr, ne0, ne1):
            _lib.check(_lib.lib.tl_model_set_tensor(h, name.encode(), typ, arr.ctypes.data_as(C.c_void_p), ne0, ne1))

        ones = np.ones(E, np.float32)
        for l in range(nL):
            p = f"blk.{l}."
            put(p + "attn_norm.weight", 0, ones, E, 1)
            put(p + "ffn_norm.weight", 0, ones, E, 1)
            for name, ne0, ne1 in (("attn_q", E, H * D), ("attn_k", E, KV * D), ("attn_v", E, KV * D),
                                   ("attn_output", H * D, E), ("ffn_gate", E, F), ("ffn_up", E, F),
                                   ("ffn_down", F, E)):
                w = synthetic_q2k(rng, ne1, ne0)
                q2k_bytes += w.nbytes
                put(p + name + ".weight", 10, w, ne0, ne1)
        put("output_norm.weight", 0, ones, E, 1)
        w = synthetic_q2k(rng, V, E)
        q2k_bytes += w.nbytes
        put("output.weight", 10, w, E, V)
        emb = (rng.standard_normal((V, E), dtype=np.float32) * np.float32(0.02))
        put("token_embd.weight", 0, emb, E, V)
        del emb, w
        prompt = rng.integers(3, V, size=n_prompt).astype(np.int32)
        ids = np.zeros(n_new, np.int32)
        gaps = np.zeros(n_new, np.float32)

        def gen():
            _lib.check(_lib.lib.tl_model_generate(h, prompt.ctypes.data_as(C.c_void_p), n_prompt, n_new,
                                                  ids.ctypes.data_as(C.c_void_p), gaps.ctypes.data_as(C.c_void_p)))

        gen()  # captures the decode-step graph
        per_step, e2e = [], []
        for _ in range(3):
            t0 = time.perf_counter()
            gen()
            e2e.append(time.perf_counter() - t0)
            pre, dec = C.c_float(), C.c_float()
            _lib.check(_lib.lib.tl_model_last_timing(h, C.byref(pre), C.byref(dec)))
            per_step.append(dec.value / (n_new - 1))
        ms = statistics.median(per_step)
        # device time per kernel (CUPTI) of one generate call, per decode step: what the step's
        # time is made of, and how much of it lies between kernels
        kt = kernel_device_ms(gen, reps=1)
        kernels = {k[:80]: round(v * 1e3 / n_new, 2) for k, v in sorted(kt.items(), key=lambda x: -x[1])[:8]}
        step_bytes = q2k_bytes + E * 4 * (2 * nL + 2)  # weights + embedding row + norm vectors
        pk = peaks()
        gbs = step_bytes / (ms / 1e3) / 1e9
        return {"workload": "TinyLlama-1.1B shapes, Q2_K weights resident in HBM (random synthetic), greedy decode "
                            "at batch 1, one CUDA graph per step (tl_model_generate)",
                "prompt": n_prompt, "decode_steps": n_new - 1, "us_per_decode_step": round(ms * 1e3, 1),
                "tok_s": round(1e3 / ms, 1), "bytes_per_step": step_bytes, "hbm_gbs": round(gbs, 1),
                "frac_of_hbm_peak": round(gbs / pk["hbm_gbs"], 4), "peak_src": pk["src"],
                "prefill_ms": round(pre.value, 3),
                "kernel_us_per_step": kernels, "kernel_us_sum": round(sum(kt.values()) * 1e3 / n_new, 1),
                "e2e_tok_s": round(n_new / statistics.median(e2e), 1),
                "e2e_note": "tl_model_generate wall clock: prompt upload, prefill, the decode steps, ids back"}
    finally:
        _lib.lib.tl_model_destroy(h)


# ------------------------------------------------------------- TinyLlama decode latency
def run_decode_tiny(args, dist, Hq=32, Hkv=4, D=64, base=10000.0, lengths=(128, 512, 2048), nslots=64):
    """TinyLlama GQA decode (32 q / 4 kv heads, head_dim 64, f32), batch 1: the cache holds L
    positions, the query is the token at position L-1 (RoPE at L-1, append, attention over L).
    1000 steps per length, replayed from a CUDA graph.  Two figures per length: the same cache
    every step (it stays in L2: latency-bound) and a rotation over 64 distinct caches (64 x
    2*4*L*64*4 B > L2 for L >= 2048) so that the K/V reads come from HBM."""
    import torch
    from tinylama_b200 import _lib
    p = lambda t: C.c_void_p(t.data_ptr())
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = C.c_void_p(stream.cuda_stream)
    steps = 1000
    out = {}
    for L in lengths:
        h = C.c_void_p()
        _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, base, L, nslots, 0,
                                           torch.cuda.current_device()))
        try:
            g = torch.Generator(device="cuda").manual_seed(L)
            for slot in range(nslots):
                k = torch.randn(L, Hkv * D, device="cuda", generator=g)
                v = torch.randn(L, Hkv * D, device="cuda", generator=g)
                _lib.check(_lib.lib.tl_kv_store(h, 0, slot, 0, p(k), p(v), L, sp))
            q = torch.randn(nslots, Hq * D, device="cuda", generator=g)
            k1 = torch.randn(nslots, Hkv * D, device="cuda", generator=g)
            v1 = torch.randn(nslots, Hkv * D, device="cuda", generator=g)
            o = torch.empty(nslots, Hq * D, device="cuda")
            pos_host = np.full(1, L - 1, np.int32)
            pos = torch.from_numpy(pos_host).cuda()
            ph = pos_host.ctypes.data_as(C.c_void_p)

            def step(slot):
                _lib.check(_lib.lib.tl_decode_step(h, 0, slot, 1, p(pos), ph, p(q[slot]), p(k1[slot]),
                                                   p(v1[slot]), p(o[slot]), sp))

            res = {}
            for mode, slots in (("l2_resident", [0]), ("hbm_rotating_64", list(range(nslots)))):
                for _ in range(3):
                    for sl in slots:
                        step(sl)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for sl in slots:
                        step(sl)
                reps = steps // len(slots)
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (reps * len(slots))
                nbytes = 2 * Hkv * D * L * 4 + 2 * Hq * D * 4
                res[mode] = {"us_per_step": round(us, 3), "tok_s": round(1e6 / us, 1),
                             "gbs": round(nbytes / (us * 1e-6) / 1e9, 1)}
                del graph
            _lib.check(_lib.lib.tl_check_device(h, sp))
            out[str(L)] = res
        finally:
            _lib.lib.tl_attn_destroy(h)
    return {"workload": "TinyLlama GQA decode (32 q / 4 kv heads, head_dim 64, f32 KV), batch 1, "
                        "1000 CUDA-graph steps per length; step = RoPE + append + attention",
            "by_ctx_len": out, "bytes_per_step": "2048*L + 16384"}


# ------------------------------------------------------------ long-context split-KV decode
def run_splitkv(args, dist, B=4, Hq=32, Hkv=8, D=128, L=131072, base=500000.0):
    """One 131072-token context per sequence, split along the sequence axis: rank r holds
    positions [r*L/N, (r+1)*L/N).  A step is the split-KV attention of one query token per
    sequence at position L-1 (tl_decode_attention_dist: one launch per rank; the decode kernel
    stores each (sequence, head) (o, m, l) into every rank's buffer over NVLink, and the last CTA
    merges after a bounded epoch-flag wait).  Strong scaling: the total work is fixed."""
    import torch
    from tinylama_b200 import _lib
    n, r = dist.world, dist.rank
    assert L % n == 0
    slice_len = L // n
    h = C.c_void_p()
    _lib.check(_lib.lib.tl_attn_create(C.byref(h), 1, Hq, Hkv, D, D, base, slice_len, B, 1,
                                       torch.cuda.current_device()))
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = C.c_void_p(stream.cuda_stream)
    p = lambda t: C.c_void_p(t.data_ptr())
    try:
        g = torch.Generator(device="cuda").manual_seed(900 + r)
        for b in range(B):
            k = torch.randn(slice_len, Hkv * D, device="cuda", generator=g)
            v = torch.randn(slice_len, Hkv * D, device="cuda", generator=g)
            _lib.check(_lib.lib.tl_kv_store(h, 0, b, 0, p(k), p(v), slice_len, sp))
            del k, v
        uid = C.create_string_buffer(128)
        if r == 0:
            _lib.check(_lib.lib.tl_dist_unique_id(uid))
        if n > 1:
            obj = [uid.raw if r == 0 else None]
            dist.pg.broadcast_object_list(obj, src=0)
            uid = C.create_string_buffer(obj[0], 128)
        _lib.check(_lib.lib.tl_dist_init(h, uid, n, r))
        gq = torch.Generator(device="cuda").manual_seed(4242)  # same q on every rank
        q = torch.randn(B, Hq * D, device="cuda", generator=gq)
        out = torch.empty(B, Hq * D, device="cuda")
        pos_host = np.full(B, L - 1, np.int32)
        pos = torch.from_numpy(pos_host).cuda()
        torch.cuda.synchronize()

        def step():
            _lib.check(_lib.lib.tl_decode_attention_dist(h, 0, 0, B, p(pos), pos_host.ctypes.data_as(C.c_void_p),
                                                         p(q), p(out), sp))

        ms = time_steps(step, args.steps, args.warmup, stream, dist)
        _lib.check(_lib.lib.tl_check_device(h, sp))
        # the same shard attended alone (no exchange, no merge across ranks): what the step
        # costs beyond it is the exchange and the ranks' skew
        shard_pos = np.full(B, slice_len - 1, np.int32)
        dshard = torch.from_numpy(shard_pos).cuda()
        local_out = torch.empty_like(out)

        def local():
            _lib.check(_lib.lib.tl_decode_attention(h, 0, 0, B, p(dshard), shard_pos.ctypes.data_as(C.c_void_p),
                                                    p(q), p(local_out), sp))

        ms_local = time_steps(local, args.steps, args.warmup, stream, dist)
        _lib.check(_lib.lib.tl_check_device(h, sp))
        kv_bytes = B * L * Hkv * D * 2 * 2
        pk = peaks()
        gbs = kv_bytes / (ms / 1e3) / 1e9
        return {
            "metric": "long-context split-KV decode attn tok/s", "value": round(B / (ms / 1e3), 1),
            "unit": "tok/s", "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16-kv/f32-math", "data": "synthetic",
            "config": {"workload": "long-context split-KV decode (Llama-3-8B-style attention)",
                       "batch": B, "ctx_len": L, "n_head": Hq, "n_head_kv": Hkv, "head_dim": D,
                       "rope_theta": base, "kv_dtype": "bf16", "parallelism": f"split-KV x{n}, fused peer-memory exchange and merge" if os.environ.get("TL_DIST_NCCL") != "1" else f"split-KV x{n} + NCCL all-gather merge",
                       "l2": f"no flush: {kv_bytes / n / 1e9:.2f} GB of KV per GPU per step > 126 MB L2"},
            "hbm_gbs_aggregate": round(gbs, 1), "hbm_gbs_per_gpu": round(gbs / n, 1),
            "local_shard_ms": round(ms_local, 4),
            "roofline": {"bound": "hbm", "achieved": round(gbs / n, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / n / pk["hbm_gbs"], 4), "peak_src": pk["src"],
                         "note": "per GPU, whole step (local attention, exchange and merge)"},
            "gpu_launches": (1 if os.environ.get("TL_DIST_NCCL") != "1" or n == 1 else 2) * args.steps,
        }
    finally:
        _lib.lib.tl_attn_destroy(h)


def run_reference(args, dist):
    """The reference arm: the oracle (C restatement of the reference's CPU attention) on all
    host threads, rank 0 only, on a bounded sample of the same workload."""
    if dist.rank != 0:
        return None
    B, Hq, Hkv, D, base = args.seqs, 32, 32, 128, 10000.0
    threads = os.cpu_count() or 1
    lens = seq_lens(1000, B)
    # size each step so that the whole run stays within a couple of minutes
    per_step_budget = max(0.3, 90.0 / max(1, args.steps + args.warmup))
    rates = []
    sample = ""
    for i in range(args.warmup + args.steps):
        r, sample = cpu_decode_sample(lens, Hq, Hkv, D, base, per_step_budget, threads, seed=i)
        if i >= args.warmup:
            rates.append(r)
    value = statistics.median(rates)
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tok/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * B / value, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": decode_config(dist.world, B, lens, Hq, Hkv, D, 0),
        "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"per step: {sample}, {threads} threads; the reference (Nim) "
                                   "cannot be built here, this is its C restatement"},
        "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="decode_batched",
                    choices=["decode_batched", "decode_batched_bf16", "decode_batched_gqa",
                             "decode_batched_gqa_bf16", "splitkv", "prefill", "decode_tiny", "model_decode"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="omit the prefill sub-measurement")
    ap.add_argument("--no-subs", action="store_true", help="omit every sub-measurement (headline only)")
    ap.add_argument("--prefill-sizes", default="512,2048,8192", help="sequence lengths of the prefill")
    ap.add_argument("--prefill-continue", default="6144:2048",
                    help="start:S points of a prefill continuing a cached prefix (comma-separated; empty: none)")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    ap.add_argument("--seqs", type=int, default=256, help="sequences per GPU (256 = the benchmark)")
    ap.add_argument("--ctx-len", type=int, default=131072, help="split-KV context length (131072 = the benchmark)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    dist = Dist()
    if args.impl == "reference":
        res = run_reference(args, dist)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    dist.init()
    try:
        if args.workload == "decode_batched":
            res = run_decode_batched(args, dist, 0)
        elif args.workload == "decode_batched_bf16":
            res = run_decode_batched(args, dist, 1)
        elif args.workload == "decode_batched_gqa":
            res = run_decode_batched(args, dist, 0, (32, 4, 64))
        elif args.workload == "decode_batched_gqa_bf16":
            res = run_decode_batched(args, dist, 1, (32, 4, 64))
        elif args.workload == "splitkv":
            res = run_splitkv(args, dist, L=args.ctx_len)
        elif args.workload == "decode_tiny":
            res = run_decode_tiny(args, dist)
        elif args.workload == "model_decode":
            res = run_model_decode(args, dist)
        else:
            res = run_prefill(args, dist)
        if dist.rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
