"""Benchmark of the in-context sparse attention call (BASELINE metric:
"sparse-attn ms/call at 65K joint tokens (40h x 128d bf16) 1/2/4/8 GPU").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload 480p|720p|config1|dit-step|sweep]
                    [--impl b200|reference]

One step is one whole call over all 40 heads.  With N GPUs (torchrun, one
process per GPU) the heads are split N ways (40/20/10/5 per GPU), every rank
runs its shard with no collective on the data path, and the step time is the
maximum over ranks: total work per call is fixed, so scaling is "strong".

* value: ms per call with q/k/v resident in HBM, timed with CUDA events on
  the launching stream around exactly K steps (barrier + synchronize on both
  sides, max over ranks); the inputs (2 GB) are larger than L2.  A step goes
  through the stage entry points with the two attention halves overlapped as
  icsa_attend overlaps them; stages_ms.attend_sparse and sequential_call come
  from the same calls with the halves in sequence, after the timed region.
* e2e: the same call through the public Python API on pinned host q/k/v
  and a pinned host result: the library streams groups of heads through the
  GPU, so every input and output byte crosses PCIe inside the timed region
  (whole-job byte counts in the line).
* roofline: the dominant kernel, the dense attention of the flat query
  blocks (tensor-core bound): algorithmic FLOPs per launch / its CUDA-event
  duration, against the measured sustained bf16 peak; the block-sparse
  kernel's figures ride along.
* cpu_baseline / --impl reference: the CPU restatement of the reference path
  (the reference's PyTorch orchestration + restated kernels) on the host
  cores: the whole call for one or two heads, scaled to all 40 heads.

--workload dit-step measures the other half of the metric, "DiT step s": one
denoising step of a random-init Wan 2.2 A14B-shaped DiT (40 blocks, CFG pair
as batch 2) on the 480p joint sequence, Ulysses sequence-parallel over the
ranks (wan_dit); its line reports seconds per step and the whole step's
tensor throughput.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "lightning-unified-video-editor-via-in-context-sparse-attention_b200")
sys.path.insert(0, REPO)
sys.path.insert(0, PKG_DIR)

from in_context_sparse_attention import _capi, editing_sparse_attention, sharding, synthetic  # noqa: E402

METRIC = "sparse-attn ms/call at 65K joint tokens (40h×128d bf16) 1/2/4/8 GPU; DiT step s"
WORKLOADS = {"480p": synthetic.WAN480P, "720p": synthetic.WAN720P, "config1": synthetic.CONFIG1}
# pool, scores GEMM, rowstats, out_c, colsum, 2x sort, extended-KV, block-score GEMM, top-k select,
# dense + sparse attention
KERNELS_PER_CALL_ALIGNED = 12


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d.get("bf16_tflops_sustained", 1373.7), d.get("bf16_tflops", 1626.6), d.get("hbm_gbs", 6546.9), "measured"
    return 1400.0, 1590.0, 6650.0, "fallback"


def attention_flops(p, n_sparse):
    """Algorithmic FLOPs of the attention kernel per call (2 FLOP per MAC):
    flat 4*Tq*Tkv*D, exact 4*Tq*(top_k*64)*D, interval 4*Tq*nkv*D."""
    D, BH = p.D, p.B * p.H
    flat = 4.0 * p.num_flat * 64 * p.tkv * D
    exact = 4.0 * n_sparse * 64 * p.top_k * 64 * D
    interval = 4.0 * n_sparse * 64 * p.nkv * D
    return BH * (flat + exact + interval), BH * flat, BH * (exact + interval)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, read through NVML
    every 5 ms in a background thread (read-only queries; nothing is set), so
    that even a timed region of a few tens of milliseconds is sampled.  Falls
    back to `nvidia-smi -lms 100` when NVML is not importable."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device):
        self.uuid = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device).uuid)
        except Exception:  # noqa: BLE001
            pass
        self.rows, self.proc, self.thread, self.stop_flag, self.nvml = [], None, None, False, None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            uid = self.uuid if self.uuid.startswith("GPU-") else "GPU-" + self.uuid
            self.handle = pynvml.nvmlDeviceGetHandleByUUID(uid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            self.masks = [(n, getattr(pynvml, c)) for n, c in self.REASONS]
            self.nvml = pynvml
        except Exception:  # noqa: BLE001
            self.nvml = None
        if self.nvml is not None:
            self.thread = threading.Thread(target=self._poll_nvml, daemon=True)
            self.thread.start()
            return
        try:
            fields = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                      "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                      "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read_smi, daemon=True)
        self.thread.start()

    def _poll_nvml(self):
        nv = self.nvml
        while not self.stop_flag:
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.rows.append((float(mhz), float(self.max_mhz), [n for n, m in self.masks if bits & m]))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def _read_smi(self):
        names = [n for n, _ in self.REASONS]
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and (not self.uuid or self.uuid.replace("GPU-", "") in parts[0]):
                try:
                    self.rows.append((float(parts[1]), float(parts[2]),
                                      [n for n, v in zip(names, parts[5:9]) if v.lower().startswith("active")]))
                except ValueError:
                    pass

    def stop(self):
        self.stop_flag = True
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        rows = self.rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted({n for r in rows for n in r[2]}), "samples": len(rows),
                "source": "nvml" if self.nvml is not None else "nvidia-smi"}


# ---------------------------------------------------------------------------
# device-resident runner through the stage entry points of the C ABI
# ---------------------------------------------------------------------------
class Runner:
    def __init__(self, q, k, v, t_seq_len, select_ratio=0.125, flat_ratio=0.5):
        self.lib = _capi.load()
        B, S, H, D = q.shape
        self.p = _capi.problem(B, S, H, D, t_seq_len, select_ratio=select_ratio, flat_ratio=flat_ratio)
        # input and result dtypes as the drop-in sets them (bf16 for the 480p /
        # 720p workloads; f32 for configuration 1)
        import importlib
        esa = importlib.import_module("in_context_sparse_attention.editing_sparse_attention")
        dt = {torch.bfloat16: _capi.ICSA_BF16, torch.float32: _capi.ICSA_F32}
        outc_dt, ca_dt, out_dt = esa._result_dtypes(q.dtype, k.dtype, v.dtype, 1.0)
        self.p.q_dtype, self.p.k_dtype, self.p.v_dtype = dt[q.dtype], dt[k.dtype], dt[v.dtype]
        self.p.out_dtype = dt[out_dt]
        self.p.outc_bf16 = int(outc_dt == torch.bfloat16)
        self.p.ca_bf16 = int(ca_dt == torch.bfloat16)
        self.L = _capi.workspace_layout(self.p)
        self.size = self.lib.icsa_workspace_size(ctypes.byref(self.p))
        self.ws = torch.empty(self.size, dtype=torch.uint8, device=q.device)
        self.out = torch.empty(q.shape, dtype=out_dt, device=q.device)
        self.q, self.k, self.v = q, k, v
        self.side = torch.cuda.Stream(device=q.device)
        self.fork, self.join = torch.cuda.Event(), torch.cuda.Event()

    def step(self, ev=None, overlap=True):
        """One call through the stage entry points.  With `overlap` the two
        attention halves run as icsa_attend runs them: the dense kernel first
        on the current stream, the block-sparse kernel on a side stream that
        forks after the selection and joins before the next call, so sparse
        CTAs fill the SMs of the dense kernel's last wave.  ev[3] (after the
        dense launch, on its stream) times the dense kernel."""
        lib, pp, cur = self.lib, ctypes.byref(self.p), torch.cuda.current_stream()
        st = cur.cuda_stream
        a = (self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr())
        if ev is not None:
            ev[0].record()
        _capi.check(lib.icsa_pool(pp, *a, self.ws.data_ptr(), self.size, st), "icsa_pool")
        if ev is not None:
            ev[1].record()
        _capi.check(lib.icsa_select(pp, a[1], a[2], self.ws.data_ptr(), self.size, st), "icsa_select")
        if ev is not None:
            ev[2].record()
        both = overlap and self.p.num_flat > 0 and self.L.n_sparse > 0
        if both:
            self.fork.record(cur)
            self.side.wait_event(self.fork)
        _capi.check(lib.icsa_attend_dense(pp, *a, None, self.out.data_ptr(), self.ws.data_ptr(), self.size, st),
                    "icsa_attend_dense")
        if ev is not None:
            ev[3].record()
        sst = self.side.cuda_stream if both else st
        _capi.check(lib.icsa_attend_sparse(pp, *a, None, self.out.data_ptr(), self.ws.data_ptr(), self.size, sst),
                    "icsa_attend_sparse")
        if both:
            self.join.record(self.side)
            cur.wait_event(self.join)
        if ev is not None:
            ev[4].record()


# ---------------------------------------------------------------------------
# CPU baseline: the oracle port on a bounded sample
# ---------------------------------------------------------------------------
_CPU_INPUTS = {}


def cpu_reference_sample(w, head_count=2, seed_base=0):
    """Run the CPU restatement of the whole call (oracle.icsa_oracle.
    editing_sparse_attention: the reference's orchestration,
    editing_sparse_attention.py:67-232, with the TileLang kernel and
    flash_attn_func restated; pinned bit for bit against the reference's own
    orchestrator on configuration 1) for the first `head_count` heads of
    workload `w` at its full sequence length, and scale to all heads (every
    stage is independent per head).  The dense part runs in fp32, flash-attn's
    accumulation type.  Returns (ms/call, seconds spent, description)."""
    from oracle import icsa_oracle as orc
    torch.set_num_threads(os.cpu_count() or 1)
    key = (w.name, head_count, seed_base)
    if key not in _CPU_INPUTS:
        _CPU_INPUTS[key] = synthetic.make_inputs(w, heads=range(head_count), seed_base=seed_base, device="cpu")
    q, k, v = _CPU_INPUTS[key]
    t0 = time.perf_counter()
    r = orc.editing_sparse_attention(q, k, v, w.t_seq_len, dense_dtype=torch.float32)
    spent = time.perf_counter() - t0
    c = r.counts
    desc = (f"the whole call for {head_count} of {w.H} heads at the full sequence length (pooling, compressed "
            f"attention, selections, extended KV, all {c.num_flat} flat and {c.n_sparse} sparse query blocks), "
            f"scaled x{w.H / head_count:g} to {w.H} heads; the oracle's restatement of the reference orchestration "
            f"(torch, fp32 dense part) on {torch.get_num_threads()} threads")
    return spent / head_count * w.H * 1e3, spent, desc


def run_reference_arm(args, rank):
    """--impl reference: the CPU restatement of the reference path, timed on
    the host cores (rank 0 only)."""
    if rank != 0:
        return
    if args.workload == "dit-step":
        print(json.dumps({"impl": "reference", "unavailable": "the reference's DiT step runs its attention in "
                          "GPU-only TileLang/flash-attn kernels, and a CPU restatement of a 40-block A14B step "
                          "is hours of host time"}), flush=True)
        return
    w = WORKLOADS[args.workload]
    heads = min(args.ref_heads, w.H)
    for _ in range(args.warmup):
        cpu_reference_sample(w, head_count=heads)
    vals, secs = [], []
    for _ in range(args.steps):
        ms, sec, desc = cpu_reference_sample(w, head_count=heads)
        vals.append(ms)
        secs.append(sec)
    value = statistics.mean(vals)
    # a timed step is the bounded sample (heads of the call); `value` is the
    # whole call, scaled from it
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "ms/call", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(secs) * 1e3,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded blurred-field generator)", "config": config_dict(w, args.gpus),
            "extrapolation": {"heads_per_step": heads, "heads_per_call": w.H, "factor": w.H / heads,
                              "note": "ms_per_step is the measured time of one step (the sample); value is "
                                      "ms_per_step scaled to all heads of one call"},
            "cpu_baseline": {"value": value, "unit": "ms/call", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": desc},
            "e2e": {"value": value, "unit": "ms/call", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# DiT step: one denoising step of the A14B-shaped DiT
# ---------------------------------------------------------------------------
DIT_LATENT = (16, 21, 60, 104)   # 480p latent (VAE stride 4x8x8): 21 x 30 x 52 = 32760 patches per video


def dit_seq_len(latent):
    """Joint tokens: target | source | padding to a multiple of 512 (65536 for
    the 480p latent: 32760 | 32760 | 16), so that 8 ranks hold whole blocks."""
    t = latent[1] * (latent[2] // 2) * (latent[3] // 2)
    return -(-2 * t // 512) * 512
DIT_LAUNCHES_PER_BLOCK = 9 + 1 + 13  # 3 LayerNorm, 3 RMSNorm/RoPE, 3 projections with the residual update, the cross-attention + one
                                     # unaligned attention call


def dit_step_flops(cfg, B, S, t_seq_len):
    """Algorithmic FLOPs of one step (2 FLOP per MAC): the block GEMMs, the
    cross-attention, the sparse self-attention and the embeddings/head."""
    C, Fd, L, H, D = cfg.dim, cfg.ffn_dim, cfg.text_len, cfg.num_heads, cfg.head_dim
    T = B * S
    gemm = 2.0 * T * C * (3 * C + 1) + 2.0 * T * C * C          # q, k, v, alpha_1; o
    gemm += 2.0 * 2 * T * C * C + 2.0 * B * L * C * 2 * C        # cross q, o; cross k | v
    gemm += 2.0 * 2 * T * C * Fd                                 # FFN
    cross = 4.0 * B * S * L * C
    attn = attention_flops(_capi.problem(B, S, H, D, t_seq_len), _capi.workspace_layout(
        _capi.problem(B, S, H, D, t_seq_len)).n_sparse)[0]
    per_block = gemm + cross + attn
    outer = 2.0 * S * 64 * C + 2.0 * B * L * (cfg.text_dim * C + C * C) + 2.0 * T * C * 64
    return cfg.num_layers * per_block + outer, cfg.num_layers * attn


def run_dit_step(args, world, rank, local):
    """Seconds per denoising step of the Wan 2.2 A14B-shaped DiT (40 layers,
    dim 5120, 40 heads, FFN 13824; CFG pair as batch 2; 512 text tokens) on
    the 480p joint 65,536-token sequence, with Ulysses sequence parallelism
    over the ranks.  Random-init weights, synthetic latents and text."""
    import datetime

    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # the Ulysses exchanges overlap full-GPU kernels: on high-priority
        # streams their CTAs are scheduled ahead of the compute kernel's
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = not args.dit_normal_priority
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local), pg_options=opts)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from wan_dit import WanDiT, WanDiTConfig
    cfg = WanDiTConfig(num_layers=args.dit_layers)
    model = WanDiT(cfg, device=dev, seed=0, pipelined=not args.dit_no_pipeline,
                   pooled_exchange=not args.dit_f32_exchange)
    g = torch.Generator().manual_seed(0)
    shape = (DIT_LATENT[0], args.dit_frames, DIT_LATENT[2], DIT_LATENT[3])
    seq = dit_seq_len(shape)
    latent = torch.randn(*shape, generator=g)
    source = 0.8 * latent + 0.6 * torch.randn(*shape, generator=g)
    context = torch.randn(2, cfg.text_len, cfg.text_dim, generator=g)
    hl, hs, hc = (x.pin_memory() for x in (latent, source, context))
    dl, ds, dc = (x.to(dev) for x in (latent, source, context))
    hout = torch.empty(shape).pin_memory()
    t_seq_len = shape[1] * (shape[2] // 2) * (shape[3] // 2)

    def step(l_, s_, c_):
        return model.denoise_step(l_, s_, 999.0, 1.0, 31.0 / 32.0, c_, seq)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(dl, ds, dc)
    barrier()
    clocks = ClockSampler(dev)
    clocks.start()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = step(dl, ds, dc)
    e1.record()
    barrier()
    clk = clocks.stop()
    sec = e0.elapsed_time(e1) / 1e3 / args.steps
    del out

    # e2e: latents and text from pinned host memory in, the updated latent out
    e2e_sec = None
    if not args.no_e2e:
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        f0.record()
        for _ in range(args.steps):
            nl = step(hl.to(dev, non_blocking=True), hs.to(dev, non_blocking=True), hc.to(dev, non_blocking=True))
            hout.copy_(nl, non_blocking=True)
        f1.record()
        barrier()
        e2e_sec = f0.elapsed_time(f1) / 1e3 / args.steps
    if dist is not None:
        t = torch.tensor([sec, e2e_sec or 0.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        sec, e2e_sec = float(t[0]), (float(t[1]) if e2e_sec is not None else None)
    flops, attn_flops = dit_step_flops(cfg, 2, seq, t_seq_len)
    sustained, burst, _, src = peaks()
    achieved = flops / sec / 1e12 / world
    if rank == 0:
        line = {"metric": METRIC, "value": sec, "unit": "s/step", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, N(0,1) latents and text)",
                "config": {"workload": "wan22_a14b_dit_step_480p_cfg2" if args.dit_frames == DIT_LATENT[1] and
                           cfg.num_layers == 40 else f"wan22_a14b_dit_step_f{args.dit_frames}_l{cfg.num_layers}",
                           "layers": cfg.num_layers, "dim": cfg.dim,
                           "heads": cfg.num_heads, "ffn": cfg.ffn_dim, "text_tokens": cfg.text_len, "cfg_batch": 2,
                           "seq_len": seq, "t_seq_len": t_seq_len, "latent": list(shape),
                           "parallelism": f"ulysses x{world}",
                           "exchange": "one all-to-all per tensor" if args.dit_no_pipeline or world == 1
                           else "per batch element, overlapped with compute",
                           "nccl_stream_priority": "normal" if args.dit_normal_priority else "high",
                           "qk_exchange": "f32" if args.dit_f32_exchange or args.dit_no_pipeline
                           else "bf16 + f32 block means",
                           "l2": "every step streams 28 GB of weights; no flush"},
                "roofline": {"bound": "tensor", "kernel": "whole step (cuBLAS GEMMs for q|k|v, cross q, cross k|v and FFN-in; this library for the rest)",
                             "achieved": achieved, "peak": sustained, "unit": "TFLOP/s per GPU",
                             "frac": achieved / sustained, "peak_kind": f"{src} sustained bf16",
                             "flops_per_step": flops, "attention_flops_per_step": attn_flops, "traffic": None},
                "clocks": clk, "gpu_launches": (DIT_LAUNCHES_PER_BLOCK * cfg.num_layers + 1) * args.steps,
                "cpu_baseline": None}
        if e2e_sec is not None:
            line["e2e"] = {"value": e2e_sec, "unit": "s/step", "path": "WanDiT.denoise_step on pinned host latents",
                           "h2d_bytes_per_step": (hl.numel() + hs.numel() + hc.numel()) * 4,
                           "d2h_bytes_per_step": hout.numel() * 4}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# stage sweep: every stage timed on its own over joint
# length x flat ratio x source-selection ratio x batch, 40 heads x 128 d bf16
# ---------------------------------------------------------------------------
SWEEP_GRIDS = {4096: (4, 32, 32), 8192: (8, 32, 32), 16384: (16, 32, 32), 32768: (21, 30, 52),
               65536: (16, 64, 64)}  # tokens per video -> latent grid of the blurred-field generator
SWEEP_FLAT = (0.0, 0.5, 1.0)
SWEEP_SRR = (0.0625, 0.125, 0.25)
SWEEP_BATCH = (1, 2)


def run_sweep(args, local):
    """One JSON line with a row per configuration: the median CUDA-event time
    of each stage (pool, select, attend_dense, attend_sparse) over K steps
    after W warm-up steps, with each stage's achieved rate against the
    measured peaks (HBM GB/s for the pooling pass, TFLOP/s for the two
    attention kernels; the selection stage is latency-bound and reported in
    ms).  Inputs of one (joint length, batch) pair are generated once and
    shared by its flat-ratio / selection-ratio rows."""
    import dataclasses
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    sustained, burst, hbm, src = peaks()
    halves = [h for h in SWEEP_GRIDS if not args.sweep_max_joint or 2 * h <= args.sweep_max_joint]
    rows, launches = [], 0
    for half in halves:
        for B in SWEEP_BATCH:
            w = dataclasses.replace(synthetic.WAN480P, name=f"sweep_joint{2 * half}_b{B}", B=B,
                                    grid=SWEEP_GRIDS[half], half_len=half)
            q, k, v = synthetic.make_inputs(w, device=dev)
            for fr in SWEEP_FLAT:
                for srr in SWEEP_SRR:
                    r = Runner(q, k, v, half, select_ratio=srr, flat_ratio=fr)
                    for _ in range(args.warmup):
                        r.step(overlap=False)
                    torch.cuda.synchronize()
                    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
                    for i in range(args.steps):
                        r.step(evs[i], overlap=False)
                    torch.cuda.synchronize()
                    _capi.check(r.lib.icsa_device_status(r.ws.data_ptr(), torch.cuda.current_stream().cuda_stream),
                                "icsa_device_status")
                    st = {n: statistics.median(e[j].elapsed_time(e[j + 1]) for e in evs) for j, n in
                          enumerate(("pool", "select", "attend_dense", "attend_sparse"))}
                    _, fl, sp = attention_flops(r.p, r.L.n_sparse)
                    p = r.p
                    pool_bytes = 3 * q.numel() * q.element_size() + 3 * B * w.H * p.num_blocks * w.D * 6
                    row = {"joint": 2 * half, "B": B, "flat_ratio": fr, "select_ratio": srr,
                           "num_flat": p.num_flat, "n_sparse": r.L.n_sparse, "topK": p.topK, "top_k": p.top_k,
                           "tkv": p.tkv, "ms": st, "ms_call": sum(st.values()),
                           "pool_gbs": pool_bytes / (st["pool"] * 1e-3) / 1e9,
                           "dense_tflops": fl / (st["attend_dense"] * 1e-3) / 1e12 if fl else None,
                           "sparse_tflops": sp / (st["attend_sparse"] * 1e-3) / 1e12 if sp else None}
                    row["pool_frac"] = row["pool_gbs"] / hbm
                    row["dense_frac"] = row["dense_tflops"] / sustained if fl else None
                    row["sparse_frac"] = row["sparse_tflops"] / sustained if sp else None
                    rows.append(row)
                    # pool, scores, rowstats, outc, colsum, 2 sorts, extended KV; top-k and the sparse kernel only with
                    # sparse blocks, the dense kernel only with flat blocks
                    launches += (8 + (3 if r.L.n_sparse else 0) + (1 if p.num_flat else 0)) * args.steps
                    del r
            del q, k, v
            torch.cuda.empty_cache()
    print(json.dumps({"workload": "stage-sweep", "unit": "ms", "steps": args.steps, "warmup": args.warmup,
                      "dtype": "bf16", "data": "synthetic (seeded blurred-field generator)", "H": 40, "D": 128,
                      "peaks": {"hbm_gbs": hbm, "bf16_tflops_sustained": sustained, "kind": src},
                      "l2": "inputs of 0.13-10.7 GB; the small joint lengths fit in L2 (no flush)",
                      "gpu_launches": launches, "rows": rows}), flush=True)


class NumaLocal:
    """Within the block, the calling thread runs on the CPUs of the NUMA node
    the GPU hangs off (sysfs local_cpulist of its PCI function), so pinned
    host buffers allocated and first touched there live in that node's
    memory.  The previous affinity is restored on exit; `node` is the CPU
    list used, or None when it could not be read or binding is disabled."""

    def __init__(self, dev, enabled=True):
        self.dev, self.enabled, self.saved, self.node = dev, enabled, None, None

    def __enter__(self):
        if not self.enabled or not hasattr(os, "sched_setaffinity"):
            return self
        try:
            pr = torch.cuda.get_device_properties(self.dev)
            bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            with open(f"/sys/bus/pci/devices/{bus}/local_cpulist") as f:
                text = f.read().strip()
            cpus = set()
            for part in text.split(","):
                a, _, b = part.partition("-")
                cpus.update(range(int(a), int(b or a) + 1))
            self.saved = os.sched_getaffinity(0)
            cpus &= self.saved
            if cpus and cpus != self.saved:
                os.sched_setaffinity(0, cpus)
                self.node = text
            elif cpus:
                self.node = f"{text} (every CPU this process may use is local)"
        except Exception:  # noqa: BLE001
            self.node = None
        return self

    def __exit__(self, *exc):
        if self.saved is not None:
            os.sched_setaffinity(0, self.saved)
        return False


def measure_link(host_in, host_out, dev, barrier, reps=3):
    """Pinned host <-> device copies of this rank's step bytes, with every
    rank copying at the same time (barrier before each measurement): the
    H2D rate and the D2H rate alone (GB/s), and the time (ms) of both
    directions at once on two streams, which is what an e2e step needs at
    the least (its copies in and out overlap)."""
    dins = [torch.empty_like(h, device=dev) for h in host_in]
    dout = torch.empty_like(host_out, device=dev)
    h2d = list(zip(dins, host_in))
    d2h = [(host_out, dout)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def run(pairs):
        for _ in range(reps):
            for dst, src in pairs:
                dst.copy_(src, non_blocking=True)

    rates = []
    for pairs in (h2d, d2h):
        nbytes = sum(src.numel() * src.element_size() for _, src in pairs)
        run(pairs[:1])  # untimed
        barrier()
        e0.record()
        run(pairs)
        e1.record()
        barrier()
        rates.append(reps * nbytes / (e0.elapsed_time(e1) * 1e-3) / 1e9)
    # both directions at once
    side = torch.cuda.Stream(device=dev)
    barrier()
    e0.record()
    side.wait_event(e0)
    with torch.cuda.stream(side):
        run(d2h)
    run(h2d)
    done = torch.cuda.Event()
    done.record(side)
    torch.cuda.current_stream().wait_event(done)
    e1.record()
    barrier()
    both_ms = e0.elapsed_time(e1) / reps
    del dins, dout
    return rates[0], rates[1], both_ms


def time_reference_dense(q, k, v, num_flat, tkv, steps):
    """The reference's dense part on this GPU: flash_attn_func (the library
    call of editing_sparse_attention.py:211-215, flash-attn 2.8 as installed
    in this image) on the flat half's shapes -- num_flat*64 queries against
    the tkv rows of the extended KV -- timed with CUDA events; torch SDPA is
    timed beside it.  It is the 93 % of the reference call's FLOPs that a
    library already does on the GPU, so it bounds the reference's GPU time
    from below.  Query rows and KV rows are slices of q, k and v: the work
    depends only on the shapes."""
    import torch.nn.functional as F
    qf = q[:, :num_flat * 64].contiguous()
    kf, vf = k[:, :tkv].contiguous(), v[:, :tkv].contiguous()
    res = {"shape": {"q": list(qf.shape), "kv": list(kf.shape)}}

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    try:
        import flash_attn
        from flash_attn import flash_attn_func
        res["flash_attn_ms"] = timed(lambda: flash_attn_func(qf, kf, vf))
        res["flash_attn_version"] = flash_attn.__version__
    except Exception as e:  # noqa: BLE001
        res["flash_attn_unavailable"] = f"{type(e).__name__}: {str(e)[:200]}"
    try:
        qt, kt, vt = (x.transpose(1, 2) for x in (qf, kf, vf))
        res["torch_sdpa_ms"] = timed(lambda: F.scaled_dot_product_attention(qt, kt, vt))
    except Exception as e:  # noqa: BLE001
        res["torch_sdpa_unavailable"] = f"{type(e).__name__}: {str(e)[:200]}"
    return res


def config_dict(w, n):
    return {"workload": w.name, "B": w.B, "H": w.H, "D": w.D, "S": w.S, "t_seq_len": w.t_seq_len,
            "grid": list(w.grid), "heads_per_gpu": w.H // n, "parallelism": f"head-sharded x{n}",
            "sparsity_ratio": 0.0625, "select_ratio": 0.125, "flat_ratio": 0.5,
            "l2": "inputs (q,k,v) larger than L2; no flush"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="480p", choices=list(WORKLOADS) + ["dit-step", "sweep"])
    ap.add_argument("--sweep-max-joint", type=int, default=0, help="sweep: largest joint length (0: all)")
    ap.add_argument("--dit-layers", type=int, default=40, help="blocks of the DiT step (40 is the A14B model)")
    ap.add_argument("--dit-no-pipeline", action="store_true", help="DiT step: unpipelined Ulysses exchanges")
    ap.add_argument("--dit-f32-exchange", action="store_true",
                    help="DiT step: exchange q and k as f32 (default: bf16 with their f32 block means)")
    ap.add_argument("--dit-normal-priority", action="store_true",
                    help="DiT step: NCCL on normal-priority streams (default: high priority)")
    ap.add_argument("--dit-frames", type=int, default=DIT_LATENT[1],
                    help="latent frames of the DiT step (21 is 480p video; fewer give a small profiling case)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-heads", type=int, default=4, help="heads the CPU baseline runs in full")
    ap.add_argument("--ref-heads", type=int, default=2, help="heads per step of --impl reference")
    ap.add_argument("--no-numa-bind", action="store_true",
                    help="e2e: do not place the pinned host buffers on the GPU's NUMA node")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's dense-part library (flash-attn) on this GPU")
    ap.add_argument("--heads", type=int, default=0, help="run only this many heads (profiling of a small case)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return
    if args.workload == "dit-step":
        run_dit_step(args, world, rank, local)
        return
    if args.workload == "sweep":
        if rank == 0:
            run_sweep(args, local)
        return

    import datetime
    dist = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = WORKLOADS[args.workload]
    if args.heads:
        import dataclasses
        w = dataclasses.replace(w, H=args.heads, name=f"{w.name}_h{args.heads}")
    heads = list(sharding.head_range(w.H, rank, world))
    hp = len(heads)
    q, k, v = synthetic.make_inputs(w, heads=heads, device=dev)
    runner = Runner(q, k, v, w.t_seq_len)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        runner.step()
    barrier()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    clocks = ClockSampler(dev)
    clocks.start()
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for i in range(args.steps):
        runner.step(evs[i])
    t_end.record()
    barrier()
    clk = clocks.stop()
    elapsed = t_start.elapsed_time(t_end)
    stage = {n: statistics.mean(e[i].elapsed_time(e[i + 1]) for e in evs) for i, n in
             enumerate(("pool", "select", "attend_dense", "attend_sparse_exposed"))}
    # the block-sparse kernel on its own: the same calls with the two attention
    # halves in sequence, after the timed region
    seq = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    for i in range(args.steps):
        runner.step(seq[i], overlap=False)
    torch.cuda.synchronize()
    stage["attend_sparse"] = statistics.mean(e[3].elapsed_time(e[4]) for e in seq)
    stage["sequential_call"] = statistics.mean(e[0].elapsed_time(e[4]) for e in seq)
    rc = runner.lib.icsa_device_status(runner.ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _capi.check(rc, "icsa_device_status")

    # e2e through the public API with host buffers: pinned q, k, v in, pinned
    # result out; the call streams head groups through the GPU (copy in,
    # compute and copy out overlap) and every byte crosses PCIe inside the
    # timed region
    e2e = None
    if not args.no_e2e:
        with NumaLocal(dev, enabled=not args.no_numa_bind) as numa:
            hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
            hout = torch.empty(q.shape, dtype=q.dtype).pin_memory()
            hout.zero_()

        def e2e_step():
            editing_sparse_attention(hq, hk, hv, w.t_seq_len, w.t_seq_len, out=hout, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        e2e = {"value": e2e_ms, "unit": "ms/call", "path": "editing_sparse_attention on pinned host tensors",
               "h2d_bytes_per_step": 3 * q.numel() * q.element_size() * world,
               "d2h_bytes_per_step": q.numel() * q.element_size() * world}
        # the host link's rates with every rank copying at once, and the floor
        # they put under e2e: the slower direction of this rank's bytes
        h2d_gbs, d2h_gbs, floor = measure_link((hq, hk, hv), hout, dev, barrier)
        link = [h2d_gbs, d2h_gbs, floor]
        if dist is not None:
            gathered = [torch.zeros(3, device=dev) for _ in range(world)]
            dist.all_gather(gathered, torch.tensor(link, device=dev))
            link = torch.stack(gathered).cpu().tolist()
        else:
            link = [link]
        e2e["link"] = {"h2d_gbs_per_rank": [r[0] for r in link], "d2h_gbs_per_rank": [r[1] for r in link],
                       "floor_ms": max(r[2] for r in link),
                       "measured": "pinned contiguous copies of each rank's step bytes, all ranks at once; rates "
                                   "per direction alone, floor_ms = both directions at once on two streams "
                                   "(max over ranks)",
                       "numa_bound_cpus": numa.node}

    ms = elapsed / args.steps
    # time x clock of this rank (the power cap moves the clock with the load)
    ms_x_mhz = ms * (clk["sm_mhz"] or 0.0)
    if dist is not None:
        names = sorted(stage)
        t = torch.tensor([ms, e2e["value"] if e2e else 0.0, ms_x_mhz] + [stage[n] for n in names], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        if e2e:
            e2e["value"] = float(t[1])
        ms_x_mhz = float(t[2])
        stage = {n: float(x) for n, x in zip(names, t[3:])}
        mhz = torch.zeros(world, device=dev)
        mhz[rank] = clk["sm_mhz"] or 0.0
        dist.all_reduce(mhz)
        clk["sm_mhz_per_rank"] = mhz.cpu().tolist()
    sustained, burst, hbm, src = peaks()
    _, flops, sparse_flops = attention_flops(runner.p, runner.L.n_sparse)
    # dominant kernel: the dense attention of the flat query blocks (one launch per call)
    achieved = flops / (stage["attend_dense"] * 1e-3) / 1e12
    sparse_achieved = sparse_flops / (stage["attend_sparse"] * 1e-3) / 1e12
    traffic = None
    tpath = os.path.join(REPO, "profiles", "dense_pair_kernel_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            tr = json.load(f)
        # measured on a smaller head count; DRAM bytes grow in proportion to the heads
        if tr.get("workload") == w.name.split("_h")[0] and tr.get("heads"):
            traffic = tr["dram_bytes_per_launch"] * hp / tr["heads"]

    if rank == 0:
        line = {"metric": METRIC, "value": ms, "unit": "ms/call", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32" if w.dtype == torch.float32 else "bf16",
                "data": "synthetic (seeded blurred-field generator)",
                "config": config_dict(w, world),
                "stages_ms": stage,
                "roofline": {"bound": "tensor", "kernel": "dense_pair_kernel (dense attention of the flat blocks, SM pairs)",
                             "achieved": achieved, "peak": sustained, "unit": "TFLOP/s", "frac": achieved / sustained,
                             "peak_kind": f"{src} sustained bf16", "frac_of_burst": achieved / burst,
                             "traffic": traffic, "flops_per_launch": flops,
                             "sparse_kernel": {"achieved": sparse_achieved, "frac": sparse_achieved / sustained,
                                               "flops_per_launch": sparse_flops}},
                "clocks": clk, "gpu_launches": KERNELS_PER_CALL_ALIGNED * args.steps}
        if ms_x_mhz and clk.get("sm_max_mhz"):
            line["clock_normalised"] = {
                "ms_x_mhz": ms_x_mhz, "ms_at_sm_max_mhz": ms_x_mhz / clk["sm_max_mhz"],
                "note": "max over ranks of (ms per call x median SM MHz under load); compare across N to factor "
                        "out the power cap's clock"}
        if e2e:
            line["e2e"] = e2e
        if world == 1 and not args.no_reference_gpu:
            line["reference_gpu"] = time_reference_dense(q, k, v, runner.p.num_flat, runner.p.tkv,
                                                         max(3, args.steps // 2))
            line["reference_gpu"]["note"] = (
                "the reference's dense part alone (flash_attn_func, 93% of the call's FLOPs) on this GPU; its "
                "TileLang/Triton kernels are JIT-compiled from the reference's sources, which this repository "
                "does not carry to the GPU box")
        if world == 1 and not args.no_cpu_baseline:
            cms, secs, desc = cpu_reference_sample(w, head_count=args.cpu_heads)
            line["cpu_baseline"] = {"value": cms, "unit": "ms/call", "cores": torch.get_num_threads(),
                                    "kind": "port", "sample": desc, "sample_seconds": secs}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
