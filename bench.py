#!/usr/bin/env python
"""Benchmark of vidax's attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

Workload (every N): the Ulysses self-attention layer of Wan2.1-14B at
720p/81 frames -- B=1, S=75600 tokens, H=40 heads, head_dim 128, bf16, scale
1/sqrt(128) -- with the sequence sharded evenly over the N ranks (strong
scaling: total work fixed). At N=1 the layer is one local attention call; at
N>1 it is the tokens->heads exchange -> attention on H/N heads over the full
sequence -> the heads->tokens exchange, pipelined by head slices, the
exchanges done by the pack / unpack kernels storing into / loading from the
other ranks' slabs over NVLink (`--exchange peer`, default) or as pack ->
NCCL all-to-all -> unpack (`--exchange nccl`). Inputs are seeded N(0,1)
synthetic tensors (no dataset exists for this path); every input exceeds the
126 MB L2, so no flush is needed between steps.

One JSON line (rank 0): value = whole-job attention TFLOP/s (vidax's FLOP
convention 4*B*H*S*S*D over the max-over-ranks step time), `e2e` = the same
through the public API with pinned host inputs copied in and the output
copied out every step, `roofline` = the attention kernel against the
measured bf16 peak, `cpu_baseline` = the CPU oracle on a bounded sample;
`secondary` = (N=1) cfg2, cfg4 and fused pre-step kernel timings and the
numpy restatement of vidax's NA scan timed on cfg4 row steps; (every N) one
Wan2.1-1.3B DiT step at BASELINE config 5, B=1 and the CFG B=2 step, with
the attention kernels' share; `parity` = seeded rows of the timed output
against a float32 softmax reference computed on the GPU.

`--impl reference` times the reference's CPU path (vidax's JAX CPU attention
is `jax.nn.dot_product_attention`; JAX is absent, so its numpy restatement in
oracle/ runs) on rank 0 with all host cores, one bounded sample per step.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, S_GLOBAL, H, D = 1, 75600, 40, 128
WORKLOAD = "cfg3: Ulysses self-attention layer, Wan2.1-14B 720p/81f (B=1, S=75600, H=40, D=128, bf16)"
FALLBACK_PEAK_TFLOPS = 1590.0
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of one attn_fwd_kernel launch
# per (head x token), from the ncu capture of the (1, 32760, 8, 128) case
# (profiles/attn_fwd_dense_h8.md: 248.6 MB / (8 x 32760)); traffic grows with
# heads x tokens, so it scales to a full launch.
TRAFFIC_BYTES_PER_HEAD_TOKEN = 948.6


def flops(b, h, sq, sk, d):
    return 4.0 * b * h * sq * sk * d


def load_hbm_peak():
    """Measured HBM copy bandwidth (GB/s) and its source."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return FALLBACK_HBM_GBS, "fallback"


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return pk.get("bf16_tflops"), pk.get("bf16_tflops_sustained"), "measured"
    except (OSError, ValueError):
        return FALLBACK_PEAK_TFLOPS, 1400.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons of one GPU every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None}


def gpu_id_for(dev) -> str:
    import torch
    p = torch.cuda.get_device_properties(dev)
    try:
        return f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except AttributeError:
        return str(dev)


def host_cpu() -> dict:
    """The host the CPU baseline ran on: CPU model and logical core count."""
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    model = ln.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "logical_cpus": os.cpu_count()}


def blas_threads() -> int:
    """Threads numpy's BLAS runs with (the host cores a CPU baseline uses)."""
    try:
        from threadpoolctl import threadpool_info
        return max((i.get("num_threads", 1) for i in threadpool_info()), default=os.cpu_count())
    except Exception:
        return os.cpu_count()


def cpu_sample(seconds: float, rows_per_chunk: int = 256):
    """Times the oracle (numpy restatement of jax.nn.dot_product_attention) on
    head 0 of the workload: chunks of query rows against all S keys, until
    `seconds` of CPU time have run. Returns (TFLOP/s, threads, description)."""
    import numpy as np
    from oracle.attention_ref import sdpa, seeded_qkv
    threads = blas_threads()
    q, k, v = seeded_qkv((1, S_GLOBAL, 1, D), 3)
    done_rows, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds and done_rows < S_GLOBAL:
        rows = np.arange(done_rows, min(done_rows + rows_per_chunk, S_GLOBAL))
        sdpa(q, k, v, q_rows=rows, chunk=rows_per_chunk)
        done_rows += len(rows)
    dt = time.perf_counter() - t0
    tf = flops(1, 1, done_rows, S_GLOBAL, D) / dt / 1e12
    desc = (f"numpy oracle, head 0 of cfg3: {done_rows} query rows x {S_GLOBAL} keys "
            f"({flops(1, 1, done_rows, S_GLOBAL, D) / 1e9:.1f} GFLOP in {dt:.1f} s)")
    return tf, threads, desc


def na_cpu_sample(seconds: float):
    """Times the oracle's restatement of vidax's NA scan step (one (t, h) row
    of diffusion_vae.py:206-225: gather the row's 5x9 frame/row windows, the
    W-window of every w, two einsums) for cfg4's shapes: W = 52, 24 heads,
    head_dim 128, window 5x9x9. Every cfg4 row does the same work (windows
    shift at the borders, they do not shrink), so the rows are timed on the
    centre row of a 5 x 9 x 52 grid, whose window is that whole grid, and the
    full scan is the per-row time x 630 rows. Returns a secondary-line dict."""
    import numpy as np
    from oracle.attention_ref import to_bf16
    from oracle.na3d_ref import na3d
    kernel, rows_full = (5, 9, 9), 21 * 30
    shape = (1, 5, 9, 52, 24, D)
    rng = np.random.Generator(np.random.PCG64(4))
    q = to_bf16(to_bf16(rng.standard_normal(shape, dtype=np.float32)) * D ** -0.5)
    k = to_bf16(rng.standard_normal(shape, dtype=np.float32))
    v = to_bf16(rng.standard_normal(shape, dtype=np.float32))
    na3d(q, k, v, kernel, round_logits=True, round_probs=True, rows=[(2, 4)])  # warm-up
    done, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        na3d(q, k, v, kernel, round_logits=True, round_probs=True, rows=[(2, 4)])
        done += 1
    dt = time.perf_counter() - t0
    row_flops = 4.0 * 52 * 405 * D * 24
    return {"desc": f"numpy restatement of vidax's NA scan, cfg4 row steps: {done} rows in "
                    f"{dt:.1f} s (the full scan is 630 rows)", "rows": done,
            "est_full_ms": round(dt / done * rows_full * 1e3, 1),
            "tflops": round(row_flops * done / dt / 1e12, 5), "cores": blas_threads()}


def add_na_cpu_line(secondary: dict, seconds: float) -> None:
    """vidax's NA on the host cores (its scan restated in numpy) as the
    `cfg4_cpu_scan` secondary entry, next to the kernel's cfg4 line."""
    na_cpu = na_cpu_sample(seconds)
    if "cfg4" in secondary:
        na_cpu["est_full_over_kernel"] = round(na_cpu["est_full_ms"] / secondary["cfg4"]["ms"])
    secondary["cfg4_cpu_scan"] = na_cpu


def time_launches(fn, steps: int, warmup: int):
    """Device time (ms) per launch of `fn`, CUDA events on the current stream."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


NVLINK_NOMINAL_GBS = 900.0      # per direction per GPU (NVLink 5)
NVLINK_MEASURED_GBS = 770.0     # peer copy per direction measured on this pool's B200s


def measure_all_to_all(numel: int, reps: int, dev, dtype, group=None) -> dict:
    """One equal-split `all_to_all_single` of `numel` elements per rank (the
    exchange the Ulysses layer runs four times: q, k, v tokens -> heads and
    o heads -> tokens), timed `reps` times after 3 warm-up calls: device time
    with CUDA events on the current stream (wall clock on a CPU group), max
    over ranks. Bytes per GPU per direction = (P-1)/P of the buffer (the
    rank's own share does not cross a link)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    numel -= numel % world
    send = torch.ones(numel, dtype=dtype, device=dev)
    recv = torch.empty_like(send)
    for _ in range(3):
        dist.all_to_all_single(recv, send, group=group)
    dist.barrier(group=group)
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            dist.all_to_all_single(recv, send, group=group)
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / reps
    else:
        t0 = time.perf_counter()
        for _ in range(reps):
            dist.all_to_all_single(recv, send, group=group)
        ms = (time.perf_counter() - t0) * 1e3 / reps
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    ms = float(t.item())
    link_bytes = (world - 1) / world * numel * send.element_size()
    gbs = link_bytes / (ms / 1e3) / 1e9
    return {"buffer_bytes_per_gpu": numel * send.element_size(),
            "bytes_per_gpu_per_direction": link_bytes, "ms": round(ms, 4),
            "gbs_per_direction": round(gbs, 1),
            "frac_of_nvlink_nominal": round(gbs / NVLINK_NOMINAL_GBS, 4),
            "frac_of_peer_copy_measured": round(gbs / NVLINK_MEASURED_GBS, 4)}


def parity_sample(out, q, k, v, world: int, dev, rows_per_rank: int = 32) -> dict:
    """Checks seeded rows of the layer's output (this rank's local tokens,
    all heads) against a float32-softmax attention computed with torch on
    the GPU over the global sequence (the ranks' k / v gathered when N > 1).
    Returns the max / mean absolute error over ranks and whether they meet
    the tolerance (max-abs 2e-2, mean-abs 2e-3)."""
    import torch
    import torch.distributed as dist
    b, s_loc, h, d = q.shape
    if world > 1:
        # (world * s_loc, H, D): the ranks' chunks in rank order
        kg = torch.empty((world * s_loc, h, d), dtype=k.dtype, device=dev)
        vg = torch.empty_like(kg)
        dist.all_gather_into_tensor(kg, k[0].contiguous())
        dist.all_gather_into_tensor(vg, v[0].contiguous())
    else:
        kg, vg = k[0], v[0]
    gen = torch.Generator().manual_seed(11)
    idx = torch.cat([torch.arange(0, 2), torch.arange(s_loc - 2, s_loc),
                     torch.randint(0, s_loc, (rows_per_rank - 4,), generator=gen)]).to(dev)
    logits = torch.einsum("nhd,shd->hns", q[0, idx].float(), kg.float()) * (d ** -0.5)
    ref = torch.einsum("hns,shd->nhd", torch.softmax(logits, dim=-1), vg.float())
    del logits
    diff = (out[0, idx].float() - ref).abs()
    stats = torch.tensor([diff.max().item(), diff.mean().item()], dtype=torch.float64, device=dev)
    if world > 1:
        mx = stats[:1].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(stats, op=dist.ReduceOp.SUM)
        stats = torch.stack([mx[0], stats[1] / world])
    mx, mean = float(stats[0]), float(stats[1])
    return {"max_abs": round(mx, 6), "mean_abs": round(mean, 7), "rows_per_rank": rows_per_rank,
            "heads": h, "reference": "float32 softmax attention in torch on the GPU",
            "tolerance": {"max_abs": 2e-2, "mean_abs": 2e-3},
            "pass": bool(mx <= 2e-2 and mean <= 2e-3)}


def kernel_case(name: str, dev):
    """Named single-kernel cases (profiling and secondary measurements).

    attn:B,S,H    dense attention, N(0,1) inputs, D=128
    cfg1          BASELINE config 1: (1, 4680, 12, 128) -- 228 work units on 148 SMs
    cfg2          BASELINE config 2: (1, 32760, 40, 128), per-head factors U[0.5, 2]
    cfg4          BASELINE config 4: NA over (1, 21, 30, 52, 24, 128), window 5x9x9
    na3d:T,H,W,NH window 5x9x9
    na3d64:T,H,W,NH,kt,kh,kw  head_dim-64 neighborhood attention (LTX-2.5 decoder stages)
    prologue:S,H,P  fused RMSNorm(dim) + RoPE + Ulysses send packing of q, k, v
                  (S tokens, H heads, D=128, P destination ranks); its work is
                  algorithmic HBM bytes, not FLOPs (see kernel_case_bytes)
    Returns (callable, algorithmic FLOPs per launch, description).
    """
    import torch
    import vidax_b200 as vx
    gen = torch.Generator(device=dev)
    gen.manual_seed(12345)

    def rnd(shape):
        return torch.randn(shape, generator=gen, device=dev, dtype=torch.float32).bfloat16()

    if name in ("cfg1", "cfg2") or name.startswith("attn:"):
        if name == "cfg2":
            b, s, h = 1, 32760, 40
        elif name == "cfg1":
            b, s, h = 1, 4680, 12
        else:
            b, s, h = (int(x) for x in name.split(":")[1].split(","))
        q, k, v = rnd((b, s, h, D)), rnd((b, s, h, D)), rnd((b, s, h, D))
        if name == "cfg2":
            f = torch.empty(3, h, device=dev).uniform_(0.5, 2.0, generator=gen)
            q = (q.float() * f[0, :, None]).bfloat16()
            k = (k.float() * f[1, :, None]).bfloat16()
            v = (v.float() * f[2, :, None]).bfloat16()
        return (lambda: vx.flash_attention(q, k, v, D ** -0.5)), flops(b, h, s, s, D), \
            f"attention (B={b}, S={s}, H={h}, D={D})"
    if name == "cfg4" or name.startswith("na3d:"):
        if name == "cfg4":
            t, hh, w, nh = 21, 30, 52, 24
        else:
            t, hh, w, nh = (int(x) for x in name.split(":")[1].split(","))
        shape = (1, t, hh, w, nh, D)
        q = (rnd(shape).float() * D ** -0.5).bfloat16()
        k, v = rnd(shape), rnd(shape)
        fl = vx.na3d_flops(1, t, hh, w, nh, D, (5, 9, 9))
        return (lambda: vx.neighborhood_attention_3d(q, k, v, (5, 9, 9))), fl, \
            f"neighborhood attention (1, {t}, {hh}, {w}, {nh}, {D}), window 5x9x9"
    if name.startswith("na3d64:"):
        # head_dim 64 (LTX-2.5 decoder): na3d64:T,H,W,NH,kt,kh,kw
        t, hh, w, nh, kt, kh, kw = (int(x) for x in name.split(":")[1].split(","))
        shape = (1, t, hh, w, nh, 64)
        q = (rnd(shape).float() * 64 ** -0.5).bfloat16()
        k, v = rnd(shape), rnd(shape)
        fl = vx.na3d_flops(1, t, hh, w, nh, 64, (kt, kh, kw))
        return (lambda: vx.neighborhood_attention_3d(q, k, v, (kt, kh, kw))), fl, \
            f"neighborhood attention (1, {t}, {hh}, {w}, {nh}, 64), window {kt}x{kh}x{kw}"
    if name.startswith("prologue:"):
        from vidax_b200.prologue import norm_rope_pack
        from vidax_b200.ulysses import _pieces
        s, h, p = (int(x) for x in name.split(":")[1].split(","))
        xs = [rnd((1, s, h * D)) for _ in range(3)]
        wq, wk = (1.0 + 0.1 * torch.randn(h * D, generator=gen, device=dev) for _ in range(2))
        ang = torch.rand((s, D // 2), generator=gen, device=dev) * 100.0
        rope = (torch.cos(ang), torch.sin(ang))
        hg = -(-h // p)
        slices = _pieces(hg) if p > 1 else None
        out = [torch.empty((1, p * s * hg * D), dtype=torch.bfloat16, device=dev) for _ in range(3)]
        return (lambda: norm_rope_pack(xs, h, norm_weights=[wq, wk, None], rope=rope, groups=p,
                                       slices=slices, out=out)), 0.0, \
            f"norm+rope+pack of q, k, v (S={s}, H={h}, D={D}, P={p})"
    raise SystemExit(f"unknown --kernel-only case {name!r}")


def na_case_bytes(name: str) -> float:
    """Algorithmic HBM bytes of a neighborhood-attention case: q, k, v read
    once and o written once (bf16). cfg4: 805.1 MB."""
    if name == "cfg4":
        t, hh, w, nh, hd = 21, 30, 52, 24, D
    elif name.startswith("na3d64:"):
        t, hh, w, nh = (int(x) for x in name.split(":")[1].split(",")[:4])
        hd = 64
    else:
        t, hh, w, nh = (int(x) for x in name.split(":")[1].split(","))
        hd = D
    return 4 * t * hh * w * nh * hd * 2


def kernel_case_bytes(name: str) -> float:
    """Algorithmic HBM bytes of a prologue case: read q, k, v once (bf16),
    write the packed slabs once (P * Hg heads, padding included), read the
    cos / sin tables once (float32, D/2 each per token); weights stay in L2."""
    s, h, p = (int(x) for x in name.split(":")[1].split(","))
    hg = -(-h // p)
    return 3 * s * h * D * 2 + 3 * s * p * hg * D * 2 + 2 * s * (D // 2) * 4


def run_kernel_only(args):
    import torch
    from vidax_b200 import _lib
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.load()
    fn, fl, desc = kernel_case(args.kernel_only, dev)
    ms = time_launches(fn, args.steps, args.warmup)
    assert _lib.device_status() == 0
    rec = {"case": args.kernel_only, "desc": desc, "ms_per_launch": round(ms, 4)}
    if args.kernel_only.startswith("prologue:"):
        rec["gbs"] = round(kernel_case_bytes(args.kernel_only) / (ms / 1e3) / 1e9, 1)
    else:
        rec["tflops"] = round(fl / (ms / 1e3) / 1e12, 2)
    if args.kernel_only == "cfg4" or args.kernel_only.startswith("na3d"):
        rec["gbs_algorithmic"] = round(na_case_bytes(args.kernel_only) / (ms / 1e3) / 1e9, 1)
    rec["launches"] = args.steps
    print(json.dumps(rec), flush=True)


def dit_measure(world: int, dev, batch: int = 1, steps: int = 3, warmup: int = 2) -> dict:
    """One Wan2.1-1.3B DiT forward step at BASELINE config 5 (latent
    (B, 21, 60, 104, 16) -> 32760 tokens, 512 text tokens, t = 500; random
    weights and inputs): Ulysses sequence parallelism over the `world` ranks
    of the default group (axis "sp", registered by the caller when world >
    1), 12 heads padded to a multiple of the rank count. batch = 2 is the
    reference's classifier-free-guidance step (conditional and
    unconditional rows in one batch, generate_wan2_1_t2v.py:453-456).
    Device time per step with CUDA events, max over ranks, plus the
    attention kernels' share of it (every self- and cross-attention launch
    bracketed by events). All ranks must call it together."""
    import torch
    import torch.distributed as dist
    import vidax_b200 as vx
    from vidax_b200 import _lib
    from vidax_b200 import attention as vx_attention
    from vidax_b200.wan_dit import T2V_1_3B, init_params, step_flops, wan_dit_forward
    cfg = T2V_1_3B
    sp = "sp" if world > 1 else None
    p = init_params(cfg, dev, seed=5, on_device=True)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    latents = torch.randn((batch, 21, 60, 104, cfg.in_dim), generator=gen, device=dev).bfloat16()
    context = torch.randn((batch, cfg.text_len, cfg.text_dim), generator=gen, device=dev).bfloat16()
    t = torch.full((batch,), 500.0, device=dev)
    rope = vx.rope3d_freqs(21, 30, 52, cfg.head_dim, device=dev)

    def step():
        return wan_dit_forward(p, cfg, latents, t, context, rope, sp_axis_name=sp)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    if world > 1:
        dist.barrier()
    events = []
    vx_attention.KERNEL_EVENTS = events
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        out = step()
    e1.record()
    torch.cuda.synchronize()
    vx_attention.KERNEL_EVENTS = None
    ms = e0.elapsed_time(e1) / steps
    attn_ms = sum(a.elapsed_time(b) for a, b in events) / steps
    if world > 1:
        tt = torch.tensor([ms, attn_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, attn_ms = float(tt[0]), float(tt[1])
        dist.barrier()
    fl = batch * step_flops(cfg, 21 * 30 * 52)
    status = _lib.device_status()
    shape = list(out.shape)
    del p, out
    return {"desc": f"Wan2.1-1.3B DiT forward step (cfg5), B={batch}"
                    + (" (CFG: conditional + unconditional)" if batch == 2 else "")
                    + f", 32760 tokens, 30 blocks, {'ulysses-sp%d' % world if world > 1 else 'single GPU'}",
            "ms": round(ms, 3), "tflops": round(fl / (ms / 1e3) / 1e12, 2),
            "flops_per_step": fl, "attention_kernel_ms": round(attn_ms, 3),
            "attention_share": round(attn_ms / ms, 4), "steps": steps, "warmup": warmup,
            "out_shape": shape, "device_status": status}


def run_dit(args, rank: int, world: int, local_rank: int):
    """--dit: the cfg5 DiT step as the whole benchmark line (B = 1)."""
    import torch
    import vidax_b200 as vx
    from vidax_b200 import _lib
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    _lib.load()
    if world > 1:
        vx.register_axis("sp", None, exchange=args.exchange)
    try:
        rec = dit_measure(world, dev, batch=1, steps=args.steps, warmup=args.warmup)
    except Exception as e:   # the peer mapping failed on every rank alike: NCCL instead
        from vidax_b200.ulysses_peer import PeerUnavailable
        if not isinstance(e, PeerUnavailable):
            raise
        print(f"peer exchange unavailable, NCCL used: {e}", file=sys.stderr, flush=True)
        args.exchange = "nccl"
        vx.register_axis("sp", None, exchange="nccl")
        rec = dit_measure(world, dev, batch=1, steps=args.steps, warmup=args.warmup)
    if world > 1:
        vx.unregister_axis("sp")
        if args.exchange == "peer":
            from vidax_b200 import ulysses_peer
            ulysses_peer.release_workspaces()   # collective, every rank
    if rank == 0:
        print(json.dumps({
            "metric": "Wan2.1-1.3B DiT forward step (cfg5), matmul TFLOP/s", "value": rec["tflops"],
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": rec["ms"], "higher_is_better": True, "scaling": "strong",
            "dtype": "bf16", "data": "synthetic (random weights and inputs)",
            "config": {"workload": "cfg5: Wan2.1-1.3B t2v DiT step, latent (1, 21, 60, 104, 16), "
                                   "32760 tokens, 30 blocks, text 512, CFG off (B=1)",
                       "parallelism": f"ulysses-sp{world}" if world > 1 else "single",
                       "flops_per_step": rec["flops_per_step"]},
            "attention_share": rec["attention_share"], "out_shape": rec["out_shape"],
            "device_status": rec["device_status"]}), flush=True)


def run_reference(args, rank: int):
    """Reference arm: vidax's CPU attention path (restated) on the host cores."""
    if rank != 0:
        return
    import numpy as np
    from oracle.attention_ref import sdpa, seeded_qkv
    threads = blas_threads()
    q, k, v = seeded_qkv((1, S_GLOBAL, 1, D), 3)
    rows_per_step = 2048

    def step(i):
        r0 = (i * rows_per_step) % (S_GLOBAL - rows_per_step)
        sdpa(q, k, v, q_rows=np.arange(r0, r0 + rows_per_step), chunk=512)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i)
    dt = (time.perf_counter() - t0) / args.steps
    fl = flops(1, 1, rows_per_step, S_GLOBAL, D)
    value = fl / dt / 1e12
    sample = (f"per step: {rows_per_step} query rows x {S_GLOBAL} keys of one head of cfg3 "
              f"({fl / 1e9:.1f} GFLOP); numpy restatement of jax.nn.dot_product_attention "
              "(JAX not installed)")
    line = {
        "impl": "reference", "metric": "attention TFLOP/s (Ulysses attn layer, Wan2.1-14B 720p)",
        "value": round(value, 5), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": "bounded CPU sample per step"},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port", "sample": sample, **host_cpu()},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist
    import vidax_b200 as vx
    from vidax_b200 import _lib, ulysses, ulysses_peer

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    _lib.load()
    if world > 1:
        vx.register_axis("sp", None, exchange=args.exchange)
    if S_GLOBAL % world != 0:
        raise SystemExit(f"S={S_GLOBAL} does not split evenly over {world} ranks")
    s_loc = S_GLOBAL // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(3 * 1000 + rank)
    q = torch.randn((B, s_loc, H, D), generator=gen, device=dev, dtype=torch.float32).bfloat16()
    k = torch.randn((B, s_loc, H, D), generator=gen, device=dev, dtype=torch.float32).bfloat16()
    v = torch.randn((B, s_loc, H, D), generator=gen, device=dev, dtype=torch.float32).bfloat16()

    kernel_ms = []
    ulysses_events = []

    def layer(qq, kk, vv):
        if world == 1:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            o = vx.dot_product_attention(qq, kk, vv)
            e1.record()
            ulysses_events.append((e0, e1))
            return o
        return vx.sequence_parallel_self_attention(qq, kk, vv, "sp")   # exchange: the axis's

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    exchange_note = None
    if world > 1 and args.exchange == "peer":
        try:
            layer(q, k, v)   # the first call maps the ranks' workspaces (collective)
        except ulysses_peer.PeerUnavailable as e:   # raised on every rank alike
            exchange_note = f"peer exchange unavailable, NCCL used: {e}"
            print(exchange_note, file=sys.stderr, flush=True)
            args.exchange = "nccl"
            vx.register_axis("sp", None, exchange="nccl")
    for _ in range(args.warmup):
        layer(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0, "device status word set during warm-up"
    ulysses_events.clear()
    ulysses.KERNEL_EVENTS = ulysses_events if world > 1 else None

    sampler = ClockSampler(gpu_id_for(dev))
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(args.steps):
        out = layer(q, k, v)
    t_end.record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ulysses.KERNEL_EVENTS = None
    ms = max_over_ranks(t_start.elapsed_time(t_end) / args.steps)
    kernel_ms = [a.elapsed_time(b) for a, b in ulysses_events]
    # attention-kernel time per layer (all pipelined slices of a step)
    kern_avg = max_over_ranks(sum(kernel_ms) / args.steps) if kernel_ms else float("nan")
    status = _lib.device_status()
    # the timed output's values: sampled rows against a float32 reference
    parity = parity_sample(out, q, k, v, world, dev)

    total_flops = flops(B, H, S_GLOBAL, S_GLOBAL, D)
    value = total_flops / (ms / 1e3) / 1e12
    hg = -(-H // world)
    launch_flops = flops(B, hg, S_GLOBAL, S_GLOBAL, D)
    achieved = launch_flops / (kern_avg / 1e3) / 1e12
    burst, sustained, peak_src = load_peaks()
    per_layer = (ulysses_peer.launches_per_layer(H, world, B) if args.exchange == "peer"
                 else ulysses.launches_per_layer(H, world, B))
    gpu_launches = args.steps * (1 if world == 1 else per_layer)

    # ---- end to end through the public API: pinned host in, host out
    hq = q.cpu().pin_memory()
    hk = k.cpu().pin_memory()
    hv = v.cpu().pin_memory()
    hout = torch.empty_like(hq).pin_memory()

    def e2e_step():
        if world == 1:
            # public host-buffer path: transfers pipelined against the kernel
            vx.attention_from_host(hq, hk, hv, D ** -0.5, out=hout, device=dev)
            return
        # public host-buffer path: per-slice uploads land directly in the
        # all-to-all send slabs, downloads leave from the receive slabs
        vx.sequence_parallel_self_attention_from_host(hq, hk, hv, "sp", out=hout, device=dev)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    ulysses_events.clear()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_value = total_flops / (e2e_ms / 1e3) / 1e12
    # the host-buffer path computes the same output bits as the device path
    same = torch.tensor([1.0 if torch.equal(hout, out.cpu()) else 0.0], device=dev)
    if world > 1:
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
    parity["e2e_output_equals_device"] = bool(same.item() == 1.0)
    del out
    elem = 2
    h2d = 3 * B * s_loc * H * D * elem
    d2h = B * s_loc * H * D * elem
    a2a = None
    if world > 1:
        # one q-sized exchange (padded heads) on its own, for the NVLink figure
        a2a = measure_all_to_all(B * s_loc * (-(-H // world) * world) * D, 10, dev,
                                 torch.bfloat16)
        if args.exchange == "peer":
            a2a = {"nccl_all_to_all": a2a,
                   "peer_pack": ulysses_peer.measure_exchange(q[0], 10)}
            a2a["ms"] = a2a["peer_pack"]["ms"]

    secondary = {}
    if world == 1 and not args.no_secondary:
        burst_peak = load_peaks()[0]
        for case in ("cfg1", "cfg2", "cfg4"):
            fn, fl, desc = kernel_case(case, dev)
            # idle a second first: right after the power-capped dense runs a
            # short launch sequence would still run at their reduced clock
            torch.cuda.synchronize()
            time.sleep(1.0)
            kms = time_launches(fn, 5 if case == "cfg2" else 50, 3)
            tf = fl / (kms / 1e3) / 1e12
            secondary[case] = {"desc": desc, "ms": round(kms, 4), "tflops": round(tf, 2),
                               "frac_of_burst_peak": round(tf / burst_peak, 4)}
            if case == "cfg4":
                # below the ridge point: the HBM view (q, k, v read, o written once)
                gbs = na_case_bytes(case) / (kms / 1e3) / 1e9
                hbm_peak = load_hbm_peak()[0]
                secondary[case].update(gbs_algorithmic=round(gbs, 1),
                                       frac_of_hbm=round(gbs / hbm_peak, 4))
        # the fused pre-attention step (RMSNorm + RoPE + send packing) of this
        # layer, per rank at N = 1 and N = 8: HBM-bound
        hbm, hbm_src = load_hbm_peak()
        for case in (f"prologue:{S_GLOBAL},{H},1", f"prologue:{S_GLOBAL // 8},{H},8"):
            fn, _, desc = kernel_case(case, dev)
            torch.cuda.synchronize()
            time.sleep(1.0)
            kms = time_launches(fn, 20, 3)
            gbs = kernel_case_bytes(case) / (kms / 1e3) / 1e9
            secondary[case] = {"desc": desc, "ms": round(kms, 4), "gbs": round(gbs, 1),
                               "frac_of_hbm": round(gbs / hbm, 4), "hbm_peak_source": hbm_src}
        assert _lib.device_status() == 0

    if not args.no_dit:
        # BASELINE config 5 at this N: one DiT step, B = 1 and the CFG B = 2 step
        torch.cuda.synchronize()
        time.sleep(1.0)
        for bsz in (1, 2):
            secondary[f"dit_cfg5_b{bsz}"] = dit_measure(world, dev, batch=bsz)
        assert _lib.device_status() == 0

    if secondary and world == 1 and not args.no_cpu_baseline:
        add_na_cpu_line(secondary, args.cpu_seconds / 2)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, threads, desc = cpu_sample(args.cpu_seconds)
        cpu = {"value": round(tf, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": desc, **host_cpu()}

    if world > 1:
        vx.unregister_axis("sp")
        if args.exchange == "peer":
            ulysses_peer.release_workspaces()   # collective: every rank, before returning
    if rank != 0:
        return
    traffic = None
    if TRAFFIC_BYTES_PER_HEAD_TOKEN is not None:
        traffic = round(TRAFFIC_BYTES_PER_HEAD_TOKEN * B * hg * S_GLOBAL)
    peak = sustained if sustained else burst
    line = {
        "metric": "attention TFLOP/s (Ulysses attn layer, Wan2.1-14B 720p)",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": B, "seq_len": S_GLOBAL, "heads": H,
                   "head_dim": D, "parallelism": f"ulysses-sp{world}" if world > 1 else "single",
                   "exchange": (args.exchange if world > 1 else None),
                   **({"exchange_note": exchange_note} if exchange_note else {}),
                   "l2": "inputs larger than L2 (774 MB per tensor), no flush"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                     "frac_of_burst": round(achieved / burst, 4) if burst else None,
                     "peak_source": f"{peak_src} bf16 dense (sustained; burst {burst})",
                     "kernel": "attn_fwd_kernel<DenseGeo>",
                     "kernel_ms_per_step": round(kern_avg, 3),
                     "kernel_flops_per_step": launch_flops,
                     "traffic": traffic},
        "e2e": {"value": round(e2e_value, 2), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 3),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": gpu_launches,
        "clocks": clocks,
        "device_status": status,
        "parity": parity,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if secondary:
        line["secondary"] = secondary
    if world > 1:
        a2a_bytes = 4 * (world - 1) / world * B * s_loc * hg * world * D * elem
        line["a2a"] = {"bytes_sent_per_gpu": a2a_bytes,
                       "single_exchange": a2a,
                       "layer_a2a_ms_if_serial": round(4 * a2a["ms"], 4),
                       "exchange": args.exchange,
                       "note": "4 all-to-alls (q, k, v, o) per layer, pipelined by head "
                               f"slices against the kernel; NVLink {NVLINK_NOMINAL_GBS:.0f} "
                               f"GB/s/dir nominal, {NVLINK_MEASURED_GBS:.0f} measured peer copy"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=["nccl", "peer"], default="peer",
                    help="N > 1: the Ulysses all-to-alls done by the slab kernels over "
                         "NVLink peer memory (vidax_b200.ulysses_peer; default, 3.5-5 %% "
                         "faster at N = 2 and 4), or over NCCL")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the extra cfg2 / cfg4 single-kernel measurements")
    ap.add_argument("--no-dit", action="store_true",
                    help="skip the cfg5 DiT step secondary measurement")
    ap.add_argument("--dit", action="store_true",
                    help="time one Wan2.1-1.3B DiT forward step (BASELINE config 5) instead")
    ap.add_argument("--kernel-only", default=None,
                    help="time one kernel case (cfg2, cfg4, attn:B,S,H, na3d:T,H,W,NH, "
                         "prologue:S,H,P) and exit")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.kernel_only:
        run_kernel_only(args)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.dit:
            run_dit(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
