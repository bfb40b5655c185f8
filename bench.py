"""Benchmark of the Palu decode-attention hot path on B200 (one JSON line on rank 0).

Default workload (the north star's target): one Llama-3.1-8B-shaped attention layer, M-LRD rank_k =
rank_v = 64, 32 query / 8 KV heads, head_dim 128, batch 32 per GPU, cached context 8192 (every row attends
all 8192 positions), bf16 latents ~ N(0,1), U ~ N(0, 1/64), wo ~ N(0, 1/4096), llama3 RoPE table.
Synthetic, seeded, created on the device (no dataset or checkpoint is involved).

A step is the attention layer's decode tail on this GPU's shard (palu_tt/attention.py:633-639, 718-733):
the fused decode op (decode kernel + split merge) over the local KV heads, the ``wo_fused`` projection of
the local heads' latent outputs (a bf16 library GEMM) and, with N > 1 GPUs, the one NCCL all-reduce of
the [B, 4096] layer output. Multi-GPU (torchrun, one rank per GPU): KV heads are sharded, 8/N per rank,
over a global batch of 32*N rows, so every rank reads the same latent bytes (weak scaling); the
all-reduce grows with N. ``value`` is global batch rows per second; the line also carries each part's
device time and share (decode op, wo GEMM, all-reduce), the decode op's roofline against
MEASURED_PEAKS.json, e2e (host buffers through the reference-facing call), clocks, and the CPU baseline.

``--config`` selects another BASELINE config (identity rank 128 with the plain GQA comparison arm;
G-LRD 2 groups x 4 KV heads at rank 256, split groups with replicated latents past 2 GPUs; the r_k 32 /
r_v 128 sweep cells ``sweep_b{B}_s{S}``). ``--workload decoder`` times the 32-layer decoder.
``--impl reference`` times the reference's CPU implementation of the same step (the oracle restatement
of palu_tt/fused.py:reference_decode plus the wo projection) on the host's cores.
"""
from __future__ import annotations

import argparse
import json
import re
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "tt-cadlab_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "decode-attn µs/layer & latent HBM GB/s vs 8 TB/s; tokens/s at 1/2/4/8 B200"
N_Q, N_KV, DIM, HD = 32, 8, 4096, 128
THETA = 500000.0
LLAMA3 = {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_max_position_embeddings": 8192}
L2_BYTES = 126 * 1024 * 1024


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_record(workload: str):
    """dram read+write bytes per launch of the decode kernel for this workload, from the committed ncu
    summaries (profiles/traffic.json: {workload: record})."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
    except ValueError:
        return None
    return d.get(workload) if isinstance(d, dict) else None


class ClockSampler:
    """nvidia-smi clocks + throttle reasons, sampled every 200 ms while the timed region runs."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}



@dataclass(frozen=True)
class Workload:
    """One BASELINE config as a bench workload: per-GPU batch rows, cached positions, latent widths, latent
    groups (8 = one per KV head, M-LRD; 2 = G-LRD with 4 KV heads per group and V rebuilt per head)."""
    name: str
    batch: int
    seq: int
    r_k: int
    r_v: int
    n_groups: int = N_KV
    identity: bool = False

    @property
    def grouped(self) -> bool:
        return self.n_groups < N_KV

    def model(self) -> str:
        kind = ("identity factorisation (U = I)" if self.identity else
                "G-LRD, V rebuilt per head" if self.grouped else "M-LRD, absorbed V")
        return f"Llama-3.1-8B attention layer ({kind})"


WORKLOADS = {w.name: w for w in (
    Workload("mlrd_r64_b32_s8192", 32, 8192, 64, 64),
    Workload("identity_r128_b32_s8192", 32, 8192, 128, 128, identity=True),
    Workload("glrd_gs4_r256_b16_s16384", 16, 16384, 256, 256, n_groups=2),
)}
DEFAULT = "mlrd_r64_b32_s8192"


def workload(name: str) -> Workload:
    if name in WORKLOADS:
        return WORKLOADS[name]
    m = re.fullmatch(r"sweep_b(\d+)_s(\d+)", name)
    if m:  # BASELINE config 5's mixed-path layer: r_k 32, r_v 128
        return Workload(f"sweep_rk32_rv128_b{m[1]}_s{m[2]}", int(m[1]), int(m[2]), 32, 128)
    raise SystemExit(f"unknown --config {name!r}: {sorted(WORKLOADS)} or sweep_b<B>_s<S>")


def make_layer(dev, W: Workload, B: int, shard, seed: int) -> dict:
    """This rank's shard of one layer on the device: latent caches of its groups [B, g, S, r], U of its KV
    heads, q of its query heads, every row at position S - 1, the packed RoPE table, and the nonzero
    columns of wo_fused for its query heads (M-LRD: r_v per head; G-LRD: wo's 128 per head)."""
    from palu_b200 import fused
    g = torch.Generator(device=dev).manual_seed(seed)
    bf = torch.bfloat16
    n_g, n_kv, n_q = len(shard.groups), len(shard.kv), len(shard.q)
    S = W.seq
    k = torch.randn(B, n_g, S, W.r_k, generator=g, device=dev, dtype=bf)
    v = torch.randn(B, n_g, S, W.r_v, generator=g, device=dev, dtype=bf)
    if W.identity:
        u = torch.eye(HD, device=dev, dtype=bf).expand(n_kv, HD, HD).contiguous()
    else:
        u = (torch.randn(n_kv, W.r_k, HD, generator=g, device=dev) / W.r_k ** 0.5).to(bf)
    u_v = (torch.randn(n_kv, W.r_v, HD, generator=g, device=dev) / W.r_v ** 0.5).to(bf) if W.grouped else None
    q = torch.randn(B, n_q, HD, generator=g, device=dev, dtype=bf)
    pos = torch.full((B,), S - 1, dtype=torch.int32, device=dev)
    cos, sin = fused.cos_sin_tables(HD, S, THETA, LLAMA3)
    cs_tab = fused.cs_table(cos, sin, S).to(dev, bf)[None, None]        # the reference's [1, 1, S, 256]
    w_rot = fused.w_rot_from_u_k(u.float()).to(bf)[None]                # the reference's [1, n_kv, r_k, 256]
    width = HD if W.grouped else W.r_v
    wo = (torch.randn(DIM, n_q * width, generator=g, device=dev) / (N_Q * HD) ** 0.5).to(bf)
    return dict(k=k, v=v, u=u, u_v=u_v, q=q, pos=pos, cs=fused.pack_cs_table(cs_tab), cs_tab=cs_tab, w_rot=w_rot,
                wo=wo, width=width, cos=cos[:S], sin=sin[:S])


class CpuStep:
    """One step of a workload on the host: the reference's CPU implementation of the op
    (palu_tt/fused.py:82-107, restated as ``oracle.reference_decode``) over ALL ``rows`` batch rows, in
    chunks of ``chunk`` rows (rows are independent; chunking only bounds the host memory of the
    reference's repeat_interleave expansion), then the layer's wo_fused projection of the head-slotted
    output (attention.py:718-727). Seeded inputs with the workload's shapes and distributions."""

    def __init__(self, W: Workload, rows: int, chunk: int = 1):
        import oracle
        self.oracle, self.W = oracle, W
        self.rows, self.chunk = rows, chunk
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        g = torch.Generator().manual_seed(5)
        bf = lambda t: t.to(torch.bfloat16).float()
        S = W.seq
        self.q = bf(torch.randn(1, rows, N_Q, HD, generator=g))
        self.k = bf(torch.randn(rows, W.n_groups, S, W.r_k, generator=g))
        self.v = bf(torch.randn(rows, W.n_groups, S, W.r_v, generator=g))
        self.u = torch.eye(HD).expand(N_KV, HD, HD) if W.identity else bf(torch.randn(N_KV, W.r_k, HD, generator=g) / W.r_k ** 0.5)
        self.u_v = bf(torch.randn(N_KV, W.r_v, HD, generator=g) / W.r_v ** 0.5) if W.grouped else None
        self.wo = torch.randn(DIM, N_Q * HD, generator=g) / (N_Q * HD) ** 0.5
        cos, sin = oracle.cos_sin_tables(HD, S, THETA, LLAMA3)
        self.cos, self.sin = bf(cos[:S]), bf(sin[:S])
        self.pos = torch.full((rows,), S - 1)
        self.gs = N_KV // W.n_groups

    def __call__(self):
        outs = []
        for r0 in range(0, self.rows, self.chunk):
            r1 = min(self.rows, r0 + self.chunk)
            k = self.oracle.expand_groups(self.k[r0:r1], self.gs)
            v = self.oracle.expand_groups(self.v[r0:r1], self.gs)
            outs.append(self.oracle.reference_decode(self.q[:, r0:r1], k, self.u, v, self.pos[r0:r1], self.cos,
                                                     self.sin, HD ** -0.5, u_v=self.u_v)[0])
        o = torch.cat(outs)                                   # [rows, n_q, width]
        slots = o.new_zeros(self.rows, N_Q, HD)
        slots[..., :o.shape[-1]] = o
        return slots.reshape(self.rows, N_Q * HD) @ self.wo.t()

    def sample(self, steps: int) -> str:
        return (f"whole steps of {self.W.name}: all {self.rows} batch rows x {N_KV} KV heads, S={self.W.seq}, "
                f"r_k={self.W.r_k}, r_v={self.W.r_v}, in chunks of {self.chunk} rows, + the wo projection; "
                f"{steps} timed steps; palu_tt/fused.py:reference_decode restated in fp32 torch on "
                f"{self.threads} threads")


def cpu_oracle_rate(W: Workload, budget_s: float):
    """The CPU baseline of the b200 arm: whole steps of the workload (all batch rows of one GPU) timed until
    the budget is spent (at least 2 steps); returns (rows/s, threads, description)."""
    step = CpuStep(W, W.batch)
    step()  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return step.rows / med, step.threads, step.sample(len(times)) + f", median of {len(times)}"


def run_reference(args, ws, rank):
    """--impl reference: the reference's CPU implementation of the step, rank 0 only; each step is one whole
    step of one GPU's share of the workload (all its batch rows), timed on the host's cores."""
    if rank != 0:
        return
    W = workload(args.config)
    step = CpuStep(W, args.batch or W.batch)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    ms = statistics.mean(times) * 1e3
    value = step.rows / (ms * 1e-3)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "ms_per_step_median": statistics.median(times) * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, host)",
            "config": workload_config(W, 1, step.rows),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": step.threads, "kind": "port",
                             "sample": step.sample(args.steps)},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(W: Workload, ws: int, batch: int, paged: int = 0, shard=None, latent: str = "bf16",
                    rope: str = "") -> dict:
    name = W.name if batch == W.batch else re.sub(r"_b\d+_", f"_b{batch}_", W.name)
    extra = {}
    if rope:
        extra["rope"] = ("chunk-relative (the reference op's Phase 2: keys by table rows 0..127, the query "
                         "rotated per 128-position chunk)" if rope == "relative"
                         else "absolute (Phase 1: every key rotated by its own table row)")
    elem = 2
    if latent == "f8":
        name += "_f8"
        elem = 1
        extra["cache"] = ("fp8 latent caches: e4m3 codes + one int8 power-of-two exponent per (position, latent "
                          "head), quantized from the bf16 latents (palu_quantize_latents_f8)")
    elif latent == "f4":
        name += "_f4"
        elem = 0.5
        extra["cache"] = ("fp4 latent caches: e2m1 codes, two per byte, + one int8 power-of-two exponent per 16 "
                          "values, quantized from the bf16 latents (palu_quantize_latents_f4)")
    if paged:
        name += f"_paged{paged}"
        extra["cache"] = (f"paged: blocks of {paged} positions, each row's blocks a seeded random permutation of "
                          "the physical blocks")
    lat_bytes = int(batch * ws * (len(shard.groups) if shard else W.n_groups) * W.seq * (W.r_k + W.r_v) * elem)
    return {"workload": name, **extra, "model": W.model(), "global_batch": batch * ws, "seq_len": W.seq,
            "rank_k": W.r_k, "rank_v": W.r_v, "n_q_heads": N_Q, "n_kv_heads": N_KV, "latent_groups": W.n_groups,
            "kv_heads_per_gpu": N_KV // ws, "latent_replicas": shard.latent_replicas if shard else 1,
            "parallelism": f"kv-head shard x{ws}",
            "step": "decode op + wo projection" + (" + NCCL all-reduce of [B, 4096]" if ws > 1 else ""),
            "l2": f"no flush: each step reads {lat_bytes / 1e6:.0f} MB of latents per GPU (L2 is 126 MB)"}


def run_layer(args, ws, rank, local):
    """The default: the attention layer's decode tail on this GPU's KV-head shard (see the module doc)."""
    import torch.distributed as dist
    from palu_b200 import _lib, fused
    from palu_b200.shard import KVShard
    W = workload(args.config)
    _lib.set_kernel({"auto": _lib.PALU_KERNEL_AUTO, "tc": _lib.PALU_KERNEL_TC, "mma": _lib.PALU_KERNEL_MMA}[args.kernel])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    shard = KVShard(rank, ws, N_KV, N_Q, W.n_groups)
    b_gpu = args.batch or W.batch
    B = b_gpu * ws                       # weak scaling: every rank attends all global rows for its heads
    n_kv, n_q, n_g = len(shard.kv), len(shard.q), len(shard.groups)
    L = make_layer(dev, W, B, shard, seed=1234 + rank)
    S = W.seq
    f8 = args.latent in ("f8", "f4")
    if f8:
        if args.paged:
            raise SystemExit("--latent f8 / f4 run on contiguous caches (no --paged)")
        quant = fused.quantize_latents_f4 if args.latent == "f4" else fused.quantize_latents_f8
        L["k"], L["v"] = quant(L["k"]), quant(L["v"])
        torch.cuda.synchronize()
    append = fused.append_latents_f8 if f8 else (lambda nk, nv, p_, kc, vc, page_table=None:
                                                 fused.append_latents(nk, nv, p_, kc, vc, page_table=page_table))
    pt = None
    if args.paged:
        # the same latents, each row's blocks scattered over the physical blocks by a seeded permutation
        bs = args.paged
        per_row = S // bs
        g = torch.Generator(device=dev).manual_seed(99 + rank)
        pt = torch.randperm(B * per_row, generator=g, device=dev).view(B, per_row).to(torch.int32)
        for name in ("k", "v"):
            c = L[name]
            r = c.shape[-1]
            paged = torch.empty(B * per_row, n_g, bs, r, dtype=c.dtype, device=dev)
            paged[pt.long().view(-1)] = c.view(B, n_g, per_row, bs, r).transpose(1, 2).reshape(-1, n_g, bs, r)
            L[name] = paged
            del c, paged
    width = L["width"]
    out = torch.empty(B, n_q, width, dtype=torch.bfloat16, device=dev)
    y = torch.empty(B, DIM, dtype=torch.bfloat16, device=dev)
    d = _lib.dims(B, n_q, n_kv, n_g, W.r_k, W.r_v, S)
    ws_buf = _lib.new_workspace(d, dev)
    stream = torch.cuda.current_stream(dev)

    rel = args.rope == "relative"
    p2_kw = ({"rot_step": fused.rot_step_table(L["cos"], L["sin"], 128).to(dev), "trans_mat": fused.trans_mat_tile()}
             if rel else {})

    def op():
        fused.decode(L["q"], L["k"], L["v"], L["u"], L["cs"], L["pos"], u_v=L["u_v"], out=out, workspace=ws_buf,
                     page_table=pt, chunk_relative=rel)

    def step(ev=None):
        if ev:
            ev[0].record(stream)
        op()
        if ev:
            ev[1].record(stream)
        # x @ wo^T in the layout of a linear layer's weight, as PaluAttention._out computes it
        torch.mm(out.view(B, n_q * width), L["wo"].t(), out=y)
        if ev:
            ev[2].record(stream)
        if ws > 1:
            dist.all_reduce(y)
        if ev:
            ev[3].record(stream)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):
        step()
    barrier()

    # ---- device-resident timing -------------------------------------------------------------------
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        # The timed region can be a few ms, shorter than nvidia-smi's 200 ms sampling period, so the
        # sampler also covers a soak of the same step (same load, untimed) right before it. Every rank runs
        # the same number of soak steps (each step holds a collective at N > 1): sized from 5 steps' wall
        # time, the largest count over ranks.
        n_soak = 0
        if args.clock_soak > 0:
            torch.cuda.synchronize()
            t_s = time.perf_counter()
            for _ in range(5):
                step()
            torch.cuda.synchronize()
            per_step = max((time.perf_counter() - t_s) / 5, 1e-6)
            n = torch.tensor([float(min(100000, int(args.clock_soak / per_step) + 1))], device=dev)
            if ws > 1:
                dist.all_reduce(n, op=dist.ReduceOp.MAX)
            n_soak = int(n.item())
        for i in range(n_soak):
            step()
            if i % 20 == 19:
                torch.cuda.synchronize()
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            step(evs[i])
        t1.record(stream)
        barrier()
    total_ms = t0.elapsed_time(t1)
    parts = [statistics.mean(e[j].elapsed_time(e[j + 1]) for e in evs) for j in range(3)]  # op, GEMM, all-reduce
    status = _lib.read_status(ws_buf)
    red = torch.tensor([total_ms, *parts, float(status)], device=dev)
    if ws > 1:
        dist.all_reduce(red, op=dist.ReduceOp.MAX)
    total_ms, op_ms, gemm_ms, ar_ms, status = red.tolist()
    ms = total_ms / args.steps
    value = B / (ms * 1e-3)   # global batch rows per second

    # ---- plain GQA comparison arm (identity config): the stock flash-decode over the rotated full K ----
    plain_ms = None
    if W.identity and ws == 1 and not args.paged and not f8:
        kf = L["k"].float()
        kr = torch.stack([-kf[..., 1::2], kf[..., 0::2]], dim=-1).flatten(-2)
        k_rot = (kf * L["cos"].to(dev) + kr * L["sin"].to(dev)).to(torch.bfloat16)
        del kf, kr
        q4 = L["q"][None]
        for _ in range(3):
            fused.plain_gqa_decode(q4, k_rot, L["v"], L["pos"])
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fused.plain_gqa_decode(q4, k_rot, L["v"], L["pos"])
        e1.record(stream)
        torch.cuda.synchronize()
        plain_ms = e0.elapsed_time(e1) / args.steps
        del k_rot

    # ---- e2e through the reference-facing call with host buffers ------------------------------------
    # Each step: the step's inputs (q, the new token's K and V latents, positions) from one pinned host
    # buffer in one copy; the two appends and palu_sdpa_decode called from Python with the reference's 4-D
    # tensors (argument checks, table-pack cache lookup and the C-ABI call every step, no graph); the wo
    # projection and the all-reduce; the [B, 4096] layer output copied back; the host waits for it before the
    # next step, as a decode loop whose next token depends on this output does.
    sizes = [B * n_q * HD * 2, B * n_g * W.r_k * 2, B * n_g * W.r_v * 2, B * 4]
    offs = [0]
    for n_b in sizes:
        offs.append(offs[-1] + (n_b + 255) // 256 * 256)
    in_h = torch.empty(offs[-1], dtype=torch.uint8).pin_memory()
    in_d = torch.empty(offs[-1], dtype=torch.uint8, device=dev)
    views = lambda buf: (buf[offs[0]:offs[0] + sizes[0]].view(torch.bfloat16).view(B, n_q, HD),
                         buf[offs[1]:offs[1] + sizes[1]].view(torch.bfloat16).view(B, n_g, W.r_k),
                         buf[offs[2]:offs[2] + sizes[2]].view(torch.bfloat16).view(B, n_g, W.r_v),
                         buf[offs[3]:offs[3] + sizes[3]].view(torch.int32))
    q_h, nk_h, nv_h, pos_h = views(in_h)
    q_h.copy_(torch.randn(B, n_q, HD).to(torch.bfloat16))
    nk_h.copy_(torch.randn(B, n_g, W.r_k).to(torch.bfloat16))
    nv_h.copy_(torch.randn(B, n_g, W.r_v).to(torch.bfloat16))
    pos_h.fill_(S - 1)
    q_d, nk_d, nv_d, pos_d = views(in_d)
    y_h = torch.empty(B, DIM, dtype=torch.bfloat16).pin_memory()
    pt_kw = {} if pt is None else {"page_table_tensor": pt}
    u_v4 = None if L["u_v"] is None else L["u_v"][None]

    def plugin_step():
        in_d.copy_(in_h, non_blocking=True)
        append(nk_d, nv_d, pos_d, L["k"], L["v"], **({"page_table": pt} if pt is not None else {}))
        o = fused.palu_sdpa_decode(q_d[None], L["k"], L["w_rot"], L["cs_tab"], L["v"], width, pos_d, u_v=u_v4,
                                   scale=HD ** -0.5, **pt_kw, **p2_kw)
        torch.mm(o[0].view(B, n_q * width), L["wo"].t(), out=y)
        if ws > 1:
            dist.all_reduce(y)
        y_h.copy_(y, non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        plugin_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        plugin_step()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    graph_ms = None
    if ws == 1:
        # the same step without the host wait, captured once as a CUDA graph and replayed back to back
        def graph_body():
            in_d.copy_(in_h, non_blocking=True)
            append(nk_d, nv_d, pos_d, L["k"], L["v"], **({"page_table": pt} if pt is not None else {}))
            fused.decode(q_d, L["k"], L["v"], L["u"], L["cs"], pos_d, u_v=L["u_v"], out=out, workspace=ws_buf,
                         page_table=pt, chunk_relative=rel)
            torch.mm(out.view(B, n_q * width), L["wo"].t(), out=y)
            y_h.copy_(y, non_blocking=True)
        graph_body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            graph_body()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        graph_ms = e0.elapsed_time(e1) / args.steps
        del graph
    red = torch.tensor([e2e_ms], device=dev)
    if ws > 1:
        dist.all_reduce(red, op=dist.ReduceOp.MAX)
    e2e_ms = float(red.item())
    h2d = in_h.numel()
    d2h = y_h.numel() * y_h.element_size()

    # ---- roofline of the decode op on this rank ------------------------------------------------------
    # fp8: one byte per code and one exponent byte per cached row of each cache; fp4: half a byte per code
    # and one exponent byte per 16 codes
    if args.latent == "f4":
        latent_bytes = B * n_g * S * ((W.r_k + W.r_v) // 2 + (W.r_k + W.r_v) // 16)
    else:
        latent_bytes = B * n_g * S * ((W.r_k + W.r_v + 2) if f8 else (W.r_k + W.r_v) * 2)
    u_bytes = n_kv * W.r_k * HD * 2 + (n_kv * W.r_v * HD * 2 if W.grouped else 0)
    alg_bytes = latent_bytes + u_bytes
    achieved = alg_bytes / (op_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    tr = traffic_record(W.name + ("_" + args.latent if f8 else ""))
    kern = _lib.kernel_for(d)
    kernel_name = ("palu_decode_tc_kernel + palu_combine_tc_kernel" if kern == _lib.PALU_KERNEL_TC
                   else "palu_decode_mma_kernel + palu_combine_kernel")

    if rank == 0:
        cpu = None
        if ws == 1 and args.cpu_budget > 0:
            rate, cores, sample = cpu_oracle_rate(W, args.cpu_budget)
            cpu = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
        clocks = clk.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, on device)",
            "config": workload_config(W, ws, b_gpu, args.paged, shard, args.latent, args.rope),
            "latent_dtype": {"f8": "e4m3 + per-row exponent", "f4": "e2m1 + per-16 exponent"}.get(args.latent, "bf16"),
            "us_per_layer": ms * 1e3,
            "parts_us": {"decode_op": op_ms * 1e3, "wo_gemm": gemm_ms * 1e3,
                         "all_reduce": ar_ms * 1e3 if ws > 1 else None},  # one GPU: no collective in the step
            "all_reduce_share": ar_ms / ms if ms > 0 and ws > 1 else None,
            "decode_op_us": op_ms * 1e3, "latent_GBps": achieved,
            "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                    "how": "headline: per step, pinned H2D copy, append + palu_sdpa_decode called from Python "
                           "(reference surface) + wo GEMM" + (" + all-reduce" if ws > 1 else "") +
                           ", D2H of the [B, 4096] output, host waits for it",
                    "graph_replay": None if graph_ms is None else {
                        "value": B / (graph_ms * 1e-3), "unit": "tokens/s", "ms_per_step": graph_ms,
                        "how": "the same step captured once as a CUDA graph and replayed back to back (no host "
                               "wait per step)"}},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": (tr or {}).get("bytes_per_launch"),
                         "kernel": kernel_name + " (one decode op; CUDA events around each op in the timed region)",
                         "algorithmic_bytes": alg_bytes},
            "cpu_baseline": cpu,
            "gpu_launches": 2 * args.steps,
            "clocks": clocks,
            "us_x_mhz": (op_ms * 1e3 * clocks["sm_mhz"]) if clocks.get("sm_mhz") else None,
            "status": int(status),
        }
        if plain_ms is not None:
            line["plain_gqa"] = {"us": plain_ms * 1e3, "kernel": "palu_plain_gqa_decode (mma.sync) over bf16 K_rot",
                                 "identity_over_plain": op_ms / plain_ms}
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_decoder(args, ws, rank, local):
    """``--workload decoder``: BASELINE config 4, the 32-layer Llama-3.1-8B-shaped Palu decoder
    (palu_b200/model.py; the reference's generation loop, palu_tt/generate.py:28-62) with random bf16 weights
    (seeded), M-LRD ranks drawn per layer AND per KV head from {32, 48, 64, 96, 128} (seed 7; each layer's
    caches padded to its largest head rank rounded to 32, as the reference's loader pads), batch 64, a
    4096-token prompt of random token ids prefilled through every layer (untimed, a few rows at a time),
    then ``--gen`` (128) greedy decode steps, each one replayed CUDA graph fed with the previous step's
    argmax. ``value`` is generated tokens per second over the timed decode steps. Tensor parallel over N
    GPUs: KV heads and the MLP hidden dimension sharded, two all-reduces per layer (strong scaling: the
    same batch at every N). With ``--paged BLOCK`` every layer's caches are paged (each row's blocks a
    seeded random permutation of the physical blocks; the page table is a buffer the graph reads)."""
    from palu_b200.attention import PagedAttentionConfig
    from palu_b200.model import DecoderConfig, PaluDecoder, mixed_head_ranks, padded_rank
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    cfg = DecoderConfig()
    B, ctx, gen = args.batch, args.context, args.gen
    ranks = mixed_head_ranks(cfg.n_layers, cfg.n_kv_heads, seed=7)
    max_seq = ctx + gen + 8
    pc, pt = None, None
    if args.paged:
        per_row = -(-max_seq // args.paged)
        pc = PagedAttentionConfig(block_size=args.paged, max_num_blocks=B * per_row)
        gp = torch.Generator(device=dev).manual_seed(99)
        pt = torch.randperm(B * per_row, generator=gp, device=dev).view(B, per_row).to(torch.int32)
    model = PaluDecoder(cfg, ranks, max_batch=B, max_seq=max_seq, seed=11, device=str(dev), rank=rank, world=ws,
                        paged_attention_config=pc, latent_dtype=args.latent,
                        cs_recurrence=args.rope == "relative")
    # the prompt: random token ids (every rank draws the same), prefilled a few rows at a time
    prompt = torch.randint(0, cfg.vocab, (B, ctx), generator=torch.Generator().manual_seed(8)).to(dev)
    t_pre = time.perf_counter()
    first = []
    rows = max(1, args.prefill_rows)
    for r0 in range(0, B, rows):
        first.append(model.prefill_logits(prompt[r0:r0 + rows], page_table=pt, row0=r0).argmax(-1))
    tok = torch.cat(first)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pre
    graph = model.capture_decode(B, page_table=pt)
    graph.tokens.copy_(tok)
    generated = []

    def step(i):
        graph.pos.fill_(ctx + i)
        nxt = graph.replay()
        graph.tokens.copy_(nxt)
        return nxt

    warm = max(3, args.warmup)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # the first steps are the warm-up (untimed), the rest of the gen tokens are timed
        for i in range(warm):
            generated.append(step(i).clone())
        torch.cuda.synchronize()
        e0.record()
        for i in range(warm, gen):
            generated.append(step(i).clone())
        e1.record()
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
    timed = gen - warm
    ms = e0.elapsed_time(e1) / max(1, timed)
    if ws > 1:
        tt = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        ms = float(tt.item())
    del graph
    toks = torch.stack(generated, 1).cpu()        # [B, gen]
    widths = [(padded_rank(k), padded_rank(v)) for k, v in ranks]
    if rank == 0:
        print(json.dumps({
            "metric": "decode tokens/s, 32-layer Llama-3.1-8B-shaped Palu decoder (greedy, CUDA graph per step)",
            "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": timed,
            "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random weights, random prompt token ids, greedy generation)",
            "config": {"workload": f"decoder_32l_b{B}_ctx{ctx}_gen{gen}" + (f"_paged{args.paged}" if args.paged else "")
                       + ("" if args.latent == "bf16" else f"_{args.latent}"),
                       "layers": cfg.n_layers, "batch": B, "prompt": ctx, "generated": gen,
                       "ranks": "per layer and per KV head from {32,48,64,96,128}, seed 7",
                       "layer_widths_rk_rv": widths,
                       "latent_bytes_per_token_step": sum(8 * (rk + rv) * 2 for rk, rv in widths),
                       "parallelism": f"tp{ws} (KV heads + MLP hidden)",
                       "rope": "chunk-relative (Phase 2)" if args.rope == "relative" else "absolute (Phase 1)",
                       "cache": (f"paged, blocks of {args.paged}" if args.paged else "contiguous")
                       + ("" if args.latent == "bf16" else f", {args.latent} latents")},
            "prefill_s": prefill_s, "generated_tokens_sample": toks[:2, :8].tolist(),
            "gpu_launches": None, "clocks": clk.summary()}), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default=DEFAULT,
                    help=f"workload: {', '.join(WORKLOADS)} or sweep_b<B>_s<S> (r_k 32 / r_v 128)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--clock-soak", type=float, default=2.0, help="seconds of untimed steps sampled for clocks")
    ap.add_argument("--batch", type=int, default=0, help="batch rows per GPU (0: the config's)")
    ap.add_argument("--workload", default="layer", choices=["layer", "decoder"],
                    help="layer: the attention layer's decode tail (the default bench line); decoder: the "
                         "32-layer Palu decoder's greedy decode steps")
    ap.add_argument("--context", type=int, default=4096, help="decoder workload: prompt tokens")
    ap.add_argument("--gen", type=int, default=128, help="decoder workload: generated tokens (warm-up steps included)")
    ap.add_argument("--prefill-rows", type=int, default=8, help="decoder workload: batch rows per prefill call")
    ap.add_argument("--paged", type=int, default=0, metavar="BLOCK",
                    help="paged caches with blocks of BLOCK positions (0: contiguous caches)")
    ap.add_argument("--latent", default="bf16", choices=["bf16", "f8", "f4"],
                    help="latent cache format of the layer workload (f8: e4m3 codes + per-row exponent; "
                         "f4: e2m1 codes + per-16 exponent)")
    ap.add_argument("--rope", default="relative", choices=["relative", "absolute"],
                    help="the op's RoPE form: chunk-relative (the reference's Phase 2, rot_step passed: its "
                         "published kernel) or absolute (Phase 1: every key's own table row)")
    ap.add_argument("--kernel", default="auto", choices=["auto", "tc", "mma"],
                    help="decode kernel family: tcgen05 (tc), legacy mma.sync (mma) or the library's choice")
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, ws, rank)
    if args.workload == "decoder":
        if not args.batch:
            args.batch = 64
        return run_decoder(args, ws, rank, local)
    return run_layer(args, ws, rank, local)


if __name__ == "__main__":
    main()
