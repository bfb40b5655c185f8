"""Benchmark of the Palu decode-attention hot path on B200 (one JSON line on rank 0).

Workload (the north star's target): one Llama-3.1-8B-shaped attention layer, M-LRD rank_k = rank_v = 64,
32 query / 8 KV heads, head_dim 128, batch 32, cached context 8192 (every row attends all 8192
positions), bf16 latents ~ N(0,1), U ~ N(0, 1/64), llama3 RoPE table. Synthetic, seeded, created on
the device. A step is one decode-attention call (fused kernel + split merge) over the whole cache.

Multi-GPU (torchrun, one rank per GPU): KV heads are sharded, 8/N per rank, over a global batch of
32*N rows, so every rank holds the same latent bytes (weak scaling; no collective inside the op).

Also reported: e2e (the same op through the C ABI with host buffers: the step's query and new latents
copied in from pinned memory, the latents appended, the output copied back, all inside the timed
region), the roofline of the decode kernel against MEASURED_PEAKS.json, and the CPU oracle timed on a
bounded sample on this host. ``--impl reference`` times the reference's CPU implementation of the path
(the oracle restatement of palu_tt/fused.py:reference_decode) on the same workload.
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

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "tt-cadlab_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

METRIC = "decode-attn µs/layer & latent HBM GB/s vs 8 TB/s; tokens/s at 1/2/4/8 B200"
B_PER_GPU, N_Q, N_KV, S, R = 32, 32, 8, 8192, 64
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


def traffic_record():
    """dram read+write bytes per launch of the decode kernel, from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except ValueError:
        return None


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


def make_layer(dev, B, n_q, n_kv, seed):
    from palu_b200 import fused
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(B, n_kv, S, R, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn(B, n_kv, S, R, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    u = (torch.randn(n_kv, R, 128, generator=g, device=dev) / R ** 0.5).to(torch.bfloat16)
    q = torch.randn(B, n_q, 128, generator=g, device=dev).to(torch.bfloat16)
    pos = torch.full((B,), S - 1, dtype=torch.int32, device=dev)
    cos, sin = fused.cos_sin_tables(128, S, THETA, LLAMA3)
    cs = fused.pack_cs_table(fused.cs_table(cos, sin, S).to(dev, torch.bfloat16))
    return dict(k=k, v=v, u=u, q=q, pos=pos, cs=cs)


def cpu_oracle_rate(budget_s: float, rows_per_sample: int = 1):
    """Time the oracle (reference_decode restated) on whole batch rows of the workload until the
    budget is spent; returns (rows/s, threads, description)."""
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(5)
    bf = lambda t: t.to(torch.bfloat16).float()
    q = bf(torch.randn(1, rows_per_sample, N_Q, 128, generator=g))
    k = bf(torch.randn(rows_per_sample, N_KV, S, R, generator=g))
    v = bf(torch.randn(rows_per_sample, N_KV, S, R, generator=g))
    u = bf(torch.randn(N_KV, R, 128, generator=g) / R ** 0.5)
    cos, sin = oracle.cos_sin_tables(128, S, THETA, LLAMA3)
    cos, sin = bf(cos[:S]), bf(sin[:S])
    pos = torch.full((rows_per_sample,), S - 1)
    oracle.reference_decode(q, k, u, v, pos, cos, sin, 128 ** -0.5)   # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        oracle.reference_decode(q, k, u, v, pos, cos, sin, 128 ** -0.5)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return rows_per_sample / med, threads, (f"{rows_per_sample} of {B_PER_GPU} batch rows (all {N_KV} KV heads, "
                                            f"S={S}, r=64) per sample, median of {len(times)} samples, "
                                            f"reference_decode (fp32 torch) on {threads} threads")


def run_reference(args, ws, rank):
    """--impl reference: the reference's CPU implementation on the same workload, rank 0 only."""
    if rank != 0:
        return
    rows = 1
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(5)
    bf = lambda t: t.to(torch.bfloat16).float()
    q = bf(torch.randn(1, rows, N_Q, 128, generator=g))
    k = bf(torch.randn(rows, N_KV, S, R, generator=g))
    v = bf(torch.randn(rows, N_KV, S, R, generator=g))
    u = bf(torch.randn(N_KV, R, 128, generator=g) / R ** 0.5)
    cos, sin = oracle.cos_sin_tables(128, S, THETA, LLAMA3)
    cos, sin = bf(cos[:S]), bf(sin[:S])
    pos = torch.full((rows,), S - 1)
    for _ in range(args.warmup):
        oracle.reference_decode(q, k, u, v, pos, cos, sin, 128 ** -0.5)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.reference_decode(q, k, u, v, pos, cos, sin, 128 ** -0.5)
        times.append(time.perf_counter() - t0)
    t_row = statistics.median(times) / rows
    # whole-job rate on the bench's workload: global batch rows / time, extrapolated per row
    rows_total = B_PER_GPU * ws
    value = rows_total / (t_row * rows_total)
    cores = torch.get_num_threads()
    sample = (f"{rows} of {B_PER_GPU} batch rows per step (all {N_KV} KV heads, S={S}, r=64); "
              f"palu_tt/fused.py:reference_decode restated in fp32 torch on {cores} threads")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_row * B_PER_GPU * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": workload_config(ws),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(ws, batch=B_PER_GPU, paged=0):
    name = "mlrd_r64_b32_s8192" if batch == B_PER_GPU else f"mlrd_r64_b{batch}_s8192"
    extra = {}
    if paged:
        name += f"_paged{paged}"
        extra = {"cache": f"paged: blocks of {paged} positions, each row's blocks a seeded random permutation "
                          f"of the physical blocks"}
    return {"workload": name, **extra, "model": "Llama-3.1-8B attention layer (M-LRD, absorbed V)",
            "global_batch": batch * ws, "seq_len": S, "rank_k": R, "rank_v": R, "n_q_heads": N_Q,
            "n_kv_heads": N_KV, "kv_heads_per_gpu": N_KV // ws, "parallelism": f"kv-head shard x{ws}",
            "l2": f"no flush: each step reads {batch * ws * (N_KV // ws) * S * 2 * R * 2 / 1e6:.0f} MB of latents per GPU "
                  f"(L2 is 126 MB)"}


def run_decoder(args, ws, rank, local):
    """``--workload decoder``: greedy decode steps of the 32-layer Llama-3.1-8B-shaped Palu decoder
    (palu_b200/model.py; the reference's decode loop, palu_tt/generate.py:40-62) at batch 64 per GPU
    group with 4096 cached positions, per-layer ranks drawn from {32, 48, 64, 96, 128} (seed 7). Weights
    random (seeded); the latent caches hold seeded N(0, 1) values for positions 0..4095 (a step's cost does
    not depend on them); the step (all layers, LM head, argmax) is one CUDA graph, replayed with the step's
    tokens and positions. Tensor parallel over N GPUs: KV heads and the MLP hidden dimension sharded, two
    all-reduces per layer. With ``--paged BLOCK`` every layer's caches are paged (each row's blocks a seeded
    random permutation of the physical blocks; the page table is a buffer the graph reads). Prints one JSON
    line with decode tokens/s for the whole job."""
    from palu_b200.attention import PagedAttentionConfig
    from palu_b200.model import DecoderConfig, PaluDecoder, mixed_ranks
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    cfg = DecoderConfig()
    B, ctx = args.batch, 4096
    ranks = mixed_ranks(cfg.n_layers, seed=7)
    max_seq = ctx + args.steps + args.warmup + 8
    pc, pt = None, None
    if args.paged:
        per_row = -(-max_seq // args.paged)
        pc = PagedAttentionConfig(block_size=args.paged, max_num_blocks=B * per_row)
        gp = torch.Generator(device=dev).manual_seed(99)
        pt = torch.randperm(B * per_row, generator=gp, device=dev).view(B, per_row).to(torch.int32)
    model = PaluDecoder(cfg, ranks, max_batch=B, max_seq=max_seq, seed=11, device=str(dev), rank=rank, world=ws,
                        paged_attention_config=pc)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    for L in model.layers:
        a = L["attn"]
        if pc is None:
            a.k_cache[:, :, :ctx].normal_(generator=g)
            a.v_cache[:, :, :ctx].normal_(generator=g)
        else:
            a.k_cache.normal_(generator=g)  # every block holds seeded latents (positions past ctx are rewritten)
            a.v_cache.normal_(generator=g)
    graph = model.capture_decode(B, page_table=pt)
    tok = torch.randint(0, cfg.vocab, (B,), generator=g, device=dev)
    graph.tokens.copy_(tok)

    def step(i):
        graph.pos.fill_(ctx + i)
        nxt = graph.replay()
        graph.tokens.copy_(nxt)

    for i in range(max(3, args.warmup)):
        step(i)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record()
        for i in range(args.steps):
            step(args.warmup + 3 + i)
        e1.record()
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    if ws > 1:
        tt = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        ms = float(tt.item())
    del graph
    if rank == 0:
        print(json.dumps({
            "metric": "decode tokens/s, 32-layer Llama-3.1-8B-shaped Palu decoder (greedy, CUDA graph per step)",
            "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random weights, seeded latent caches)",
            "config": {"workload": "decoder_32l_b64_ctx4096" + (f"_paged{args.paged}" if args.paged else ""),
                       "layers": cfg.n_layers, "batch": B, "context": ctx, "ranks_seed": 7,
                       "parallelism": f"tp{ws} (KV heads + MLP hidden)",
                       "cache": f"paged, blocks of {args.paged}" if args.paged else "contiguous"},
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
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--clock-soak", type=float, default=2.0, help="seconds of untimed steps sampled for clocks")
    ap.add_argument("--batch", type=int, default=B_PER_GPU, help="batch rows per GPU (profiling cases)")
    ap.add_argument("--workload", default="decode_op", choices=["decode_op", "decoder"],
                    help="decode_op: the fused decode-attention op (the default bench line); decoder: the "
                         "32-layer Palu decoder's greedy decode steps")
    ap.add_argument("--paged", type=int, default=0, metavar="BLOCK",
                    help="decode_op over paged caches with blocks of BLOCK positions (0: contiguous caches)")
    ap.add_argument("--kernel", default="auto", choices=["auto", "tc", "mma"],
                    help="decode kernel family: tcgen05 (tc), legacy mma.sync (mma) or the library's choice")
    args = ap.parse_args()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, ws, rank)
    if args.workload == "decoder":
        if args.batch == B_PER_GPU:
            args.batch = 64
        return run_decoder(args, ws, rank, local)

    from palu_b200 import _lib, fused
    _lib.set_kernel({"auto": _lib.PALU_KERNEL_AUTO, "tc": _lib.PALU_KERNEL_TC, "mma": _lib.PALU_KERNEL_MMA}[args.kernel])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    if N_KV % ws:
        raise SystemExit(f"{N_KV} KV heads do not shard over {ws} GPUs")
    B = args.batch * ws
    n_kv = N_KV // ws
    n_q = N_Q // ws
    L = make_layer(dev, B, n_q, n_kv, seed=1234 + rank)
    pt = None
    if args.paged:
        # the same latents, each row's blocks scattered over the physical blocks by a seeded permutation
        bs = args.paged
        per_row = S // bs
        g = torch.Generator(device=dev).manual_seed(99 + rank)
        pt = torch.randperm(B * per_row, generator=g, device=dev).view(B, per_row).to(torch.int32)
        for name in ("k", "v"):
            c = L[name]
            paged = torch.empty(B * per_row, n_kv, bs, R, dtype=c.dtype, device=dev)
            paged[pt.long().view(-1)] = c.view(B, n_kv, per_row, bs, R).transpose(1, 2).reshape(-1, n_kv, bs, R)
            L[name] = paged
            del c, paged
    out = torch.empty(B, n_q, R, dtype=torch.bfloat16, device=dev)
    d = _lib.dims(B, n_q, n_kv, n_kv, R, R, S)
    ws_buf = _lib.new_workspace(d, dev)

    def step():
        fused.decode(L["q"], L["k"], L["v"], L["u"], L["cs"], L["pos"], out=out, workspace=ws_buf, page_table=pt)

    stream = torch.cuda.current_stream(dev)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    def barrier():
        if ws > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    # ---- device-resident timing -------------------------------------------------------------------
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    barrier()
    with ClockSampler(local) as clk:
        # The timed region can be a few ms, shorter than nvidia-smi's 200 ms sampling period, so the
        # sampler also covers a soak of the same step (same load, untimed) right before it.
        soak_end = time.perf_counter() + args.clock_soak
        while time.perf_counter() < soak_end:
            for _ in range(50):
                step()
            torch.cuda.synchronize()
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(args.steps):
            evs[2 * i].record(stream)
            step()
            evs[2 * i + 1].record(stream)
        t1.record(stream)
        barrier()
    total_ms = t0.elapsed_time(t1)
    per_launch = [evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(args.steps)]
    if ws > 1:
        tt = torch.tensor([total_ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(tt.item())
    ms = total_ms / args.steps
    value = B / (ms * 1e-3)   # global batch rows per second (each rank does the same per-rank work)

    # ---- e2e through the C ABI with host buffers ---------------------------------------------------
    # One step = the step's inputs (q, new K/V latents, positions) from one pinned host buffer to the GPU in
    # one copy, append, decode + merge, and the output back to pinned host memory; steps run back to back
    # (each step's inputs would depend on the previous step's output in a decode loop, so nothing overlaps
    # across steps). The step is captured once as a CUDA graph and replayed, as a serving loop would.
    sizes = [B * n_q * 128 * 2, B * n_kv * R * 2, B * n_kv * R * 2, B * 4]
    offs = [0]
    for n_b in sizes:
        offs.append(offs[-1] + (n_b + 255) // 256 * 256)
    in_h = torch.empty(offs[-1], dtype=torch.uint8).pin_memory()
    in_d = torch.empty(offs[-1], dtype=torch.uint8, device=dev)
    views = lambda buf: (buf[offs[0]:offs[0] + sizes[0]].view(torch.bfloat16).view(B, n_q, 128),
                         buf[offs[1]:offs[1] + sizes[1]].view(torch.bfloat16).view(B, n_kv, R),
                         buf[offs[2]:offs[2] + sizes[2]].view(torch.bfloat16).view(B, n_kv, R),
                         buf[offs[3]:offs[3] + sizes[3]].view(torch.int32))
    q_h, nk_h, nv_h, pos_h = views(in_h)
    q_h.copy_(torch.randn(B, n_q, 128).to(torch.bfloat16))
    nk_h.copy_(torch.randn(B, n_kv, R).to(torch.bfloat16))
    nv_h.copy_(torch.randn(B, n_kv, R).to(torch.bfloat16))
    pos_h.fill_(S - 1)
    q_d, nk_d, nv_d, pos_d = views(in_d)
    out_h = torch.empty(B, n_q, R, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        in_d.copy_(in_h, non_blocking=True)
        fused.append_latents(nk_d, nv_d, pos_d, L["k"], L["v"], page_table=pt)
        fused.decode(q_d, L["k"], L["v"], L["u"], L["cs"], pos_d, out=out, workspace=ws_buf, page_table=pt)
        out_h.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        e2e_step()
    for _ in range(3):
        graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if ws > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    del graph
    h2d = in_h.numel()
    d2h = out_h.numel() * out_h.element_size()

    # ---- roofline of the op on this rank -----------------------------------------------------------
    per_launch_ms = statistics.mean(per_launch)
    latent_bytes = B * n_kv * S * (R + R) * 2
    u_bytes = n_kv * R * 128 * 2
    alg_bytes = latent_bytes + u_bytes
    achieved = alg_bytes / (per_launch_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    tr = traffic_record()
    kernel_name = ("palu_decode_tc_kernel + palu_combine_tc_kernel" if _lib.kernel_for(d) == _lib.PALU_KERNEL_TC
                   else "palu_decode_mma_kernel + palu_combine_kernel")

    if rank == 0:
        cpu = None
        if ws == 1:
            rate, cores, sample = cpu_oracle_rate(args.cpu_budget)
            cpu = {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, on device)",
            "config": workload_config(ws, args.batch, args.paged),
            "us_per_layer": ms * 1e3, "latent_GBps": achieved,
            "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": (tr or {}).get("bytes_per_launch"),
                         "kernel": kernel_name + " (one decode op)",
                         "algorithmic_bytes": alg_bytes},
            "cpu_baseline": cpu,
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
