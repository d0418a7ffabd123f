#!/usr/bin/env python
"""MoE decode benchmark of the B200 NVFP4 expert path.

Workload: one decode token (batch 1) through 24 stacked routed-MoE layers of
the Nemotron 30B-A3B shape -- 128 NVFP4 experts per layer (up 1856x2688,
relu^2, down 2688x1856), all HBM-resident (17.24 GB), sigmoid top-6 routing
from random logits per layer and token, x_{L+1} = x_L + moe_L(x_L) in fp32.
A "step" is one token through all 24 layers.  Weights are seeded synthetic
(N(0, 0.02) quantised to NVFP4 on the device): the real checkpoint is not
available.  With --gpus N the experts are sharded by id (e % N) and every
rank runs the token in one launch that writes its route slots' rows into
every rank's memory over NVLink and sums them in route order
(--exchange nccl: per-layer launches with an NCCL all-gather and a
route-sum launch instead).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
HIDDEN, INTER, N_EXPERTS, TOP_K, N_LAYERS = 2688, 1856, 128, 6, 24
METRIC = "moe_decode_tok_s"
UNIT = "tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="only the decode-step line (no per-kernel, GEMV, batch-32 or router keys)")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--bank", choices=["quantized", "random"], default="quantized",
                    help="random: expert records of seeded random bytes (same shapes and "
                         "bytes, a few launches to build; for profiler runs)")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="expert-parallel exchange of the slot outputs (N > 1)")
    ap.add_argument("--gemv", type=int, nargs=2, metavar=("ROWS", "COLS"),
                    help="time one NVFP4 GEMV shape instead of the decode step")
    ap.add_argument("--bf16-tc", type=int, nargs=3, metavar=("ROWS", "COLS", "N"),
                    help="time one BF16 tensor-core GEMM shape and exit")
    ap.add_argument("--gemm-tc", type=int, nargs=3, metavar=("ROWS", "COLS", "N"),
                    help="time the tensor-core batched NVFP4 GEMM (N <= 16 tokens)")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_setup(n):
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, torch.device("cuda", local if world > 1 else 0)


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}",
                                       f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None
        # nvidia-smi takes a moment to start: wait (bounded) for its first
        # sample so that the timed region that follows is covered.
        t_end = time.time() + 5.0
        while self.p is not None and time.time() < t_end and self.p.poll() is None:
            self.f.flush()
            if Path(self.f.name).stat().st_size > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        self.f.flush()
        rows = []
        for line in Path(self.f.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def time_region(fn, steps, device):
    """CUDA-event time of `steps` calls of fn on the current stream (ms)."""
    torch.cuda.synchronize(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        fn(i)
    b.record()
    b.synchronize()
    return a.elapsed_time(b)


def time_graph(fn, steps, device, barrier=None):
    """Device time per call (ms) of `steps` calls of fn captured in one CUDA
    graph, so that host launch cost does not hide short kernels; replayed
    once untimed, then timed with CUDA events.  `barrier` (ranks that wait
    for one another inside fn): called before the timed replay so that every
    rank starts it together."""
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        fn(0)
    torch.cuda.current_stream(device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(steps):
            fn(i)
    g.replay()
    torch.cuda.synchronize(device)
    if barrier is not None:
        barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    b.synchronize()
    del g
    return a.elapsed_time(b) / steps


def random_bank(L, device):
    """A bank of seeded random code bytes and scale bytes 0x28..0x37 (E4M3
    0.25..0.47) with global scale 1/64: the bench's shapes and bytes in a
    handful of launches, for profiler runs whose time goes into every launch."""
    from ervf_b200.moe import ExpertBank

    bank = ExpertBank(L, N_EXPERTS, HIDDEN, INTER, device)
    g = torch.Generator(device=device)
    for l in range(L):
        g.manual_seed(7000 + l)
        for t in (bank.up_codes[l], bank.dn_codes[l]):
            t.copy_(torch.randint(0, 256, t.shape, generator=g, device=device, dtype=torch.int32).to(torch.uint8))
        for t in (bank.up_scales[l], bank.dn_scales[l]):
            t.copy_(torch.randint(0x28, 0x38, t.shape, generator=g, device=device, dtype=torch.int32).to(torch.uint8))
        bank.globals[l].fill_(1.0 / 64.0)
    torch.cuda.synchronize(device)
    return bank


def kernel_roofline(dec, bank, device, hbm, iters=192):
    """Average device time of the two grouped expert kernels (a CUDA graph of
    `iters` launches each, timed with CUDA events), each launch on a
    different (layer, token) routing so that weights come from HBM."""
    from ervf_b200 import _lib

    f = dec.fused
    g = torch.Generator(device=device)
    g.manual_seed(12345)
    L = bank.n_layers
    ids = torch.stack([torch.randperm(N_EXPERTS, generator=g, device=device)[:TOP_K]
                       for _ in range(iters)]).to(torch.int32)
    w = torch.full((TOP_K,), 1.0 / TOP_K, device=device)
    x = torch.randn(HIDDEN, device=device)
    act = torch.zeros(TOP_K * INTER, device=device)
    out = torch.zeros(HIDDEN, device=device)

    def up(i):
        l = i % L
        f.moe_up_grouped(bank.up_codes[l], bank.up_scales[l], bank.up_code_bytes,
                         bank.up_scale_bytes, ids[i], bank.globals[l], TOP_K, x, act, INTER, HIDDEN)

    def down(i):  # the decode chain's variant: PDL launch, group-counter route sum
        l = i % L
        f.moe_down_routesum(bank.dn_codes[l], bank.dn_scales[l], bank.dn_code_bytes,
                            bank.dn_scale_bytes, ids[i], bank.globals[l], w, TOP_K, act, out,
                            HIDDEN, INTER, resid=x, flags=_lib.LAUNCH_PDL | _lib.LAUNCH_IDS_READY)

    for fn in (up, down):
        for i in range(8):
            fn(i)
    t_up = time_graph(up, iters, device)
    t_dn = time_graph(down, iters, device)
    rec = INTER * HIDDEN // 2 + INTER * HIDDEN // 16
    up_bytes = TOP_K * rec + HIDDEN * 4 + TOP_K * INTER * 4
    dn_bytes = TOP_K * rec + TOP_K * INTER * 4 + 2 * HIDDEN * 4
    res = {
        "moe_up_grouped": {"ms": t_up, "bytes": up_bytes, "gbs": up_bytes / t_up / 1e6},
        "moe_down_routesum": {"ms": t_dn, "bytes": dn_bytes, "gbs": dn_bytes / t_dn / 1e6},
    }
    if dec.token:
        # the one-launch token kernel (the decode step's kernel on one GPU):
        # every launch on its own routing of all L layers
        tok_ids = ids[: (iters // L) * L].view(-1, L, TOP_K)[:8]
        tok_w = torch.full((L, TOP_K), 1.0 / TOP_K, device=device)
        xt = (x * 0.0625).contiguous()
        yt = torch.zeros(HIDDEN, device=device)

        def token(i):
            dec.token_step(xt, yt, tok_ids[i % tok_ids.shape[0]], tok_w)

        for i in range(4):
            token(i)
        t_tok = time_graph(token, 16, device)
        tok_bytes = L * (TOP_K * 2 * rec + 3 * HIDDEN * 4 + 2 * TOP_K * INTER * 4)
        res["moe_token"] = {"ms": t_tok, "bytes": tok_bytes, "gbs": tok_bytes / t_tok / 1e6}
    for v in res.values():
        v["frac"] = v["gbs"] / hbm
    return res


def gemv_shape(device, hbm, rows=INTER, cols=HIDDEN, min_iters=64):
    """One NVFP4 GEMV [rows x cols] (config 0 by default) cycling over a
    replica pool of >= 8 x L2 (L2-cold weights; two copies when a single
    matrix already exceeds 2 x L2), B200 schedule, device time per call from
    a CUDA graph of the calls.
    Algorithmic bytes per call: codes + scales + global scale + x + out."""
    from ervf_b200 import FusedNVFP4
    from ervf_b200.formats import quantize_nvfp4_torch

    f = FusedNVFP4(device=device)
    if (rows, cols) == (1856, 2688):  # BASELINE config 0's exact inputs
        from ervf_b200.formats import config0_inputs

        c0, s0, g0, x0 = config0_inputs()
        codes, scales = torch.from_numpy(c0).to(device), torch.from_numpy(s0).to(device)
        x, gsc = torch.from_numpy(x0).to(device), g0
    else:
        gen = torch.Generator(device=device)
        gen.manual_seed(0)
        codes, scales, gsc = quantize_nvfp4_torch(torch.randn(rows, cols, generator=gen,
                                                              device=device) * 0.02)
        x = torch.randn(cols, device=device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    rec = codes.numel() + scales.numel()
    n = max(1, (8 * l2) // rec + 1) if rec < 2 * l2 else 2
    pc = codes.reshape(1, -1).repeat(n, 1)
    ps = scales.reshape(1, -1).repeat(n, 1)
    del codes, scales
    out = torch.zeros(rows, device=device)
    g = float(gsc)

    def call(i):
        j = i % n
        f.gemv_into(out, pc[j], ps[j], x, g, rows, cols, apply_relu2=True)

    for i in range(10):
        call(i)
    iters = max(min_iters, 4 * n)
    ms = time_graph(call, iters, device)
    algo = rec + 4 + cols * 4 + rows * 4
    return {"rows": rows, "cols": cols, "us": ms * 1e3, "gbs": algo / ms / 1e6,
            "frac": algo / ms / 1e6 / hbm, "pool_replicas": n, "bytes_per_call": algo}


def gemm_tc_shape(device, hbm, rows, cols, n):
    """Batched NVFP4 GEMM on the tensor cores: one matrix [rows x cols] times
    n <= 16 activation rows, L2-cold replica pool, device time per call from a
    CUDA graph.  Algorithmic bytes: codes + scales + n*cols*4 + n*rows*4; the
    same weights through n batch-1 GEMVs are reported beside it."""
    from ervf_b200 import FusedNVFP4
    from ervf_b200.formats import quantize_nvfp4_torch

    f = FusedNVFP4(device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    codes, scales, gsc = quantize_nvfp4_torch(torch.randn(rows, cols, generator=gen,
                                                          device=device) * 0.02)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    rec = codes.numel() + scales.numel()
    m = max(1, (8 * l2) // rec + 1) if rec < 2 * l2 else 2
    pc = codes.reshape(1, -1).repeat(m, 1)
    ps = scales.reshape(1, -1).repeat(m, 1)
    del codes, scales
    x = torch.randn(n * cols, device=device)
    out = torch.zeros(n * rows, device=device)
    g = float(gsc)
    iters = max(16, 4 * m)
    ms = time_graph(lambda i: f.gemm_tc(out, pc[i % m], ps[i % m], x, g, rows, cols, n), iters, device)
    o1 = torch.zeros(rows, device=device)
    ms1 = time_graph(lambda i: f.gemv_into(o1, pc[i % m], ps[i % m], x[:cols], g, rows, cols),
                     iters, device)
    algo = rec + n * cols * 4 + n * rows * 4
    return {"rows": rows, "cols": cols, "n": n, "us": round(ms * 1e3, 2),
            "gbs": round(algo / ms / 1e6, 1), "frac": round(algo / ms / 1e6 / hbm, 4),
            "tokens_per_s": round(n / (ms * 1e-3), 1),
            "batch1_gemv_us": round(ms1 * 1e3, 2),
            "speedup_vs_n_batch1_gemvs": round(n * ms1 / ms, 2)}


def bf16_gemvs(device, hbm):
    """Config 3: BF16 dense GEMVs [4096x2688], [2688x4096] and the output head
    [131072x2688] at batch 1 and 8, cycling an L2-cold replica pool (>= 8 x
    L2; the head alone exceeds L2), device time per call from a CUDA graph.  Algorithmic
    bytes: 2*rows*cols + 4*cols*B + 4*rows*B."""
    from ervf_b200 import GPUKernels

    k = GPUKernels(device=device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    res = {}
    for rows, cols in ((4096, 2688), (2688, 4096), (131072, 2688)):
        nbytes = 2 * rows * cols
        n = max(1, (8 * l2) // nbytes + 1) if nbytes < 2 * l2 else 2
        w1 = (torch.randn(rows * cols, device=device) * 0.02).to(torch.bfloat16).view(torch.int16)
        W = w1.reshape(1, -1).repeat(n, 1)
        del w1
        for batch in (1, 8):
            x = torch.randn(batch * cols, device=device)
            out = torch.zeros(batch * rows, device=device)

            def call(i):
                k.mv_bf16_batched(out, W[i % n], x, rows, cols, batch)

            for i in range(3):
                call(i)
            iters = max(16, 4 * n)
            ms = time_graph(call, iters, device)
            algo = nbytes + 4 * cols * batch + 4 * rows * batch
            res[f"{rows}x{cols}_b{batch}"] = {"us": round(ms * 1e3, 2), "gbs": round(algo / ms / 1e6, 1),
                                              "frac": round(algo / ms / 1e6 / hbm, 4)}
            if batch > 1:  # the tensor-core path (tolerance) beside the SIMT one

                def call_tc(i):
                    k.mm_bf16_tc(out, W[i % n], x, rows, cols, batch)

                ms = time_graph(call_tc, iters, device)
                res[f"{rows}x{cols}_b{batch}_tc"] = {"us": round(ms * 1e3, 2),
                                                     "gbs": round(algo / ms / 1e6, 1),
                                                     "frac": round(algo / ms / 1e6 / hbm, 4)}
        del W
    return res


def bf16_tc_shape(device, hbm, rows, cols, n):
    """One BF16 tensor-core GEMM shape [rows x cols] at batch n (config 3's
    batched path), L2-cold replica pool, device time per call from a CUDA
    graph; bytes as in bf16_gemvs."""
    from ervf_b200 import GPUKernels

    k = GPUKernels(device=device)
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    nbytes = 2 * rows * cols
    reps = max(1, (8 * l2) // nbytes + 1) if nbytes < 2 * l2 else 2
    w1 = (torch.randn(rows * cols, device=device) * 0.02).to(torch.bfloat16).view(torch.int16)
    W = w1.reshape(1, -1).repeat(reps, 1)
    del w1
    x = torch.randn(n * cols, device=device)
    out = torch.zeros(n * rows, device=device)

    def call(i):
        k.mm_bf16_tc(out, W[i % reps], x, rows, cols, n)

    for i in range(3):
        call(i)
    ms = time_graph(call, max(16, 4 * reps), device)
    algo = nbytes + 4 * cols * n + 4 * rows * n
    return {"rows": rows, "cols": cols, "n": n, "us": round(ms * 1e3, 2), "gbs": round(algo / ms / 1e6, 1),
            "frac": round(algo / ms / 1e6 / hbm, 4)}


def batched_decode(dec, device, hbm, world=1, tokens=32, steps=20):
    """Config 4 at batch 32: a decode batch through all layers, expert-major on
    the tensor cores (each routed expert read once per layer for all its
    tokens), CUDA graph of the whole step, device time (max over ranks).  With
    N GPUs every rank streams only its experts (e % N) and one peer-memory
    exchange per layer feeds the route-order sum.  Bytes per step: the
    distinct (layer, expert) records the routing touches plus activations;
    frac is against the aggregate HBM roofline (N x measured), frac_busiest
    against the busiest rank's bytes per layer."""
    L, E = dec.bank.n_layers, dec.bank.n_experts
    g = torch.Generator(device=device)
    g.manual_seed(7)
    xb = torch.randn(tokens, HIDDEN, generator=g, device=device)
    rb = torch.randn(L, tokens, E, generator=g, device=device)
    dec.step_batch(xb, rb)
    torch.cuda.synchronize(device)
    ids = dec.bids.view(L, tokens, TOP_K)
    rec = 2 * (INTER * HIDDEN // 2 + INTER * HIDDEN // 16)
    act_bytes = tokens * TOP_K * (HIDDEN + INTER) * 4
    distinct, busiest = 0, 0
    for l in range(L):
        u = torch.unique(ids[l]).cpu()
        distinct += int(u.numel())
        busiest += max(int((u % world == r).sum()) for r in range(world))
    step_bytes = distinct * rec + L * act_bytes
    busiest_bytes = busiest * rec + L * act_bytes
    sync = None
    if world > 1:
        import torch.distributed as dist

        def sync():
            dist.barrier()
            torch.cuda.synchronize(device)

    ms = time_graph(lambda i: dec.step_batch(xb, rb), steps, device, barrier=sync)
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return {"tokens_per_step": tokens, "n_gpus": world, "ms_per_step": round(ms, 4),
            "tok_s": round(tokens / (ms * 1e-3), 1),
            "distinct_experts_per_layer": round(distinct / L, 1),
            "step_bytes": step_bytes, "gbs": round(step_bytes / ms / 1e6, 1),
            "frac": round(step_bytes / ms / 1e6 / (hbm * world), 4),
            "frac_busiest": round(busiest_bytes / ms / 1e6 / hbm, 4),
            "path": "expert-major tcgen05 (tolerance), route-order sum"
                    + (", peer-memory exchange" if world > 1 else "")}


def qwen_block_b16(device, hbm, tokens=16, layers=48, pools=4, steps=5):
    """Config 2 at batch 16: the Qwen3-30B-A3B-shaped MoE layer (128 experts,
    hidden 2048, moe intermediate 768, gate / up rows interleaved, softmax
    top-8) as the expert-major batched block on the tensor cores with the
    SwiGLU epilogue, `layers` layers per step cycling over `pools` expert
    banks of seeded random record bytes (each bank 340 MB, larger than L2),
    fresh router logits per layer; CUDA graph, device time.  Bytes per step:
    the distinct (layer, expert) records the routing touches plus the
    activations."""
    from ervf_b200.fused_nvfp4 import FusedNVFP4

    H, I, E, K = 2048, 768, 128, 8
    up_c, up_s = 2 * I * H // 2, 2 * I * H // 16
    dn_c, dn_s = H * I // 2, H * I // 16
    g = torch.Generator(device=device)
    banks = []
    for p in range(pools):
        g.manual_seed(9100 + p)
        rb = lambda n, lo, hi: torch.randint(lo, hi, (n,), generator=g, device=device,
                                             dtype=torch.int32).to(torch.uint8)
        banks.append((rb(E * up_c, 0, 256), rb(E * up_s, 0x28, 0x38), rb(E * dn_c, 0, 256),
                      rb(E * dn_s, 0x28, 0x38), torch.full((E, 2), 1.0 / 64.0, device=device)))
    g.manual_seed(9200)
    rlogs = torch.randn(layers, tokens, E, generator=g, device=device)
    x0 = torch.randn(tokens, H, generator=g, device=device) * 0.1
    ids = torch.zeros(layers, tokens, K, dtype=torch.int32, device=device)
    w = torch.zeros(layers, tokens, K, device=device)
    xs = [torch.empty(tokens, H, device=device) for _ in range(2)]
    f = FusedNVFP4(device=device)

    def step(i):
        xs[0].copy_(x0)
        for l in range(layers):
            uc, us, dc, ds, gl = banks[l % pools]
            f.route_topk_softmax(rlogs[l], ids[l], w[l], tokens, E, K)
            f.moe_batched(uc, us, up_c, up_s, dc, ds, dn_c, dn_s, gl, ids[l], w[l], tokens, K, E,
                          xs[l % 2], xs[(l + 1) % 2], H, I, swiglu=True)

    step(0)
    torch.cuda.synchronize(device)
    distinct = sum(int(torch.unique(ids[l]).numel()) for l in range(layers))
    rec = up_c + up_s + dn_c + dn_s
    step_bytes = distinct * rec + layers * tokens * K * (H + I) * 4
    ms = time_graph(step, steps, device)
    return {"tokens_per_step": tokens, "layers": layers, "ms_per_step": round(ms, 4),
            "us_per_layer": round(ms * 1e3 / layers, 2), "tok_s": round(tokens / (ms * 1e-3), 1),
            "distinct_experts_per_layer": round(distinct / layers, 1), "step_bytes": step_bytes,
            "gbs": round(step_bytes / ms / 1e6, 1), "frac": round(step_bytes / ms / 1e6 / hbm, 4),
            "path": "softmax top-8 router + expert-major tcgen05 block, SwiGLU epilogue "
                    "(tolerance), route-order sum; seeded random record bytes"}


def busiest_rank_slots(rlogs, world, top_k=TOP_K):
    """Per token (rlogs [T][L][E] router logits), the sum over layers of the
    most route slots that any one rank owns (expert e on rank e % world,
    slots = the top_k experts of the layer's logits): the records the
    busiest rank streams, which bounds an expert-parallel step.  [T] floats;
    top_k * L for one rank."""
    top = rlogs.topk(top_k, dim=-1).indices                                # [T, L, K]
    counts = torch.nn.functional.one_hot(top % world, world).sum(dim=-2)   # [T, L, world]
    return counts.max(dim=-1).values.sum(dim=-1).to(torch.float64)


def routed_decode(dec, device, hbm, steps=50):
    """Config 4 at batch 1 with the router on the device between the layers
    (per layer: router GEMV fp32 [128 x 2688] + top-k in one launch, then up
    and down + routed sum), graph-timed: the decode step as the reference's
    runtime runs it (runtime.py:705-746), minus the trunk."""
    L, E = dec.bank.n_layers, dec.bank.n_experts
    g = torch.Generator(device=device)
    g.manual_seed(11)
    gate_w = torch.randn(L, E, HIDDEN, generator=g, device=device) * 0.02
    x = torch.randn(HIDDEN, generator=g, device=device)
    ms = time_graph(lambda i: dec.step_with_router(x, gate_w), steps, device)
    router_bytes = E * HIDDEN * 4 + HIDDEN * 4
    token_bytes = L * (TOP_K * dec.bank.expert_bytes() + router_bytes)
    one = dec.token and dec.token_router and E <= 256
    res = {"ms_per_token": round(ms, 4), "tok_s": round(1e3 / ms, 1),
           "launches_per_token": 1 if one else 3 * L,
           "path": "one launch (router items in the token kernel)" if one else "per-layer launches",
           "token_bytes": token_bytes,
           "frac": round(token_bytes / ms / 1e6 / hbm, 4)}
    if dec.token:
        # the same step on the other path
        dec.token_router = not one
        ms1 = time_graph(lambda i: dec.step_with_router(x, gate_w), steps, device)
        dec.token_router = one
        res["per_layer_ms_per_token" if one else "one_launch_ms_per_token"] = round(ms1, 4)
    return res


def cpu_sample(bank, layers_sampled=4, tokens=2):
    """Reference-path CPU baseline on a bounded sample: `tokens` tokens x
    `layers_sampled` layers of the same workload (8 rounds by default), torch
    FP32 dequant + matmul with all host threads; p50 over the rounds of one
    layer's time (dequant + matmul = the headline, and matmul alone),
    extrapolated to tok/s over 24 layers."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_baseline as cb

    cores = cb.use_all_cores()
    g = np.random.default_rng(7)
    full, mm = [], []
    for t in range(tokens):
        x = torch.from_numpy(g.standard_normal(HIDDEN).astype(np.float32))
        for l in range(layers_sampled):
            ids = g.choice(N_EXPERTS, TOP_K, replace=False)
            experts = {}
            for e in ids:
                (uc, us, ug), (dc, ds, dg) = bank.expert_host(l, int(e))
                experts[int(e)] = ((torch.from_numpy(uc), torch.from_numpy(us), float(ug)),
                                   (torch.from_numpy(dc), torch.from_numpy(ds), float(dg)))
            w = np.full(TOP_K, 1.0 / TOP_K, np.float32)
            x, t_dq, t_mm = cb.moe_layer_timed(x, experts, ids, w, HIDDEN, INTER)
            full.append(t_dq + t_mm)
            mm.append(t_mm)
    per_layer = statistics.median(full)
    per_layer_mm = statistics.median(mm)
    return {"value": 1.0 / (per_layer * N_LAYERS), "unit": UNIT, "cores": cores, "kind": "port",
            "matmul_only_value": 1.0 / (per_layer_mm * N_LAYERS), "rounds": len(full),
            "sample": f"{tokens} tokens x {layers_sampled} of {N_LAYERS} layers (6 experts each), "
                      f"p50 of {len(full)} rounds: {per_layer * 1e3:.1f} ms/layer dequant + matmul "
                      f"({per_layer_mm * 1e3:.1f} ms matmul only), extrapolated x{N_LAYERS} layers"}


def reference_arm(args, rank, world):
    """CPU reference path (torch FP32 dequant-then-matmul, all host cores) on
    the same workload: each step is one token through a bounded sample of one
    layer, extrapolated to 24 layers."""
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import cpu_baseline as cb
    from ervf_b200.formats import synthetic_nvfp4

    cores = cb.use_all_cores()
    g = np.random.default_rng(11)
    n_pool = 12
    pool = {}
    for e in range(n_pool):
        uc, us, ug = synthetic_nvfp4(INTER, HIDDEN, seed=e)
        dc, ds, dg = synthetic_nvfp4(HIDDEN, INTER, seed=500 + e)
        pool[e] = ((torch.from_numpy(uc.reshape(-1)), torch.from_numpy(us.reshape(-1)), float(ug)),
                   (torch.from_numpy(dc.reshape(-1)), torch.from_numpy(ds.reshape(-1)), float(dg)))
    times, mm = [], []
    for step in range(args.warmup + args.steps):
        x = torch.from_numpy(g.standard_normal(HIDDEN).astype(np.float32))
        ids = g.choice(n_pool, TOP_K, replace=False)
        w = np.full(TOP_K, 1.0 / TOP_K, np.float32)
        _, t_dq, t_mm = cb.moe_layer_timed(x, pool, ids, w, HIDDEN, INTER)
        if step >= args.warmup:
            times.append(t_dq + t_mm)
            mm.append(t_mm)
    per_layer = statistics.median(times)  # p50 over the K steps
    value = 1.0 / (per_layer * N_LAYERS)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_layer * N_LAYERS * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": "config4: 24 MoE layers x 128 NVFP4 experts (2688/1856), top-6, "
                               "batch 1", "parallelism": "cpu", "l2": "n/a"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "matmul_only_value": 1.0 / (statistics.median(mm) * N_LAYERS),
                         "sample": f"each step: 1 token x 1 of 24 layers (6 experts, dequant + "
                                   f"matmul), p50 of {len(times)} steps, extrapolated x24"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", 0))
        world = int(os.environ.get("WORLD_SIZE", 1))
        reference_arm(args, rank, world)
        return
    rank, world, device = dist_setup(args.gpus)
    sys.path.insert(0, str(ROOT))
    from ervf_b200 import build
    from ervf_b200.moe import ExpertBank, MoEDecoder

    build.build()
    hbm, peak_kind = peaks()
    if args.gemv:
        r = gemv_shape(device, hbm, args.gemv[0], args.gemv[1])
        r.update({"peak_gbs": hbm, "peak_kind": peak_kind})
        print(json.dumps({"gemv": r}))
        return
    if args.bf16_tc:
        r = bf16_tc_shape(device, hbm, *args.bf16_tc)
        r.update({"peak_gbs": hbm, "peak_kind": peak_kind})
        print(json.dumps({"bf16_tc": r}))
        return
    if args.gemm_tc:
        r = gemm_tc_shape(device, hbm, *args.gemm_tc)
        r.update({"peak_gbs": hbm, "peak_kind": peak_kind})
        print(json.dumps({"gemm_tc": r}))
        return
    L = args.layers
    t0 = time.time()
    # every rank builds only the experts it owns (e % world == rank); seeds
    # 1000 * layer + expert (+500 for down), N(0, 0.02), quantised on the device
    if args.bank == "random":
        bank = random_bank(L, device)
    else:
        bank = ExpertBank.synthetic(L, N_EXPERTS, HIDDEN, INTER, device, rank=rank, world=world)
    torch.cuda.synchronize(device)
    build_s = time.time() - t0

    group = None
    if world > 1:
        import torch.distributed as dist

        group = dist.group.WORLD
    dec = MoEDecoder(bank, TOP_K, ep_ranks=world, ep_rank=rank, group=group,
                     exchange=args.exchange)

    T = args.warmup + args.steps
    g = torch.Generator(device=device)
    g.manual_seed(2)
    rlogs = torch.randn(T, L, N_EXPERTS, generator=g, device=device)
    xs = torch.randn(T, HIDDEN, generator=g, device=device)
    xs = (xs.view(torch.int32) & -65536).view(torch.float32)  # bf16-valued hidden states
    x_buf = torch.zeros(HIDDEN, device=device)
    r_buf = torch.zeros(L, N_EXPERTS, device=device)

    # the whole token (the exchanges included when world > 1) is one graph
    use_graph = not args.no_graph
    graph = None
    if use_graph:
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            for _ in range(2):
                y = dec.step(x_buf, r_buf)
        torch.cuda.current_stream(device).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y_graph = dec.step(x_buf, r_buf)

    def step(i):
        x_buf.copy_(xs[i])
        r_buf.copy_(rlogs[i])
        if graph is not None:
            graph.replay()
        else:
            dec.step(x_buf, r_buf)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize(device)

    for i in range(args.warmup):
        step(i)
    barrier()
    with Clocks(device.index) as clk:
        # every rank's sampler is running: the ranks start the timed region
        # together (they are coupled every token, so a rank that started
        # late would otherwise add its delay to the others' time)
        barrier()
        ms = time_region(lambda i: step(args.warmup + i), args.steps, device)
        barrier()
    clocks = clk.summary()
    ms_t = torch.tensor([ms], device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    value = args.steps / (ms / 1e3)

    # ---- end to end through the public API with host buffers
    xh = xs.cpu().pin_memory()
    rh = rlogs.cpu().pin_memory()
    yh = torch.zeros(args.steps, HIDDEN, pin_memory=True)
    out_dev = y_graph if graph is not None else dec.xs[(L - 1) & 1]

    def e2e_step(i):
        x_buf.copy_(xh[i], non_blocking=True)
        r_buf.copy_(rh[i], non_blocking=True)
        if graph is not None:
            graph.replay()
        else:
            dec.step(x_buf, r_buf)
        yh[i % args.steps].copy_(out_dev, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()

    for i in range(min(3, args.warmup)):
        e2e_step(i)
    barrier()
    e2e_ms = time_region(lambda i: e2e_step(args.warmup + i), args.steps, device)
    barrier()
    e_t = torch.tensor([e2e_ms], device=device)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e2e_value = args.steps / (float(e_t.item()) / 1e3)

    full = not args.no_extras
    kern = kernel_roofline(dec, bank, device, hbm) if (world == 1 and full) else None
    gemv0 = gemv_shape(device, hbm) if (world == 1 and rank == 0 and full) else None
    # the lm_head shape (131072 x 2688, L2-cold replicas), one launch per call
    lmhead = gemv_shape(device, hbm, 131072, HIDDEN) if (world == 1 and rank == 0 and full) else None
    batch32 = batched_decode(dec, device, hbm, world) if full else None
    routed = routed_decode(dec, device, hbm) if (world == 1 and full) else None
    extra = None
    if world == 1 and rank == 0 and full:
        # config 2 (Qwen shapes) GEMVs and config 3 BF16 GEMVs, L2-cold
        extra = {"gemv_config2": {f"{r}x{c}": gemv_shape(device, hbm, r, c) for r, c in
                                  ((1536, 2048), (2048, 768))},
                 "bf16_gemv_config3": bf16_gemvs(device, hbm),
                 # config 2 batch-16 variant on the tensor cores
                 "gemm_tc_config2_b16": {f"{r}x{c}": gemm_tc_shape(device, hbm, r, c, 16) for r, c in
                                         ((1536, 2048), (2048, 768))},
                 # the whole config-2 MoE layer at batch 16 on the tensor cores
                 "qwen_block_b16": qwen_block_b16(device, hbm)}

    # records of the busiest rank per timed token (load-imbalance-aware roofline)
    busiest = float(busiest_rank_slots(rlogs[args.warmup:args.warmup + args.steps], world).mean())
    if rank == 0:
        # bytes one token streams: distinct (layer, expert) pairs x expert bytes
        token_bytes = L * TOP_K * bank.expert_bytes()
        busiest_bytes = busiest * bank.expert_bytes()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "nvfp4-w/f32-acc", "data": "synthetic",
            "config": {"workload": f"config4: {L} MoE layers x {N_EXPERTS} NVFP4 experts "
                                   f"(hidden {HIDDEN}, inter {INTER}), top-{TOP_K} sigmoid, batch 1",
                       "global_batch": 1, "parallelism": f"ep{world}",
                       "exchange": args.exchange if world > 1 else None,
                       "l2": "inputs larger than L2 (17.2 GB bank, 808 MB streamed per token)",
                       "cuda_graph": graph is not None},
            # router + the one-launch token kernel (on every rank with N > 1:
            # the expert-parallel token, slot rows exchanged inside it);
            # without it router + per layer up, down(+route sum) on one GPU,
            # up, down, exchange(+route sum) with N > 1
            "gpu_launches": (2 if dec.token else (2 * L + 1 if world == 1 else 3 * L + 1)) * args.steps,
            "token_bytes": token_bytes,
            "token_roofline_frac": (token_bytes / (ms / args.steps / 1e3) / 1e9) / (hbm * world),
            # against the busiest rank's records per token and one GPU's HBM
            # (equal to token_roofline_frac on one GPU)
            "busiest_rank_records_per_token": busiest,
            "token_roofline_frac_busiest": (busiest_bytes / (ms / args.steps / 1e3) / 1e9) / hbm,
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": (HIDDEN + L * N_EXPERTS) * 4,
                    "d2h_bytes_per_step": HIDDEN * 4},
            "bank_build_s": build_s,
        }
        if kern is not None:
            dom = max(kern, key=lambda k: kern[k]["ms"])
            traffic = None
            tfile = ROOT / "profiles" / "traffic.json"
            if tfile.exists():
                traffic = json.loads(tfile.read_text()).get(dom)
            line["roofline"] = {"bound": "hbm", "kernel": dom, "achieved": kern[dom]["gbs"],
                                "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                                "frac": kern[dom]["frac"], "traffic": traffic,
                                "algorithmic_bytes": kern[dom]["bytes"]}
            line["kernels"] = kern
        if gemv0 is not None:
            line["gemv_config0"] = gemv0
        if lmhead is not None:
            line["gemv_lmhead_nvfp4"] = lmhead
        if extra is not None:
            line.update(extra)
        if batch32 is not None:
            line["batched_decode_b32"] = batch32
        if routed is not None:
            line["decode_with_device_router"] = routed
        if world == 1 and not args.no_cpu_baseline and full:
            line["cpu_baseline"] = cpu_sample(bank)
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if world > 1:
        import torch.distributed as dist

        torch.cuda.synchronize(device)
        dec.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
