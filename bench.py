#!/usr/bin/env python
"""ResonanceNet training-step benchmark on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 is launched by torchrun (RANK / LOCAL_RANK / WORLD_SIZE / MASTER_* from
the environment); the library's own NCCL communicator all-reduces gradient
buckets during backward, torch.distributed is only used for the barrier, the
max-over-ranks timing reduction and the NCCL id broadcast.

Workload: d_model 512, 8 layers, d_ff 1024, 1024 slots,
top-2, vocab 256, fp32; per GPU batch 64 x seq 256 of synthetic Zipf(1.1)
byte tokens (a pool of 8 batches per rank, seed 7 + rank), weights N(0, 0.02)
(seed 1234). One step = zero_grad + forward + cross-entropy + backward
(+ bucketed all-reduce) + clipped SGD. Prints ONE JSON line on rank 0.

--impl reference times the reference's own CUDA implementation
(oracle/_ref/libref.so: its sources compiled unmodified for sm_100a) through
its ResonanceNet class on the same config and data, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "train tok/s (d512 L8 B64 T256)"
UNIT = "tok/s"
CFG = dict(d_model=512, n_layers=8, d_ff=1024, n_slots=1024, top_k=2, vocab=256, seq_len=256)
# the scaled model, bf16 GEMM operands, per-GPU B16 x T2048
CFG5 = dict(d_model=2048, n_layers=24, d_ff=5632, n_slots=8192, top_k=2, vocab=256, seq_len=2048)
METRIC5 = "train tok/s (d2048 L24 F5632 S8192, B16 T2048 per GPU, bf16)"
LR, CLIP = 3e-4, 1.0
# Algorithmic bytes per [N, D] element of one launch (fp32): scan fwd reads
# pz, ph, writes h, z; scan bwd reads dy, z, h, h~, writes dz, dh~; conv fwd
# reads x, writes S; conv bwd reads dS, x, writes dx; RMSNorm fwd reads x,
# writes y; RMSNorm bwd reads dy, x, writes dx.
ALG_BYTES_PER_ELEM = {"scan_fwd": 16, "scan_bwd": 24, "conv_fwd": 8, "conv_bwd": 12,
                      "rms_fwd": 8, "rms_bwd": 12}
POOL = 8


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=["c2", "c5"], default="c2",
                    help="c2: config 2 (default, fp32); c5: config 5 (d2048 L24, bf16, "
                         "activation recompute)")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--bf16", action="store_true",
                    help="bf16 GEMM operands with fp32 accumulation (default: fp32-accurate)")
    # single-operation mode (profiling captures of one kernel class)
    ap.add_argument("--op", default=None,
                    help="gemm | gemm16 | scan_fwd | scan_bwd | conv_fwd | conv_bwd | rms_fwd | rms_bwd")
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=512)
    ap.add_argument("--k", type=int, default=512)
    ap.add_argument("--amn", type=int, default=0)
    ap.add_argument("--cg", type=int, default=0, help="--op: GEMM CTA group (0 auto, 1, 2)")
    ap.add_argument("--decode", action="store_true",
                    help="config 4: prefill + batched greedy decode instead of training")
    ap.add_argument("--no-bf16", action="store_true",
                    help="skip the bf16-mode object of the default (1-GPU) line")
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the config-4 decode object of the default (1-GPU) line")
    ap.add_argument("--streams", type=int, default=256, help="--decode: streams over all GPUs")
    ap.add_argument("--prompt", type=int, default=4096, help="--decode: prefill length")
    ap.add_argument("--gen", type=int, default=1024, help="--decode: decode steps")
    ap.add_argument("--epi", type=int, default=0, help="--op gemm: 0 store, 1 accumulate, 2 residual")
    ap.add_argument("--bmn", type=int, default=0)
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", os.environ.get("RANK", 0))))


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return dict(hbm=p["hbm_gbs"], bf16=p["bf16_tflops"],
                    bf16_sust=p.get("bf16_tflops_sustained", p["bf16_tflops"]), src="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sust=1400.0, src="fallback")


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def start(self):
        if self.gpu is None:
            return
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # the first sample arrives only after nvidia-smi has initialised
        t_end = time.time() + 5.0
        while time.time() < t_end and os.path.getsize(self.path) == 0:
            time.sleep(0.02)

    def mark(self, begin: bool):
        """Wall-clock bounds of the timed region; samples outside are dropped."""
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 10:
                    rows.append(parts[1:])
                    try:
                        ts = parts[0].replace("/", "-")
                        rows[-1].insert(0, time.mktime(time.strptime(ts[:19], "%Y-%m-%d %H:%M:%S"))
                                        + float("0" + ts[19:]))
                    except ValueError:
                        rows[-1].insert(0, None)
        os.unlink(self.path)
        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if r[0] is not None and self.t0 - 0.05 <= r[0] <= self.t1 + 0.05]
            if inside:
                rows = inside
        rows = [r[1:] for r in rows]
        if not rows:
            return None
        def num(x):
            try:
                return float(x)
            except ValueError:
                return float("nan")
        sm = [num(r[1]) for r in rows]
        mx = max(num(r[2]) for r in rows)
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return dict(sm_mhz=statistics.median(loaded), sm_max_mhz=mx, reasons=reasons,
                    samples=len(rows), power_w_max=max(num(r[3]) for r in rows))


def zipf_pool(rdata, B, T, seed):
    toks, tgts = [], []
    for i in range(POOL):
        a, b = rdata.zipf_tokens(B, T, seed=seed * 1000 + i)
        toks.append(a.reshape(-1))
        tgts.append(b.reshape(-1))
    return toks, tgts


def cpu_baseline(rdata):
    """The CPU oracle (scalar C++/OpenMP restatement of the reference math),
    one full training step of the config-2 model on a bounded sample."""
    import numpy as np
    import oracle
    cfg = oracle.make_config(**CFG)
    params = rdata.init_params_normal(cfg, seed=1234)
    B, T = 1, 256
    tok, tgt = rdata.zipf_tokens(B, T, seed=7)
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    oracle.train_step(cfg, params, tok[:, :32], tgt[:, :32], 1, 32)  # warm the pool
    # ~10 s of CPU work: repeat B=1 x T=256 steps (the token rate of one step
    # does not depend on the batch size in the oracle)
    steps, dt = 0, 0.0
    while dt < 10.0 and steps < 64:
        t0 = time.perf_counter()
        oracle.train_step(cfg, params, tok, tgt, B, T, LR, CLIP)
        dt += time.perf_counter() - t0
        steps += 1
    return dict(value=steps * B * T / dt, unit=UNIT, cores=threads, kind="port",
                sample=f"{steps} full train steps (fwd+bwd+SGD) of the d512/L8 model on B=1 x "
                       f"T=256 Zipf tokens ({dt:.1f} s, {threads} OpenMP threads)")


def run_ours(args, rank, world, local):
    import numpy as np
    import torch
    rnet = importlib.import_module("resonance-net_b200")
    rdata = importlib.import_module("resonance-net_b200.data")
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        pg = dist
    B, T = args.batch, args.seq
    c5 = args.model == "c5"
    C = CFG5 if c5 else CFG
    cfg = rnet.ModelConfig.make(d_model=C["d_model"], n_layers=C["n_layers"],
                                d_ff=C["d_ff"], n_slots=C["n_slots"], top_k=C["top_k"],
                                vocab=C["vocab"], seq_len=C["seq_len"])
    model = rnet.Model(cfg, device=local, reference_init=False)
    if c5:
        # 2.14B parameters: N(0, 0.02) drawn on the device (same rule as
        # init_params_normal: norm gains 1, biases 0), one seeded generator
        flat = torch.empty(model.num_params, device="cuda")
        g = torch.Generator(device="cuda").manual_seed(1234)
        off = 0
        for name, n in rdata.tensor_layout(cfg):
            base = name.split(".")[-1]
            if base.startswith("norm") or base == "final_norm":
                flat[off:off + n].fill_(1.0)
            elif base in ("bz", "bh"):
                flat[off:off + n].zero_()
            else:
                flat[off:off + n].normal_(0.0, 0.02, generator=g)
            off += n
        model.set_params_device(flat)
        del flat
        model.set_recompute(True)
    else:
        model.set_params(rdata.init_params_normal(cfg, seed=1234))
    model.set_precision(args.bf16)
    dist_h = None
    if world > 1:
        uid = [rnet.Dist.unique_id() if rank == 0 else None]
        pg.broadcast_object_list(uid, src=0)
        dist_h = rnet.Dist(rank, world, local, uid[0])
        model.set_dist(dist_h)
    toks, tgts = zipf_pool(rdata, B, T, seed=7 + rank)
    d_in = [torch.from_numpy(t).cuda() for t in toks]
    d_tg = [torch.from_numpy(t).cuda() for t in tgts]
    h_in = [torch.from_numpy(t).pin_memory() for t in toks]
    h_tg = [torch.from_numpy(t).pin_memory() for t in tgts]
    d_loss = torch.zeros(1, device="cuda")
    stream = torch.cuda.ExternalStream(model.stream())

    def barrier():
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not pg:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    for i in range(args.warmup):
        model.train_step(d_in[i % POOL], d_tg[i % POOL], B, T, LR, CLIP, d_loss)
    model.synchronize()

    # ---- device-resident timed region (value) ------------------------------
    # one sampler (rank 0, its own GPU): NVML polling from every rank at once
    # measurably slows the other ranks' steps
    clocks = ClockSampler(local) if rank == 0 else ClockSampler(None)
    clocks.start()  # returns after its first sample, before the ranks align
    barrier()
    n0 = rnet.kernel_launches()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per_step = os.environ.get("RNET_BENCH_PER_STEP") == "1"
    step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)] if per_step else []
    clocks.mark(True)
    ev0.record(stream)
    for i in range(args.steps):
        if per_step:
            step_ev[i].record(stream)
        model.train_step(d_in[i % POOL], d_tg[i % POOL], B, T, LR, CLIP, d_loss)
    if per_step:
        step_ev[args.steps].record(stream)
    ev1.record(stream)
    ev1.synchronize()
    clocks.mark(False)
    if per_step:
        print(f"rank {rank} step ms: " + " ".join(f"{step_ev[i].elapsed_time(step_ev[i + 1]):.2f}"
                                                  for i in range(args.steps)), file=sys.stderr)
    launches = rnet.kernel_launches() - n0
    barrier()
    ck = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    model.synchronize()
    loss = float(d_loss.item()) / (B * T)

    # ---- the same steps again with per-kernel-class CUDA events (roofline) -
    barrier()
    model.profile_enable(True)
    model.profile_read(reset=True)
    for i in range(args.steps):
        model.train_step(d_in[i % POOL], d_tg[i % POOL], B, T, LR, CLIP, d_loss)
    prof = model.profile_read(reset=True)
    model.profile_enable(False)
    barrier()

    # ---- end-to-end through the public API with host buffers (e2e) --------
    barrier()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record(stream)
    for i in range(args.steps):
        model.train_step_host(h_in[i % POOL].numpy(), h_tg[i % POOL].numpy(), B, T, LR, CLIP)
    ev3.record(stream)
    ev3.synchronize()
    barrier()
    ms_e2e = max_over_ranks(ev2.elapsed_time(ev3))

    if rank != 0:
        _finish(pg, model, dist_h)
        return
    tokens = world * B * T * args.steps
    peaks = measured_peaks()
    g = prof["gemm"]
    gemm_tflops = g["flops"] / (g["ms"] * 1e-3) / 1e12 if g["ms"] > 0 else 0.0
    per_launch_ms = g["ms"] / max(1, g["launches"])
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gemm_traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    kernels = {}
    for k, v in prof.items():
        if v["launches"]:
            kernels[k] = dict(ms_per_step=round(v["ms"] / args.steps, 4),
                              share=round(v["ms"] / max(1e-9, sum(x["ms"] for x in prof.values())), 4))
            if v["ms"] > 0 and v["bytes"] > 0 and k != "gemm":
                kernels[k]["GBps"] = round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1)
                kernels[k]["hbm_frac"] = round(kernels[k]["GBps"] / peaks["hbm"], 3)
            # the same time against the algorithmic bytes per [N, D] element (reads
            # of the inputs and writes of the outputs the math needs; the kernels' own
            # extra outputs, e.g. the scan's saved e and second residual copy, excluded)
            if k in ALG_BYTES_PER_ELEM and v["ms"] > 0:
                alg = ALG_BYTES_PER_ELEM[k] * B * T * C["d_model"] * v["launches"]
                kernels[k]["alg_GBps"] = round(alg / (v["ms"] * 1e-3) / 1e9, 1)
                kernels[k]["alg_hbm_frac"] = round(kernels[k]["alg_GBps"] / peaks["hbm"], 3)
    out = {
        "metric": METRIC5 if c5 else METRIC, "value": round(tokens / (ms * 1e-3), 1), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": ("bf16 GEMM operands, fp32 accumulate (tcgen05 kind::f16)" if args.bf16
                  else "fp32 (3xTF32 tcgen05)"),
        "data": "synthetic Zipf(1.1) byte tokens, N(0,0.02) weights",
        "config": ({"workload": "config 5 train step, d2048 L24 F5632 S8192 top2 V256, bf16 GEMM "
                                "operands, fp32 master weights, activation recompute, "
                                + ("bf16 gradient all-reduce" if world > 1 else "1 GPU"),
                    "model": "ResonanceNet", "global_batch": world * B, "seq_len": T,
                    "parallelism": f"dp{world}", "per_gpu_batch": B,
                    "l2": "working set per step ~45 GB >> 126 MB L2 (no flush)"} if c5 else
                   {"workload": "train step, d512 L8 F1024 S1024 top2 V256", "model": "ResonanceNet",
                    "global_batch": world * B, "seq_len": T, "parallelism": f"dp{world}",
                    "per_gpu_batch": B, "l2": "working set per step ~6.5 GB >> 126 MB L2 (no flush)"}),
        "e2e": {"value": round(tokens / (ms_e2e * 1e-3), 1), "unit": UNIT,
                "h2d_bytes_per_step": 2 * B * T * 4, "d2h_bytes_per_step": 4},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "kernel": "gemm_tf32x3 (all GEMMs of the step)",
                     "achieved": round(gemm_tflops, 2), "peak": peaks["bf16_sust"],
                     "unit": "TFLOP/s", "frac": round(gemm_tflops / peaks["bf16_sust"], 4),
                     "peak_src": f"{peaks['src']} bf16 dense, sustained",
                     **({} if args.bf16 else {
                         "ceiling_3xtf32": round(peaks["bf16_sust"] / 6, 1),
                         "frac_of_3xtf32_ceiling": round(gemm_tflops / (peaks["bf16_sust"] / 6),
                                                         4)}),
                     "ms_per_launch": round(per_launch_ms, 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": round(g["bytes"] / max(1, g["launches"]))},
        "kernels": kernels, "loss": round(loss, 4),
        "clocks": ck,
    }
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(importlib.import_module("resonance-net_b200.data"))
    if world == 1 and not args.bf16 and args.model == "c2" and not args.no_bf16:
        out["bf16"] = bf16_measure(model, rnet, torch, stream, d_in, d_tg, B, T, args, peaks)
    _finish(pg, model, dist_h)
    if world == 1 and not args.no_decode:
        out["decode"] = decode_measure(rnet, rdata, torch, None, 0, 1, local, args.streams,
                                       args.prompt, args.gen, args.warmup, args.steps)
    print(json.dumps(out), flush=True)


def bf16_measure(model, rnet, torch, stream, d_in, d_tg, B, T, args, peaks):
    """The same config-2 step with bf16 GEMM operands (rnet_model_set_precision
    1): device-resident tok/s and the GEMM class against the bf16 peak."""
    model.set_precision(True)
    d_loss = torch.zeros(1, device="cuda")
    for i in range(args.warmup):
        model.train_step(d_in[i % POOL], d_tg[i % POOL], B, T, LR, CLIP, d_loss)
    model.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        model.train_step(d_in[i % POOL], d_tg[i % POOL], B, T, LR, CLIP, d_loss)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    model.profile_enable(True)
    model.profile_read(reset=True)
    for i in range(args.steps):
        model.train_step(d_in[i % POOL], d_tg[i % POOL], B, T, LR, CLIP, d_loss)
    g = model.profile_read(reset=True)["gemm"]
    model.profile_enable(False)
    model.set_precision(False)
    tf = g["flops"] / (g["ms"] * 1e-3) / 1e12 if g["ms"] > 0 else 0.0
    return {"metric": METRIC + " with bf16 GEMM operands", "value":
            round(B * T * args.steps / (ms * 1e-3), 1), "unit": UNIT,
            "ms_per_step": round(ms / args.steps, 3),
            "dtype": "bf16 GEMM operands (bf16 copies in memory), fp32 accumulate, fp32 master "
                     "weights and non-GEMM work",
            "gemm_ms_per_step": round(g["ms"] / args.steps, 3),
            "roofline": {"bound": "tensor", "kernel": "gemm_tf32x3 MODE 2 (bf16 tiles)",
                         "achieved": round(tf, 2), "peak": peaks["bf16_sust"],
                         "unit": "TFLOP/s", "frac": round(tf / peaks["bf16_sust"], 4)}}


def _finish(pg, model, dist_h):
    model.synchronize()
    model.close()
    if dist_h:
        dist_h.close()
    if pg:
        pg.destroy_process_group()


def run_reference(args, rank, world, local):
    if rank != 0:
        return
    import numpy as np
    import torch
    import oracle
    rdata = importlib.import_module("resonance-net_b200.data")
    base = {"impl": "reference", "metric": METRIC, "unit": UNIT}
    if args.model == "c5":
        print(json.dumps({**base, "metric": METRIC5, "unavailable":
                          "config 5 is not safely runnable on the reference: its per-layer cache "
                          "is sized from free memory (src/resonance_net.cpp:91-101) while forward "
                          "still uses it for N <= 64*seq_len (src/resonance_net.cpp:245)"}),
              flush=True)
        return
    if not oracle.ref_available():
        print(json.dumps({**base, "unavailable": "oracle/_ref/libref.so (reference CUDA build) "
                                                 "not built"}), flush=True)
        return
    torch.cuda.set_device(local)
    B, T = args.batch, args.seq
    cfg = oracle.make_config(**CFG)
    R = oracle.ref_lib()
    fd, path = tempfile.mkstemp(suffix=".bin")
    os.close(fd)
    rdata.write_checkpoint(path, cfg, rdata.init_params_normal(cfg, seed=1234))
    saved = os.dup(1)
    os.dup2(2, 1)  # the reference prints to stdout; keep ours to one JSON line
    try:
        h = R.ref_model_load(path.encode())
        toks, tgts = zipf_pool(rdata, B, T, seed=7)
        d_in = [torch.from_numpy(t).cuda() for t in toks]
        d_tg = [torch.from_numpy(t).cuda() for t in tgts]
        for i in range(args.warmup):
            R.ref_train_step_device(h, d_in[i % POOL].data_ptr(), d_tg[i % POOL].data_ptr(), B, T,
                                    ctypes.c_float(LR), ctypes.c_float(CLIP))
        torch.cuda.synchronize()
        clocks = ClockSampler(local)
        clocks.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks.mark(True)
        e0.record()
        for i in range(args.steps):
            R.ref_train_step_device(h, d_in[i % POOL].data_ptr(), d_tg[i % POOL].data_ptr(), B, T,
                                    ctypes.c_float(LR), ctypes.c_float(CLIP))
        e1.record()
        torch.cuda.synchronize()
        clocks.mark(False)
        ck = clocks.stop()
        ms = e0.elapsed_time(e1)
        dec = None if args.no_decode else reference_infer(R, h, torch, np)
        R.ref_model_destroy(h)
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
        os.unlink(path)
    v = round(B * T * args.steps / (ms * 1e-3), 1)
    out = {**base, "value": v, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "fp32 (cuBLAS SGEMM)",
           "data": "synthetic Zipf(1.1) byte tokens, N(0,0.02) weights",
           "config": {"workload": "train step, d512 L8 F1024 S1024 top2 V256",
                      "model": "ResonanceNet", "global_batch": B, "seq_len": T,
                      "parallelism": "dp1"},
           "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "cpu_baseline": {"value": v, "unit": UNIT, "cores": None, "kind": "reference",
                            "sample": "the reference has no CPU implementation; this is its own "
                                      "CUDA build (unmodified sources, sm_100a) timed on the "
                                      "same B200, full config"},
           "clocks": ck}
    if dec is not None:
        out["decode"] = dec
    print(json.dumps(out), flush=True)


def reference_infer(R, h, torch, np, prompt_len=5):
    """The reference's only inference path, as-is (src/main.cpp:266-384
    infer): batch 1, and for every generated token the context (prompt plus
    tokens so far, up to seq_len = 256) is uploaded and the WHOLE prefix is
    recomputed by ResonanceNet::forward; the last row's logits come back to
    the host. Greedy choice stands in for its host top-p sampling (host-side,
    not timed differently). Timed with CUDA events around the loop."""
    S = CFG["seq_len"]
    rng = np.random.default_rng(3)
    ctx = list(rng.integers(32, 127, size=prompt_len))
    logits = np.empty((S, CFG["vocab"]), np.float32)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    n = 0
    while len(ctx) < S:
        tok = np.ascontiguousarray(ctx, np.int32)
        R.ref_forward(h, tok.ctypes.data, 1, len(ctx), logits.ctypes.data)
        ctx.append(int(np.argmax(logits[len(ctx) - 1])))
        n += 1
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    return {"metric": "decode tok/s, batch 1, full-prefix recompute (reference infer path)",
            "value": round(n / (ms * 1e-3), 1), "unit": "tok/s", "tokens": n,
            "context": f"{prompt_len}-token prompt grown to {S} (the checkpoint's seq_len cap)",
            "ms_per_token": round(ms / n, 3)}


def run_op(args):
    """One operation in a loop at config-2 shapes through the C ABI (used for
    ncu captures of one kernel class); prints the device time per call."""
    import torch
    rnet = importlib.import_module("resonance-net_b200")
    torch.cuda.set_device(0)
    F32 = ctypes.c_float
    p = rnet.ptr
    B, T, D = args.batch, args.seq, CFG["d_model"]
    N = B * T
    g = torch.Generator(device="cuda").manual_seed(0)
    rnet.call("rnet_gemm_set_cta_group", args.cg)

    def rnd(*shape, scale=1.0):
        return torch.randn(*shape, device="cuda", generator=g) * scale

    def z(*shape):
        return torch.zeros(*shape, device="cuda")

    if args.op == "gemm":
        M, Nn, K = args.m, args.n, args.k
        A = rnd(K, M) if args.amn else rnd(M, K)
        Bm = rnd(K, Nn) if args.bmn else rnd(Nn, K)
        C = z(M, Nn)
        lda, ldb = (M if args.amn else K), (Nn if args.bmn else K)
        R = rnd(M, Nn)
        fn = lambda: rnet.call("rnet_gemm_f32", M, Nn, K, p(A), lda, args.amn, p(Bm), ldb,
                               args.bmn, p(C), Nn, p(R), Nn, args.epi, F32(1.0), None)
        work = (f"gemm M={M} N={Nn} K={K} a_mn={args.amn} b_mn={args.bmn} cg={args.cg} "
                f"epi={args.epi}")
    elif args.op == "gemm16":
        M, Nn, K = args.m, args.n, args.k
        A = (rnd(K, M) if args.amn else rnd(M, K)).bfloat16()
        Bm = (rnd(K, Nn) if args.bmn else rnd(Nn, K)).bfloat16()
        C = z(M, Nn)
        lda, ldb = (M if args.amn else K), (Nn if args.bmn else K)
        R = rnd(M, Nn)
        fn = lambda: rnet.call("rnet_gemm_bf16", M, Nn, K, p(A), lda, args.amn, p(Bm), ldb,
                               args.bmn, p(C), Nn, p(R), Nn, args.epi, F32(1.0), None, None)
        work = (f"gemm bf16 M={M} N={Nn} K={K} a_mn={args.amn} b_mn={args.bmn} cg={args.cg} "
                f"epi={args.epi}")
    elif args.op in ("scan_fwd", "scan_bwd"):
        x = rnd(N, D)
        Wz, Wh = rnd(D, D, scale=D ** -0.5), rnd(D, D, scale=D ** -0.5)
        bz, bh = rnd(D), rnd(D)
        y, zc, h = z(N, D), z(N, D), z(N, D)
        fwd = lambda: rnet.call("rnet_min_gru_forward", p(x), p(y), p(Wz), p(Wh), p(bz), p(bh),
                                p(zc), p(h), B, T, D, None)
        fwd()
        if args.op == "scan_fwd":
            fn = fwd
        else:
            dy, dx = rnd(N, D), z(N, D)
            gz, gh, gbz, gbh = z(D, D), z(D, D), z(D), z(D)
            fn = lambda: rnet.call("rnet_min_gru_backward", p(dy), p(x), p(Wz), p(Wh), p(bz),
                                   p(bh), p(zc), p(h), p(dx), p(gz), p(gh), p(gbz), p(gbh), B, T,
                                   D, None)
        work = f"min_gru {args.op[5:]} B={B} T={T} D={D}"
    elif args.op in ("conv_fwd", "conv_bwd"):
        x = rnd(N, D)
        w3, w7, w15, mix = rnd(3, D), rnd(7, D), rnd(15, D), rnd(D, D, scale=D ** -0.5)
        y, cb = z(N, D), z(3, N, D)
        fwd = lambda: rnet.call("rnet_causal_conv_forward", p(x), p(y), p(w3), p(w7), p(w15),
                                p(mix), p(cb), B, T, D, None)
        fwd()
        if args.op == "conv_fwd":
            fn = fwd
        else:
            dy, dx = rnd(N, D), z(N, D)
            gw = [z(3, D), z(7, D), z(15, D), z(D, D)]
            fn = lambda: rnet.call("rnet_causal_conv_backward", p(dy), p(x), p(w3), p(w7),
                                   p(w15), p(mix), p(cb), p(dx), *(p(a) for a in gw), B, T, D, 1,
                                   None)
        work = f"causal_conv {args.op[5:]} B={B} T={T} D={D}"
    elif args.op in ("swiglu_fwd", "swiglu_bwd"):
        Fd = CFG["d_ff"]
        x = rnd(N, D)
        gu = rnd(2 * Fd, D, scale=D ** -0.5)  # gate|up contiguous -> paired GEMM
        down = rnd(D, Fd, scale=Fd ** -0.5)
        y, gc, uc = z(N, D), z(N, Fd), z(N, Fd)
        gate, up = gu[:Fd], gu[Fd:]
        fwd = lambda: rnet.call("rnet_swiglu_forward", p(x), p(y), p(gate), p(up), p(down),
                                p(gc), p(uc), N, D, Fd, None)
        fwd()
        if args.op == "swiglu_fwd":
            fn = fwd
        else:
            dy, dx = rnd(N, D), z(N, D)
            gg, gup, gd = z(Fd, D), z(Fd, D), z(D, Fd)
            fn = lambda: rnet.call("rnet_swiglu_backward", p(dy), p(x), p(gate), p(up), p(down),
                                   p(gc), p(uc), p(dx), p(gg), p(gup), p(gd), N, D, Fd, None)
        work = f"swiglu {args.op[7:]} N={N} D={D} F={Fd} cg={args.cg}"
    elif args.op in ("rms_fwd", "rms_bwd"):
        x, w, y, ri = rnd(N, D), rnd(D), z(N, D), z(N)
        fwd = lambda: rnet.call("rnet_rms_norm_forward", p(x), p(w), p(y), p(ri), N, D,
                                F32(1e-6), None)
        fwd()
        if args.op == "rms_fwd":
            fn = fwd
        else:
            dy, dx, dw = rnd(N, D), z(N, D), z(D)
            fn = lambda: rnet.call("rnet_rms_norm_backward", p(dy), p(x), p(w), p(ri), p(dx),
                                   p(dw), N, D, None)
        work = f"rms_norm {args.op[4:]} N={N} D={D}"
    else:
        raise SystemExit(f"unknown --op {args.op}")
    for _ in range(max(1, args.warmup)):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps({"op": args.op, "workload": work,
                      "ms_per_call": round(e0.elapsed_time(e1) / args.steps, 4)}), flush=True)


def decode_measure(rnet, rdata, torch, pg, rank, world, local, streams, T, G, warmup, steps):
    """Config 4 on this rank's share of `streams`: prefill of Zipf-byte prompts of
    length T through the chunked scan, then G greedy decode steps carrying the
    O(1) recurrent state (graph-replayed step). Returns the result dict on
    rank 0 (None elsewhere)."""
    import numpy as np
    M = streams // world
    cfg = rnet.ModelConfig.make(d_model=CFG["d_model"], n_layers=CFG["n_layers"],
                                d_ff=CFG["d_ff"], n_slots=CFG["n_slots"], top_k=CFG["top_k"],
                                vocab=CFG["vocab"], seq_len=T)
    model = rnet.Model(cfg, device=local, reference_init=False)
    model.set_params(rdata.init_params_normal(cfg, seed=1234))
    dec = rnet.Decoder(model, M)
    tok, _ = rdata.zipf_tokens(M, T, seed=11 + rank)
    h_tok = torch.from_numpy(np.ascontiguousarray(tok.reshape(-1))).pin_memory()
    d_tok = h_tok.cuda()
    d_out = torch.zeros(G, M, dtype=torch.int32, device="cuda")
    h_out = torch.zeros(G, M, dtype=torch.int32).pin_memory()
    stream = torch.cuda.ExternalStream(model.stream())

    def barrier():
        torch.cuda.synchronize()
        if pg:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not pg:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, reps):
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        e1.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / reps

    reps = max(1, min(steps, 3))
    for _ in range(max(1, warmup)):
        dec.prefill(d_tok, T)
    dec.generate(8, d_out, True)  # captures the decode-step graph
    n0 = rnet.kernel_launches()
    clocks = ClockSampler(local) if rank == 0 else ClockSampler(None)
    clocks.start()
    ms_prefill = timed(lambda: dec.prefill(d_tok, T), reps)
    # untimed decode steps first: the power cap's running average (and the
    # clocks it sets) then reflect the decode steps, not the prefill before
    dec.generate(G, d_out, True)
    clocks.mark(True)  # the clocks reported are the decode steps' own
    ms_decode = timed(lambda: dec.generate(G, d_out, True), 1)
    clocks.mark(False)
    ck = clocks.stop()
    launches = rnet.kernel_launches() - n0

    # end to end: prompt from pinned host memory, generated tokens back to host
    def e2e():
        d_tok.copy_(h_tok, non_blocking=True)
        dec.prefill(d_tok, T)
        dec.generate(G, d_out, True)
        h_out.copy_(d_out, non_blocking=True)
    ms_e2e = timed(e2e, 1)
    dec.close()
    model.close()
    if rank != 0:
        return None
    peaks = measured_peaks()
    # one decode step streams every weight once and reads + writes each
    # stream's state (14 conv rows + h per layer)
    weight_bytes = 4.0 * model.num_params
    state_bytes = 2 * 4.0 * M * CFG["n_layers"] * 15 * CFG["d_model"]
    step_ms = ms_decode / G
    hbm_gbs = (weight_bytes + state_bytes) / (step_ms * 1e-3) / 1e9
    # forward FLOPs per token: 10 D^2 + 2 D S + 6 D F per layer + 2 D V (head)
    D_, F_, S_, V_ = CFG["d_model"], CFG["d_ff"], CFG["n_slots"], CFG["vocab"]
    flops_tok = CFG["n_layers"] * (10 * D_ * D_ + 2 * D_ * S_ + 6 * D_ * F_) + 2 * D_ * V_
    tflops = M * flops_tok / (step_ms * 1e-3) / 1e12
    return {
        "metric": f"decode tok/s (d512 L8, {streams} streams x {G} greedy steps after a "
                  f"{T}-token prefill)",
        "value": round(streams * G / (ms_decode * 1e-3), 1), "unit": "tok/s",
        "n_gpus": world, "ms_per_step": round(step_ms, 4),
        "dtype": "fp32 (3xTF32 tcgen05)",
        "config": {"workload": "config 4: prefill + greedy decode", "model": "ResonanceNet d512 L8",
                   "streams": streams, "streams_per_gpu": M, "prompt": T, "decode_steps": G,
                   "parallelism": f"streams sharded over {world} GPU(s), no collective"},
        "prefill": {"value": round(streams * T / (ms_prefill * 1e-3), 1), "unit": "tok/s",
                    "ms": round(ms_prefill, 3)},
        "e2e": {"value": round(streams * G / (ms_e2e * 1e-3), 1), "unit": "generated tok/s",
                "note": "prompt H2D + prefill + decode + tokens D2H",
                "h2d_bytes_per_step": int(4 * M * T), "d2h_bytes_per_step": int(4 * M * G)},
        "gpu_launches": int(launches),
        # at 256 streams a step is compute-bound in fp32 (3xTF32 ceiling =
        # bf16 peak / 6); the weight + state stream is reported beside it
        "roofline": {"bound": "tensor", "kernel": "decode step (all kernels of one graph replay)",
                     "achieved": round(tflops, 2), "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": round(tflops / peaks["bf16"], 4),
                     "ceiling_3xtf32": round(peaks["bf16"] / 6, 1),
                     "frac_of_3xtf32_ceiling": round(tflops / (peaks["bf16"] / 6), 4),
                     "flops_per_step": M * flops_tok,
                     "hbm": {"achieved_GBps": round(hbm_gbs, 1),
                             "frac": round(hbm_gbs / peaks["hbm"], 4),
                             "bytes_per_step": weight_bytes + state_bytes}},
        "reference_note": "the reference has no recurrent decode: its only inference path "
                          "(src/main.cpp:266-384 infer) recomputes the whole prefix at batch 1 "
                          "for every token; bench.py --impl reference reports that reading "
                          "as-is in its own line's 'decode' object",
        "clocks": ck,
    }


def run_decode(args, rank, world, local):
    """Config 4 alone (--decode): strong scaling of a fixed stream count."""
    import torch
    rnet = importlib.import_module("resonance-net_b200")
    rdata = importlib.import_module("resonance-net_b200.data")
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        pg = dist
    out = decode_measure(rnet, rdata, torch, pg, rank, world, local, args.streams, args.prompt,
                         args.gen, args.warmup, args.steps)
    if out is not None:
        out.update({"steps": 1, "warmup": args.warmup, "higher_is_better": True,
                    "scaling": "strong", "vs_baseline": None,
                    "data": "synthetic Zipf(1.1) byte prompts, N(0,0.02) weights"})
        print(json.dumps(out), flush=True)
    if pg:
        pg.destroy_process_group()


def main():
    args = parse()
    if args.model == "c5":
        args.batch = args.batch or 16
        args.seq = args.seq or 2048
        args.bf16 = True
        args.no_decode = True
        args.no_cpu_baseline = True
    else:
        args.batch = args.batch or 64
        args.seq = args.seq or 256
    rank, world, local = env_rank()
    if args.op:
        run_op(args)
        return
    if args.decode:
        run_decode(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference(args, rank, world, local)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
