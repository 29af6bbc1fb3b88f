"""Benchmark of the flow-matching denoise loop (p50 denoise-loop latency at bs=1;
action chunks/s at bs=64 across 1-8 B200).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--model pi05|molmoact2]
                  [--impl ours|reference] [--wfmt bf16|fp8] [--prefix P]

Default workload: pi0.5 C1. --model molmoact2 runs C3 (configs[3]: 36 DiT
blocks, width 768, T=30 with 6 valid action dims, 493 context tokens, 10 steps, seed 1).
--wfmt fp8 streams the pi0.5 GEMM weights as E4M3 codes with per-row scales (
C4, with --prefix 1736); the codes are made on the GPU by flashact_b200.quant.

One "step" = one call of the public API that runs the whole 10-step x 18-layer Euler loop for
the rank's batch (fa_sample_actions). Synthetic inputs follow BASELINE.json configs[1]
(C1): seeded N(0, 0.02) weights, N(0, 1) prefix KV of 968 tokens and noise, T=50, AD=32.
Under torchrun every rank drives one GPU with its own engine and its own batch shard; the only
inter-rank traffic is the barrier around the timed region and the max-over-ranks reduction of
the measured times (no collective in the loop).

--impl reference times the reference's CPU path on the host cores: openpi's PyTorch model is
not available, so the CPU fp32 restatement in oracle/ stands in for it.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L, T, AD, LP, NSTEPS = 18, 50, 32, 968, 10
W_BYTES_BF16 = 622_854_144            # expert GEMM weights streamed per Euler step (bf16)
PI05_ROWS = 2560 + 1024 + 8192 + 1024  # packed GEMM rows per layer (QKV, O, gate/up, down)
W_BYTES_FP8 = W_BYTES_BF16 // 2 + L * PI05_ROWS * 4  # E4M3 codes + fp32 row scales: 312,348,672
KV_BYTES = 2 * L * LP * 256 * 2       # prefix K+V read per Euler step per observation (bf16)
GEMM_PARAMS = W_BYTES_BF16 // 2
# MolmoAct2 C3: 36 blocks x (qkv 2304x768 + 3 x 768x768 + gate/up 2x3072x768 + down 768x3072) bf16
MA2_L, MA2_T, MA2_LK = 36, 30, 493
MA2_W_BYTES = MA2_L * (2304 * 768 + 3 * 768 * 768 + 2 * 3072 * 768 + 768 * 3072) * 2  # 764,411,904
MA2_BIAS_BYTES = MA2_L * (2304 + 3 * 768 + 2 * 3072 + 768) * 4
MA2_KV_BYTES = 2 * MA2_L * MA2_LK * 768 * 2  # cross-attention K+V per Euler step per observation


# DRAM bytes (read + write) of one megakernel launch on the bench workload, from one ncu capture
# of `bench.py [--model molmoact2] --steps 1 --warmup 3 --no-cpu-baseline` (metrics
# dram__bytes_read.sum and dram__bytes_write.sum, -k regex:<kernel> -s 3 -c 1; summaries kept
# under profiles/).
NCU_TRAFFIC = {("pi05", 1): 6_246_001_408 + 3_208_704, ("molmoact2", 1): 7_739_515_904 + 3_610_112,
               ("pi05-fp8", 1): 3_134_528_512 + 3_190_016}


def set_shape(layers, euler_steps, prefix=0):
    """Smaller cases for profiling (--layers / --euler-steps) and the pi0.5 prefix length
    (--prefix); the defaults are the BASELINE ones."""
    global L, NSTEPS, W_BYTES_BF16, W_BYTES_FP8, KV_BYTES, GEMM_PARAMS, MA2_L, MA2_W_BYTES, MA2_BIAS_BYTES, MA2_KV_BYTES
    global LP
    if prefix:
        KV_BYTES = KV_BYTES // LP * prefix
        LP = prefix
    if layers:
        W_BYTES_BF16 = W_BYTES_BF16 // L * layers
        W_BYTES_FP8 = W_BYTES_FP8 // L * layers
        KV_BYTES = KV_BYTES // L * layers
        GEMM_PARAMS = W_BYTES_BF16 // 2
        MA2_W_BYTES = MA2_W_BYTES // MA2_L * layers
        MA2_BIAS_BYTES = MA2_BIAS_BYTES // MA2_L * layers
        MA2_KV_BYTES = MA2_KV_BYTES // MA2_L * layers
        L = MA2_L = layers
    if euler_steps:
        NSTEPS = euler_steps


def algorithmic_bytes(batch, model="pi05", wfmt="bf16"):
    if model == "molmoact2":
        return NSTEPS * (MA2_W_BYTES + MA2_BIAS_BYTES + batch * MA2_KV_BYTES)
    return NSTEPS * ((W_BYTES_FP8 if wfmt == "fp8" else W_BYTES_BF16) + batch * KV_BYTES)


def algorithmic_flops(batch):
    attn = 4 * T * 8 * (LP + T) * 256 * L
    return batch * NSTEPS * (2 * T * GEMM_PARAMS + attn)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 100 ms from before the warm-up so that
    the sampler is running when the timed region starts; summary() keeps the samples received
    between mark_start() and mark_end() (the timed region, host clock)."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 6:
                self.rows.append((time.monotonic(), parts))

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()
        time.sleep(0.15)  # the sample taken just before the end is still in the pipe

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = [r for t, r in self.rows if self.t0 is not None and self.t0 <= t <= (self.t1 or t) + 0.15]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[2:]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group(backend=backend, device_id=torch.device("cuda", local))
        else:
            dist.init_process_group(backend=backend)
    return world, rank, local


def max_over_ranks(x, world, device):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_chunk(case, threads, model="pi05", mods=None):
    """Times one whole 10-step bs=1 action chunk of the CPU fp32 oracle on the host cores (seconds)."""
    torch.set_num_threads(threads)
    if model == "molmoact2":
        from oracle import molmoact2_oracle as M
        one = M.Ma2Case(**{**case.__dict__, "B": 1})
        t0 = time.perf_counter()
        M.flow(one, max_obs=1)
        return time.perf_counter() - t0
    from oracle import pi05_oracle as O
    one = O.Pi05Case(**{**case.__dict__, "B": 1})
    mods, mod_final = mods
    t0 = time.perf_counter()
    O.denoise(one, mods=mods, mod_final=mod_final)
    return time.perf_counter() - t0


def cpu_chunks(case, threads, model, warmup, timed):
    """`warmup` untimed then `timed` timed whole chunks; the conditioning (modulation precompute,
    outside the denoise loop in both arms) is computed once before."""
    mods = None
    if model != "molmoact2":
        from oracle import pi05_oracle as O
        mods = O.modulations(case.w, case.L, case.num_steps)
    for _ in range(warmup):
        cpu_chunk(case, threads, model, mods)
    return [cpu_chunk(case, threads, model, mods) for _ in range(timed)]


def make_case(model, seed, B):
    if model == "molmoact2":
        from oracle import molmoact2_oracle as M
        return M.make_case(seed=1 + seed, L=MA2_L, T=MA2_T, Lk=MA2_LK, B=B, num_steps=NSTEPS)
    from oracle import pi05_oracle as O
    return O.make_case(seed=seed, L=L, T=T, AD=AD, Lp=LP, B=B, num_steps=NSTEPS)


def shard_case(model, case, lo, hi):
    """Observations [lo, hi) of a seeded global case (weights shared)."""
    import copy
    sub = copy.copy(case)
    sub.B = hi - lo
    sub.noise = case.noise[lo:hi]
    if model == "molmoact2":
        sub.kctx, sub.vctx = case.kctx[lo:hi], case.vctx[lo:hi]
    else:
        sub.k, sub.v, sub.valid_len = case.k[lo:hi], case.v[lo:hi], case.valid_len[lo:hi]
    return sub


WORKLOAD = {
    "pi05": "pi0.5 action-expert denoise, BASELINE configs[1] (C1): 18 layers, width 1024, 8q/1kv heads x 256, "
            "GeGLU 4096, T=50, AD=32, prefix 968, 10 Euler steps",
    "molmoact2": "MolmoAct2 action-expert flow, BASELINE configs[3] (C3): 36 DiT blocks, width 768, 8 heads x 96, "
                 "SiLU MLP 3072, T=30 (6 valid action dims), AD=32, cross-attention context 493, 10 Euler steps",
}
METRICS = {
    "pi05": "pi0.5 10-step denoise throughput, action chunks/s (bs per GPU; ms_per_step = mean latency of one chunk batch)",
    "molmoact2": "MolmoAct2 10-step denoise throughput, action chunks/s (bs per GPU; ms_per_step = mean latency of one chunk batch)",
}


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    case = make_case(args.model, 0, 1)
    times = cpu_chunks(case, threads, args.model, max(args.warmup, 0), args.steps)
    chunk_s = statistics.mean(times)  # whole 10-step chunks of one observation, each timed
    value = 1.0 / chunk_s
    line = {"metric": METRICS[args.model], "value": value, "unit": "chunks/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": chunk_s * 1000,
            "p50_ms": statistics.median(times) * 1000, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD[args.model] + " (CPU fp32 restatement of the reference path)",
                       "batch_per_rank": 1},
            "cpu_baseline": {"value": value, "unit": "chunks/s", "cores": threads, "kind": "port",
                             "sample": "each step = one whole 10-step bs=1 chunk, timed on its own"},
            "e2e": {"value": value, "unit": "chunks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)



def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1, help="observations per GPU (weak scaling)")
    ap.add_argument("--global-batch", type=int, default=0,
                    help="observations in total, sharded across the GPUs (strong scaling; BASELINE C2 = 64)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="pi05", choices=["pi05", "molmoact2"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="profiling only: fewer expert layers than the config")
    ap.add_argument("--euler-steps", type=int, default=0, help="profiling only: fewer Euler steps than the config")
    ap.add_argument("--wfmt", default="bf16", choices=["bf16", "fp8"],
                    help="pi0.5 weight stream: bf16, or E4M3 codes + per-row scales (BASELINE C4)")
    ap.add_argument("--prefix", type=int, default=0, help="pi0.5 prefix tokens (default 968; C4 uses 1736)")
    args = ap.parse_args()
    if args.model == "molmoact2" and (args.wfmt != "bf16" or args.prefix):
        ap.error("--wfmt / --prefix apply to pi0.5 only")
    set_shape(args.layers, args.euler_steps, args.prefix)
    if args.impl == "reference":  # host-CPU arm: rank 0 alone works, no process group needed
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup()

    from flashact_b200 import MolmoAct2ActionExpert, Pi05ActionExpert
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.global_batch > 0:  # one global batch, contiguous shards (flashact_b200.sharding)
        from flashact_b200.sharding import shard_range
        lo, hi = shard_range(args.global_batch, world, rank)
        B = hi - lo
        full = make_case(args.model, 0, args.global_batch)
        case = shard_case(args.model, full, lo, hi)
    else:
        B = args.batch
        case = make_case(args.model, rank, B)  # each rank: its own observations (prefix KV / context, noise)
    if args.model == "molmoact2":
        eng = MolmoAct2ActionExpert(case.w, case.mods, case.mod_final, num_layers=MA2_L, horizon=MA2_T, action_dim=AD,
                                    valid_action_dim=case.adim, max_context=MA2_LK, max_batch=B, num_steps=NSTEPS,
                                    device=local, rope_cos=case.rope_cos, rope_sin=case.rope_sin)
        eng.bind_context(case.kctx, case.vctx, [MA2_LK] * B)
    elif args.wfmt == "fp8":  # E4M3 codes + row scales made on the GPU (flashact_b200.quant)
        from flashact_b200.pi05 import quantized_weights
        w, qs = quantized_weights(case.w, dev)
        eng = Pi05ActionExpert(w, num_layers=L, horizon=T, action_dim=AD, max_prefix=LP, max_batch=B,
                               num_steps=NSTEPS, device=local, wfmt="fp8", qscales=qs)
        eng.bind_prefix_kv(case.k.to(torch.bfloat16).to(dev), case.v.to(torch.bfloat16).to(dev), case.valid_len)
    else:
        eng = Pi05ActionExpert(case.w, num_layers=L, horizon=T, action_dim=AD, max_prefix=LP, max_batch=B,
                               num_steps=NSTEPS, device=local)
        eng.bind_prefix_kv(case.k.to(torch.bfloat16).to(dev), case.v.to(torch.bfloat16).to(dev), case.valid_len)
    noise_d = case.noise.to(dev)
    out_d = torch.empty_like(noise_d)
    noise_h = case.noise.clone().pin_memory()
    out_h = torch.empty_like(noise_h).pin_memory()
    stream = torch.cuda.current_stream()

    clk = ClockSampler(local).__enter__()  # running before the timed region starts
    for _ in range(max(args.warmup, 3)):
        eng.sample_actions(noise_d, out_d)

    # device-resident inputs: kernel + in-HBM copies only
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    clk.mark_start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for e0, e1 in ev:
        e0.record()
        eng.sample_actions(noise_d, out_d, sync=False)
        e1.record()
    t_end.record()
    torch.cuda.synchronize()
    clk.mark_end()
    clk.__exit__()
    eng.sync()
    barrier(world)
    total_ms = max_over_ranks(t_start.elapsed_time(t_end), world, dev)
    per = sorted(a.elapsed_time(b) for a, b in ev)
    p50 = per[len(per) // 2]
    launches = args.steps * eng.launch_count()

    # end to end through the public API with pinned host buffers (H2D noise + D2H actions)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.sample_actions(noise_h, out_h, sync=False)
    e1.record()
    torch.cuda.synchronize()
    eng.sync()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    barrier(world)

    ms_step = total_ms / args.steps
    total_batch = args.global_batch if args.global_batch > 0 else world * B
    value = total_batch * 1000.0 / ms_step
    e2e_value = total_batch * 1000.0 / (e2e_ms / args.steps)
    if world > 1 and args.global_batch > 0:  # the one data exchange: gather the action chunks (untimed)
        from flashact_b200.sharding import gather_actions
        gathered = gather_actions(out_d, args.global_batch)
        assert gathered.shape[0] == args.global_batch
    peak, peak_kind = measured_peaks()
    achieved = algorithmic_bytes(B, args.model, args.wfmt) / (ms_step * 1e-3) / 1e9
    workload = WORKLOAD[args.model]
    if args.prefix:
        workload = workload.replace("prefix 968", f"prefix {LP}")
    if args.wfmt == "fp8":
        workload = workload.replace("configs[1] (C1)", "configs[4] (C4, FP8 E4M3 weights with per-row scales)")
    line = {
        "metric": METRICS[args.model], "value": value, "unit": "chunks/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "p50_ms": p50, "min_ms": per[0],
        "higher_is_better": True, "scaling": "strong" if args.global_batch > 0 else "weak", "vs_baseline": None,
        "dtype": "bf16" if args.wfmt == "bf16" else "e4m3 weights x bf16 activations, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) prefix KV and noise)",
        "config": {"workload": workload + (f" [profiling case: {L} layers, {NSTEPS} Euler steps]"
                                                       if args.layers or args.euler_steps else ""),
                   "batch_per_gpu": B, "global_batch": total_batch, "parallelism": f"batch shards x{world}",
                   "l2": "no flush: the bf16 weight stream per Euler step (623 MB pi0.5, 764 MB MolmoAct2) exceeds "
                         "the 126 MB L2"},
        "e2e": {"value": e2e_value, "unit": "chunks/s", "h2d_bytes_per_step": int(noise_h.numel() * 4),
                "d2h_bytes_per_step": int(out_h.numel() * 4)},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": (NCU_TRAFFIC.get((args.model + ("-fp8" if args.wfmt == "fp8" else ""), B))
                                 if not (args.layers or args.euler_steps or args.prefix) else None),
                     "algorithmic_bytes_per_launch": algorithmic_bytes(B, args.model, args.wfmt),
                     "note": f"achieved = N x ({args.wfmt} weights + B x prefix KV) per launch / mean launch time"},
        "clocks": clk.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        ref_case = case if B == 1 else make_case(args.model, 0, 1)
        times = cpu_chunks(ref_case, threads, args.model, 1, 3)
        line["cpu_baseline"] = {"value": 1.0 / statistics.median(times), "unit": "chunks/s", "cores": threads,
                                "kind": "port",
                                "sample": "p50 of 3 whole 10-step bs=1 chunks of the CPU fp32 oracle, after 1 warm-up "
                                          f"(chunk seconds: {', '.join(f'{t:.3f}' for t in times)})"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
