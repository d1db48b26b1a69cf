"""Benchmark: GKR matmul-sumcheck prove time per layer on B200.

Workload: A = 64 x 5120 activations, B = 5120 x 13824
weights (Qwen2.5-14B MLP up-projection), int8 values embedded in M31, MLEs
padded to 64 x 8192 and 8192 x 16384.  One step = one
``reduce_matmul_layer_with_backend`` (gkr/prover.rs:5959-6073): transcript
seeding, the W.eq(r) restrictions, 13 sumcheck rounds with the Poseidon
channel on the host, and the final evaluation mixes.

Multi-GPU: one process per GPU (torchrun).  The headline value keeps N = 1
comparable: each rank proves its own independent C2 layer (different seeded
weights), the timed region is bracketed by barriers and the max over ranks is
reported ("scaling": "weak").  The same JSON line carries, under "sharded",
the splits of one proof across the N GPUs, each timed the same way:
  c5           one 2^30-element product sumcheck (config 5) with the MLEs split by
               the low index bits; the 12 round words are added across the GPUs
               inside the round kernels and the folded vectors are gathered by
               peer stores (the peer mesh); strong scaling;
  c5_sweep     the same split proof at 2^20, 2^22, ..., 2^28 elements (config 5's
               sweep; 2^30 is c5), each with its HBM fraction per GPU;
  c2_colsplit  one C2 layer with B split by column blocks, the partial words
               exchanged by peer stores; strong scaling;
and "parity_vs_1gpu": rank 0 recomputes both proofs on one GPU (untimed) and
compares them bit for bit.  The reference arm (--impl reference) times the CPU
restatement of the reference prover (the oracle, materialised restriction as
in engine/src/backend.rs:110-197) on the host cores, rank 0 only.
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "stwo-ml_b200"))
sys.path.insert(0, str(ROOT / "tests"))

M, K, N = 64, 5120, 13824
METRIC = "matmul-sumcheck prove s/layer (config 2: 64x5120 . 5120x13824 M31, padded 64x8192 . 8192x16384)"
WORKLOAD = "C2 batched matmul sumcheck, Qwen2.5-14B MLP up-proj at 64 tokens"


def log2(x):
    return x.bit_length() - 1


def npow2(x):
    return 1 << max(0, (x - 1).bit_length())


PM, PK, PN = npow2(M), npow2(K), npow2(N)
# MLE elements folded per layer: the restriction folds every real (unpadded) element of A
# and B -- the zero padding is never read -- and the rounds fold both length-pk vectors.
ELEMS_FOLDED = M * K + K * N + 2 * (2 * PK - 2)


def make_inputs(rank):
    from helpers import int_matrix_m31

    a = int_matrix_m31(M, K, 1000 + 2 * rank)
    b = int_matrix_m31(K, N, 1001 + 2 * rank)
    return a, b


def seeded_channel_state(Z, rank):
    ch = Z.PoseidonChannel()
    seed = int.from_bytes(bytes(range(32)), "big") % Z.STARK_P
    ch.mix_felt(seed)
    ch.mix_u64(rank)
    point = ch.draw_qm31s(log2(PM) + log2(PN))
    return ch, point


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[4 + i] == "Active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic_per_launch():
    """dram bytes per restrict_cols launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "restrict_cols_c2.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":")[1].split()[0])
    return None


def host_cores():
    """Every host core this process may run on, before any narrowing to the GPU-local CPUs."""
    return len(HOST_AFFINITY) if HOST_AFFINITY else (os.cpu_count() or 1)


HOST_AFFINITY = set(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else set()


def cpu_reference_layer(threads):
    """One C2 layer through the oracle's materialised (reference) CPU path, its threads spread
    over all host cores (the process affinity is widened back for the call)."""
    import oracle_lib as O

    a, b = make_inputs(0)
    rng = np.random.default_rng(0)
    r_i = rng.integers(0, (1 << 31) - 1, (log2(PM), 4), dtype=np.uint32)
    r_j = rng.integers(0, (1 << 31) - 1, (log2(PN), 4), dtype=np.uint32)
    ch = O.new_channel()
    narrowed = set(os.sched_getaffinity(0)) if HOST_AFFINITY else set()
    if HOST_AFFINITY and narrowed != HOST_AFFINITY:
        os.sched_setaffinity(0, HOST_AFFINITY)
    try:
        t0 = time.perf_counter()
        O.reduce_matmul_layer(a, b, r_i, r_j, ch, mode=0, nthreads=threads)
        return time.perf_counter() - t0
    finally:
        if HOST_AFFINITY and narrowed != HOST_AFFINITY:
            os.sched_setaffinity(0, narrowed)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = host_cores()
    for _ in range(args.warmup):
        cpu_reference_layer(threads)
    times = [cpu_reference_layer(threads) for _ in range(args.steps)]
    s_per_layer = float(np.mean(times))
    line = {
        "impl": "reference", "metric": METRIC, "value": s_per_layer, "unit": "s/layer", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": s_per_layer * 1e3, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "u32 (M31/QM31 integer)", "data": "synthetic",
        "config": {"workload": WORKLOAD, "m": M, "k": K, "n": N, "l2": "inputs larger than L2 (B = 283 MB)"},
        "cpu_baseline": {"value": s_per_layer, "unit": "s/layer", "cores": threads, "kind": "port",
                         "sample": "one full C2 layer per step through the C restatement of the reference CPU "
                                   "prover (materialised pad + MLE + restrict_mle, backend.rs:110-197)"},
        "e2e": {"value": s_per_layer, "unit": "s/layer", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "mle_elems_folded_per_s_per_gpu": ELEMS_FOLDED / s_per_layer,
    }
    print(json.dumps(line), flush=True)


def bind_to_gpu_cpus(dev):
    """Pin this rank's process to the CPUs NVML reports as local to its GPU: the round loop
    spins on mapped host memory and its pinned buffers are allocated near the running CPU."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(dev)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, 16)
        cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception:
        return None


def run_b200(args):
    import torch
    import torch.distributed as dist

    import zkml_b200 as Z

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.cuda.current_device()
    if world > 1:  # one rank alone keeps every host CPU: the packed upload of B runs on them
        bind_to_gpu_cpus(dev)
        # several ranks share the host's memory bandwidth, which packing spends more of than
        # the plain copy (it reads every word on the CPUs): B goes over as words
        os.environ.setdefault("ZKML_PACK_H2D", "0")
    stream = torch.cuda.current_stream()
    ctx = Z.Context(dev)
    ctx.set_stream(stream.cuda_stream)
    backend = Z.GpuBackend.__new__(Z.GpuBackend)
    backend.ctx = ctx

    a, b = make_inputs(rank)
    ta = torch.from_numpy(a.view(np.int32)).cuda()
    tb = torch.from_numpy(b.view(np.int32)).cuda()
    # pinned host copies for the end-to-end leg
    ha = torch.from_numpy(a.view(np.int32)).pin_memory()
    hb = torch.from_numpy(b.view(np.int32)).pin_memory()
    A_dev, B_dev = Z.M31Matrix(M, K, ta), Z.M31Matrix(K, N, tb)
    A_host, B_host = Z.M31Matrix(M, K, ha), Z.M31Matrix(K, N, hb)
    ch0, point = seeded_channel_state(Z, rank)
    # true claim: p(0) + p(1) of round 0 = sum_k f_a f_b (evaluated once, untimed)
    probe = backend.reduce_matmul_layer(A_dev, B_dev, point[:log2(PM)], point[log2(PM):], PK, ch0.clone())
    rp = probe.round_polys[0]
    P = Z.M31_P
    claim = ((2 * rp.c0.astype(np.int64) + rp.c1 + rp.c2) % P).astype(np.uint32)

    def step(Amat, Bmat):
        ch = ch0.clone()
        return Z.reduce_matmul_layer_with_backend(Z.GKRClaim(point, claim), Amat, Bmat, M, K, N, ch, backend)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def timed(Amat, Bmat, profile):
        for _ in range(args.warmup):
            step(Amat, Bmat)
        if profile:
            ctx.enable_timing(True, classes=["restrict_cols"])
        barrier()
        l0 = ctx.kernel_launches()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                step(Amat, Bmat)
            e1.record(stream)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        launches = ctx.kernel_launches() - l0
        kt = ctx.kernel_time("restrict_cols") if profile else (0.0, 0)
        if profile:
            ctx.enable_timing(False)
        rank_ms = [ms]
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            rank_ms = [float(p.item()) for p in parts]
            ms = max(rank_ms)
            lt = torch.tensor([launches], device="cuda", dtype=torch.int64)
            dist.all_reduce(lt)
            launches = int(lt.item())
        barrier()
        timed.rank_ms = rank_ms
        return ms, launches, kt, clk.summary()

    ms, launches, (rc_ms, rc_n), clocks = timed(A_dev, B_dev, profile=True)
    rank_ms = timed.rank_ms
    if args.headline_only:
        args.no_sharded = True
        ms_e2e = float("nan")
        h2d_step = 4 * (M * K + K * N)
    else:
        h0 = backend.ctx.h2d_bytes()
        ms_e2e, _, _, _ = timed(A_host, B_host, profile=False)
        # bytes the library actually copied per step (B packed to one byte per word when its
        # values fit a signed byte, as the config-2 int8 weights do)
        h2d_step = (backend.ctx.h2d_bytes() - h0) // (args.warmup + args.steps)

    # CPU baseline: rank 0 at N=1 only, one full layer through the oracle
    cpu = None
    if world == 1 and not args.headline_only:
        threads = host_cores()
        t = cpu_reference_layer(threads)
        cpu = {"value": t, "unit": "s/layer", "cores": threads, "kind": "port",
               "sample": "one full C2 layer through the C restatement of the reference CPU prover "
                         "(materialised restriction, backend.rs:110-197), all host threads"}

    nxt = time_next_rows(Z, torch, ta, tb) if world == 1 and not args.headline_only else None
    sharded = (measure_sharded(Z, torch, dist, world, rank, ctx, stream, cpu_sample=(world == 1))
               if not args.no_sharded else None)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    peak, peak_kind = measured_peak_hbm()
    rc_bytes = 4.0 * K * N + 32.0 * K  # B read once + per-row accumulators
    rc_avg_ms = rc_ms / max(rc_n, 1)
    achieved = rc_bytes / (rc_avg_ms * 1e-3) / 1e9
    traffic = ncu_traffic_per_launch()
    s_per_layer = ms / 1e3 / world
    rounds = log2(PK)
    line = {
        "metric": METRIC, "value": s_per_layer, "unit": "s/layer", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "u32 (M31/QM31 integer)",
        "data": "synthetic (SplitMix64-seeded int8 embedded in M31)",
        "config": {"workload": WORKLOAD, "m": M, "k": K, "n": N, "padded": [PM, PK, PN],
                   "layers_per_step": world, "parallelism": f"independent layer per GPU x{world}",
                   "ms_per_step_by_rank": [round(x, 4) for x in rank_ms],
                   "l2": "inputs larger than L2 (B = 283 MB > 126 MB L2)"},
        "e2e": {"value": ms_e2e / 1e3 / world, "unit": "s/layer",
                "h2d_bytes_per_step": int(h2d_step), "h2d_packed": h2d_step < 4 * (M * K + K * N),
                "d2h_bytes_per_step": rounds * 52 + 36},
        "gpu_launches": launches,
        "mle_elems_folded_per_s_per_gpu": ELEMS_FOLDED / (ms / 1e3),
        "roofline": {"bound": "hbm", "kernel": "restrict_cols", "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "algorithmic_bytes": rc_bytes, "avg_launch_ms": rc_avg_ms},
        "clocks": clocks,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    if sharded:
        line["parity_vs_1gpu"] = sharded.pop("parity_vs_1gpu")
        line["sharded"] = sharded
    if nxt:
        line["next_rows"] = nxt
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


C5_LOG_N = 30
C5_SWEEP = (20, 22, 24, 26, 28)  # the rest of config 5's 2^20 ... 2^30 sweep
# config 4: Qwen2.5-14B decoder layer at 64 tokens (hidden 5120, 40 x 128 query width, SwiGLU 13824)
C4_M, C4_D, C4_Q, C4_FF = 64, 5120, 5120, 13824


# config 3: SmolLM2-135M, 30 blocks (hidden 576, 9 x 64 query width, SwiGLU 1536), one token
C3_D, C3_Q, C3_FF, C3_BLOCKS = 576, 576, 1536, 30


def c3_inputs(torch, Z, blocks=C3_BLOCKS):
    """int8 input and weights in M31 from fixed seeds on the GPU, the reference recipe's layers."""
    from zkml_b200.circuits import hf_transformer_layers
    g = torch.Generator(device="cuda").manual_seed(0xC3)

    def m31(rows, cols):
        v = torch.randint(-127, 128, (rows, cols), dtype=torch.int64, device="cuda", generator=g)
        return torch.where(v < 0, v + Z.M31_P, v).to(torch.int32)

    x = m31(1, C3_D)
    return x, hf_transformer_layers(C3_D, C3_Q, C3_FF, blocks, lambda i, r, c: m31(r, c), "silu")


def c3_cpu_sample(torch, Z):
    """The oracle (the C restatement of the reference prover) on the first block of the same
    recipe, all host cores: the CPU baseline's bounded sample, scaled by the block count."""
    import oracle_lib as O
    x, layers = c3_inputs(torch, Z, blocks=1)
    xh = x.cpu().numpy().view(np.uint32)
    lh = [(k, a.cpu().numpy().view(np.uint32) if k == "linear" else a) for k, a in layers]
    narrowed = set(os.sched_getaffinity(0)) if HOST_AFFINITY else set()
    if HOST_AFFINITY:
        os.sched_setaffinity(0, HOST_AFFINITY)
    try:
        t0 = time.perf_counter()
        rc, _, _, _ = O.prove_gkr_chain(xh, lh, n_queries=10, activation_logup=True, cap=1 << 22)
        dt = time.perf_counter() - t0
    finally:
        if HOST_AFFINITY:
            os.sched_setaffinity(0, narrowed)
    assert rc == 0
    return dt


def c4_inputs(torch, Z):
    """16-bit activations and int8 weights embedded in M31, drawn on the GPU from fixed seeds;
    the layer list of the reference recipe for one block (zkml_b200.circuits)."""
    from zkml_b200.circuits import hf_transformer_layers
    g = torch.Generator(device="cuda").manual_seed(0xC4)

    def m31(rows, cols, bound):
        v = torch.randint(-bound, bound + 1, (rows, cols), dtype=torch.int64, device="cuda", generator=g)
        return torch.where(v < 0, v + Z.M31_P, v).to(torch.int32)

    x = m31(C4_M, C4_D, 32767)
    return x, hf_transformer_layers(C4_D, C4_Q, C4_FF, 1, lambda i, r, c: m31(r, c, 127), "silu")


def c5_inputs(torch, n, world, rank):
    """The config-5 MLEs: uniform M31 from a fixed torch generator on the GPU; every rank
    draws the same global vectors and keeps the elements with index = rank mod world."""
    g = torch.Generator(device="cuda").manual_seed(0xC5)
    a = torch.randint(0, 2**31 - 1, (n,), dtype=torch.int32, device="cuda", generator=g)
    b = torch.randint(0, 2**31 - 1, (n,), dtype=torch.int32, device="cuda", generator=g)
    if world == 1:
        return a, b, a, b
    return a, b, a[rank::world].contiguous(), b[rank::world].contiguous()


def timed_steps(torch, dist, world, stream, fn, steps, warmup):
    """fn() `steps` times between barriers, CUDA events on `stream`; the max over ranks (ms)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    out = None
    for _ in range(steps):
        out = fn()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, out


def proof_words(round_polys, final_a, final_b):
    return np.concatenate([np.concatenate([p.c0, p.c1, p.c2]) for p in round_polys] +
                          [np.asarray(final_a, np.uint32), np.asarray(final_b, np.uint32)])


def measure_sharded(Z, torch, dist, world, rank, ctx, stream, steps=5, warmup=3, cpu_sample=False):
    """The north star's splits of one proof over the `world` GPUs (see the module docstring),
    with rank 0's one-GPU recomputation of both proofs for the parity check."""
    from zkml_b200.distributed import (P2PInbox, PeerMesh, ShmExchange, column_block, prove_product_sharded_mesh,
                                       prove_product_sharded_native, reduce_matmul_layer_colsharded_p2p)
    out, parity = {}, True
    peak, _ = measured_peak_hbm()
    # ---- C5: 2^30-element product sumcheck split by the low index bits -----------------
    n = 1 << C5_LOG_N
    ga, gb, la, lb = c5_inputs(torch, n, world, rank)
    mesh = PeerMesh(ctx=ctx, max_gather_bytes=32 << 17) if world > 1 else None
    # one GPU: the same library loop with a one-rank exchange (no split, no exchange)
    solo = ShmExchange(f"zkml_solo_{os.getpid()}", 1, 0, max_gather_bytes=64, nonce=os.getpid()) \
        if (world == 1 or rank == 0) else None
    backend = Z.GpuBackend.__new__(Z.GpuBackend)
    backend.ctx = ctx
    if mesh is not None:
        def c5():
            return prove_product_sharded_mesh(la, lb, n, Z.PoseidonChannel(), mesh)
    else:
        def c5():
            return prove_product_sharded_native(la, lb, n, Z.PoseidonChannel(), solo, ctx=ctx)
    l0 = ctx.kernel_launches()
    ms, proof = timed_steps(torch, dist, world, stream, c5, steps, warmup)
    launches = (ctx.kernel_launches() - l0) // (steps + warmup)
    n_loc = n // world
    per_gpu = product_bytes(n_loc)
    out["c5"] = {"log_n": C5_LOG_N, "ms": round(ms, 4), "elems_folded_per_s_per_gpu": 2 * (2 * n - 2) / (ms * 1e-3) / world,
                 "hbm_frac_per_gpu": per_gpu / (ms * 1e-3) / 1e9 / peak, "algorithmic_bytes_per_gpu": per_gpu,
                 "launches_per_proof": launches,
                 "exchange": "peer mesh (round words reduced in the round kernels, gather by peer stores)"
                 if world > 1 else "none (one GPU)"}
    if world > 1:
        out["c5"]["gathered_at"] = proof.gathered_at
        got = proof_words(proof.round_polys, proof.final_a, proof.final_b)
        if rank == 0:
            ref = prove_product_sharded_native(ga, gb, n, Z.PoseidonChannel(), solo, ctx=ctx)
            parity &= bool((proof_words(ref.round_polys, ref.final_a, ref.final_b) == got).all())
        mesh.close()
    del ga, gb, la, lb
    torch.cuda.empty_cache()
    # ---- C5 sweep: the same split proof at 2^20 ... 2^28 elements -----------------------------
    sweep = []
    for lg in C5_SWEEP:
        ns = 1 << lg
        ga, gb, la, lb = c5_inputs(torch, ns, world, rank)
        mesh = PeerMesh(ctx=ctx, max_gather_bytes=32 << 17) if world > 1 else None
        if mesh is not None:
            def c5s():
                return prove_product_sharded_mesh(la, lb, ns, Z.PoseidonChannel(), mesh)
        else:
            def c5s():
                return prove_product_sharded_native(la, lb, ns, Z.PoseidonChannel(), solo, ctx=ctx)
        mss, proof = timed_steps(torch, dist, world, stream, c5s, 10, 3)
        per_gpu = product_bytes(ns // world)
        sweep.append({"log_n": lg, "ms": round(mss, 4), "elems_folded_per_s_per_gpu": 2 * (2 * ns - 2) / (mss * 1e-3) / world,
                      "hbm_frac_per_gpu": per_gpu / (mss * 1e-3) / 1e9 / peak})
        if world > 1:
            got = proof_words(proof.round_polys, proof.final_a, proof.final_b)
            if rank == 0:
                ref = prove_product_sharded_native(ga, gb, ns, Z.PoseidonChannel(), solo, ctx=ctx)
                parity &= bool((proof_words(ref.round_polys, ref.final_a, ref.final_b) == got).all())
            torch.cuda.synchronize()
            dist.barrier()
            mesh.close()
        del ga, gb, la, lb
        torch.cuda.empty_cache()
    out["c5_sweep"] = sweep
    if solo is not None:
        solo.close()
    # ---- C2 layer split by column blocks ---------------------------------------------------
    if world > 1:
        a, b = make_inputs(0)
        lo, hi = column_block(N, rank, world)
        A = Z.M31Matrix(M, K, torch.from_numpy(a.view(np.int32)).cuda().reshape(-1))
        blk = torch.from_numpy(np.ascontiguousarray(b[:, lo:hi]).view(np.int32)).cuda() if hi > lo else None
        ch0, point = seeded_channel_state(Z, 0)
        claim = np.zeros(4, np.uint32)
        inbox = P2PInbox(K, ctx=ctx)

        def c2():
            ch = ch0.clone()
            red, nxt = reduce_matmul_layer_colsharded_p2p(Z.GKRClaim(point, claim), A, blk, lo, M, K, N, ch, inbox)
            return red, nxt, ch

        ms2, (red, nxt, ch) = timed_steps(torch, dist, world, stream, c2, 10, warmup)
        out["c2_colsplit"] = {"ms": round(ms2, 4), "columns_per_gpu": hi - lo,
                              "exchange": "peer stores of the 4k partial words into every rank's inbox"}
        if rank == 0:
            chr_ = ch0.clone()
            ref, rnxt = Z.reduce_matmul_layer_with_backend(Z.GKRClaim(point, claim), A,
                                                           Z.M31Matrix(K, N, torch.from_numpy(b.view(np.int32)).cuda()),
                                                           M, K, N, chr_, backend)
            parity &= bool((proof_words(ref.round_polys, ref.final_a_eval, ref.final_b_eval) ==
                            proof_words(red.round_polys, red.final_a_eval, red.final_b_eval)).all())
            parity &= chr_.digest() == ch.digest() and bool((rnxt.point == nxt.point).all())
        torch.cuda.synchronize()
        dist.barrier()
        inbox.close()
    # ---- C2 full layer: prove_gkr of the one-layer circuit, Sequential weight opening included ----
    a, b = make_inputs(0)
    xa = torch.from_numpy(a.view(np.int32)).cuda()
    wb = torch.from_numpy(b.view(np.int32)).cuda()
    mesh = PeerMesh(ctx=ctx, max_gather_bytes=32 << 17) if world > 1 else None

    def full():
        return Z.prove_gkr_chain(xa, [("linear", wb)], mesh=mesh, device=ctx.device)

    msf, proof = timed_steps(torch, dist, world, stream, full, 2, 1)
    out["c2_full_layer"] = {"s": round(msf / 1e3, 4), "felts": int(proof.raw.size // 4),
                            "includes": "forward GEMM, output claim, matmul sumcheck, Sequential weight opening "
                                        "(2^27-leaf Merkle trees of every folded layer), io commitment",
                            "split": "weight-opening Merkle hashing over the peer mesh" if world > 1 else "none"}
    if world > 1:
        if rank == 0:
            ref = Z.prove_gkr_chain(xa, [("linear", wb)], device=ctx.device)
            parity &= ref.raw.size == proof.raw.size and bool((ref.raw == proof.raw).all())
        torch.cuda.synchronize()
        dist.barrier()
        mesh.close()
    del xa, wb, proof
    torch.cuda.empty_cache()
    # ---- C3: the 30-block SmolLM2-135M proof (one token), openings split over the mesh ---------
    x, layers = c3_inputs(torch, Z)
    mesh = PeerMesh(ctx=ctx, max_gather_bytes=32 << 17) if world > 1 else None

    def c3():
        return Z.prove_gkr_chain(x, layers, mesh=mesh, device=ctx.device, activation_logup=True)

    ms3, proof = timed_steps(torch, dist, world, stream, c3, 2, 1)
    out["c3_30_layer"] = {"s": round(ms3 / 1e3, 4), "blocks": C3_BLOCKS, "d": C3_D, "d_ff": C3_FF,
                          "felts": int(proof.raw.size // 4),
                          "activation": "SiLU through LogUp (the STWO_PIECEWISE_ACTIVATION=0 pin)",
                          "recipe": "build_hf_transformer_graph: RMSNorm, q, o, RMSNorm, gate, SiLU, down per "
                                    "block, final RMSNorm (no K/V, attention, RoPE, embedding or lm_head, as the "
                                    "reference graph)",
                          "split": "weight-opening Merkle hashing over the peer mesh" if world > 1 else "none"}
    if world > 1:
        if rank == 0:
            ref = Z.prove_gkr_chain(x, layers, device=ctx.device, activation_logup=True)
            parity &= ref.raw.size == proof.raw.size and bool((ref.raw == proof.raw).all())
        torch.cuda.synchronize()
        dist.barrier()
        mesh.close()
    elif cpu_sample:
        t1 = c3_cpu_sample(torch, Z)
        out["c3_30_layer"]["cpu_baseline"] = {
            "value": round(t1 * C3_BLOCKS, 2), "unit": "s", "cores": host_cores(), "kind": "port",
            "sample": f"the first of the 30 blocks through the oracle chain prover ({t1:.1f} s), times 30"}
    del x, layers, proof
    torch.cuda.empty_cache()
    # ---- C4: one Qwen2.5-14B decoder layer, weight openings' Merkle hashing split over the mesh ----
    x, layers = c4_inputs(torch, Z)
    mesh = PeerMesh(ctx=ctx, max_gather_bytes=32 << 17) if world > 1 else None

    def c4():
        return Z.prove_gkr_chain(x, layers, mesh=mesh, device=ctx.device, activation_logup=True)

    ms4, proof = timed_steps(torch, dist, world, stream, c4, 2, 1)
    out["c4_layer"] = {"s": round(ms4 / 1e3, 4), "m": C4_M, "d": C4_D, "q_dim": C4_Q, "d_ff": C4_FF,
                       "felts": int(proof.raw.size // 4),
                       "activation": "SiLU through LogUp (the STWO_PIECEWISE_ACTIVATION=0 pin)",
                       "split": "weight-opening Merkle hashing over the peer mesh" if world > 1 else "none (one GPU)"}
    if world > 1:
        if rank == 0:
            ref = Z.prove_gkr_chain(x, layers, device=ctx.device, activation_logup=True)
            parity &= ref.raw.size == proof.raw.size and bool((ref.raw == proof.raw).all())
        torch.cuda.synchronize()
        dist.barrier()
        mesh.close()
    del x, layers
    torch.cuda.empty_cache()
    out["parity_vs_1gpu"] = parity if world > 1 else None
    return out


def run_colsharded(args):
    """One C2 layer per step, B split by column blocks over the ranks: per rank the block
    restriction, one NCCL all-reduce of the 4k partial words, and the (replicated) sumcheck."""
    import torch
    import torch.distributed as dist

    import zkml_b200 as Z
    from zkml_b200.distributed import (P2PInbox, column_block, reduce_matmul_layer_colsharded,
                                       reduce_matmul_layer_colsharded_p2p)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.cuda.current_device()
    bind_to_gpu_cpus(dev)
    ctx = Z.context(dev)
    a, b = make_inputs(0)
    lo, hi = column_block(N, rank, world)
    A = Z.M31Matrix(M, K, torch.from_numpy(a.view(np.int32)).cuda().reshape(-1))
    blk = torch.from_numpy(np.ascontiguousarray(b[:, lo:hi]).view(np.int32)).cuda() if hi > lo else None
    ch0, point = seeded_channel_state(Z, 0)
    claim = np.zeros(4, np.uint32)
    inbox = P2PInbox(K, ctx=ctx) if (args.p2p and world > 1) else None

    def step():
        if inbox is not None:
            return reduce_matmul_layer_colsharded_p2p(Z.GKRClaim(point, claim), A, blk, lo, M, K, N, ch0.clone(),
                                                      inbox)
        return reduce_matmul_layer_colsharded(Z.GKRClaim(point, claim), A, blk, lo, M, K, N, ch0.clone(), ctx=ctx)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record()
        for _ in range(args.steps):
            step()
        e1.record()
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device="cuda") if world > 1 else None
    rank_ms = [ms]
    if world > 1:
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        rank_ms = [float(x.item()) for x in parts]
    ms = max(rank_ms)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC + " [one layer split by column blocks]", "value": ms / 1e3, "unit": "s/layer",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "u32 (M31/QM31 integer)",
            "data": "synthetic (SplitMix64-seeded int8 embedded in M31)",
            "config": {"workload": "C2 layer, B column blocks of next_pow2(n)/G columns, " +
                       ("peer-memory exchange of the 4k partial words" if inbox is not None else
                        "NCCL all-reduce of the 4k partial words"),
                       "m": M, "k": K, "n": N, "ms_per_step_by_rank": [round(x, 4) for x in rank_ms]},
            "clocks": clk.summary()}), flush=True)
    if inbox is not None:
        torch.cuda.synchronize()
        dist.barrier()
        inbox.close()
    if world > 1:
        dist.destroy_process_group()


def time_next_rows(Z, torch, ta, tb, reps=5):
    """Wall time per call (host transcript included, inputs resident in HBM) of the layer
    reductions beside the matmul path, on config-2-shaped data: the forward GEMM, the SiLU
    activation (LogUp and piecewise) and the RMSNorm of the C2 input, and the aggregated
    binding of the C2 weight."""
    import time

    from helpers import random_qm31

    rng = np.random.default_rng(7)
    out = {}

    def wall(fn, n):
        fn()
        torch.cuda.synchronize()
        t = time.perf_counter()
        for _ in range(n):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t) / n * 1e3

    A, B = Z.M31Matrix(M, K, ta), Z.M31Matrix(K, N, tb)
    tc = torch.empty(M * N, dtype=torch.int32, device="cuda")
    out["forward_gemm_ms"] = wall(lambda: Z.matmul_m31(A, B, out=tc), reps)
    C = Z.M31Matrix(M, N, tc)
    pt_c = random_qm31(log2(PM) + log2(PN), rng)
    val = random_qm31(1, rng)[0]
    out["logup_silu_ms"] = wall(lambda: Z.reduce_activation_layer(Z.GKRClaim(pt_c, val), C, 5,
                                                                  Z.PoseidonChannel()), reps)
    out["piecewise_silu_ms"] = wall(lambda: Z.reduce_activation_layer_piecewise(Z.GKRClaim(pt_c, val), C, 5,
                                                                                Z.PoseidonChannel()), reps)
    pt_a = random_qm31(log2(PM) + log2(PK), rng)
    out["rmsnorm_ms"] = wall(lambda: Z.reduce_rmsnorm_layer(Z.GKRClaim(pt_a, val), A, K, Z.PoseidonChannel()), reps)
    com = Z.weight_commitment(tb)
    out["weight_commitment_ms"] = wall(lambda: Z.weight_commitment(tb), 1)
    claim = Z.AggregatedWeightClaim(B, 0, random_qm31(log2(PK) + log2(PN), rng), val, com)
    out["aggregated_binding_ms"] = wall(lambda: Z.prove_aggregated_binding([claim], Z.PoseidonChannel()), 1)
    out["merkle_2e24"] = time_merkle_vs_reference(Z, torch)
    out["merkle_sweep"] = [time_merkle_vs_reference(Z, torch, log_n=lg, with_reference=False) for lg in (20, 22, 26)]
    out["shapes"] = {"gemm": [M, K, N], "activation": [M, N], "rmsnorm": [M, K], "binding_weight": [K, N]}
    return {k: (round(v, 3) if isinstance(v, float) else v) for k, v in out.items()}


def time_merkle_vs_reference(Z, torch, log_n=24, reps=3, with_reference=True):
    """Poseidon-252 Merkle commitment of 2^log_n QM31 leaves: this library's kernels against the
    reference's own layer kernel compiled from its source (oracle/_ref, a measuring stick; leaf
    felts precomputed for it, as the reference converts leaves on the CPU), both on this GPU,
    CUDA events, after one warm-up each; the roots are compared."""
    import ref_merkle as R
    n = 1 << log_n
    g = torch.Generator(device="cuda").manual_seed(24)
    leaves = torch.randint(0, 2**31 - 1, (n, 4), dtype=torch.int32, device="cuda", generator=g)

    def events(fn):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            r = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, r

    ms, root = events(lambda: Z.commit_mle_root(leaves))
    res = {"leaves": n, "ms": round(ms, 3), "hashes_per_s": (n - 1) / (ms * 1e-3)}
    if with_reference and R.available():
        felts = torch.from_numpy(R.leaf_felts(leaves.cpu().numpy().view(np.uint32)).view(np.int64)).cuda()
        rc = torch.from_numpy(R.limbs(R.compressed_round_keys()).view(np.int64)).cuda()
        scratch = torch.zeros((n, 4), dtype=torch.int64, device="cuda")

        def ref():
            R.lib().ref_merkle_root(felts.data_ptr(), n, scratch.data_ptr(), rc.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
            return scratch[0]
        rms, rroot = events(ref)
        rroot = rroot.cpu().numpy().view(np.uint64)
        res.update({"reference_kernel_ms": round(rms, 3), "reference_kernel_hashes_per_s": (n - 1) / (rms * 1e-3),
                    "speedup_vs_reference_kernel": rms / ms,
                    "roots_equal": sum(int(rroot[j]) << (64 * j) for j in range(4)) == root})
    return res


def product_bytes(n):
    """Algorithmic HBM bytes of one length-n M31 product sumcheck on one device.

    Round 0 reads both M31 vectors (8n); the fused fold+round from M31 reads
    them again and writes two QM31 halves (8n + 16n); each later fused
    fold+round over length L reads 32L and writes 16L.
    """
    total = 8 * n + 8 * n + 16 * n
    length = n // 2
    while length > 2:
        total += 48 * length
        length //= 2
    return total


def run_product(args):
    """The MLE-sweep product sumcheck (config 5) split across the GPUs (strong scaling)."""
    import torch
    import torch.distributed as dist

    import zkml_b200 as Z

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local if world > 1 else 0)
    dist.init_process_group("nccl" if world > 1 else "gloo", rank=rank, world_size=world,
                            **({"device_id": torch.device("cuda", local)} if world > 1 else
                               {"init_method": "tcp://127.0.0.1:%d" % (29500 + os.getpid() % 1000)}))
    dev = torch.cuda.current_device()
    stream = torch.cuda.current_stream()
    ctx = Z.Context(dev)
    ctx.set_stream(stream.cuda_stream)
    from zkml_b200.distributed import ShmExchange, job_nonce, prove_product_sharded_native
    port = os.environ.get("MASTER_PORT", "0")
    ex = ShmExchange(f"zkml_bench_{port}_{world}", world, rank, max_gather_bytes=32 << 17, nonce=job_nonce())
    n = 1 << args.log_n
    n_loc = n // world
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    a = torch.randint(0, 2**31 - 1, (n_loc,), dtype=torch.int32, device="cuda", generator=g)
    b = torch.randint(0, 2**31 - 1, (n_loc,), dtype=torch.int32, device="cuda", generator=g)

    def step():  # the library's round loop; round words and the final gather go through shared memory
        return prove_product_sharded_native(a, b, n, Z.PoseidonChannel(), ex, ctx=ctx)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    l0 = ctx.kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            proof = step()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], dtype=torch.float64, device="cuda" if world > 1 else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    launches = ctx.kernel_launches() - l0
    dist.barrier()
    merkle = None
    if world == 1:
        # config 5's commitment: Poseidon-252 Merkle root of the first MLE (QM31 leaves (a, 0, 0, 0)),
        # 2^min(L, 26) leaves
        lg = min(args.log_n, 26)
        leaves = torch.zeros((1 << lg, 4), dtype=torch.int32, device="cuda")
        leaves[:, 0] = a[: 1 << lg]
        Z.commit_mle_root(leaves)
        torch.cuda.synchronize()
        m0, m1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 2
        m0.record(stream)
        for _ in range(reps):
            Z.commit_mle_root(leaves)
        m1.record(stream)
        torch.cuda.synchronize()
        mms = m0.elapsed_time(m1) / reps
        merkle = {"leaves": 1 << lg, "ms": mms, "hashes_per_s": ((1 << lg) - 1) / (mms * 1e-3),
                  "bound": "integer pipe (Hades, radix-2^26 Montgomery multiply-add columns)"}
        del leaves
    if rank == 0:
        peak, peak_kind = measured_peak_hbm()
        # per-GPU bytes until the gather, then one GPU's share of the tail
        per_gpu = product_bytes(n_loc)
        achieved = per_gpu / (ms * 1e-3) / 1e9
        elems = 2 * (2 * n - 2)
        print(json.dumps({
            "metric": f"product sumcheck MLE elems folded/s (config 5, N = 2^{args.log_n} M31, two MLEs)",
            "value": elems / (ms * 1e-3), "unit": "elems/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "u32 (M31/QM31 integer)", "data": "synthetic (torch-seeded M31)",
            "config": {"workload": "C5 degree-2 product sumcheck, MLE split by low index bits",
                       "exchange": "host shared memory between the ranks (12 words per round, one gather)",
                       "log_n": args.log_n, "gathered_at": proof.gathered_at,
                       "l2": "inputs larger than L2" if 8 * n_loc > 126e6 else "inputs fit in L2"},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": "sumcheck rounds (whole proof)", "achieved": achieved,
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "algorithmic_bytes_per_gpu": per_gpu},
            "clocks": clk.summary(),
            **({"merkle_commitment": merkle} if merkle else {}),
        }), flush=True)
    ex.close()
    dist.destroy_process_group()


def run_case(name):
    """Small fixed workloads for ncu captures (one kernel class each)."""
    import torch

    import zkml_b200 as Z
    from helpers import int_matrix_m31, random_qm31

    torch.cuda.set_device(0)
    if name == "restrict_c2":  # three C2 reductions; restrict_cols launch 2 is the steady-state one
        be = Z.GpuBackend(0)
        a, b = make_inputs(0)
        ta = torch.from_numpy(a.view(np.int32)).cuda()
        tb = torch.from_numpy(b.view(np.int32)).cuda()
        rng = np.random.default_rng(0)
        r_i, r_j = random_qm31(log2(PM), rng), random_qm31(log2(PN), rng)
        for _ in range(3):
            be.reduce_matmul_layer(Z.M31Matrix(M, K, ta), Z.M31Matrix(K, N, tb), r_i, r_j, PK, Z.PoseidonChannel())
    elif name.startswith("merkle_"):  # Poseidon Merkle root over 2^L QM31 leaves, twice
        lg = int(name.split("_")[1])
        ev = torch.randint(0, 2**31 - 1, (1 << lg, 4), dtype=torch.int64).to(torch.int32).cuda()
        for _ in range(2):
            Z.commit_mle_root(ev)
    elif name.startswith("logup_"):  # SiLU LogUp layer at C4's activation size 64 x 13824
        x = int_matrix_m31(64, 13824, 3, bound=60000)
        rng = np.random.default_rng(0)
        pt, val = random_qm31(20, rng), random_qm31(1, rng)[0]
        for _ in range(2):
            Z.reduce_activation_layer(Z.GKRClaim(pt, val), Z.M31Matrix.from_numpy(x), 5, Z.PoseidonChannel())
    elif name.startswith("rmsnorm_"):  # RMSNorm layer R x C (e.g. rmsnorm_64x5120) with an affine scale, twice
        rows, cols = (int(v) for v in name.split("_")[1].split("x"))
        x = int_matrix_m31(rows, cols, 3, bound=300)
        nv = (rows - 1).bit_length() + (cols - 1).bit_length()
        rng = np.random.default_rng(0)
        pt, val = random_qm31(nv, rng), random_qm31(1, rng)[0]
        g = (np.arange(cols, dtype=np.uint32) % 1000) + 1
        for _ in range(2):
            Z.reduce_rmsnorm_layer(Z.GKRClaim(pt, val), Z.M31Matrix.from_numpy(x), cols, Z.PoseidonChannel(), gamma=g)
    elif name.startswith("gemm_"):  # forward M31 GEMM M x K x N (e.g. gemm_64x5120x13824), three times
        m_, k_, n_ = (int(v) for v in name.split("_")[1].split("x"))
        a = torch.randint(-127, 128, (m_, k_), dtype=torch.int32, device="cuda")
        b = torch.randint(-127, 128, (k_, n_), dtype=torch.int32, device="cuda")
        a = torch.where(a < 0, a + (2**31 - 1), a)
        b = torch.where(b < 0, b + (2**31 - 1), b)
        c = torch.empty(m_ * n_, dtype=torch.int32, device="cuda")
        for _ in range(3):
            Z.matmul_m31(Z.M31Matrix(m_, k_, a.reshape(-1)), Z.M31Matrix(k_, n_, b.reshape(-1)), out=c)
    elif name.startswith("piecewise_"):  # piecewise SiLU layer R x C (e.g. piecewise_64x13824), twice
        rows, cols = (int(v) for v in name.split("_")[1].split("x"))
        x = int_matrix_m31(rows, cols, 3, bound=60000)
        nv = (rows - 1).bit_length() + (cols - 1).bit_length()
        rng = np.random.default_rng(0)
        pt, val = random_qm31(nv, rng), random_qm31(1, rng)[0]
        for _ in range(2):
            Z.reduce_activation_layer_piecewise(Z.GKRClaim(pt, val), Z.M31Matrix.from_numpy(x), 5,
                                                Z.PoseidonChannel())
    elif name.startswith("binding_"):  # aggregated binding of one R x C weight (e.g. binding_5120x13824)
        rows, cols = (int(v) for v in name.split("_")[1].split("x"))
        w = torch.randint(0, 255, (rows, cols), dtype=torch.int32, device="cuda")
        nv = (rows - 1).bit_length() + (cols - 1).bit_length()
        rng = np.random.default_rng(0)
        claim = Z.AggregatedWeightClaim(w, 0, random_qm31(nv, rng), random_qm31(1, rng)[0], Z.weight_commitment(w))
        Z.prove_aggregated_binding([claim], Z.PoseidonChannel())
    elif name.startswith("la_"):  # native 1 x 2^L . 2^L x 1 reduction (look-ahead rounds), four times
        lg = int(name.split("_")[1])
        be = Z.GpuBackend(0)
        a = torch.randint(0, 2**31 - 1, (1 << lg,), dtype=torch.int32).cuda()
        b = torch.randint(0, 2**31 - 1, (1 << lg,), dtype=torch.int32).cuda()
        for _ in range(4):
            be.reduce_matmul_layer(Z.M31Matrix(1, 1 << lg, a), Z.M31Matrix(1 << lg, 1, b), [], [], 1 << lg,
                                   Z.PoseidonChannel())
    elif name.startswith("product_"):  # the product sumcheck of 2^L M31 elements, twice
        from zkml_b200.distributed import GpuSumcheckSession, LocalCollective, prove_product_sharded
        lg = int(name.split("_")[1])
        g = torch.Generator(device="cuda").manual_seed(1234)
        a = torch.randint(0, 2**31 - 1, (1 << lg,), dtype=torch.int32, device="cuda", generator=g)
        b = torch.randint(0, 2**31 - 1, (1 << lg,), dtype=torch.int32, device="cuda", generator=g)
        for _ in range(2):
            prove_product_sharded(a, b, 1 << lg, Z.PoseidonChannel(), session=GpuSumcheckSession(),
                                  collective=LocalCollective())
    else:
        raise SystemExit(f"unknown case {name}")
    torch.cuda.synchronize()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="run a small profiling workload instead of the benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=["c2", "c2-colsharded", "product"], default="c2",
                    help="c2: the headline matmul layer (one independent layer per GPU); c2-colsharded: one C2 "
                         "layer with B split by column blocks across the GPUs (strong scaling); product: the "
                         "config-5 product sumcheck split across GPUs")
    ap.add_argument("--log-n", type=int, default=28, help="product workload: log2 of the MLE length")
    ap.add_argument("--no-sharded", action="store_true", help="skip the split-proof measurements")
    ap.add_argument("--headline-only", action="store_true",
                    help="only the headline C2 layer (no e2e leg, CPU baseline, next rows or splits): for launch lists")
    ap.add_argument("--p2p", action="store_true",
                    help="c2-colsharded: exchange the partial words over peer memory instead of NCCL")
    args = ap.parse_args()
    if args.case:
        run_case(args.case)
        return
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.workload == "product" and args.impl == "b200":
        run_product(args)
    elif args.workload == "c2-colsharded" and args.impl == "b200":
        run_colsharded(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
