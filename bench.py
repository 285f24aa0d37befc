#!/usr/bin/env python
"""Benchmark of the B200 W4A4 prefix LM (BASELINE config 2 / 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--batch B] [--prefix M]
    torchrun --nproc-per-node N bench.py --gpus N ...      (N > 1)

One step = the full 18-layer W4A4 prefix-LM forward (PaliGemma's Gemma-2B,
fp16, every projection W4A4) of B robot-observation prefixes of M tokens per
GPU: per layer residual add + RMSNorm + Hadamard/INT4 quant, the fused q/k/v
GEMM, RoPE, bidirectional attention over the prefix with its padding mask,
quant + o_proj GEMM, residual add + RMSNorm + quant, the gate/up GEMM, GeGLU +
quant, the down GEMM; then the final residual add + norm.  The prefix is
config 2's: 256 + 256 + 64 image-token embeddings ~ N(0, 1) and M - 576
language tokens, 52 of them real.  Weights are random-init N(0, 0.02) (norm
weights N(0, 0.1)) packed in the reference's format; there is no dataset.
The 18 layers' ~1 GB of packed weights stream through HBM every step, far
more than the 126 MB L2, so no L2 flush is needed between steps.

Printed JSON (rank 0): ``value`` = prefixes/s of the whole job measured on
the device (CUDA graph of the forward, inputs resident), ``e2e`` = the same
through the model's public entry point with pinned-host inputs copied in and
the final hidden states copied out inside the timed region, ``roofline`` =
the gate/up GEMM (61 % of the prefix's integer ops) against the int8 tensor
peak, ``kernels`` = every kernel of a layer timed alone, ``w4a4_ops`` = the
72 W4A4 ops of a prefix chained without the glue (the path of the
pi05_w4a4 custom ops), ``cpu_baseline`` = the CPU oracle port of the
reference's int4_gemm_ref.  With N > 1, every rank runs its own
observations (data parallel, weak scaling); the step time is the max over
ranks.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "W4A4 prefix-LM ms per 776-tok prefix; GEMM int TOPS; obs/s at 1/2/4/8 B200"
UNIT = "obs/s (776-token W4A4 prefix-LM forwards per second)"
HIDDEN, INTER, N_Q, N_KV = 2048, 16384, 2048, 256
N_IMG = 576  # 256 + 256 + 64 image tokens
# dram__bytes_read.sum + dram__bytes_write.sum of one gate/up GEMM launch at
# M=776 (the CTA-pair kernel, which the default variant picks for it), from
# one `ncu --set full` capture of `bench.py --case gateup` (cold L2; most of
# the fp16 output is still in L2 when the kernel ends, so writes read low).
GATE_UP_DRAM_BYTES = 35_340_288 + 8_771_328


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=1, help="observations per GPU per step")
    ap.add_argument("--prefix", type=int, default=776, help="tokens per observation prefix (>= 628)")
    ap.add_argument("--layers", type=int, default=18)
    ap.add_argument("--staging", choices=("fp16", "fp32"), default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel timings")
    ap.add_argument("--sweep", action="store_true",
                    help="config 3: time the forward at prefix M in {640, 768, 776} x batch B in "
                         "{1, 8, 32, 64} on one GPU, one JSON line per point")
    ap.add_argument("--shard-mlp", action="store_true",
                    help="with N > 1: every rank runs the SAME observations and holds 1/N of gate/up "
                         "(tensor-parallel MLP, NCCL all-to-all + all-gather; strong scaling)")
    ap.add_argument("--int8", default="",
                    help="comma-separated projections (q,k,v,o,gate,up,down) repacked once into the "
                         "int8 layout (SS CTA-pair GEMM); default: none")
    ap.add_argument("--roofline-reps", type=int, default=20)
    ap.add_argument("--snapflow", action="store_true",
                    help="config 4: the SnapFlow 1-NFE action chunk (SigLIP + the W4A4 prefix LM + the "
                         "action expert); --batch observations per GPU (config 4: 64 over 8 GPUs)")
    ap.add_argument("--case", choices=("qkv", "o", "gateup", "down", "quant2k", "quant16k",
                                       "normquant", "geglu", "attn", "forward", "snapflow"),
                    default=None, help="run one op (or one forward) 3 times at the bench shape and "
                                       "exit (a small, self-contained case for ncu)")
    return ap.parse_args()


# ----------------------------------------------------------------------------- helpers
def ops_per_prefix(m: int, layers: int) -> float:
    """Algorithmic integer ops (2 per MAC) of one prefix's W4A4 GEMMs."""
    per_layer = 2 * m * HIDDEN * (N_Q + 2 * N_KV) + 2 * m * HIDDEN * HIDDEN \
        + 2 * m * HIDDEN * 2 * INTER + 2 * m * INTER * HIDDEN
    return float(per_layer * layers)


def quant_bytes(m: int, k: int) -> int:
    """Algorithmic bytes of one activation quant: fp16 in, packed INT4
    codes (K/2 bytes a row) and an fp32 scale out: 2MK + MK/2 + 4M."""
    return 2 * m * k + m * k // 2 + 4 * m


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.isfile(path):
        with open(path) as f:
            d = json.load(f)
        d["_source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "_source": "fallback"}


class ClockSampler:
    """Polls NVML (SM clock, clock-event reasons) every 10 ms on a thread."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device_index: int):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._handle = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self._nvml = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid if not uuid.startswith("GPU-") else uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001 - clocks are reported as unavailable
            self.error = repr(e)
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _reasons(self):
        n = self._nvml
        fn = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            n.nvmlDeviceGetCurrentClocksThrottleReasons
        return fn(self._handle)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self._nvml.nvmlDeviceGetClockInfo(self._handle, self._nvml.NVML_CLOCK_SM)
                self.samples.append((mhz, int(self._reasons())))
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        if self._handle is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._handle is not None:
            self._thread.join()

    def summary(self) -> dict:
        if self._handle is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "error": getattr(self, "error", "nvml unavailable")}
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = sorted(name for bit, name in self.REASONS.items() if mask & bit and bit != 0x1)
        mhz = [s for s, _ in self.samples]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(mhz)}


# ----------------------------------------------------------------------------- the W4A4 op chain
def layer_weights(lw) -> dict:
    return {"q": lw.q, "k": lw.k, "v": lw.v, "o": lw.o, "gate": lw.gate, "up": lw.up, "down": lw.down}


def w4a4_op_chain(x, layers):
    """The 72 pi05_w4a4 ops of one prefix pass chained through their outputs
    (q -> o_proj input, o -> gate/up input, gate -> down input, down -> next
    layer), without the glue between them."""
    import torch

    ops = torch.ops.pi05_w4a4
    for lw in layers:
        q, _, _ = ops.int4_gemm3(x, lw["q"], lw["k"], lw["v"])
        o = ops.int4_gemm(q, lw["o"])
        g, _ = ops.int4_gemm2_tiled(o, lw["gate"], lw["up"])
        x = ops.int4_gemm(g, lw["down"])
    return x


def synthetic_activations(rows: int, k: int, device, seed: int):
    import torch

    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(rows, k, device=device, generator=gen)
    ch = torch.randperm(k, device=device, generator=gen)[: k // 100]
    x[:, ch] *= 20
    return x.half()


# ----------------------------------------------------------------------------- timing
def time_device(fn, steps: int, warmup: int, dist_on: bool, device) -> float:
    """ms per step: events on the current stream, barrier + sync both sides,
    max over ranks."""
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / steps
    if dist_on:
        dist.barrier()
        ms = max_over_ranks(ms, device)
    return ms


def time_e2e(graphs, emb_host, pad_host, steps: int, warmup: int, dist_on: bool, device) -> float:
    """ms per step of the forward through GraphedPrefixLM with every step's
    inputs (embeddings and pad mask) copied in from pinned host memory and its
    final hidden states copied back, inside the timed region.  The copies run
    on a copy stream and two graph instances (each with its own static
    inputs and outputs) alternate, so step i+1's input copy and step i's
    output copy overlap the neighbouring steps' compute, as a serving loop
    runs them.  Events on the compute stream, barrier + sync both sides, max
    over ranks."""
    import torch
    import torch.distributed as dist

    compute = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device)
    out_host = [torch.empty(g.out.hidden.shape, dtype=torch.float16).pin_memory() for g in graphs]
    h2d = [torch.cuda.Event() for _ in graphs]
    done = [torch.cuda.Event() for _ in graphs]
    d2h = [torch.cuda.Event() for _ in graphs]

    def load(b, after):
        with torch.cuda.stream(copy):
            if after is not None:
                copy.wait_event(after)
            graphs[b].embeds.copy_(emb_host, non_blocking=True)
            graphs[b].pad.copy_(pad_host, non_blocking=True)
            h2d[b].record(copy)

    def run(n: int, after=None):
        load(0, after)
        for i in range(n):
            b = i & 1
            if i + 1 < n:
                load(b ^ 1, done[b ^ 1] if i >= 1 else None)  # step i-1 has consumed its inputs
            compute.wait_event(h2d[b])
            if i >= 2:
                compute.wait_event(d2h[b])  # step i-2's output has been copied out
            graphs[b].replay()
            done[b].record(compute)
            with torch.cuda.stream(copy):
                copy.wait_event(done[b])
                out_host[b].copy_(graphs[b].out.hidden, non_blocking=True)
                d2h[b].record(copy)
        compute.wait_stream(copy)

    run(warmup)
    torch.cuda.synchronize(device)
    if dist_on:
        dist.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(compute)
    run(steps, after=start)
    end.record(compute)
    torch.cuda.synchronize(device)
    ms = start.elapsed_time(end) / steps
    if dist_on:
        dist.barrier()
        ms = max_over_ranks(ms, device)
    return ms


def max_over_ranks(value: float, device) -> float:
    """The largest of every rank's `value` (the step time of the slowest
    rank); every rank must call it at the same point."""
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(ms_per_step: float, per_rank_prefixes: int, world: int) -> float:
    """Whole-job prefixes/s: every rank runs `per_rank_prefixes` independent
    observations per step (weak scaling), the job's step lasts as long as its
    slowest rank's."""
    return per_rank_prefixes * world / (ms_per_step * 1e-3)


def graph_ms(fn, reps: int, dist_on: bool, device, per_graph: int = 1) -> float:
    """ms per call of fn, captured `per_graph` times in one CUDA graph."""
    import torch

    g = torch.cuda.CUDAGraph()
    fn()
    torch.cuda.synchronize(device)
    with torch.cuda.graph(g):
        for _ in range(per_graph):
            fn()
    ms = time_device(g.replay, reps, 3, dist_on, device) / per_graph
    del g
    return ms


# ----------------------------------------------------------------------------- CPU reference
def set_host_threads(n: int) -> int:
    """All BLAS / OpenMP pools to n threads, whatever OMP_NUM_THREADS a
    launcher (torchrun sets 1) left behind."""
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n)
    except Exception:  # noqa: BLE001 - threadpoolctl is optional
        pass
    return n


def oracle_layer(m: int, staging: str):
    """One decoder layer's W4A4 ops through the CPU oracle port (numpy; exact
    integer products in fp32 BLAS), with weights in the reference's layouts:
    q/k/v as one N=2560 GEMM (shared quant, like int4_gemm3), o_proj, gate and
    up fragment-major, down_proj.  Returns a zero-argument callable."""
    from oracle import w4a4_oracle as orc

    qkv = orc.random_packed_weight(N_Q + 2 * N_KV, HIDDEN, 1)
    o = orc.random_packed_weight(HIDDEN, HIDDEN, 2)
    gate = orc.preshuffle_wmma_weight(orc.random_packed_weight(INTER, HIDDEN, 3), HIDDEN)
    up = orc.preshuffle_wmma_weight(orc.random_packed_weight(INTER, HIDDEN, 4), HIDDEN)
    down = orc.random_packed_weight(HIDDEN, INTER, 5)
    x = orc.make_activations(m, HIDDEN, 0)
    h = orc.make_activations(m, INTER, 1)

    def run():
        orc.int4_gemm_ref(x, qkv, staging=staging)
        orc.int4_gemm_ref(x, o, staging=staging)
        orc.int4_gemm_ref(x, gate, staging=staging, layout="fragment")
        orc.int4_gemm_ref(x, up, staging=staging, layout="fragment")
        orc.int4_gemm_ref(h, down, staging=staging)

    return run


def cpu_baseline_sample(m: int, staging: str, layers: int, batch: int) -> dict:
    """The CPU oracle port timed on this host for ONE decoder layer at M=m
    (median of 3), scaled to the prefix's layers.  A reported baseline only."""
    cores = set_host_threads(os.cpu_count() or 1)
    run = oracle_layer(m, staging)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    per_step = statistics.median(times) * layers
    return {"value": batch / per_step, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"1 decoder layer's W4A4 ops (qkv, o, gate, up, down) at M={m}, median of 3, "
                      f"x{layers} layers; numpy oracle port of int4_gemm_ref (BLAS threads = cores, "
                      "elementwise numpy on 1 thread); the glue (norms, attention, GeGLU) not included",
            "ms_per_prefix": per_step * 1e3 / batch}


# ----------------------------------------------------------------------------- arms
def run_ours(args, rank, world, local_rank, dist_on):
    import torch

    from pi05_pytorch_fast_b200 import _native as nat
    from pi05_pytorch_fast_b200 import prefix_lm as plm
    from pi05_pytorch_fast_b200.shard import MlpShard, exchange_row_blocks, gather_row_blocks
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    if args.staging:
        os.environ["PI05_W4A4_STAGING"] = args.staging
    staging_name = os.environ.get("PI05_W4A4_STAGING", "fp16")
    staging = nat.STAGING_FP32 if staging_name == "fp32" else nat.STAGING_FP16
    if args.prefix < N_IMG + 52:
        raise SystemExit(f"--prefix must be >= {N_IMG + 52} (576 image tokens + 52 real language tokens)")
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ext.preload()
    cfg = plm.PrefixLMConfig(layers=args.layers)
    sharded = args.shard_mlp and world > 1
    shard = MlpShard(rank, world) if sharded else None
    model = plm.W4A4PrefixLM.random(cfg, device, seed=1234, staging=staging, shard=shard)
    if args.int8:
        model.repack_int8(tuple(args.int8.split(",")))
    lang = args.prefix - N_IMG
    # data parallel: each rank its own observations; sharded: the same ones on every rank
    in_seed = 100 if sharded else 100 + rank
    embeds, pad = plm.synthetic_prefix(args.batch, lang_tokens=lang, device=device, seed=in_seed)
    m = args.batch * args.prefix
    torch.cuda.synchronize(device)

    # --- the forward as one CUDA graph, inputs resident on the device
    with torch.no_grad():
        graphs = [plm.GraphedPrefixLM(model, args.batch, args.prefix) for _ in range(2)]
        graphs[0].run(embeds, pad)
        with ClockSampler(local_rank) as clocks:
            ms = time_device(graphs[0].replay, args.steps, args.warmup, dist_on, device)

        # --- end to end: pinned host inputs in, final hidden states out, every step
        emb_host = plm.synthetic_prefix(args.batch, lang_tokens=lang,
                                        seed=200 if sharded else 200 + rank)[0].pin_memory()
        pad_host = pad.cpu().pin_memory()
        e2e_steps = max(5, min(args.steps, 50))
        ms_e2e = time_e2e(graphs, emb_host, pad_host, e2e_steps, max(3, args.warmup), dist_on, device)
        del graphs

        # --- the 72 W4A4 ops alone (the pi05_w4a4 op path), one CUDA graph
        ms_ops = None
        coll_ms = None
        if not sharded:
            lws = [layer_weights(lw) for lw in model.layers]
            x_static = synthetic_activations(m, HIDDEN, device, seed=100 + rank)
            ms_ops = graph_ms(lambda: w4a4_op_chain(x_static, lws), max(5, args.steps // 4), dist_on, device)
        else:
            # the step's collectives alone: per layer the all-to-all of the
            # GeGLU shards and the all-gather of the down_proj rows
            ws = model.workspace(args.batch, args.prefix)

            def collectives():
                for _ in model.layers:
                    exchange_row_blocks(ws.h_part, ws.h_recv, shard)
                    gather_row_blocks(ws.down_part, ws.down, shard)
            coll_ms = time_device(collectives, max(5, args.steps // 4), 3, dist_on, device)

    job_obs = 1 if sharded else world  # observation sets the job runs per step, per rank's batch
    result = {
        "metric": METRIC,
        "value": job_throughput(ms, args.batch, job_obs),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "prefix_lm_ms": ms / args.batch,
        "gemm_int_tops": ops_per_prefix(m, args.layers) / (ms * 1e-3) / 1e12,
        "higher_is_better": True,
        "scaling": "strong" if sharded else "weak",
        "vs_baseline": None,
        "dtype": "int4 codes x int4 codes -> int32 (tcgen05 kind::i8) for every projection; "
                 "fp16 activations, glue and attention",
        "data": "synthetic: random-init weights N(0,0.02) packed in the reference's format, norm weights "
                "N(0,0.1); prefix = 576 image-token embeddings N(0,1) + language tokens (52 real ids, "
                "rest padding) as config 2 builds it",
        "config": {
            "workload": f"config 2: full {args.layers}-layer W4A4 Gemma-2B prefix-LM forward, prefix "
                        f"M={args.prefix} tokens, {args.batch} observation(s) per GPU per step",
            "rows_per_gpu": m,
            "layers": args.layers,
            "staging": staging_name,
            "staging_parity": "fp32: pinned to the reference's golden vectors; fp16: the HIP kernel's "
                              "rounding, pinned to the reference's quant_rot_rb source compiled for host "
                              "threads (oracle/ref_quant)",
            "parallelism": (f"tp{world} MLP (N-sharded gate/up; per layer an NCCL all-to-all of the GeGLU "
                            "shards and an all-gather of the down_proj rows; attention replicated)")
                           if sharded else
                           f"dp{world} (independent observations per GPU, no collective in the step)",
            "l2": "working set ~1.0 GB of packed weights per step >> 126 MB L2 (no flush needed)",
            "timing": "CUDA graph replay of the whole forward, CUDA events, max over ranks",
        },
        "gpu_launches": model.launches_per_forward() * args.steps,
        "gpu_launches_note": "kernels of libw4a4_sm100.so per timed region: per forward the positions / "
                             "mask / cos-sin tables, 10 per layer (11 with --shard-mlp) and the final "
                             "norm; nothing else runs on the device (NCCL's kernels under --shard-mlp "
                             "not counted)",
        "clocks": clocks.summary(),
        "e2e": {
            "value": job_throughput(ms_e2e, args.batch, job_obs),
            "unit": UNIT,
            "h2d_bytes_per_step": int(emb_host.numel() * 2 + pad_host.numel()),
            "d2h_bytes_per_step": int(emb_host.numel() * 2),
            "mode": "GraphedPrefixLM.run semantics: every step's pinned-host embeddings and pad mask "
                    "copied in and its final hidden states copied out inside the timed region, on a "
                    "copy stream, two graph instances alternating so copies overlap compute",
            "steps": e2e_steps,
        },
    }
    if ms_ops is not None:
        result["w4a4_ops"] = {
            "ms_per_prefix": ms_ops / args.batch,
            "obs_per_s": job_throughput(ms_ops, args.batch, 1),
            "what": "the 72 pi05_w4a4 ops of a prefix (int4_gemm3, int4_gemm, int4_gemm2_tiled, "
                    "int4_gemm x 18) chained without the glue, one CUDA graph, torch op path",
        }
    if coll_ms is not None:
        result["collectives"] = {"ms_per_step": coll_ms, "share_of_step": coll_ms / ms,
                                 "what": "the step's NCCL all-to-alls and all-gathers timed alone "
                                         "(max over ranks)"}
    if not args.no_kernels and not sharded:
        result.update(kernel_figures(args, model, m, staging, dist_on, device))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference's CPU path is int4_gemm_ref: fp32 FWHT staging
        result["cpu_baseline"] = cpu_baseline_sample(m, "fp32", args.layers, args.batch)
    return result


def kernel_figures(args, model, m: int, staging: int, dist_on: bool, device) -> dict:
    """Every kernel of a layer timed alone (CUDA graphs cycling over the
    layers' weights, so weights come from HBM), with roofline fractions."""
    import torch

    from pi05_pytorch_fast_b200 import _native as nat
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    lib = nat.lib()
    peaks = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    hbm = peaks["hbm_gbs"]
    reps = args.roofline_reps
    x = synthetic_activations(m, HIDDEN, device, seed=7)
    h = synthetic_activations(m, INTER, device, seed=8)
    codes, scales = ext.quantize(x, fmt="gemm", staging=staging)
    codes16, scales16 = ext.quantize(h, fmt="gemm", staging=staging)
    lws = [layer_weights(lw) for lw in model.layers]
    out: dict = {}

    def cycle(fn):
        def run():
            for lw in lws:  # outputs dropped at once: the graph pool reuses their memory
                fn(lw)
        return run

    gemms = {
        "gemm_qkv": (lambda lw: ext.gemm_from_codes(codes, scales, [lw["q"], lw["k"], lw["v"]]),
                     2.0 * m * (N_Q + 2 * N_KV) * HIDDEN),
        "gemm_o": (lambda lw: ext.gemm_from_codes(codes, scales, [lw["o"]]), 2.0 * m * HIDDEN * HIDDEN),
        "gemm_gateup": (lambda lw: ext.gemm_from_codes(codes, scales, [lw["gate"], lw["up"]],
                                                       fragment_major=True),
                        2.0 * m * 2 * INTER * HIDDEN),
        "gemm_down": (lambda lw: ext.gemm_from_codes(codes16, scales16, [lw["down"]]),
                      2.0 * m * HIDDEN * INTER),
    }
    for name, (fn, ops) in gemms.items():
        t = graph_ms(cycle(fn), reps, dist_on, device, per_graph=1) / len(lws)
        out[name] = {"ms": t, "tops": ops / (t * 1e-3) / 1e12, "frac": ops / (t * 1e-3) / 1e12 / int8_peak}

    def bw(name, fn, nbytes, note):
        t = graph_ms(fn, reps, dist_on, device, per_graph=10)
        gbs = nbytes / (t * 1e-3) / 1e9
        out[name] = {"ms": t, "gbs": gbs, "peak_gbs": hbm, "frac": gbs / hbm, "bytes": nbytes, "note": note}

    for sname, st in (("", staging), ("_fp32", nat.STAGING_FP32)):
        if sname and st == staging:
            continue
        bw("quant_k2048" + sname, lambda st=st: ext.quantize(x, fmt="gemm", staging=st),
           quant_bytes(m, HIDDEN), "2MK + MK/2 + 4M algorithmic bytes (packed codes); 4.0 MB at M=776, "
                                   "L2-resident, launch-latency bound")
        bw("quant_k16384" + sname, lambda st=st: ext.quantize(h, fmt="gemm", staging=st),
           quant_bytes(m, INTER), "2MK + MK/2 + 4M algorithmic bytes (packed codes); repeated on one "
                                  "input, mostly L2-resident as in the forward")
    gate = synthetic_activations(m, INTER, device, seed=9)
    up = synthetic_activations(m, INTER, device, seed=10)
    gain = torch.ones(HIDDEN, dtype=torch.float32, device=device)
    xo = torch.empty_like(x)
    cb = torch.empty((m, INTER), dtype=torch.int8, device=device)
    sb = torch.empty((m,), dtype=torch.float32, device=device)
    stream = lambda: torch.cuda.current_stream(device).cuda_stream  # noqa: E731

    def geglu():
        nat.check(lib.w4a4_geglu_quant(gate.data_ptr(), up.data_ptr(), m, INTER, INTER, staging,
                                       nat.CODES_GEMM, cb.data_ptr(), sb.data_ptr(), None, INTER, stream()))

    def normq():
        nat.check(lib.w4a4_rmsnorm_quant(x.data_ptr(), HIDDEN, h.data_ptr(), INTER, gain.data_ptr(), 1e-6,
                                         xo.data_ptr(), HIDDEN, None, HIDDEN, m, HIDDEN, staging,
                                         nat.CODES_GEMM, cb.data_ptr(), sb.data_ptr(), stream()))

    bw("geglu_quant_k16384", geglu, 2 * 2 * m * INTER + m * INTER // 2 + 4 * m,
       "gate + up fp16 in, packed codes + scale out; replaces F.gelu(gate)*up and the down_proj quant")
    bw("rmsnorm_quant_k2048", normq, 3 * 2 * m * HIDDEN + m * HIDDEN // 2 + 4 * m,
       "x + delta in, x out (residual), packed codes + scale out; replaces add, RMSNorm and quant")
    # prep + attention as the forward runs them (RoPE of q and k, V^T, the
    # padded-prefix attention on CTA pairs), one observation batch
    from pi05_pytorch_fast_b200 import prefix_lm as plm

    batch, seq = args.batch, args.prefix
    _, pad = plm.synthetic_prefix(batch, lang_tokens=seq - N_IMG, device=device, seed=3)
    q = synthetic_activations(m, N_Q, device, seed=11)
    kk = synthetic_activations(m, N_KV, device, seed=12)
    vv = synthetic_activations(m, N_KV, device, seed=13)
    key_valid = pad.to(torch.uint8).contiguous()
    kv_len = (pad * torch.arange(1, seq + 1, device=device)).amax(dim=1).to(torch.int32)
    pos = (torch.cumsum(pad.long(), 1) - 1).clamp_min(0).reshape(-1).float()
    fr = pos[:, None] * model.inv_freq[None].float()
    emb = torch.cat((fr, fr), dim=-1)
    cos_t, sin_t = emb.cos().half().contiguous(), emb.sin().half().contiguous()
    vt = torch.empty((batch, N_KV, nat.attn_vt_stride(seq)), dtype=torch.float16, device=device)
    ao = torch.empty((m, N_Q), dtype=torch.float16, device=device)
    kc = torch.empty_like(kk)

    def attention():
        nat.check(lib.w4a4_prefix_attention(q.data_ptr(), N_Q, kk.data_ptr(), N_KV, vv.data_ptr(), N_KV,
                                            key_valid.data_ptr(), kv_len.data_ptr(), batch, seq, N_Q // N_KV,
                                            vt.data_ptr(), ao.data_ptr(), N_Q, cos_t.data_ptr(), sin_t.data_ptr(),
                                            kc.data_ptr(), N_KV, stream()))

    t = graph_ms(attention, reps, dist_on, device, per_graph=10)
    real = int(pad.sum())
    flops = 4.0 * real * (N_Q // N_KV) * int(kv_len.max()) * N_KV  # S and P V of the real queries
    out["attention_rope"] = {"ms": t, "tflops": flops / (t * 1e-3) / 1e12,
                             "note": "RoPE + V transpose launch and the attention on CTA pairs; latency bound "
                                     "at one observation (98 CTAs), tflops over the real queries' keys"}
    gu = out["gemm_gateup"]
    return {
        "roofline": {
            "kernel": "w4a4_gemm_pair_kernel<fragment-major> (gate+up, one launch on CTA pairs)",
            "bound": "tensor",
            "achieved": gu["tops"],
            "peak": int8_peak,
            "unit": "TFLOP/s",
            "op_kind": "int8 tensor ops (1 MAC = 2 ops); peak = 2 x bf16 dense "
                       f"({peaks['_source']}: {peaks['bf16_tflops']} TFLOP/s), the i8:f16 rate ratio",
            "frac": gu["frac"],
            "traffic": GATE_UP_DRAM_BYTES,
            "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch at M=776",
            "ms_per_launch": gu["ms"],
            "algorithmic_ops_per_launch": 2.0 * m * 2 * INTER * HIDDEN,
        },
        "kernels": out,
    }


def run_snapflow(args, rank, world, local_rank, dist_on) -> dict:
    """Config 4 on each rank: B observations per GPU through the whole
    SnapFlow step in one CUDA graph (independent observations per GPU)."""
    import torch

    from pi05_pytorch_fast_b200 import prefix_lm as plm
    from pi05_pytorch_fast_b200 import snapflow as sf
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    ext.preload()
    cfg = sf.SnapFlowConfig()
    lm = plm.W4A4PrefixLM.random(cfg.lm, device, seed=1234)
    policy = sf.SnapFlowPolicy(cfg, lm, device, seed=4321)
    b = args.batch
    obs = sf.synthetic_observation(cfg, b, seed=300 + rank, device=device)
    with torch.no_grad():
        # the three stages, each captured alone in a CUDA graph: SigLIP + the
        # prefix assembly, the W4A4 prefix LM, the action expert
        images, ids, mask, noise = obs
        embeds, pad = policy.embed_prefix(images, ids, mask)
        out = lm.forward(embeds, pad)
        x_t, t1 = noise.to(policy.dtype), torch.ones(b, device=device)
        reps = max(5, args.steps // 2)
        stages = {
            "siglip_and_prefix_assembly": graph_ms(lambda: policy.embed_prefix(images, ids, mask), reps,
                                                   dist_on, device),
            "w4a4_prefix_lm": graph_ms(lambda: lm.forward(embeds, pad, out=out), reps, dist_on, device),
            "action_expert": graph_ms(lambda: policy.expert(x_t, t1, t1, pad, out.keys, out.values), reps,
                                      dist_on, device),
        }
        g = sf.GraphedSnapFlow(policy, b)
        g.run(*obs)
        with ClockSampler(local_rank) as clocks:
            ms = time_device(g.replay, args.steps, args.warmup, dist_on, device)
        # end to end: pinned host observations in, actions out, every step
        host = [t.cpu().pin_memory() for t in sf.synthetic_observation(cfg, b, seed=400 + rank)]
        act_host = torch.empty(g.actions.shape, dtype=g.actions.dtype).pin_memory()

        def e2e_step():
            g.run(*host)
            act_host.copy_(g.actions, non_blocking=True)
        e2e_steps = max(5, min(args.steps, 30))
        ms_e2e = time_device(e2e_step, e2e_steps, max(3, args.warmup), dist_on, device)
    unit = "action chunks/s (observations/s; 50 x 32 actions each)"
    return {
        "metric": "pi0.5 SnapFlow 1-NFE action chunks per second (config 4)",
        "value": job_throughput(ms, b, world),
        "unit": unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16 SigLIP-So400m and action expert (cuBLAS / SDPA); the prefix LM W4A4 (int4 x int4 "
                 "-> int32 on tcgen05, fp16 activations)",
        "data": "synthetic: random-init weights (N(0, 0.02)); 2 real cameras of 224 x 224 pixels ~ U[-1, 1], "
                "the empty camera cached and pooled 4:1, 200 language tokens (52 real ids), noise ~ N(0, 1)",
        "config": {
            "workload": f"config 4: SnapFlow 1-NFE action chunk, {b} observation(s) per GPU per step "
                        "(SigLIP on 2 cameras, 776-token W4A4 prefix LM, 18-layer expert over 50 "
                        "action tokens)",
            "batch_per_gpu": b,
            "parallelism": f"dp{world} (independent observations per GPU, no collective in the step)",
            "timing": "CUDA graph replay of the whole step, CUDA events, max over ranks",
            "l2": "weights ~2.9 GB per step >> 126 MB L2 (no flush needed)",
        },
        "stages_ms": stages,
        "gpu_launches": lm.launches_per_forward() * args.steps,
        "gpu_launches_note": "kernels of libw4a4_sm100.so per timed region (the prefix LM); SigLIP and "
                             "the expert run cuBLAS / PyTorch kernels",
        "clocks": clocks.summary(),
        "e2e": {
            "value": job_throughput(ms_e2e, b, world),
            "unit": unit,
            "h2d_bytes_per_step": int(sum(t.numel() * t.element_size() for t in host)),
            "d2h_bytes_per_step": int(act_host.numel() * act_host.element_size()),
            "mode": "GraphedSnapFlow.run: every step's pinned-host images, language ids, mask and noise "
                    "copied in and the actions copied out inside the timed region (one stream)",
            "steps": e2e_steps,
        },
    }


def run_sweep(args) -> None:
    """Config 3 on one GPU: the forward at every (prefix, batch) of the
    sweep, one model, one JSON line per point with its own clock record and
    the per-GEMM fractions at that row count."""
    import torch

    from pi05_pytorch_fast_b200 import _native as nat
    from pi05_pytorch_fast_b200 import prefix_lm as plm
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    ext.preload()
    staging = nat.STAGING_FP32 if args.staging == "fp32" else nat.STAGING_FP16
    model = plm.W4A4PrefixLM.random(plm.PrefixLMConfig(layers=args.layers), device, seed=1234,
                                    staging=staging)
    peaks = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    lws = [layer_weights(lw) for lw in model.layers]
    for prefix in (640, 768, 776):
        for batch in (1, 8, 32, 64):
            m = batch * prefix
            embeds, pad = plm.synthetic_prefix(batch, lang_tokens=prefix - N_IMG, device=device, seed=7)
            steps = max(5, args.steps // batch)
            with torch.no_grad():
                g = plm.GraphedPrefixLM(model, batch, prefix)
                g.run(embeds, pad)
                with ClockSampler(0) as clocks:
                    ms = time_device(g.replay, steps, args.warmup, False, device)
                del g
                x = synthetic_activations(m, HIDDEN, device, seed=1)
                h = synthetic_activations(m, INTER, device, seed=2)
                codes, scales = ext.quantize(x, fmt="gemm", staging=staging)
                codes16, scales16 = ext.quantize(h, fmt="gemm", staging=staging)
                fr = {}
                for name, fn, ops in (
                        ("qkv", lambda lw: ext.gemm_from_codes(codes, scales, [lw["q"], lw["k"], lw["v"]]),
                         2.0 * m * (N_Q + 2 * N_KV) * HIDDEN),
                        ("o", lambda lw: ext.gemm_from_codes(codes, scales, [lw["o"]]), 2.0 * m * HIDDEN * HIDDEN),
                        ("gateup", lambda lw: ext.gemm_from_codes(codes, scales, [lw["gate"], lw["up"]],
                                                                  fragment_major=True),
                         2.0 * m * 2 * INTER * HIDDEN),
                        ("down", lambda lw: ext.gemm_from_codes(codes16, scales16, [lw["down"]]),
                         2.0 * m * HIDDEN * INTER)):
                    def cyc(fn=fn):
                        for lw in lws:  # outputs dropped at once: the graph pool reuses their memory
                            fn(lw)
                    t = graph_ms(cyc, 3, False, device) / len(lws)
                    fr[name] = {"us": round(t * 1e3, 2), "frac": ops / (t * 1e-3) / 1e12 / int8_peak}
                del x, h, codes, scales, codes16, scales16
            model._ws.clear()
            torch.cuda.empty_cache()
            print(json.dumps({"sweep": "config 3", "prefix": prefix, "batch": batch, "rows": m,
                              "ms_per_step": ms, "ms_per_prefix": ms / batch, "obs_per_s": batch / (ms * 1e-3),
                              "gemm_int_tops": ops_per_prefix(m, args.layers) / (ms * 1e-3) / 1e12,
                              "gemm_frac_of_int8": fr, "int8_peak_tops": int8_peak,
                              "clocks": clocks.summary(), "steps": steps}), flush=True)


def run_reference(args, rank, world):
    """The reference's CPU implementation of the path (this repo's oracle port
    of int4_gemm_ref; the reference itself is Python + HIP and cannot run
    here), timed on the host cores.  Rank 0 only; BLAS on every core."""
    import numpy as np

    if rank != 0:
        return None
    cores = set_host_threads(os.cpu_count() or 1)
    staging = "fp32"  # int4_gemm_ref's arithmetic (pack.py:113-145)
    m = args.batch * args.prefix
    one_layer = oracle_layer(m, staging)

    t0 = time.perf_counter()
    one_layer()
    t_first = time.perf_counter() - t0
    budget = 150.0
    steps = max(1, min(args.steps, int(budget / max(t_first, 1e-3)) - args.warmup))
    for _ in range(max(0, args.warmup - 1)):
        one_layer()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_layer()
    t_layer = (time.perf_counter() - t0) / steps
    value = 1.0 / (t_layer * args.layers) * args.batch
    sample = (f"each step = 1 decoder layer's W4A4 ops at M={m} (q/k/v as one N=2560 GEMM), "
              f"scaled x{args.layers} layers; numpy oracle port of int4_gemm_ref, {cores} BLAS threads")
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": t_layer * 1e3,
        "ms_per_prefix": t_layer * args.layers * 1e3 / args.batch,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int32 codes in fp32 BLAS (exact), fp16 out", "data": "synthetic",
        "config": {"workload": f"config 2 W4A4 path, {args.layers} layers, prefix M={args.prefix}, "
                               f"{args.batch} observation(s); one CPU process for the whole job",
                   "rows": m, "staging": staging},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "numpy": np.__version__,
    }


def run_case(args):
    """One op (or one forward) of one layer, 3 launches, for profiling (no
    timing, no JSON)."""
    import torch

    from pi05_pytorch_fast_b200 import _native as nat
    from pi05_pytorch_fast_b200 import prefix_lm as plm
    from pi05_pytorch_fast_b200.w4a4 import extension as ext

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    if args.case == "snapflow":
        # three eager config-4 steps, each in an NVTX range snapflow_step<i>
        # (ncu --nvtx --nvtx-include "snapflow_step2/" keeps the last)
        from pi05_pytorch_fast_b200 import snapflow as sf

        cfg = sf.SnapFlowConfig()
        policy = sf.SnapFlowPolicy(cfg, plm.W4A4PrefixLM.random(cfg.lm, device, seed=1234), device, seed=4321)
        obs = sf.synthetic_observation(cfg, args.batch, seed=300, device=device)
        for i in range(3):
            with torch.cuda.nvtx.range(f"snapflow_step{i}"):
                policy.sample_actions(*obs)
        torch.cuda.synchronize(device)
        print(f"case snapflow done (batch {args.batch})")
        return
    if args.staging:
        os.environ["PI05_W4A4_STAGING"] = args.staging
    staging = nat.STAGING_FP32 if os.environ.get("PI05_W4A4_STAGING", "fp16") == "fp32" else nat.STAGING_FP16
    m = args.batch * args.prefix
    layers = 1 if args.case != "forward" else args.layers
    model = plm.W4A4PrefixLM.random(plm.PrefixLMConfig(layers=layers), device, seed=1234, staging=staging)
    if args.int8:
        model.repack_int8(tuple(args.int8.split(",")))
    lw = layer_weights(model.layers[0])
    x = synthetic_activations(m, HIDDEN, device, seed=100)
    h = synthetic_activations(m, INTER, device, seed=101)
    codes, scales = ext.quantize(x, fmt="gemm")
    codes_h, scales_h = ext.quantize(h, fmt="gemm")
    lib = nat.lib()
    st = torch.cuda.current_stream(device).cuda_stream
    cb = torch.empty((m, INTER), dtype=torch.int8, device=device)
    sb = torch.empty((m,), dtype=torch.float32, device=device)
    gain = torch.ones(HIDDEN, dtype=torch.float32, device=device)
    embeds, pad = plm.synthetic_prefix(args.batch, lang_tokens=args.prefix - N_IMG, device=device)
    if args.case == "attn":  # the forward's key mask and spans
        with torch.no_grad():
            model.forward(embeds, pad)
        torch.cuda.synchronize(device)
    for _ in range(3):
        if args.case == "qkv":
            ext.gemm_from_codes(codes, scales, [lw["q"], lw["k"], lw["v"]])
        elif args.case == "o":
            ext.gemm_from_codes(codes, scales, [lw["o"]])
        elif args.case == "gateup":
            ext.gemm_from_codes(codes, scales, [lw["gate"], lw["up"]], fragment_major=True)
        elif args.case == "down":
            ext.gemm_from_codes(codes_h, scales_h, [lw["down"]])
        elif args.case == "quant2k":
            ext.quantize(x, fmt="gemm")
        elif args.case == "quant16k":
            ext.quantize(h, fmt="gemm")
        elif args.case == "geglu":
            nat.check(lib.w4a4_geglu_quant(h.data_ptr(), h.data_ptr(), m, INTER, INTER, staging,
                                           nat.CODES_GEMM, cb.data_ptr(), sb.data_ptr(), None, INTER, st))
        elif args.case == "normquant":
            nat.check(lib.w4a4_rmsnorm_quant(x.data_ptr(), HIDDEN, None, HIDDEN, gain.data_ptr(), 1e-6,
                                             None, HIDDEN, None, HIDDEN, m, HIDDEN, staging,
                                             nat.CODES_GEMM, cb.data_ptr(), sb.data_ptr(), st))
        elif args.case == "attn":
            ws = model.workspace(args.batch, args.prefix)
            nat.check(lib.w4a4_prefix_attention(
                x.data_ptr(), HIDDEN, h.data_ptr(), INTER, h.data_ptr() + 2 * 256, INTER,
                ws.key_valid.data_ptr(), ws.kv_len.data_ptr(), args.batch, args.prefix, 8,
                ws.vt.data_ptr(), ws.attn.data_ptr(), HIDDEN, None, None, None, 0, st))
        elif args.case == "forward":
            with torch.no_grad():
                model.forward(embeds, pad)
    torch.cuda.synchronize(device)
    print(f"case {args.case} done (M={m})")


def main():
    args = parse_args()
    if args.case:
        run_case(args)
        return
    if args.sweep:
        run_sweep(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference" and args.snapflow:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "config 4 runs lerobot's PI05 policy "
                              "(SigLIP, expert, SnapFlow step), which is not part of the reference "
                              "checkout; only its W4A4 path has a CPU implementation"}), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    import torch
    import torch.distributed as dist

    dist_on = world > 1
    if dist_on:
        from datetime import timedelta

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        res = (run_snapflow if args.snapflow else run_ours)(args, rank, world, local_rank, dist_on)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if dist_on:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
