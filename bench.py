#!/usr/bin/env python
"""MoE-layer benchmark on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--precision bf16x3|3xtf32|bf16] [--workload c2|c2small|c5|c4]

Workload: a Mixtral-shaped MoE FFN layer in prefill,
T=4096 tokens per GPU, d_model=4096, d_ff=14336, 8 experts, top-2 softmax
routing, SwiGLU experts, fp32 weights N(0, 0.02) (seed 1) and N(0, 1)
activations -- synthetic, drawn on the GPU by a seeded torch generator.

One step = one forward of the layer over the step's T tokens: router,
dispatch (histogram / scan / permute), gate/up grouped GEMM with the SwiGLU
epilogue, down grouped GEMM (each routed row's output at its selection
slot), ordered combine.

The headline precision is fp32-faithful, as BASELINE config 2's fp32 weights
and the reference's fp32 arithmetic ask: bf16x3 (every fp32 operand split
into bf16 hi + lo, three bf16 MMAs into fp32; rel-L2 <= 1e-3).  The BF16
weight mode (rel-L2 <= 2e-2) is measured in the same run and reported under
roofline.modes.

  value       tokens/s over all ranks, x resident in HBM, CUDA events around
              each step on the launching stream; L2 is flushed (256 MiB
              write) between steps, outside the events.
  e2e         tokens/s through moe_forward_host (the reference-facing
              host-buffer call): pinned host x -> device -> layer -> host y,
              host clock around the synchronous call.
  roofline    the gate/up GEMM (2/3 of the layer's FLOPs): algorithmic FLOPs
              4*T*k*d*ff per launch / its time (the step time of the timed,
              unprofiled steps times the GEMM's share of a profiled step),
              against the measured burst dense bf16 peak in
              MEASURED_PEAKS.json.  Also holds each precision mode's numbers
              (modes), the config-3 decode HBM fractions (decode) and the
              config-4 decoder's (decoder).
  cpu_baseline  the reference's own PhiMoE::forward (src/layer.cu:80-103,
              compiled from its sources into oracle/_ref) on this host's
              cores, on a bounded sample of the same layer.

N > 1 (torchrun): expert parallel -- each rank holds E/N experts (round-robin
placement) and its own T tokens; the default transport deduplicates: one row
per (token, destination rank) stored into the destination's buffer over
NVLink by the push kernel, the rank's expert outputs summed there in
ascending expert order and one row stored back (--ep-transport nccl: NCCL
send/recv exchanges instead); weak scaling.  --parallelism dp runs
token-sharded replicas instead.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = "MoE-layer tokens/s at 1–8 B200; expert-GEMM % of TC peak; decode HBM GB/s"
WORKLOADS = {
    "c2": dict(workload="c2-mixtral-moe-prefill", T=4096, d=4096, ff=14336, E=8, k=2, seed=1),
    # Profiling case for ncu --set full: the C2 expert shapes (d 4096, d_ff
    # 14336) with 2 experts, ~2 GB on the device (weights > L2).
    "c2small": dict(workload="c2small-2expert-profile", T=2048, d=4096, ff=14336, E=2, k=2,
                    seed=1),
    # A quarter of config 2 for DRAM-traffic captures: 2 of its 8 experts with
    # its 1024 routed rows per expert, so a launch's traffic times 4 is
    # config 2's (~3 GB on the device).
    "c2slice": dict(workload="c2slice-2of8-experts", T=1024, d=4096, ff=14336, E=2, k=2, seed=1),
    # fine-grained experts, top-8, router logits ~N(0, 1)
    # (router weights N(0, 1/d)) plus the Zipf-like bias 0.5 ln(1/rank).
    "c5": dict(workload="c5-finegrained-ep", T=16384, d=2048, ff=1408, E=64, k=8, seed=3,
               zipf=True),
}
# Precision modes: the MoeConfig precision, the dtype string, and how many
# bf16-rate tensor-core passes one algorithmic FLOP costs (bf16x3: three bf16
# MMAs; 3xTF32: three tf32 MMAs at half the bf16 rate).
PRECISIONS = {
    "bf16x3": dict(prec=2, dtype="fp32 (bf16x3 tensor cores: hi*hi + hi*lo + lo*hi)", passes=3),
    "3xtf32": dict(prec=0, dtype="fp32 (3xTF32 tensor cores)", passes=6),
    "bf16": dict(prec=1, dtype="bf16", passes=1),
}
ROUTER_NOTE = ("the reference's PhiMoE routes with its quantised top-2 rule (scores rounded to "
               "1e-3, tie margin 2e-2, weights 0.5/0.5); this repo's line routes with "
               "BASELINE's softmax top-k renormalised -- the expert FLOPs per token are the same")


def _router_weights(wl, gen, dev):
    """Router weights and bias of a workload, drawn on the device."""
    import torch
    E, d = wl["E"], wl["d"]
    std = (1.0 / d ** 0.5) if wl.get("zipf") else 0.02
    wg = torch.randn(E, d, generator=gen, device=dev).mul_(std)
    bias = None
    if wl.get("zipf"):
        r = torch.arange(1, E + 1, dtype=torch.float64)
        bias = (0.5 * torch.log(1.0 / r)).to(torch.float32).to(dev)
    return wg, bias


# router, dispatch_scan, dispatch_permute, gate/up GEMM, down GEMM, combine
KERNELS_PER_FORWARD = 6
# the toy MoE decoder, end to end (prompt of 512 uniform
# ids, 128 greedy tokens, batch 1 and 16).
C4 = dict(workload="c4-toy-moe-decoder", n_layers=8, d=2048, heads=16, hd=128, vocab=32000,
          E=16, k=2, ff=5632, prompt=512, new=128, batches=(1, 16), seed=2)
DECODE_T = (1, 2, 4, 8, 16, 32, 64)
FLUSH_BYTES = 256 << 20
# Cycles of the device sleep before each timed call (about 0.2 ms at 1.965 GHz).
SLEEP_CYCLES = 400_000


def _pkg():
    import importlib.util
    name = "moe_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / "accelerating-moe-inference_b200" / "__init__.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def _gemm_variant(args, pkg):
    return {"auto": pkg.GEMM_AUTO, "single": pkg.GEMM_SINGLE_CTA,
            "ctapair": pkg.GEMM_CTA_PAIR}[args.gemm]


def _traffic_from_profile(workload: str, precision: str):
    """dram bytes per launch of the gate/up GEMM from the committed ncu summary."""
    f = ROOT / "profiles" / f"expert_gemm_gateup_{workload}_{precision}.md"
    if not f.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", f.read_text())
    return float(m.group(1)) if m else None


def _config(wl, args, world):
    """The config object of both arms' lines (the reference arm emits the same)."""
    par = f"dp{world} (token-sharded replicas, all experts per GPU)"
    if world > 1 and args.parallelism == "ep":
        par = (f"ep{world} (expert parallel, {wl['E'] // world} experts per GPU placed "
               "round-robin, " + ("NCCL send/recv dispatch and combine)" if args.ep_transport == "nccl"
                                  else "deduplicated NVLink peer-store dispatch and return)"))
    return {"workload": wl["workload"], "T_per_gpu": wl["T"], "d_model": wl["d"], "d_ff": wl["ff"],
            "experts": wl["E"], "top_k": wl["k"],
            "router": "softmax_topk_renorm" + (" + zipf bias" if wl.get("zipf") else ""),
            "precision": args.precision, "seed": wl["seed"],
            "l2": "flushed between steps (256 MiB write, outside the timed events)",
            "parallelism": par}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, sampled every
    10 ms from construction to stop() by an NVML polling thread (read-only
    queries); nvidia-smi every 100 ms if NVML is unavailable."""
    Q = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits.
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40}

    def __init__(self, uuid: str):
        import threading
        self.uuid = uuid
        self.p = None
        self.samples, self.mask, self.mx = [], 0, None
        self._stop = threading.Event()
        self.t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons

            def poll():
                while not self._stop.is_set():
                    try:
                        self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(
                            h, pynvml.NVML_CLOCK_SM)))
                        self.mask |= int(reasons(h))
                    except Exception:  # noqa: BLE001 -- a failed query skips a sample
                        pass
                    self._stop.wait(0.01)

            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
            return
        except Exception:  # noqa: BLE001 -- no NVML: fall back to nvidia-smi
            self.t = None
        self.f = tempfile.TemporaryFile(mode="w+")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.t is not None:
            self._stop.set()
            self.t.join()
            reasons = sorted(n for n, b in self.BITS.items() if self.mask & b)
            return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                    "sm_max_mhz": self.mx, "samples": len(self.samples), "reasons": reasons,
                    "source": "NVML, 10 ms"}
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().splitlines():
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9 or (self.uuid and c[0] != self.uuid):
                continue
            try:
                sm.append(float(c[1]))
                mx = float(c[2])
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "samples": len(sm), "reasons": sorted(reasons), "source": "nvidia-smi, 100 ms"}



def _ref_layer(wl):
    """The workload's layer on the host for the reference CPU code (seeded
    torch CPU generator, N(0, 0.02) weights)."""
    import torch
    pkg = _pkg()
    g = torch.Generator().manual_seed(wl["seed"])
    d, ff, E = wl["d"], wl["ff"], wl["E"]
    mk = lambda *s: (torch.randn(*s, generator=g) * 0.02).numpy()  # noqa: E731
    layer = pkg.LayerWeights(mk(E, d), [mk(ff, d) for _ in range(E)],
                             [mk(ff, d) for _ in range(E)], [mk(d, ff) for _ in range(E)])
    x = torch.randn(wl["T"], d, generator=g).numpy()
    return layer, x


def _load_reference(host_layer, threads):
    """The reference's PhiMoE (oracle/_ref) loaded with this layer through a
    RAM-backed model.bin; (None, 0) when it was not built."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # checker / baseline only
    pkg = _pkg()
    if not oracle.Reference.available(host_layer.E):
        return None, 0
    ref = oracle.Reference(host_layer.E)
    cores = ref.set_threads(threads)
    fd = os.memfd_create("moe_model_bin", 0)
    path = f"/proc/self/fd/{fd}"
    try:
        pkg.write_model_bin(path, [host_layer])
        ref.load(path, 0)
    finally:
        os.close(fd)
    return ref, cores


def _ref_sample(cores, T):
    # The reference parallelises each expert's matmuls over that expert's
    # rows (OpenMP), so a sample of 4 tokens per core gives every core about
    # one row per expert at top-2 of 8 experts; fewer tokens leave cores idle.
    return int(min(T, max(8, 4 * cores)))


def cpu_reference_tokens_per_s(host_layer, x_host, threads: int):
    """Time the reference's own PhiMoE::forward on a bounded token sample.
    Returns (tokens/s, kind, tokens in the sample, threads used)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # checker / baseline only
    ref, cores = _load_reference(host_layer, threads)
    if ref is not None:
        run, kind = ref.forward, "reference"
    else:
        orc = oracle.Oracle()
        cores = threads
        run = lambda xs: orc.moe_forward(xs, host_layer, 2, oracle.POLICY_PHI, nthreads=threads)[0]  # noqa: E731
        kind = "port"
    n = _ref_sample(cores, len(x_host))
    t = time.perf_counter()
    run(x_host[:n])
    dt = time.perf_counter() - t
    if ref is not None:
        ref.close()
    return n / dt, kind, n, cores


def reference_arm(args, wl):
    """bench.py --impl reference: the reference's own CPU MoE layer (rank 0
    only; other ranks exit without work)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    layer, x = _ref_layer(wl)
    threads = len(os.sched_getaffinity(0))
    ref, cores = _load_reference(layer, threads)
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref was not built (reference sources absent at build time)"}))
        return 0
    n = _ref_sample(cores, wl["T"])
    # Warm-up steps run one token (they only page the code and the first
    # experts in); each timed step runs the n-token sample.
    for _ in range(args.warmup):
        ref.forward(x[:1])
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        ref.forward(x[:n])
        times.append(time.perf_counter() - t)
    ref.close()
    ms = 1e3 * sum(times) / len(times)
    value = n / (ms / 1e3)
    sample = (f"{n} of the workload's {wl['T']} tokens per timed step ({n // max(cores, 1)} per "
              f"core) through the reference's PhiMoE::forward, {cores} OpenMP threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded torch CPU generator, N(0,0.02) weights, N(0,1) x)",
        "config": _config(wl, args, world),
        "router_difference": ROUTER_NOTE,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }))
    return 0


def run_decoder(args, pkg, dev, reps: int = 2, new_tokens=None, profile_range=False):
    """BASELINE config 4 through moe_decoder_generate: weights N(0, 0.02)
    drawn on the device (seed 2), norms 1; per batch, prefill and decode
    time from CUDA events on the decoder's stream and the host clock around
    the whole call (prompt in, ids and logits [B][128][32000] out)."""
    import numpy as np
    import torch
    c = dict(C4)
    if new_tokens:
        c["new"] = new_tokens
    if getattr(args, "decoder_layers", None):
        c["n_layers"] = args.decoder_layers
    if getattr(args, "decoder_batches", None):
        c["batches"] = tuple(int(b) for b in args.decoder_batches.split(","))
    d, L, E, ff, V, k = c["d"], c["n_layers"], c["E"], c["ff"], c["vocab"], c["k"]
    gen = torch.Generator(device="cuda").manual_seed(c["seed"])
    rnd = lambda *s: torch.randn(*s, generator=gen, device=dev).mul_(0.02)  # noqa: E731
    keep = []

    def t(x):
        keep.append(x)
        return x.data_ptr()
    ones = torch.ones(d, device=dev)
    ptrs = {"embed": t(rnd(V, d)), "final_norm": ones.data_ptr(), "attn_norm": [], "wq": [],
            "wk": [], "wv": [], "wo": [], "ffn_norm": [], "router": [], "w1": [], "w3": [],
            "w2": []}
    for _ in range(L):
        for name in ("wq", "wk", "wv", "wo"):
            ptrs[name].append(t(rnd(d, d)))
        ptrs["attn_norm"].append(ones.data_ptr())
        ptrs["ffn_norm"].append(ones.data_ptr())
        ptrs["router"].append(t(rnd(E, d)))
        for _e in range(E):
            ptrs["w1"].append(t(rnd(ff, d)))
            ptrs["w3"].append(t(rnd(ff, d)))
            ptrs["w2"].append(t(rnd(d, ff)))
    # BASELINE config 4 names no precision: bf16, or 3xTF32 when that is the headline.
    dprec = "3xtf32" if args.precision == "3xtf32" else "bf16"
    prec = pkg.PREC_FP32 if dprec == "3xtf32" else pkg.PREC_BF16
    bmax = max(c["batches"])
    m = pkg.MoeDecoder(n_heads=c["heads"], head_dim=c["hd"], top_k=k, precision=prec,
                       max_batch=bmax, max_seq=c["prompt"] + c["new"], device=dev.index,
                       device_pointers=ptrs, dims=dict(n_layers=L, d=d, vocab=V, E=E, ff=ff))
    del keep, ptrs
    torch.cuda.empty_cache()
    prompt = pkg.synthetic_prompt(c["seed"], bmax, c["prompt"], V)
    hbm = _peaks()[0]
    wb = 4 if dprec == "3xtf32" else 2
    out = {}
    for B in c["batches"]:
        p = np.ascontiguousarray(prompt[:B])
        lbuf = np.empty((B, c["new"], V), np.float32)
        m.generate(p, c["new"], logits_out=lbuf)                      # warm-up
        if profile_range:
            # One generate inside cudaProfilerStart/Stop (ncu --profile-from-start off).
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            m.generate(p, c["new"], logits_out=lbuf)
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
        pre = dec = wall = 0.0
        for _ in range(reps):
            t0 = time.perf_counter()
            ids, _ = m.generate(p, c["new"], logits_out=lbuf)
            wall += time.perf_counter() - t0
            a, b = m.last_timing()
            pre += a
            dec += b
        pre, dec, wall = pre / reps, dec / reps, wall / reps
        steps = c["new"] - 1
        # Bytes one decode step must read at least: dense projections and the
        # output head, the experts a batch of B routes to (expected distinct
        # experts under uniform routing), the router, the KV cache (fp32) at
        # the mean position.
        e_dist = E * (1.0 - (1.0 - k / E) ** B)
        pos = c["prompt"] + steps / 2.0
        step_bytes = (L * (4 * d * d * wb + e_dist * 3 * d * ff * wb + E * d * 4
                           + 2 * B * pos * d * 4) + V * d * wb)
        ms_step = dec / steps
        out[str(B)] = {
            "prefill_ms": pre, "prefill_tokens_per_s": B * c["prompt"] / (pre / 1e3),
            "decode_ms_per_step": ms_step, "decode_tokens_per_s": B * steps / (dec / 1e3),
            "decode_step_bytes": step_bytes,
            "decode_hbm_gbs": step_bytes / (ms_step / 1e3) / 1e9,
            "decode_frac_of_hbm": step_bytes / (ms_step / 1e3) / 1e9 / hbm,
            "generate_wall_s": wall,
            "e2e_new_tokens_per_s": B * c["new"] / wall,
            "ids_valid": bool(((ids >= 0) & (ids < V)).all()),
            "logits_finite": bool(np.isfinite(lbuf).all()),
        }
        if B == 1:
            # The fused batch-1 step (one cooperative launch per decode
            # step; off by default), for comparison with the chain above.
            try:
                m.set_fused_step(True)
            except pkg.MoeError:
                pass
            if m.fused_step_active:
                m.generate(p, c["new"], logits_out=lbuf)
                m.generate(p, c["new"], logits_out=lbuf)
                fused = m.last_timing()[1] / steps
                m.set_fused_step(False)
                out[str(B)]["fused_decode_ms_per_step"] = fused
                out[str(B)]["fused_decode_frac_of_hbm"] = step_bytes / (fused / 1e3) / 1e9 / hbm
    m.close()
    return {"workload": c["workload"], "n_layers": L, "d_model": d, "heads": c["heads"],
            "head_dim": c["hd"], "vocab": V, "experts": E, "top_k": k, "d_ff": ff,
            "prompt": c["prompt"], "new_tokens": c["new"], "precision": dprec,
            "seed": c["seed"], "by_batch": out,
            "how": "moe_decoder_generate (KV-cached greedy decode); prefill/decode from CUDA "
                   "events on the decoder's stream, e2e = host clock around the call; decode "
                   "bytes use the expected distinct experts under uniform routing"}


def decoder_only(args):
    """--workload c4: the toy MoE decoder alone on GPU 0; one JSON line whose
    value is batch-16 decode tokens/s."""
    import torch
    torch.cuda.set_device(0)
    pkg = _pkg()
    dev = torch.device("cuda", 0)
    dec = run_decoder(args, pkg, dev, reps=max(1, args.steps // 25),
                      new_tokens=args.decoder_new_tokens, profile_range=args.profile_range)
    b16 = dec["by_batch"][max(dec["by_batch"], key=int)]
    print(json.dumps({
        "metric": "toy MoE decoder tokens/s (BASELINE config 4)", "value": b16["decode_tokens_per_s"],
        "unit": "tokens/s", "n_gpus": 1, "higher_is_better": True,
        "dtype": dec["precision"],
        "data": "synthetic (seeded torch CUDA generator: N(0,0.02) weights; uniform prompt ids)",
        "config": {"workload": C4["workload"], "batch": max(C4["batches"]),
                   "prompt": C4["prompt"], "new_tokens": dec["new_tokens"]},
        "decoder": dec}))
    return 0


def _ep_transport(args, pkg):
    return pkg.EP_TRANSPORT_NCCL if args.ep_transport == "nccl" else pkg.EP_TRANSPORT_P2P


def run_ep(args, wl, pkg, world, rank, local):
    """N > 1, expert parallel: each rank holds E/N experts (round-robin) and
    its own T tokens (weak scaling: tokens per GPU fixed).  Default
    transport: the deduplicated fused one -- one row per (token, destination
    rank) stored into the destination's receive buffer over NVLink, the
    rank's expert outputs summed there in ascending expert order, one row
    stored back, flags in peer memory, no NCCL call per step; --ep-transport
    nccl: NCCL send/recv exchanges."""
    import torch
    import torch.distributed as dist
    T, d, ff, E, k = wl["T"], wl["d"], wl["ff"], wl["E"], wl["k"]
    if E % world:
        raise SystemExit(f"{E} experts do not split over {world} GPUs")
    mode = PRECISIONS[args.precision]
    dev = torch.device("cuda", local)
    obj = [pkg.ep_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    gen = torch.Generator(device="cuda").manual_seed(wl["seed"])
    rnd = lambda *s: torch.randn(*s, generator=gen, device=dev).mul_(0.02)  # noqa: E731
    wg, rbias = _router_weights(wl, gen, dev)
    w1, w3, w2 = [], [], []
    El = E // world
    for e in range(E):
        mine = e % world == rank   # round-robin placement: rank r holds r, r + N, ...
        a, b, c = rnd(ff, d), rnd(ff, d), rnd(d, ff)   # every rank draws the same stream
        w1.append(a if mine else None)
        w3.append(b if mine else None)
        w2.append(c if mine else None)
        if not mine:
            del a, b, c
    ptr = lambda t: t.data_ptr() if t is not None else wg.data_ptr()  # noqa: E731
    layer = pkg.MoeLayer.expert_parallel(
        rank, world, obj[0], d=d, ff=ff, E=E, wg=wg.data_ptr(), w1=[ptr(t) for t in w1],
        w3=[ptr(t) for t in w3], w2=[ptr(t) for t in w2], device_pointers=True, top_k=k,
        bias=rbias.data_ptr() if rbias is not None else None,
        policy=pkg.ROUTER_SOFTMAX_TOPK, precision=mode["prec"], device=local, max_tokens=T,
        gemm_variant=_gemm_variant(args, pkg), ep_transport=_ep_transport(args, pkg))
    del w1, w3, w2
    torch.cuda.empty_cache()
    xgen = torch.Generator(device="cuda").manual_seed(wl["seed"] * 1000 + 17 + rank)
    x = torch.randn(T, d, generator=xgen, device=dev)
    y = torch.empty_like(x)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    step = lambda: layer.ep_forward_device(x.data_ptr(), y.data_ptr(), T, sp)  # noqa: E731
    for _ in range(args.warmup):
        step()
        flush.zero_()
    torch.cuda.synchronize()
    dist.barrier()
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    dist.barrier()
    total = 0.0
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        flush.zero_()
        b.synchronize()
        total += a.elapsed_time(b)
    torch.cuda.synchronize()
    dist.barrier()
    # One profiled step (collective: every rank runs it) for the stage
    # breakdown, and the rows each rank's experts received (load balance).
    layer.profile(True)
    step()
    ep_stages = layer.stage_ms()
    rows_here = float(layer.expert_counts().sum())
    layer.profile(False)
    torch.cuda.synchronize()
    rr = torch.tensor([rows_here, rows_here], dtype=torch.float64, device=dev)
    dist.all_reduce(rr[0:1], op=dist.ReduceOp.MAX)
    dist.all_reduce(rr[1:2], op=dist.ReduceOp.SUM)
    rows_max, rows_mean = float(rr[0]), float(rr[1]) / world
    dist.barrier()
    # e2e: pinned host x in, y out, copies inside the timed region.
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    e2e_n = max(3, args.steps // 2)
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_n):
        x.copy_(xh, non_blocking=True)
        step()
        yh.copy_(y, non_blocking=True)
    b.record(stream)
    b.synchronize()
    e2e_ms = a.elapsed_time(b) / e2e_n
    clocks = sampler.stop()
    t = torch.tensor([total, e2e_ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0]) / args.steps
    e2e_ms = float(t[1])
    if rank == 0:
        hbm, bf16_peak, _, src = _peaks()
        flops = 6.0 * T * k * d * ff          # expert FLOPs per rank (average routed rows)
        achieved = flops / (ms / 1e3) / 1e12
        print(json.dumps({
            "metric": METRIC, "value": world * T / (ms / 1e3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": mode["dtype"],
            "data": "synthetic (seeded torch CUDA generator: N(0,0.02) weights, N(0,1) x)",
            "config": _config(wl, args, world),
            "roofline": {"kernel": "whole expert-parallel step (exchanges included), per GPU",
                         "bound": "tensor", "achieved": achieved, "peak": bf16_peak,
                         "unit": "TFLOP/s", "frac": achieved / bf16_peak,
                         "frac_of_mode_ceiling": achieved * mode["passes"] / bf16_peak,
                         "traffic": None, "peak_source": f"{src} dense bf16, burst",
                         "stages_ms_rank0": {nm: round(float(v), 4) for nm, v in
                                             zip(pkg.PROFILE_STAGES, ep_stages)},
                         "expert_load": {"rows_max_rank": rows_max, "rows_mean_rank": rows_mean,
                                         "imbalance": rows_max / max(rows_mean, 1.0)}},
            "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": T * d * 4, "d2h_bytes_per_step": T * d * 4,
                    "how": "pinned host x -> device -> moe_ep_forward_device -> pinned host y, "
                           "CUDA events, max over ranks"},
            "gpu_launches": 9 * args.steps,
            "clocks": clocks,
        }))
    layer.close()
    return 0


def _timed(fn, n, warmup, flush, stream):
    """Mean device ms of fn over n calls (CUDA events on `stream`, L2
    flushed between calls outside the events), after `warmup` calls.  A
    0.2 ms device sleep precedes each start event: the host enqueues the
    call's kernels meanwhile, so the events bracket device work, not the
    host's launch latency (which the host-buffer e2e figures include)."""
    import torch
    for _ in range(warmup):
        fn()
        flush.zero_()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(SLEEP_CYCLES)
        a.record(stream)
        fn()
        b.record(stream)
        flush.zero_()
        b.synchronize()
        tot += a.elapsed_time(b)
    return tot / n


def _stages(layer, fn, n, flush):
    """Per-stage device ms of fn averaged over n profiled calls (the stage
    events sit between the kernels and turn dependent launches off, so only
    their shares are applied to the timed, unprofiled steps)."""
    import numpy as np
    import torch
    pkg = _pkg()
    layer.profile(True)
    st = np.zeros(len(pkg.PROFILE_STAGES))
    for _ in range(n):
        fn()
        st += layer.stage_ms()
        flush.zero_()
    torch.cuda.synchronize()
    layer.profile(False)
    return st / n


def measure_mode(args, wl, pkg, name, wptrs, x, y, flush, stream, decode_T, host_e2e):
    """One precision mode on this GPU: the timed prefill steps, the stage
    shares, the config-3 decode sweep and (headline mode) the host-buffer
    e2e.  Returns (numbers, layer handle)."""
    import numpy as np
    import torch
    mode = PRECISIONS[name]
    T, d, ff, E, k = wl["T"], wl["d"], wl["ff"], wl["E"], wl["k"]
    layer = pkg.MoeLayer.from_device_pointers(
        d, ff, E, wptrs["wg"], wptrs["w1"], wptrs["w3"], wptrs["w2"], wptrs["bias"], top_k=k,
        policy=pkg.ROUTER_SOFTMAX_TOPK, precision=mode["prec"], device=x.device.index,
        max_tokens=T, decode_max_tokens=args.decode_max_tokens,
        gemm_variant=_gemm_variant(args, pkg))
    layer.profile(False)
    sp = stream.cuda_stream

    def step():
        layer.forward_device(x.data_ptr(), y.data_ptr(), T, sp)

    ms = _timed(step, args.steps, args.warmup, flush, stream)
    st = _stages(layer, step, max(3, args.steps // 5), flush)
    share = dict(zip(pkg.PROFILE_STAGES, st / max(st.sum(), 1e-9)))
    _, bf16_peak, _, _ = _peaks()
    gu_ms = ms * share["gateup_gemm"]
    dn_ms = ms * share["down_gemm"]
    gu_tf = 4.0 * T * k * d * ff / (gu_ms / 1e3) / 1e12
    layer_tf = 6.0 * T * k * d * ff / (ms / 1e3) / 1e12
    out = {"tokens_per_s": T / (ms / 1e3), "ms_per_step": ms,
           "gateup_ms": gu_ms, "down_ms": dn_ms,
           "gateup_tflops": gu_tf, "gateup_frac": gu_tf / bf16_peak,
           "layer_tflops": layer_tf, "layer_frac": layer_tf / bf16_peak,
           "tc_passes": mode["passes"],
           "stage_share": {n: round(float(v), 4) for n, v in share.items() if v > 0}}
    if host_e2e:
        import ctypes
        xh = x.cpu().pin_memory()
        yh = torch.empty_like(xh).pin_memory()
        xn, yn = xh.numpy(), yh.numpy()
        lib = pkg.load_library()
        fp = ctypes.POINTER(ctypes.c_float)
        xp, yp = xn.ctypes.data_as(fp), yn.ctypes.data_as(fp)
        for _ in range(args.warmup):
            pkg._check(lib.moe_forward_host(layer._h, xp, yp, T))
        n = max(3, args.steps // 2)
        t0 = time.perf_counter()
        for _ in range(n):
            pkg._check(lib.moe_forward_host(layer._h, xp, yp, T))
        out["e2e_tokens_per_s"] = T / ((time.perf_counter() - t0) / n)
        out["output_finite"] = bool(np.isfinite(yn).all())
    dec = {}
    hbm = _peaks()[0]
    wbytes = 2 if name == "bf16" else 4
    for td in decode_T:
        xt, yt = x[:td], y[:td]
        fn = lambda: layer.forward_device(xt.data_ptr(), yt.data_ptr(), td, sp)  # noqa: E731
        ms_d = _timed(fn, max(5, args.steps), args.warmup, flush, stream)
        active = int((layer.expert_counts() > 0).sum())
        alg = active * 3 * d * ff * wbytes + E * d * 4 + 2 * td * d * 4
        gbs = alg / (ms_d / 1e3) / 1e9
        dec[str(td)] = {"ms": round(ms_d, 4), "gbs": round(gbs, 1), "frac": round(gbs / hbm, 3),
                        "path": "decode" if td <= layer.cfg.decode_max_tokens else "gemm"}
    out["decode"] = dec
    return out, layer


def run_single(args, wl, pkg, world, rank, local):
    """N = 1 (or token-sharded replicas): the headline precision and the other
    modes on this GPU, the decoder-layer block, the toy decoder, the CPU
    baseline."""
    import torch
    import torch.distributed as dist
    T, d, ff, E, k = wl["T"], wl["d"], wl["ff"], wl["E"], wl["k"]
    dev = torch.device("cuda", local)
    gen = torch.Generator(device="cuda").manual_seed(wl["seed"])
    rnd = lambda *s: torch.randn(*s, generator=gen, device=dev).mul_(0.02)  # noqa: E731
    wg, rbias = _router_weights(wl, gen, dev)
    w1 = [rnd(ff, d) for _ in range(E)]
    w3 = [rnd(ff, d) for _ in range(E)]
    w2 = [rnd(d, ff) for _ in range(E)]
    wptrs = {"wg": wg.data_ptr(), "w1": [t.data_ptr() for t in w1],
             "w3": [t.data_ptr() for t in w3], "w2": [t.data_ptr() for t in w2],
             "bias": rbias.data_ptr() if rbias is not None else None}
    host_layer = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host_layer = pkg.LayerWeights(wg.cpu().numpy(), [t.cpu().numpy() for t in w1],
                                      [t.cpu().numpy() for t in w3], [t.cpu().numpy() for t in w2])
    xgen = torch.Generator(device="cuda").manual_seed(wl["seed"] * 1000 + 17 + rank)
    x = torch.randn(T, d, generator=xgen, device=dev)
    y = torch.empty_like(x)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    decode_T = [] if args.no_decode else [t for t in DECODE_T if t <= T]
    names = [args.precision] + [m for m in args.modes.split(",")
                                if m and m != "none" and m != args.precision]
    if world > 1:
        dist.barrier()
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    sampler = ClockSampler(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
    time.sleep(0.3)
    modes, head_layer = {}, None
    for i, nm in enumerate(names):
        res, layer = measure_mode(args, wl, pkg, nm, wptrs, x, y, flush, stream, decode_T,
                                  host_e2e=(i == 0))
        modes[nm] = res
        if i == 0:
            head_layer = layer
        else:
            layer.close()
    del w1, w3, w2
    torch.cuda.empty_cache()
    head = modes[args.precision]

    # The decoder layer's MoE half: y = x + MoE(layer_norm(x)), the norm
    # fused into the router and the dispatch permute, the residual into the
    # ordered combine; and the standalone bit-exact LayerNorm.
    block = {}
    sp = stream.cuda_stream
    if not args.no_block:
        nw, nb = pkg.synthetic_post_norm(wl["seed"], d)
        head_layer.set_post_norm(nw, nb)
        wd, bd = torch.from_numpy(nw).to(dev), torch.from_numpy(nb).to(dev)
        yb = torch.empty_like(x)
        nb_steps = max(5, args.steps // 2)
        for tb in sorted({T, 1}):
            ms_b = _timed(lambda: head_layer.block_forward_device(x.data_ptr(), yb.data_ptr(), tb,
                                                                  sp), nb_steps, args.warmup,
                          flush, stream)
            block[str(tb)] = {"ms": round(ms_b, 4), "tokens_per_s": tb / (ms_b / 1e3)}
        block[str(T)]["overhead_ms_vs_moe_forward"] = block[str(T)]["ms"] - head["ms_per_step"]
        ms_ln = _timed(lambda: pkg.layer_norm_device(x.data_ptr(), wd.data_ptr(), bd.data_ptr(),
                                                     1e-5, T, d, yb.data_ptr(), sp), nb_steps,
                       args.warmup, flush, stream)
        ln_bytes = 2 * T * d * 4
        block["layer_norm_device"] = {"T": T, "ms": round(ms_ln, 4),
                                      "frac_of_hbm": ln_bytes / (ms_ln / 1e3) / 1e9 / _peaks()[0]}
    head_layer.close()

    decoder = None
    if not args.no_decoder and world == 1:
        decoder = run_decoder(args, pkg, dev)
    clocks = sampler.stop()

    ms, e2e_tps = head["ms_per_step"], head["e2e_tokens_per_s"]
    if world > 1:
        t = torch.tensor([ms, T / e2e_tps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_s = float(t[0]), float(t[1])
        e2e_tps = T / e2e_s
    if rank != 0:
        return 0
    hbm, bf16_peak, _, src = _peaks()
    mode = PRECISIONS[args.precision]
    roofline = {
        "kernel": f"gate/up grouped GEMM (tcgen05, SwiGLU epilogue), {args.precision}",
        "bound": "tensor", "achieved": head["gateup_tflops"], "peak": bf16_peak,
        "unit": "TFLOP/s", "frac": head["gateup_frac"],
        "frac_of_mode_ceiling": head["gateup_frac"] * mode["passes"],
        "traffic": _traffic_from_profile(wl["workload"], args.precision),
        "peak_source": f"{src} dense bf16, burst (the GEMM runs ~1-10 ms per step)",
        "how": "achieved = 4*T*k*d*ff / (timed step ms x the GEMM's share of a profiled step); "
               "frac counts algorithmic FLOPs once (fp32-faithful modes: ceiling 1/passes)",
        "modes": {nm: {key: (round(v, 4) if isinstance(v, float) else v)
                       for key, v in r.items() if key not in ("decode", "stage_share")}
                  for nm, r in modes.items()},
        "decode": {"hbm_peak_gbs": hbm,
                   "bytes": "routed experts x 3 x d x d_ff x weight bytes + router + x/y",
                   **{nm: {t: [v["path"], v["ms"], v["frac"]] for t, v in r["decode"].items()}
                      for nm, r in modes.items() if r["decode"]}},
    }
    if decoder is not None:
        roofline["decoder"] = {
            f"batch{b}": {"decode_ms_per_step": round(v["decode_ms_per_step"], 4),
                          "decode_tokens_per_s": round(v["decode_tokens_per_s"], 1),
                          "decode_frac_of_hbm": round(v["decode_frac_of_hbm"], 3),
                          "prefill_ms": round(v["prefill_ms"], 3),
                          **({"fused_decode_frac_of_hbm": round(v["fused_decode_frac_of_hbm"], 3)}
                             if "fused_decode_frac_of_hbm" in v else {})}
            for b, v in decoder["by_batch"].items()}
    line = {
        "metric": METRIC, "value": world * T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": mode["dtype"],
        "data": "synthetic (seeded torch CUDA generator: N(0,0.02) weights, N(0,1) x)",
        "config": _config(wl, args, world),
        "stages_share": head["stage_share"],
        "block": block,
        "decoder": decoder,
        "gpu_launches": KERNELS_PER_FORWARD * args.steps,
        "output_finite": head.get("output_finite"),
        "e2e": {"value": world * e2e_tps, "unit": "tokens/s", "h2d_bytes_per_step": T * d * 4,
                "d2h_bytes_per_step": T * d * 4,
                "how": "moe_forward_host on pinned host buffers, host clock around the "
                       "synchronous call"},
        "clocks": clocks,
        "roofline": roofline,
    }
    if host_layer is not None:
        xs = x[: min(T, 1024)].cpu().numpy()
        tps, kind, n, cores = cpu_reference_tokens_per_s(host_layer, xs,
                                                         len(os.sched_getaffinity(0)))
        line["cpu_baseline"] = {
            "value": tps, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{n} tokens of this layer through PhiMoE::forward (fp32, "
                      f"its quantised top-2 router), {cores} OpenMP threads"}
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--precision", choices=sorted(PRECISIONS), default="bf16x3",
                    help="headline precision: bf16x3 (fp32-faithful, default), 3xtf32 "
                         "(fp32-faithful) or bf16")
    ap.add_argument("--modes", default="bf16",
                    help="other precisions measured on one GPU besides the headline, "
                         "comma-separated (reported under roofline.modes), or none")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["c4"], default="c2",
                    help="c2 (default, the headline layer), c2small, c5, or c4: only the toy "
                         "MoE decoder (BASELINE config 4), one GPU")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--gemm", choices=["auto", "ctapair", "single"], default="auto",
                    help="grouped-GEMM tiling: auto (2-CTA 256x256 tiles for prefill, 1-CTA "
                         "128x256 for decode-sized T), or force one")
    ap.add_argument("--ep-transport", choices=["p2p", "nccl"], default="p2p",
                    help="expert-parallel exchange: the deduplicated NVLink peer-store "
                         "transport (default) or NCCL send/recv")
    ap.add_argument("--parallelism", choices=["ep", "dp"], default="ep",
                    help="N > 1: expert parallel (default) or token-sharded replicas")
    ap.add_argument("--no-block", action="store_true",
                    help="skip the decoder-layer block section (post-attention LayerNorm + "
                         "MoE + residual)")
    ap.add_argument("--no-decoder", action="store_true",
                    help="skip the toy MoE decoder section (BASELINE config 4)")
    ap.add_argument("--decoder-new-tokens", type=int, default=None,
                    help="generated tokens per sequence in the decoder section (default 128)")
    ap.add_argument("--decoder-layers", type=int, default=None,
                    help="decoder layers (default 8; fewer for a small profiling case)")
    ap.add_argument("--decoder-batches", default=None,
                    help="comma-separated decoder batch sizes (default 1,16)")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket one decoder generate per batch with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--decode-max-tokens", type=int, default=None,
                    help="override the handle's decode threshold (0..64)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    for m in args.modes.split(","):
        if m and m != "none" and m not in PRECISIONS:
            ap.error(f"unknown mode {m}")
    if args.workload == "c4":
        return decoder_only(args)
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return reference_arm(args, wl)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # Rank 0's stdout carries exactly one JSON line: keep NCCL's banner off it.
    if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        os.environ["NCCL_DEBUG"] = "WARN"
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    pkg = _pkg()
    if world > 1 and args.parallelism == "ep":
        rc = run_ep(args, wl, pkg, world, rank, local)
    else:
        rc = run_single(args, wl, pkg, world, rank, local)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
