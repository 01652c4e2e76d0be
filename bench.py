"""Decode throughput of the quantized-weight path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c2|c1] [--impl dz|reference]

A step is one whole job of the workload on each GPU: for C2 (the default),
64 sequences x (32 prompt tokens prefilled + 32 top-p draws) of the 4-layer
d128 INT4 model. Sequences are independent: each rank runs its own 64
(weak scaling, no collective on the data path). Prints one JSON line on rank 0.

value: generated tokens / device time with prompts, seeds and outputs resident
in HBM (CUDA events on the launching stream, L2 flushed between steps outside
the events, max over ranks). e2e: the same jobs through the public C ABI
(dz_cuda_generate) from pinned host buffers, host<->device copies inside the
events. roofline: the dominant kernel class of one eagerly launched job, timed
per launch with CUDA events. cpu_baseline: the reference's own C sources
(oracle/_ref) on this host's cores, sequence-parallel, on the same workload.
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "INT4/INT8 decode tokens/s at 1/2/4/8 B200; quant-matvec HBM GB/s vs peak"
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of one dz_seqgen_kernel launch on the
# C2 job (64 sequences x (32 + 32), INT4 d128 L4 V512), one ncu capture
SEQGEN_C2_DRAM_BYTES = 1025280 + 60672


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, 1590.0, "fallback"


# ------------------------------------------------------------------ clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = f"/tmp/dz_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.remove(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- CPU baseline

def cpu_sample(wl):
    """(sequences, prompt_len, n_new, one shared session) the CPU baseline runs."""
    if wl.cpu_sample:
        return wl.cpu_sample
    return (wl.batch, wl.prompt_len, wl.n_new, False)


def cpu_reference(wl, seqs=None, repeats=2):
    """The reference's own C path (oracle/_ref/libdzref.so: model_forward_token
    + sample_next_token in the generation loop) on the host cores: either
    sequences spread over threads (one session each, OMP 1) or, for models too
    large to hold once per thread, one session with every thread in the
    reference's OpenMP matmul. Falls back to the oracle port when the
    reference build is absent."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from dranzer_b200 import workloads as W
    from _native_oracle import REF_SO, Oracle
    cores = os.cpu_count() or 1
    n, plen, n_new, shared = cpu_sample(wl)
    if seqs is not None:
        n = seqs
    prompts, seeds = W.prompts(wl)[:n, :plen], W.seeds(wl)[:n]
    mk = np.array(W.MASKED, np.uint32)
    out = np.zeros((n, n_new), np.uint32)
    workers = 1 if shared else cores
    if os.path.exists(REF_SO):
        kind = "reference"
        L = ctypes.CDLL(REF_SO)
        L.rh_build_bundle.argtypes = [ctypes.c_char_p] + [ctypes.c_size_t] * 5 + [ctypes.c_uint64, ctypes.c_int,
                                                                                  ctypes.c_int]
        L.rh_load.restype = ctypes.c_void_p
        L.rh_load.argtypes = [ctypes.c_char_p]
        L.rh_free.argtypes = [ctypes.c_void_p]
        L.rh_set_omp_threads.argtypes = [ctypes.c_int]
        L.rh_generate.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                  ctypes.c_size_t, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_float,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                  ctypes.c_void_p]
        path = f"/tmp/dz_cpu_ref_{os.getpid()}.bin".encode()
        s = wl.spec
        assert L.rh_build_bundle(path, s.vocab, s.dim, s.heads, s.layers, s.max_seq, wl.weight_seed, wl.bits, 2) == 0
        sessions = [L.rh_load(path) for _ in range(workers)]
        os.remove(path)

        def run(t, lo, hi):
            L.rh_set_omp_threads(cores if shared else 1)
            p = np.ascontiguousarray(prompts[lo:hi])
            sd = np.ascontiguousarray(seeds[lo:hi])
            o = np.zeros((hi - lo, n_new), np.uint32)
            L.rh_generate(sessions[t], p.ctypes.data, hi - lo, plen, n_new, wl.strategy,
                          wl.temperature, wl.top_k, wl.top_p, sd.ctypes.data if wl.strategy else None,
                          mk.ctypes.data, mk.size, o.ctypes.data, None)
            out[lo:hi] = o
    else:
        kind = "port"
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from _models import Spec, quantize_params, synth_params
        o_ = Oracle()
        s = wl.spec
        spec = Spec(s.vocab, s.dim, s.heads, s.layers, s.max_seq)
        _, flat = quantize_params(o_, spec, synth_params(o_, spec, wl.weight_seed), wl.bits)
        models = [o_.model(spec, flat) for _ in range(workers)]

        def run(t, lo, hi):
            toks, _ = models[t].generate(np.ascontiguousarray(prompts[lo:hi]), n_new, wl.strategy, wl.temperature,
                                         wl.top_k, wl.top_p, seeds[lo:hi] if wl.strategy else None, W.MASKED)
            out[lo:hi] = toks
    times = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        ths = []
        for t in range(workers):
            lo, hi = W.shard(n, t, workers)
            if hi > lo:
                ths.append(threading.Thread(target=run, args=(t, lo, hi)))
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        times.append(time.perf_counter() - t0)
    if kind == "reference":
        for h in sessions:
            L.rh_free(h)
    best = min(times)
    how = (f"one session, {cores} OpenMP threads" if shared
           else f"sequences spread over {cores} threads (OMP 1 each)")
    return {"value": n * n_new / best, "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{n} sequences x ({plen} prompt + {n_new} decode), best of {repeats}, {how}",
            "seconds": best}, out


# ---------------------------------------------------------------- GPU arm

def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                 device_id=torch.device("cuda", local))
    return world, rank, local


def quant_matvec_probe(dz, torch, stream, hbm, bf16=None):
    """C3 rows: K=4096, N=32000, M in {1, 8, 64, 512}, INT8 and INT4; enough
    weight copies rotated per launch that the weights exceed L2 (126 MB)."""
    res = []
    st = np.array([dz.rng_stream(3, dz.STREAM_TESTING)], np.uint64)
    Ms = (1, 8, 64, 512)
    x = dz.synth_gaussian(st, max(Ms) * 4096, 1.0).reshape(max(Ms), 4096)
    w = dz.synth_gaussian(st, 4096 * 32000, 0.02).reshape(4096, 32000)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((max(Ms), 32000), dtype=torch.float32, device="cuda")
    for bits in (8, 4):
        s, p = dz.quantize_pack(w, bits)
        copies = 2 if bits == 8 else 4
        mats = [dz.QuantizedWeightMatrix(s, p, 4096, 32000, bits) for _ in range(copies)]
        for M in Ms:
            for i in range(6):
                mats[i % copies].matmul_async(xd.data_ptr(), yd.data_ptr(), M, stream.cuda_stream)
            reps = 24 if M <= 64 else 8
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            torch.cuda.synchronize()
            # a bounded device-side delay lets the host enqueue the whole burst
            # first, so the events see device time rather than launch cadence
            if hasattr(torch.cuda, "_sleep"):
                with torch.cuda.stream(stream):
                    torch.cuda._sleep(8_000_000)
            for i in range(reps):
                evs[i][0].record(stream)
                mats[i % copies].matmul_async(xd.data_ptr(), yd.data_ptr(), M, stream.cuda_stream)
                evs[i][1].record(stream)
            torch.cuda.synchronize()
            ms = statistics.median(a.elapsed_time(b) for a, b in evs)
            # the same launches back to back, as a decode stream issues them:
            # one event pair around the burst
            b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            if hasattr(torch.cuda, "_sleep"):
                with torch.cuda.stream(stream):
                    torch.cuda._sleep(8_000_000)
            b0.record(stream)
            for i in range(reps):
                mats[i % copies].matmul_async(xd.data_ptr(), yd.data_ptr(), M, stream.cuda_stream)
            b1.record(stream)
            torch.cuda.synchronize()
            ms_stream = b0.elapsed_time(b1) / reps
            nbytes = 4096 * 32000 * bits / 8 + 32000 * 4 + M * 4096 * 4 + M * 32000 * 4
            gbs = nbytes / (ms * 1e-3) / 1e9
            tflops = 2.0 * M * 4096 * 32000 / (ms * 1e-3) / 1e12
            r = {"bits": bits, "M": M, "K": 4096, "N": 32000, "us": round(ms * 1e3, 2),
                 "GB/s": round(gbs, 1), "frac": round(gbs / hbm, 3), "TFLOP/s": round(tflops, 1),
                 "bytes": int(nbytes), "us_stream": round(ms_stream * 1e3, 2),
                 "frac_stream": round(nbytes / (ms_stream * 1e-3) / 1e9 / hbm, 3)}
            if bf16:
                r["tensor_frac_of_bf16"] = round(tflops / bf16, 4)
            res.append(r)
        for m in mats:
            m.close()
    return res


def run_dz(args, wl):
    import torch
    import dranzer_b200 as dz
    from dranzer_b200 import _native
    from dranzer_b200 import workloads as W
    world, rank, local = dist_init()
    torch.cuda.set_device(local)
    if not dz.available():
        raise RuntimeError("no usable B200")
    hbm, bf16, peak_src = peaks()

    path = f"/tmp/dz_bench_{os.getpid()}_{rank}.bin"
    W.write_bundle(wl, path)
    bundle = dz.Bundle(path)
    model = dz.Model.from_bundle(bundle, device=local)
    cache = dz.KVCache(model, wl.batch, wl.capacity or wl.spec.max_seq)
    stream = torch.cuda.Stream()
    cache.set_stream(stream.cuda_stream)
    samp = wl.sampling()

    prompts = W.prompts(wl, rank)
    seeds = W.seeds(wl, rank)
    pd = torch.from_numpy(prompts.astype(np.int32)).cuda()
    sdv = torch.from_numpy(seeds.astype(np.int64)).cuda()
    od = torch.zeros((wl.batch, wl.n_new), dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    seeds_ptr = sdv.data_ptr() if wl.strategy else None

    def job():
        cache.generate_async(pd.data_ptr(), wl.prompt_len, wl.n_new, samp, seeds_ptr, od.data_ptr())

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            job()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            import torch.distributed as tdist
            tdist.barrier()

    clocks = ClockSampler(local)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    with torch.cuda.stream(stream):
        for k in range(args.steps):
            flush.zero_()
            evs[k][0].record(stream)
            job()
            evs[k][1].record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    dev_ms = sum(a.elapsed_time(b) for a, b in evs)
    tokens_local = wl.batch * wl.n_new * args.steps
    got = od.cpu().numpy().astype(np.uint32)

    # e2e through the public C ABI from pinned host buffers
    hp = torch.from_numpy(prompts.astype(np.int32)).pin_memory()
    hs = torch.from_numpy(seeds.astype(np.int64)).pin_memory()
    ho = torch.zeros((wl.batch, wl.n_new), dtype=torch.int32).pin_memory()
    L = _native.lib()

    def job_e2e():
        _native.check(L.dz_cuda_generate(cache.handle, hp.data_ptr(), wl.prompt_len, wl.n_new,
                                         ctypes.byref(samp.c), hs.data_ptr() if wl.strategy else None,
                                         ho.data_ptr()), "generate")

    job_e2e()
    e2e_evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    for k in range(args.steps):
        with torch.cuda.stream(stream):
            flush.zero_()
            e2e_evs[k][0].record(stream)
        job_e2e()
        with torch.cuda.stream(stream):
            e2e_evs[k][1].record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = sum(a.elapsed_time(b) for a, b in e2e_evs)
    assert np.array_equal(ho.numpy().astype(np.uint32), got), "e2e tokens differ from the device-resident run"

    if world > 1:
        import torch.distributed as tdist
        t = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device="cuda")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        dev_ms, e2e_ms = float(t[0]), float(t[1])

    # per-kernel-class CUDA-event timing of one eager job (the full prompt + 8
    # decode steps at the full batch when the real job is too long to bracket
    # every launch)
    nk = len(_native.KERNEL_CLASSES) + len(_native.FUSED_PHASES)
    stats = (_native.DzKernelStat * nk)()
    long_job = cache.generate_launches(wl.prompt_len, wl.n_new, samp) > 20000
    p_plen, p_new = (wl.prompt_len, 8) if long_job else (wl.prompt_len, wl.n_new)
    _native.check(L.dz_cuda_profile_generate(cache.handle, pd.data_ptr(), p_plen, p_new,
                                             ctypes.byref(samp.c), seeds_ptr, od.data_ptr(), stats, nk),
                  "profile_generate")
    classes = {}
    for k, name in enumerate(_native.KERNEL_CLASSES):
        s = stats[k]
        if s.launches:
            classes[name] = {"launches": int(s.launches), "total_ms": round(s.total_ms, 4),
                             "avg_us": round(1e3 * s.total_ms / s.launches, 3),
                             "bytes_per_launch": int(s.bytes / s.launches),
                             "flops_per_launch": float(s.flops / s.launches)}
    phases = {name: round(stats[len(_native.KERNEL_CLASSES) + k].total_ms, 4)
              for k, name in enumerate(_native.FUSED_PHASES) if stats[len(_native.KERNEL_CLASSES) + k].total_ms}
    dom = max(classes, key=lambda n: classes[n]["total_ms"])
    d = classes[dom]
    achieved = d["bytes_per_launch"] / (d["avg_us"] * 1e-6) / 1e9
    # arithmetic intensity above the ridge (bf16 peak / HBM peak): tensor-bound
    tensor_bound = d["flops_per_launch"] > 0 and d["flops_per_launch"] / d["bytes_per_launch"] > bf16 * 1e3 / hbm
    achieved_tf = d["flops_per_launch"] / (d["avg_us"] * 1e-6) / 1e12
    total_prof = sum(c["total_ms"] for c in classes.values())
    for c in classes.values():
        c["share"] = round(c["total_ms"] / total_prof, 3)

    launches = cache.generate_launches(wl.prompt_len, wl.n_new, samp) * args.steps
    out = None
    if rank == 0:
        tokens = tokens_local * world
        value = tokens / (dev_ms * 1e-3)
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": f"int{wl.bits} weights, fp32 compute",
            "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids; no dataset named)",
            "config": {"workload": wl.name, "model": f"DRANZER d{wl.spec.dim} h{wl.spec.heads} L{wl.spec.layers} "
                       f"V{wl.spec.vocab} T{wl.spec.max_seq}", "bits": wl.bits,
                       "sequences_per_gpu": wl.batch, "global_batch": wl.batch * world,
                       "prompt_len": wl.prompt_len, "decode_len": wl.n_new, "seq_len": wl.prompt_len + wl.n_new,
                       "sampling": {"strategy": ["greedy", "top-k", "top-p"][wl.strategy],
                                    "temperature": wl.temperature, "top_k": wl.top_k, "top_p": wl.top_p},
                       "parallelism": f"batch-sharded x{world} (independent sequences, no collective)",
                       "l2": "flushed between steps (256 MiB write on the stream, outside the timed events)",
                       "step": "prefill prompt token by token + decode, one CUDA graph per job"},
            "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(prompts.nbytes + (seeds.nbytes if wl.strategy else 0)),
                    "d2h_bytes_per_step": int(wl.batch * wl.n_new * 4)},
            "gpu_launches": int(launches),
            "roofline": ({"bound": "tensor", "kernel": dom, "achieved": round(achieved_tf, 1), "peak": bf16,
                          "unit": "TFLOP/s", "frac": round(achieved_tf / bf16, 4), "peak_source": peak_src,
                          "traffic": None,
                          "note": "flops = 2*M*K*N of the quantized GEMMs (useful work; the integer "
                                  "tensor cores run three 8-bit limb passes of it); peak = measured dense "
                                  "bf16; the profiled job is " + (f"{p_plen} + {p_new} tokens at the "
                                  "full batch" if long_job else "the measured one")}
                         if tensor_bound else
                         {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm,
                         "unit": "GB/s", "frac": round(achieved / hbm, 4), "peak_source": peak_src,
                         # DRAM bytes of one dz_seqgen_kernel launch on this workload, from one ncu
                         # capture (profiles/seqgen_c2_int4.md)
                         "traffic": SEQGEN_C2_DRAM_BYTES if dom == "seqgen" and wl.name == W.C2.name else None,
                         "note": "bytes = weight codes+scales+fp32 tensors each sequence streams per step "
                                 "x steps x sequences; all of it is L2-resident for this workload, so the "
                                 "kernel is latency/L2 bound, not HBM bound"}),
            "path": "fused" if cache.uses_fused(samp) else "layered",
            "kernels": classes,
            "fused_phases_ms": phases,
            "clocks": clk,
        }
    if rank == 0 and world == 1:
        out["quant_matvec"] = quant_matvec_probe(dz, torch, stream, hbm, bf16)
        cpu, cpu_tokens = cpu_reference(wl)
        out["cpu_baseline"] = {k: v for k, v in cpu.items() if k != "seconds"}
        if wl.cpu_sample:
            # the same sample through the device path
            n, plen, n_new, _ = cpu_sample(wl)
            sc = dz.KVCache(model, n, plen + n_new)
            sp = np.ascontiguousarray(prompts[:n, :plen])
            gs = sc.generate(sp, n_new, samp, seeds=seeds[:n] if wl.strategy else None)
            sc.close()
            out["cpu_baseline"]["tokens_match_gpu"] = bool(np.array_equal(cpu_tokens, gs))
        else:
            out["cpu_baseline"]["tokens_match_gpu"] = bool(np.array_equal(cpu_tokens, got))
    cache.close()
    model.close()
    bundle.close()
    os.remove(path)
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
        tdist.destroy_process_group()
    return out


def run_reference(args, wl):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    vals = []
    for _ in range(args.warmup):
        cpu_reference(wl, repeats=1)
    for _ in range(args.steps):
        cpu, _ = cpu_reference(wl, repeats=1)
        vals.append(cpu["value"])
    v = statistics.median(vals)
    return {"metric": METRIC, "value": round(v, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * wl.batch * wl.n_new / v, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"int{wl.bits} weights dequantized to fp32 at load (reference loader), fp32 compute",
            "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids; no dataset named)",
            "config": {"workload": wl.name, "sequences": wl.batch, "prompt_len": wl.prompt_len,
                       "decode_len": wl.n_new},
            "impl": "reference",
            "cpu_baseline": {"value": round(v, 1), "unit": "tokens/s", "cores": cpu["cores"], "kind": cpu["kind"],
                             "sample": cpu["sample"]},
            "e2e": {"value": round(v, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c2")
    ap.add_argument("--impl", default="dz", choices=["dz", "reference"])
    ap.add_argument("--probe", choices=["qmv"], help="run only the C3 quantized-matvec probe (profiling target)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.probe == "qmv":
        import torch
        import dranzer_b200 as dz
        stream = torch.cuda.Stream()
        hbm, bf16, _ = peaks()
        print(json.dumps({"quant_matvec": quant_matvec_probe(dz, torch, stream, hbm, bf16)}))
        return
    from dranzer_b200 import workloads as W
    wl = W.WORKLOADS[args.workload]
    out = run_reference(args, wl) if args.impl == "reference" else run_dz(args, wl)
    if out is not None:
        print(json.dumps(out))


if __name__ == "__main__":
    main()
