"""Decode throughput of the quantized-weight path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c4|c2|c1] [--impl dz|reference]

A step is one whole job of the workload, split over the GPUs: for config 4
(the default, the largest configuration that fits one GPU) 256 sequences of
the 24-layer d2048 INT8 model, each 512 prompt tokens prefilled then 128
greedy draws. At N GPUs each rank runs 256/N of the sequences (strong
scaling: the job is fixed, no collective on the data path). Config 2 (64 x
(32 + 32) top-p on the 4-layer d128 INT4 model) runs after it as a secondary
line, split the same way. Rank 0 prints one JSON line.

value: generated tokens of the job / device time (CUDA events on the
launching stream, prompts, seeds and outputs resident in HBM, L2 flushed
between steps outside the events, max over ranks). e2e: the same job
through the public C ABI (dz_cuda_generate) from pinned host buffers, the
host<->device copies inside the events. roofline: the kernel class with the
largest share of the job (per-launch CUDA events of eagerly launched
prefill and decode steps), its algorithmic bytes or flops per launch over
its mean launch time. cpu_baseline: the reference's own C sources
(oracle/_ref) on this host's cores, on a bounded sample of the same job.

--impl reference times that reference build alone (rank 0; the other ranks
exit), on a bounded sample per step, and imports nothing of dranzer_b200.
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
FALLBACK_BF16_TFLOPS = 1590.0
MASKED = (256, 257, 258, 259)

# The workloads as the reference arm needs them: plain data, so that arm
# loads nothing of dranzer_b200 (tests/test_bench_config.py keeps this table
# equal to dranzer_b200/workloads.py). cpu_sample: (sequences, prompt tokens,
# decode tokens, one session with every host thread) or None for the job.
REF_WORKLOADS = {
    "c1": dict(name="c1-int8-greedy-b1-16+48", vocab=512, dim=128, heads=4, layers=4, max_seq=64, bits=8,
               weight_seed=0, prompt_seed=1, batch=1, prompt_len=16, n_new=48, strategy=0, temperature=0.0,
               top_k=0, top_p=0.0, seed_base=0, cpu_sample=None),
    "c2": dict(name="c2-int4-topp0.9-64x(32+32)", vocab=512, dim=128, heads=4, layers=4, max_seq=64, bits=4,
               weight_seed=0, prompt_seed=2, batch=64, prompt_len=32, n_new=32, strategy=2, temperature=0.8,
               top_k=0, top_p=0.9, seed_base=2000, cpu_sample=None),
    "c4": dict(name="c4-int8-greedy-256x(512+128)", vocab=32000, dim=2048, heads=16, layers=24, max_seq=2048,
               bits=8, weight_seed=4, prompt_seed=4, batch=256, prompt_len=512, n_new=128, strategy=0,
               temperature=0.0, top_k=0, top_p=0.0, seed_base=0, cpu_sample=(1, 16, 4, True)),
}

# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant
# kernel on a workload, from one ncu capture (profiles/): (workload, class) ->
# bytes per launch, or absent.
NCU_TRAFFIC = {
    # dz_seqgen_kernel, the whole config-2 job (64 x (32 + 32)) in one launch
    ("c2-int4-topp0.9-64x(32+32)", "seqgen"): 1025280 + 60672,
}
# Where the dominant kernel's launches are too many and too large to capture
# each, one capture's DRAM bytes over its algorithmic bytes, applied to the
# class's algorithmic bytes per launch (the launches scale with the context).
NCU_TRAFFIC_RATIO = {
    # dz_attn_decode_kernel<4>, one C4 decode step's layer at context 516-520
    # (profiles/attn_decode_c4_b256.md): 2.284 GB read + 5.5 MB written for
    # 256 x 518 x 2048 x 8 B of K/V rows + 4 MB of q and output
    ("c4-int8-greedy-256x(512+128)", "attention"): (2.284e9 + 5.5e6) / (256 * 518 * 2048 * 8 + 4.0e6),
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def shard(n_items, rank, world):
    """Contiguous share of n_items for `rank` of `world` (balanced, no gaps)."""
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


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


# --------------------------------------------------- CPU reference (checker)

def _checker():
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import _native_oracle
    return _native_oracle


def ref_prompts(w, n, plen):
    """The first n prompts of a workload, cut to plen tokens, drawn with the
    reference build's own RNG (dranzer_rng_stream/next, rejecting the
    control ids): the same ids the device arm draws."""
    no = _checker()
    if os.path.exists(no.REF_SO):
        L = no.RefHarness().L
        stream, nxt = L.dranzer_rng_stream, L.dranzer_rng_next
    else:
        o = no.Oracle()
        stream, nxt = o.L.or_rng_stream, o.L.or_rng_next
    st = np.array([stream(w["prompt_seed"], no.STREAM_TESTING)], np.uint64)
    out = []
    while len(out) < n * w["prompt_len"]:
        t = nxt(st.ctypes.data) % w["vocab"]
        if t not in MASKED:
            out.append(t)
    return np.array(out, np.uint32).reshape(n, w["prompt_len"])[:, :plen]


class CpuReference:
    """The reference's own C path (oracle/_ref/libdzref.so: model_forward_token
    + sample_next_token in the generation loop) on the host cores, on the
    workload's bounded sample: either sequences spread over threads (one
    session each, OMP 1) or, for models too large to hold once per thread,
    one session with every thread in the reference's OpenMP matmul. The
    oracle port stands in when the reference build is absent. The model is
    built once; run() times one pass over the sample."""

    def __init__(self, w):
        no = _checker()
        self.w = w
        self.cores = os.cpu_count() or 1
        n, plen, n_new, shared = w["cpu_sample"] or (w["batch"], w["prompt_len"], w["n_new"], False)
        self.n, self.plen, self.n_new, self.shared = n, plen, n_new, shared
        self.prompts = ref_prompts(w, n, plen)
        self.seeds = np.array([w["seed_base"] + i for i in range(n)], np.uint64)
        self.workers = 1 if shared else min(self.cores, n)
        self.out = np.zeros((n, n_new), np.uint32)
        self.mk = np.array(MASKED, np.uint32)
        if os.path.exists(no.REF_SO):
            self.kind = "reference"
            self.L = no.RefHarness().L
            self.L.rh_set_omp_threads.argtypes = [ctypes.c_int]
            path = f"/tmp/dz_cpu_ref_{os.getpid()}.bin".encode()
            assert self.L.rh_build_bundle(path, w["vocab"], w["dim"], w["heads"], w["layers"], w["max_seq"],
                                          w["weight_seed"], w["bits"], 2) == 0
            self.sessions = [self.L.rh_load(path) for _ in range(self.workers)]
            os.remove(path)
        else:
            self.kind = "port"
            from _models import Spec, quantize_params, synth_params
            o_ = no.Oracle()
            spec = Spec(w["vocab"], w["dim"], w["heads"], w["layers"], w["max_seq"])
            _, flat = quantize_params(o_, spec, synth_params(o_, spec, w["weight_seed"]), w["bits"])
            self.models = [o_.model(spec, flat) for _ in range(self.workers)]

    def _run_part(self, t, lo, hi):
        w = self.w
        p = np.ascontiguousarray(self.prompts[lo:hi])
        sd = np.ascontiguousarray(self.seeds[lo:hi])
        if self.kind == "reference":
            self.L.rh_set_omp_threads(self.cores if self.shared else 1)
            o = np.zeros((hi - lo, self.n_new), np.uint32)
            self.L.rh_generate(self.sessions[t], p.ctypes.data, hi - lo, self.plen, self.n_new, w["strategy"],
                               w["temperature"], w["top_k"], w["top_p"], sd.ctypes.data if w["strategy"] else None,
                               self.mk.ctypes.data, self.mk.size, o.ctypes.data, None)
        else:
            o, _ = self.models[t].generate(p, self.n_new, w["strategy"], w["temperature"], w["top_k"], w["top_p"],
                                           sd if w["strategy"] else None, MASKED)
        self.out[lo:hi] = o

    def run(self):
        t0 = time.perf_counter()
        ths = []
        for t in range(self.workers):
            lo, hi = shard(self.n, t, self.workers)
            if hi > lo:
                ths.append(threading.Thread(target=self._run_part, args=(t, lo, hi)))
        for th in ths:
            th.start()
        for th in ths:
            th.join()
        return time.perf_counter() - t0

    def describe(self, seconds, how_many):
        w = self.w
        how = (f"one session, {self.cores} OpenMP threads" if self.shared
               else f"sequences spread over {self.workers} threads (OMP 1 each)")
        sample = f"{self.n} sequence(s) x ({self.plen} prompt + {self.n_new} decode)"
        if w["cpu_sample"]:
            sample += (f" of the {w['batch']} x ({w['prompt_len']} + {w['n_new']}) job, at the job's "
                       "prompt-to-decode ratio; prompt fed token by token as the reference's generation loop does")
        return {"value": self.n * self.n_new / seconds, "unit": "tokens/s",
                "cores": self.cores if self.shared else self.workers, "kind": self.kind,
                "sample": f"{sample}; {how_many}; {how}"}

    def close(self):
        if self.kind == "reference":
            for h in self.sessions:
                self.L.rh_free(h)
            self.sessions = []


def run_reference(args, w):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    ref = CpuReference(w)
    for _ in range(args.warmup):
        ref.run()
    secs = [ref.run() for _ in range(args.steps)]
    ref.close()
    med = statistics.median(secs)
    cpu = ref.describe(med, f"median of {args.steps} steps")
    maps = open("/proc/self/maps").read()
    assert "libdz_cuda.so" not in maps, "the reference arm loaded this repository's CUDA library"
    v = cpu["value"]
    return {"metric": METRIC, "value": round(v, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1e3 * med, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": f"int{w['bits']} weights dequantized to fp32 at load (reference loader), fp32 compute",
            "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids; no dataset named)",
            "config": {"workload": w["name"], "sequences": w["batch"], "prompt_len": w["prompt_len"],
                       "decode_len": w["n_new"]},
            "impl": "reference",
            "cpu_baseline": {"value": round(v, 2), "unit": "tokens/s", "cores": cpu["cores"], "kind": cpu["kind"],
                             "sample": cpu["sample"]},
            "e2e": {"value": round(v, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "process_maps": "no libdz_cuda.so mapped (checked)"}


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
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
    return world, rank, local


def quant_matvec_probe(dz, torch, stream, hbm, bf16=None, cpu=False, Ns=(4096, 11008, 32000),
                       Ms=(1, 8, 64, 512), K=4096):
    """C3 rows: K=4096, N in {4096, 11008, 32000}, M in {1, 8, 64, 512},
    INT8 and INT4; enough weight copies rotated per launch that the weights
    exceed L2 (126 MB). cpu: also time the reference's own
    matmul_quantized_weight (oracle/_ref, OpenMP over the host cores, median
    of 3) at M = 1 and 8, and M = 64 at N = 4096."""
    res = []
    ref = None
    if cpu:
        no = _checker()
        if os.path.exists(no.REF_SO):
            ref = no.RefHarness()
            ref.L.rh_set_omp_threads.argtypes = [ctypes.c_int]
            ref.L.rh_set_omp_threads(os.cpu_count() or 1)
    for N in Ns:
        st = np.array([dz.rng_stream(3, dz.STREAM_TESTING)], np.uint64)
        x = dz.synth_gaussian(st, max(Ms) * K, 1.0).reshape(max(Ms), K)
        w = dz.synth_gaussian(st, K * N, 0.02).reshape(K, N)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((max(Ms), N), dtype=torch.float32, device="cuda")
        for bits in (8, 4):
            s, p = dz.quantize_pack(w, bits)
            wbytes = K * N * bits // 8
            copies = max(2, -(-(256 << 20) // wbytes))
            mats = [dz.QuantizedWeightMatrix(s, p, K, N, bits) for _ in range(copies)]
            rh = ref.qmat(w, bits, 2) if ref is not None else None
            for M in Ms:
                # every copy once first: a copy grows its scratch on its first call at a new M
                for i in range(max(6, copies)):
                    mats[i % copies].matmul_async(xd.data_ptr(), yd.data_ptr(), M, stream.cuda_stream)
                reps = 24 if M <= 64 else 8
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(reps)]
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
                # the same launches back to back, as a decode stream issues them
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
                nbytes = wbytes + N * 4 + M * K * 4 + M * N * 4
                gbs = nbytes / (ms * 1e-3) / 1e9
                tflops = 2.0 * M * K * N / (ms * 1e-3) / 1e12
                r = {"bits": bits, "M": M, "K": K, "N": N, "us": round(ms * 1e3, 2),
                     "GB/s": round(gbs, 1), "frac": round(gbs / hbm, 3), "TFLOP/s": round(tflops, 1),
                     "bytes": int(nbytes), "us_stream": round(ms_stream * 1e3, 2),
                     "frac_stream": round(nbytes / (ms_stream * 1e-3) / 1e9 / hbm, 3)}
                if bf16:
                    r["tensor_frac_of_bf16"] = round(tflops / bf16, 4)
                if rh is not None and (M <= 8 or (M == 64 and N == 4096)):
                    xa = np.ascontiguousarray(x[:M])
                    c = np.empty((M, N), np.float32)
                    ts = []
                    for _ in range(3):
                        t0 = time.perf_counter()
                        ref.L.rh_qmat_matmul(rh, xa.ctypes.data, c.ctypes.data, M)
                        ts.append(time.perf_counter() - t0)
                    r["cpu_reference_us"] = round(statistics.median(ts) * 1e6, 1)
                res.append(r)
            if rh is not None:
                ref.L.rh_qmat_free(rh)
            for m in mats:
                m.close()
        del xd, yd
    if ref is not None:
        res.append({"cpu_reference": "matmul_quantized_weight of the reference build, "
                                     f"{os.cpu_count()} OpenMP threads, median of 3"})
    return res


def _class_stats(dz_native, stats):
    out = {}
    for k, name in enumerate(dz_native.KERNEL_CLASSES):
        s = stats[k]
        if s.launches:
            out[name] = {"launches": int(s.launches), "total_ms": float(s.total_ms), "bytes": float(s.bytes),
                         "flops": float(s.flops)}
    return out


def _profile(L, _native, cache, pd, plen, n_new, samp, seeds_ptr, od):
    nk = len(_native.KERNEL_CLASSES) + len(_native.FUSED_PHASES)
    stats = (_native.DzKernelStat * nk)()
    _native.check(L.dz_cuda_profile_generate(cache.handle, pd, plen, n_new, ctypes.byref(samp.c), seeds_ptr, od,
                                             stats, nk), "profile_generate")
    phases = {name: round(stats[len(_native.KERNEL_CLASSES) + k].total_ms, 4)
              for k, name in enumerate(_native.FUSED_PHASES) if stats[len(_native.KERNEL_CLASSES) + k].total_ms}
    return _class_stats(_native, stats), phases


NVLINK_GBS = 770.0   # measured peer copy per direction per GPU on this pool (900 nominal)


def roofline_of(classes, wl_name, hbm, bf16, peak_src, note):
    """Per class: achieved bytes or flops over its time against the measured
    peak of its bound (flops per byte above the ridge = tensor); the class
    with the largest time is the line's `roofline`."""
    ridge = bf16 * 1e3 / hbm   # flop per byte where the bf16 peak meets HBM
    per = {}
    for name, c in classes.items():
        t = c["total_ms"] * 1e-3
        if t <= 0:
            continue
        if name == "allreduce":
            # bytes each rank sends over NVLink, against the measured peer copy
            # of 770 GB/s per direction on this pool
            ach = c["bytes"] / t / 1e9
            per[name] = {"bound": "nvlink", "achieved": round(ach, 1), "peak": NVLINK_GBS, "unit": "GB/s",
                         "frac": round(ach / NVLINK_GBS, 4), "ms": round(c["total_ms"], 3),
                         "launches": c["launches"], "bytes_per_launch": int(c["bytes"] / c["launches"]),
                         "flops_per_launch": 0.0}
            continue
        tensor = c["flops"] > 0 and c["flops"] / max(c["bytes"], 1.0) > ridge
        if tensor:
            ach = c["flops"] / t / 1e12
            per[name] = {"bound": "tensor", "achieved": round(ach, 1), "peak": bf16, "unit": "TFLOP/s",
                         "frac": round(ach / bf16, 4)}
        else:
            ach = c["bytes"] / t / 1e9
            per[name] = {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(ach / hbm, 4)}
        per[name].update({"ms": round(c["total_ms"], 3), "launches": c["launches"],
                          "bytes_per_launch": int(c["bytes"] / c["launches"]),
                          "flops_per_launch": float(c["flops"] / c["launches"])})
    total = sum(p["ms"] for p in per.values()) or 1.0
    for p in per.values():
        p["share"] = round(p["ms"] / total, 3)
    dom = max(per, key=lambda n: per[n]["ms"])
    d = per[dom]
    roof = {"bound": d["bound"], "kernel_class": dom, "achieved": d["achieved"], "peak": d["peak"],
            "unit": d["unit"], "frac": d["frac"], "peak_source": peak_src,
            "traffic": NCU_TRAFFIC.get((wl_name, dom)), "note": note}
    ratio = NCU_TRAFFIC_RATIO.get((wl_name, dom))
    if roof["traffic"] is None and ratio is not None:
        roof["traffic"] = int(ratio * d["bytes_per_launch"])
        roof["traffic_note"] = ("ncu DRAM bytes / algorithmic bytes of one captured launch "
                                f"({ratio:.3f}) x the class's algorithmic bytes per launch")
    return roof, per


def run_job(args, wl, torch, dz, _native, W, world, rank, local, hbm, bf16, peak_src):
    """Build the workload's model on this rank, time the job (device-resident
    and end to end), split prefill from decode and profile the kernel
    classes. Returns (line dict on rank 0 else None, handles to close)."""
    lo, hi = shard(wl.batch, rank, world)
    n = hi - lo
    if n < 1:
        raise RuntimeError(f"{wl.name}: {wl.batch} sequences cannot be split over {world} GPUs")
    path = f"/tmp/dz_bench_{os.getpid()}_{rank}_{wl.spec.dim}.bin"
    W.write_bundle(wl, path)
    bundle = dz.Bundle(path)
    model = dz.Model.from_bundle(bundle, device=local)
    cap = wl.capacity or wl.spec.max_seq
    cache = dz.KVCache(model, n, cap)
    stream = torch.cuda.Stream()
    cache.set_stream(stream.cuda_stream)
    samp = wl.sampling()
    prompts = W.prompts(wl, lo, hi)
    seeds = W.seeds(wl, lo, hi)
    pd = torch.from_numpy(prompts.astype(np.int32)).cuda()
    sdv = torch.from_numpy(seeds.astype(np.int64)).cuda()
    od = torch.zeros((n, wl.n_new), dtype=torch.int32, device="cuda")
    od1 = torch.zeros((n, 1), dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    seeds_ptr = sdv.data_ptr() if wl.strategy else None

    def job(n_new=wl.n_new, out=od):
        cache.generate_async(pd.data_ptr(), wl.prompt_len, n_new, samp, seeds_ptr, out.data_ptr())

    def barrier():
        if world > 1:
            import torch.distributed as tdist
            tdist.barrier()

    def timed(fn, reps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        barrier()
        torch.cuda.synchronize()
        for k in range(reps):
            with torch.cuda.stream(stream):
                flush.zero_()
                evs[k][0].record(stream)
            fn()
            with torch.cuda.stream(stream):
                evs[k][1].record(stream)
        torch.cuda.synchronize()
        barrier()
        return sum(a.elapsed_time(b) for a, b in evs)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            job()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    dev_ms = timed(job, args.steps)
    clk = clocks.stop()
    got = od.cpu().numpy().astype(np.uint32)

    # prefill alone: the same job with one draw (prefill + one selection)
    job(1, od1)
    pre_reps = max(3, min(args.steps, 5))
    pre_ms = timed(lambda: job(1, od1), pre_reps) / pre_reps

    # e2e through the public C ABI from pinned host buffers
    hp = torch.from_numpy(prompts.astype(np.int32)).pin_memory()
    hs = torch.from_numpy(seeds.astype(np.int64)).pin_memory()
    ho = torch.zeros((n, wl.n_new), dtype=torch.int32).pin_memory()
    L = _native.lib()

    def job_e2e():
        _native.check(L.dz_cuda_generate(cache.handle, hp.data_ptr(), wl.prompt_len, wl.n_new,
                                         ctypes.byref(samp.c), hs.data_ptr() if wl.strategy else None,
                                         ho.data_ptr()), "generate")

    job_e2e()
    e2e_steps = args.steps if dev_ms / args.steps < 500 else max(3, min(args.steps, 5))
    e2e_ms = timed(job_e2e, e2e_steps)
    assert np.array_equal(ho.numpy().astype(np.uint32), got), "e2e tokens differ from the device-resident run"

    if world > 1:
        import torch.distributed as tdist
        t = torch.tensor([dev_ms, e2e_ms, pre_ms], dtype=torch.float64, device="cuda")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        dev_ms, e2e_ms, pre_ms = (float(x) for x in t)

    # kernel classes: eager launches with CUDA events; for long jobs the
    # prefill (one draw) and the prefill plus 8 decode steps, the decode
    # steps' difference scaled to the job's n_new - 1 steps
    fused = cache.uses_fused(samp)
    launches_job = cache.generate_launches(wl.prompt_len, wl.n_new, samp)
    long_job = launches_job > 20000
    if long_job:
        P = 8
        c1, ph = _profile(L, _native, cache, pd.data_ptr(), wl.prompt_len, 1, samp, seeds_ptr, od.data_ptr())
        c2, _ = _profile(L, _native, cache, pd.data_ptr(), wl.prompt_len, 1 + P, samp, seeds_ptr, od.data_ptr())
        zero = {"launches": 0, "total_ms": 0.0, "bytes": 0.0, "flops": 0.0}
        classes = {}
        scale = (wl.n_new - 1) / P
        for name in set(c1) | set(c2):
            a, b = c1.get(name, zero), c2.get(name, zero)
            classes[name] = {k: a[k] + scale * (b[k] - a[k]) for k in ("launches", "total_ms", "bytes", "flops")}
            classes[name]["launches"] = max(1, int(round(classes[name]["launches"])))
        note = (f"kernel classes of the job: the eager prefill plus {P} decode steps at the full batch, the decode "
                f"steps scaled to the job's {wl.n_new - 1}")
        # the two phases on their own: the prefill, and one decode step (the
        # mean of the P profiled steps)
        step = {}
        for name in set(c1) | set(c2):
            a, b = c1.get(name, zero), c2.get(name, zero)
            d = {k: (b[k] - a[k]) / P for k in ("launches", "total_ms", "bytes", "flops")}
            if d["total_ms"] > 0:
                d["launches"] = max(1, int(round(d["launches"])))
                step[name] = d
        phase_classes = {}
        for pname, cl in (("prefill", c1), ("decode_step", step)):
            _, per = roofline_of(cl, wl.name, hbm, bf16, peak_src, "")
            phase_classes[pname] = {k: {f: v[f] for f in ("bound", "frac", "ms", "launches", "share")}
                                    for k, v in per.items()}
    else:
        classes, ph = _profile(L, _native, cache, pd.data_ptr(), wl.prompt_len, wl.n_new, samp, seeds_ptr,
                               od.data_ptr())
        note = "kernel classes of one eagerly launched job"
        phase_classes = None
    note += ("; bytes = weight codes + scales + fp32 tensors once per batch step, KV rows read and written, "
             "activations in and out; flops = 2*M*K*N of the quantized products (useful work; the integer tensor "
             "cores run three 8-bit limb passes) plus attention")
    roof, per_class = roofline_of(classes, wl.name, hbm, bf16, peak_src, note)

    out = None
    if rank == 0:
        tokens = wl.batch * wl.n_new * args.steps
        value = tokens / (dev_ms * 1e-3)
        job_ms = dev_ms / args.steps
        dec_ms = max(job_ms - pre_ms, 1e-9)
        if fused:
            step_desc = "whole generation in one fused kernel per job (prompt token by token, then the draws)"
        elif wl.spec.dim >= 512:
            step_desc = ("batched prefill (every prompt position per layer pass, tensor-core GEMMs), then one "
                         "decode step per draw, one CUDA graph per job")
        else:
            step_desc = "prompt token by token, then one decode step per draw, one CUDA graph per job"
        per_gpu = wl.batch // world if wl.batch % world == 0 else f"{wl.batch // world}-{-(-wl.batch // world)}"
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(job_ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": f"int{wl.bits} weights, fp32 compute",
            "data": "synthetic (seeded N(0,0.02) weights, uniform prompt ids; no dataset named)",
            "config": {"workload": wl.name, "model": f"DRANZER d{wl.spec.dim} h{wl.spec.heads} L{wl.spec.layers} "
                       f"V{wl.spec.vocab} T{wl.spec.max_seq}", "bits": wl.bits,
                       "global_batch": wl.batch, "sequences_per_gpu": per_gpu,
                       "prompt_len": wl.prompt_len, "decode_len": wl.n_new, "seq_len": wl.prompt_len + wl.n_new,
                       "sampling": {"strategy": ["greedy", "top-k", "top-p"][wl.strategy],
                                    "temperature": wl.temperature, "top_k": wl.top_k, "top_p": wl.top_p},
                       "parallelism": f"batch-sharded x{world} (the job's {wl.batch} independent sequences split "
                                      "over the GPUs, no collective on the data path)",
                       "l2": "flushed between steps (256 MiB write on the stream, outside the timed events)",
                       "step": step_desc},
            "phases": {"prefill": {"ms": round(pre_ms, 3),
                                   "prompt_tokens_per_s": round(wl.batch * wl.prompt_len / (pre_ms * 1e-3), 1)},
                       "decode": {"ms": round(dec_ms, 3),
                                  "tokens_per_s": round(wl.batch * wl.n_new / (dec_ms * 1e-3), 1),
                                  "how": "job time minus the prefill-only job (prefill + one draw), max over ranks"}},
            "e2e": {"value": round(wl.batch * wl.n_new * e2e_steps / (e2e_ms * 1e-3), 1), "unit": "tokens/s",
                    "steps": e2e_steps,
                    "h2d_bytes_per_step": int(wl.batch * wl.prompt_len * 4 + (wl.batch * 8 if wl.strategy else 0)),
                    "d2h_bytes_per_step": int(wl.batch * wl.n_new * 4)},
            "gpu_launches": int(launches_job * args.steps),
            "roofline": roof,
            "kernel_classes": per_class,
            "path": "fused" if fused else "layered",
            "clocks": clk,
        }
        if ph:
            out["fused_phases_ms"] = ph
        if phase_classes:
            out["phase_kernel_classes"] = phase_classes
    os.remove(path)
    return out, (cache, model, bundle, prompts, seeds, samp)


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
    out, (cache, model, bundle, prompts, seeds, samp) = run_job(args, wl, torch, dz, _native, W, world, rank, local,
                                                                 hbm, bf16, peak_src)
    if rank == 0 and world == 1 and not args.no_cpu:
        w = REF_WORKLOADS[args.workload]
        ref = CpuReference(w)
        secs = min(ref.run() for _ in range(2))
        out["cpu_baseline"] = ref.describe(secs, "best of 2")
        # the same sample through the device path: identical tokens
        assert np.array_equal(ref.prompts, prompts[:ref.n, :ref.plen]), "CPU and device prompts differ"
        sc = dz.KVCache(model, ref.n, max(ref.plen + ref.n_new, 2))
        gs = sc.generate(np.ascontiguousarray(prompts[:ref.n, :ref.plen]), ref.n_new, samp,
                         seeds=seeds[:ref.n] if wl.strategy else None)
        sc.close()
        out["cpu_baseline"]["tokens_match_gpu"] = bool(np.array_equal(ref.out, gs))
        ref.close()
    cache.close()
    model.close()
    bundle.close()
    if args.workload == "c4" and not args.no_secondary:
        sec, (c2, m2, b2, *_) = run_job(args, W.C2, torch, dz, _native, W, world, rank, local, hbm, bf16, peak_src)
        if rank == 0:
            out["secondary"] = {k: sec[k] for k in ("value", "unit", "ms_per_step", "config", "e2e", "roofline",
                                                    "path", "gpu_launches", "clocks")}
            if "fused_phases_ms" in sec:
                out["secondary"]["fused_phases_ms"] = sec["fused_phases_ms"]
        c2.close()
        m2.close()
        b2.close()
    if rank == 0 and world == 1 and not args.no_probe:
        stream = torch.cuda.Stream()
        out["quant_matvec"] = quant_matvec_probe(dz, torch, stream, hbm, bf16, cpu=not args.no_cpu)
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
        tdist.destroy_process_group()
    return out


def tp_probe(args):
    """Tensor parallelism at the config-5 width (d 6144, 48 heads of 128,
    F 24576, V 50257, INT4, weights seed 5) with args.probe_layers layers:
    32 sequences, a 1024-token batched prefill, then 32 greedy steps, on every
    rank of a torchrun job (heads and FFN columns split over the ranks, NCCL
    all-reduces after attention-out and FFN-down). Reports the job, its
    prefill and decode parts (max over ranks) and the share of each phase
    spent in the all-reduce (eager launches bracketed by CUDA events)."""
    import torch
    import dranzer_b200 as dz
    from dranzer_b200 import _native
    from dranzer_b200 import workloads as W
    world, rank, local = dist_init()
    torch.cuda.set_device(local)
    hbm, bf16, peak_src = peaks()
    spec = W.Spec(50257, 6144, 48, args.probe_layers, 4096)
    wl = W.Workload("c5-width-tp", spec, 4, 5, 5, 32, 1024, 33, capacity=1088)
    path = f"/tmp/dz_tp_probe_{args.probe_layers}.bin"
    if rank == 0:
        W.write_bundle(wl, path)
    if world > 1:
        import torch.distributed as tdist
        tdist.barrier()
        uid = [dz.Model.tp_unique_id() if rank == 0 else None]
        tdist.broadcast_object_list(uid, src=0)
    bundle = dz.Bundle(path)
    model = dz.Model.from_bundle(bundle, device=local, tp=(rank, world, uid[0]) if world > 1 else None)
    cache = dz.KVCache(model, wl.batch, wl.capacity)
    stream = torch.cuda.Stream()
    cache.set_stream(stream.cuda_stream)
    samp = wl.sampling()
    pd = torch.from_numpy(W.prompts(wl).astype(np.int32)).cuda()
    od = torch.zeros((wl.batch, wl.n_new), dtype=torch.int32, device="cuda")

    def job(n_new):
        cache.generate_async(pd.data_ptr(), wl.prompt_len, n_new, samp, None, od.data_ptr())

    def timed(n_new, reps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        if world > 1:
            tdist.barrier()
        torch.cuda.synchronize()
        for k in range(reps):
            with torch.cuda.stream(stream):
                evs[k][0].record(stream)
            job(n_new)
            with torch.cuda.stream(stream):
                evs[k][1].record(stream)
        torch.cuda.synchronize()
        ms = sum(a.elapsed_time(b) for a, b in evs) / reps
        if world > 1:
            t = torch.tensor([ms], dtype=torch.float64, device="cuda")
            tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
            ms = float(t[0])
        return ms

    for n in (wl.n_new, 1):   # warm-up (and the graphs of both jobs)
        job(n)
    job_ms = timed(wl.n_new, args.steps)
    pre_ms = timed(1, max(3, min(args.steps, 5)))
    L = _native.lib()
    c1, _ = _profile(L, _native, cache, pd.data_ptr(), wl.prompt_len, 1, samp, None, od.data_ptr())
    c2, _ = _profile(L, _native, cache, pd.data_ptr(), wl.prompt_len, 9, samp, None, od.data_ptr())
    toks = od.cpu().numpy()
    out = None
    if rank == 0:
        def shares(cl):
            tot = sum(v["total_ms"] for v in cl.values()) or 1.0
            return {k: {"ms": round(v["total_ms"], 3), "share": round(v["total_ms"] / tot, 4)} for k, v in cl.items()}
        step = {k: {f: (c2[k][f] - c1.get(k, {}).get(f, 0.0)) / 8 for f in ("total_ms", "launches", "bytes", "flops")}
                for k in c2}
        step = {k: v for k, v in step.items() if v["total_ms"] > 0}
        ar = step.get("allreduce")
        out = {"tp_probe": {
            "world": world, "layers": args.probe_layers, "model": "d6144 h48 F24576 V50257 INT4 (config-5 width)",
            "batch": wl.batch, "prompt_len": wl.prompt_len, "decode_steps": wl.n_new - 1,
            "job_ms": round(job_ms, 3), "prefill_ms": round(pre_ms, 3),
            "decode_step_ms": round((job_ms - pre_ms) / (wl.n_new - 1), 4),
            "prefill_classes": shares(c1), "decode_step_classes": shares(step),
            "decode_allreduce_gbs_per_rank": round(ar["bytes"] / (ar["total_ms"] * 1e-3) / 1e9, 1) if ar else None,
            "how": "CUDA events on the launching stream, max over ranks; classes from eager launches each bracketed "
                   "by events (prefill alone, and prefill + 8 steps, the difference per step)",
            "first_tokens": toks[:2, :4].tolist()}}
    cache.close()
    model.close()
    bundle.close()
    if world > 1:
        tdist.barrier()
        tdist.destroy_process_group()
    if rank == 0:
        os.remove(path)
    return out


def decode_probe(dz, torch, hbm, layers=2, batch=64, steps=8):
    """The config-4 layer shapes (d 2048, 16 heads of 128, F 8192, V 32000,
    INT8) with a few layers and a smaller batch: a 512-token batched prefill,
    then `steps` decode steps, each step timed with CUDA events (a profiling
    target for the decode kernels at the job's contexts, a few GB on the
    device)."""
    from dranzer_b200 import workloads as W
    spec = W.Spec(32000, 2048, 16, layers, 2048)
    wl = W.Workload("decode-probe", spec, 8, 4, 4, batch, 512, steps + 1, capacity=640)
    path = f"/tmp/dz_probe_{os.getpid()}.bin"
    W.write_bundle(wl, path)
    bundle = dz.Bundle(path)
    os.remove(path)
    model = dz.Model.from_bundle(bundle)
    cache = dz.KVCache(model, batch, 640)
    prompts = W.prompts(wl)
    cache.prefill(prompts, want_logits=False)
    ids = prompts[:, -1].copy()
    times = []
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        cache.forward_tokens(ids, want_logits=False)
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    kv = 2.0 * layers * batch * 516 * 2048 * 4
    ms = statistics.median(times)
    cache.close()
    model.close()
    bundle.close()
    return {"decode_probe": {"layers": layers, "batch": batch, "context": "513-520", "step_ms": round(ms, 4),
                             "kv_gb_per_step": round(kv / 1e9, 3),
                             "kv_frac_of_hbm_if_alone": round(kv / (ms * 1e-3) / 1e9 / hbm, 3)}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c4", choices=sorted(REF_WORKLOADS))
    ap.add_argument("--impl", default="dz", choices=["dz", "reference"])
    ap.add_argument("--no-secondary", action="store_true", help="skip the config-2 line after config 4")
    ap.add_argument("--no-probe", action="store_true", help="skip the config-3 quantized-matmul rows")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline and the CPU matmul column")
    ap.add_argument("--probe-layers", type=int, default=2, help="with --probe tp: layers")
    ap.add_argument("--probe", choices=["qmv", "decode", "tp"],
                    help="run only the C3 quantized-matmul rows, or a few config-4 decode steps (profiling targets)")
    ap.add_argument("--probe-n", type=int, default=0, help="with --probe: one N instead of all three")
    ap.add_argument("--probe-batch", type=int, default=64, help="with --probe decode: sequences")
    ap.add_argument("--probe-m", default="", help="with --probe qmv: comma-separated row counts")
    ap.add_argument("--probe-k", type=int, default=4096, help="with --probe qmv: K")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        out = run_reference(args, REF_WORKLOADS[args.workload])
    elif args.probe == "qmv":
        import torch
        import dranzer_b200 as dz
        stream = torch.cuda.Stream()
        hbm, bf16, _ = peaks()
        Ns = (args.probe_n,) if args.probe_n else (4096, 11008, 32000)
        Ms = tuple(int(v) for v in args.probe_m.split(",")) if args.probe_m else (1, 8, 64, 512)
        out = {"quant_matvec": quant_matvec_probe(dz, torch, stream, hbm, bf16, Ns=Ns, Ms=Ms, K=args.probe_k)}
    elif args.probe == "tp":
        out = tp_probe(args)
    elif args.probe == "decode":
        import torch
        import dranzer_b200 as dz
        hbm, _, _ = peaks()
        out = decode_probe(dz, torch, hbm, batch=args.probe_batch)
    else:
        from dranzer_b200 import workloads as W
        out = run_dz(args, W.WORKLOADS[args.workload])
    if out is not None:
        print(json.dumps(out))


if __name__ == "__main__":
    main()
