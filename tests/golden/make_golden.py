"""Generate tests/golden/*.npz from the reference's own sources.

Run here, where the DRANZER tree is present:  make -C oracle ref &&
python tests/golden/make_golden.py. Every vector comes out of
oracle/_ref/libdzref.so, i.e. the reference's C sources compiled with its own
flags (-O3 -ffast-math) plus oracle/ref_harness.c. Inputs are the synthetic
generators described in tests/_models.py and the fill patterns of the
reference's tests (src/tests/core/test_quantize.c:81-90,
src/tests/core/test_quantized_matmul.c:25-29), restated here.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

from _native_oracle import (GREEDY, STREAM_DROPOUT, STREAM_INIT, STREAM_SAMPLING,  # noqa: E402
                            STREAM_TESTING, TOPP, TOPK, FLT_MAX, RefHarness)
from _margins import stream_margins, unit_draws  # noqa: E402

ref = RefHarness()
L = ref.L


def rng_stream(seed, stream):
    return L.dranzer_rng_stream(seed, stream)


def gaussian(state, count, sd):
    out = np.empty(count, np.float32)
    L.rh_fill_gaussian(state.ctypes.data, out.ctypes.data, count, sd)
    return out


def prompt_ids(state, count, vocab, excluded=(256, 257, 258, 259)):
    out = []
    while len(out) < count:
        t = L.dranzer_rng_next(state.ctypes.data) % vocab
        if t not in excluded:
            out.append(t)
    return np.array(out, np.uint32)


def fill_quantize_test(count, salt):
    i = np.arange(count, dtype=np.int64)
    base = ((i * 37 + salt * 11) % 71 - 35).astype(np.float32) / np.float32(17.0)
    base = np.where(i % 23 == 0, base * np.float32(12.0), base)
    return base.astype(np.float32)


def fill_qmm_test(count, salt):
    i = np.arange(count, dtype=np.int64)
    return (((i * 29 + salt * 17) % 97 - 48).astype(np.float32) / np.float32(31.0)).astype(np.float32)


def fnv(data):
    data = np.ascontiguousarray(data).view(np.uint8)
    h = 0xCBF29CE484222325
    # vectorised FNV-1a is sequential; chunk through numpy scalars is slow, so use the oracle
    from _native_oracle import Oracle
    return Oracle().fnv1a(data, h)


def gen_rng():
    seeds = np.array([0, 1, 2, 3, 7, 42, 2000, 2063, 12345678901234], np.uint64)
    streams = np.array([STREAM_INIT, STREAM_DROPOUT, STREAM_SAMPLING, STREAM_TESTING], np.uint64)
    init = np.zeros((len(seeds), len(streams)), np.uint64)
    draws = np.zeros((len(seeds), len(streams), 8), np.uint64)
    units = np.zeros((len(seeds), len(streams), 4), np.float64)
    for a, s in enumerate(seeds):
        for b, st in enumerate(streams):
            state = np.array([rng_stream(int(s), int(st))], np.uint64)
            init[a, b] = state[0]
            for k in range(8):
                draws[a, b, k] = L.dranzer_rng_next(state.ctypes.data)
            for k in range(4):
                units[a, b, k] = L.dranzer_rng_unit(state.ctypes.data)
    st = np.array([rng_stream(0, STREAM_TESTING)], np.uint64)
    g = gaussian(st, 4096, 0.02)
    np.savez_compressed(os.path.join(HERE, "rng.npz"), seeds=seeds, streams=streams, init=init,
                        draws=draws, units=units, gaussian_seed0=g)


def gen_quant():
    cases = {}
    shapes = [(1, 1), (1, 64), (64, 1), (3, 5), (16, 16), (7, 129)]
    n = 0
    for si, (r, c) in enumerate(shapes):
        for bits in (2, 3, 4, 5, 8, 12, 16):
            for g in (0, 1, 2):
                w = fill_quantize_test(r * c, si * 7 + bits).reshape(r, c)
                s, p = ref.quantize_pack(w, bits, g)
                cases[f"c{n}_w"] = w
                cases[f"c{n}_meta"] = np.array([r, c, bits, g], np.int64)
                cases[f"c{n}_s"] = s
                cases[f"c{n}_p"] = p
                n += 1
    # N(0, 0.02) matrix, the bundle generator's distribution
    st = np.array([rng_stream(11, STREAM_TESTING)], np.uint64)
    w = gaussian(st, 192 * 320, 0.02).reshape(192, 320)
    # adversarial columns: exact half-steps (round-half-away ties), signed zeros,
    # an all-zero column, subnormals, a lone outlier
    qmax8 = 127
    w[:, 0] = 0.0
    w[:, 1] = -0.0
    w[0, 2] = np.float32(127 * 0.001)
    w[1:, 2] = (np.arange(191, dtype=np.float32) % 127 - 63 + 0.5).astype(np.float32) * np.float32(0.001)
    w[:, 3] = np.float32(1e-40) * np.arange(192, dtype=np.float32)
    w[5, 4] = np.float32(3.0)
    cases["adv_w"] = w
    for bits in (4, 8):
        for g in (0, 1, 2):
            s, p = ref.quantize_pack(w, bits, g)
            cases[f"c{n}_meta"] = np.array([192, 320, bits, g], np.int64)
            cases[f"c{n}_s"] = s
            cases[f"c{n}_p"] = p
            n += 1
    cases["count"] = np.array(n)
    # full C3 weight matrices (K=4096 x N), codes and scales pinned by FNV-1a
    hashes = []
    for N in (4096, 11008, 32000):
        st = np.array([rng_stream(3, STREAM_TESTING)], np.uint64)
        # X[M=1..512,K] comes first in the seed-3 stream; the largest M is drawn
        # and W follows it, as bench and tests do
        gaussian(st, 512 * 4096, 1.0)
        wN = gaussian(st, 4096 * N, 0.02).reshape(4096, N)
        for bits in (8, 4):
            s, p = ref.quantize_pack(wN, bits, 2)
            hashes.append([N, bits, fnv(s), fnv(p)])
    cases["c3_hashes"] = np.array(hashes, np.uint64)
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **cases)


def gen_qmm():
    out = {}
    shapes = [(1, 64, 257), (17, 33, 47), (5, 7, 3), (16, 16, 16)]
    n = 0
    for (m, k, nn) in shapes:
        for bits in (4, 8):
            for g in (0, 1, 2):
                a = fill_qmm_test(m * k, 1).reshape(m, k)
                b = fill_qmm_test(k * nn, 2).reshape(k, nn)
                h = ref.qmat(b, bits, g)
                c = ref.qmat_matmul(h, a, nn)
                L.rh_qmat_free(h)
                out[f"t{n}_a"], out[f"t{n}_b"], out[f"t{n}_c"] = a, b, c
                out[f"t{n}_meta"] = np.array([m, k, nn, bits, g], np.int64)
                n += 1
    out["count"] = np.array(n)
    # C3 shapes at K=4096, N=4096, M in {1, 8}: reference INT8/INT4 outputs
    st = np.array([rng_stream(3, STREAM_TESTING)], np.uint64)
    x = gaussian(st, 512 * 4096, 1.0).reshape(512, 4096)
    w = gaussian(st, 4096 * 4096, 0.02).reshape(4096, 4096)
    for bits in (8, 4):
        h = ref.qmat(w, bits, 2)
        out[f"c3_m8_int{bits}"] = ref.qmat_matmul(h, x[:8], 4096)
        L.rh_qmat_free(h)
    np.savez_compressed(os.path.join(HERE, "qmm.npz"), **out)


def units_for(seeds, n_new):
    return unit_draws(lambda s, st: L.dranzer_rng_stream(s, st),
                      lambda st: L.dranzer_rng_unit(st.ctypes.data), seeds, n_new, STREAM_SAMPLING)


def gen_model(name, vocab, dim, heads, layers, max_seq, wseed, bits, prompt_seed, n_seq, plen,
              n_new, strategy, temperature, top_k, top_p, seeds, logits_seqs, prompt_logits=True, flags=0):
    path = f"/tmp/dz_golden_{name}.bin"
    rc = L.rh_build_bundle_arch(path.encode(), vocab, dim, heads, layers, max_seq, wseed, bits, 2, flags)
    assert rc == 0, rc
    h = L.rh_load(path.encode())
    st = np.array([rng_stream(prompt_seed, STREAM_TESTING)], np.uint64)
    prompts = prompt_ids(st, n_seq * plen, vocab).reshape(n_seq, plen)
    toks = np.empty((n_seq, n_new), np.uint32)
    lg = np.empty((n_seq, n_new, vocab), np.float32)
    sd = np.array(seeds, np.uint64) if seeds is not None else None
    mk = np.array([256, 257, 258, 259], np.uint32)
    rc = L.rh_generate(h, prompts.ctypes.data, n_seq, plen, n_new, strategy, temperature, top_k,
                       top_p, sd.ctypes.data if sd is not None else None, mk.ctypes.data, 4,
                       toks.ctypes.data, lg.ctypes.data)
    assert rc == 0
    # decision margin of every draw (tests/_margins.py)
    units = units_for(seeds, n_new) if seeds is not None else None
    margins = stream_margins(lg, toks, strategy, temperature, top_k, top_p, units)
    # prompt-position logits of sequence 0 (prefill parity)
    pl = np.empty((plen if prompt_logits else 0, vocab), np.float32)
    if prompt_logits:
        L.rh_reset(h)
        for i in range(plen):
            L.rh_forward_token(h, int(prompts[0, i]), pl[i].ctypes.data)
    L.rh_free(h)
    with open(path, "rb") as f:
        blob = np.frombuffer(f.read(), np.uint8)
    os.remove(path)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"),
                        spec=np.array([vocab, dim, heads, layers, max_seq, wseed, bits], np.int64),
                        architecture_flags=np.array([flags], np.int64),
                        prompts=prompts, tokens=toks, logits=lg[:logits_seqs], margins=margins,
                        prompt_logits=pl, bundle_fnv=np.array([fnv(blob)], np.uint64),
                        bundle_size=np.array([blob.size], np.int64),
                        sampling=np.array([strategy, top_k], np.int64),
                        sampling_f=np.array([temperature, top_p], np.float32),
                        seeds=np.array(seeds if seeds is not None else [], np.uint64))


def gen_bundle_small():
    path = "/tmp/dz_golden_small_bundle.bin"
    for bits in (4, 8):
        assert L.rh_build_bundle(path.encode(), 300, 16, 2, 2, 8, 9, bits, 2) == 0
        with open(path, "rb") as f:
            blob = np.frombuffer(f.read(), np.uint8)
        os.remove(path)
        blob.tofile(os.path.join(HERE, f"bundle_small_int{bits}.bin"))


def gen_pe():
    t = np.empty((64, 128), np.float32)
    assert L.compute_positional_encoding(t.ctypes.data, 64, 128) == 0
    np.savez_compressed(os.path.join(HERE, "pe.npz"), pe_64x128=t)


def gen_c1():
    # config 1: INT8 greedy, batch 1, 16 prompt + 48 decode
    gen_model("c1", 512, 128, 4, 4, 64, 0, 8, 1, 1, 16, 48, GREEDY, 0.0, 0, 0.0, None, 1)


def gen_c2():
    # config 2: INT4 top-p 0.9 at temperature 0.8, 64 x (32 + 32), seed 2*1000+i
    gen_model("c2", 512, 128, 4, 4, 64, 0, 4, 2, 64, 32, 32, TOPP, 0.8, 0, 0.9,
              [2000 + i for i in range(64)], 4)


def gen_ring():
    # a ring-eviction case: capacity 32 (max_seq 32), 24 prompt + 40 decode, top-k 5
    gen_model("ring", 400, 64, 2, 2, 32, 7, 8, 3, 2, 24, 40, TOPK, 0.8, 5, 0.0, [70, 71], 2)


def gen_c4():
    # config 4 sample: the full model (d 2048, 16 heads, 24 layers, V 32000,
    # context 2048, INT8, weights seed 4), the first 2 of its prompts (seed 4,
    # 512 tokens each), then 8 greedy draws; every draw's logits are kept
    # (the first is the last prompt position's)
    gen_model("c4s", 32000, 2048, 16, 24, 2048, 4, 8, 4, 2, 512, 8, GREEDY, 0.0, 0, 0.0, None, 2,
              prompt_logits=False)


def gen_controls():
    """The reference's own generation loop (generation_decode_with_options via
    rh_generate_ex) with repetition penalty, minimum length, EOS and stop
    sequences, on a 2-layer INT8 model whose tokenizer assigns ids 0..259
    (so ids >= 260 are masked, src/cli/generation.c:43-45). Stop sequences
    are picked from a first run without them, so that they occur."""
    from _native_oracle import Controls, Oracle
    vocab, dim, heads, layers, max_seq, wseed, bits = 512, 128, 4, 2, 64, 12, 8
    path = "/tmp/dz_golden_controls.bin"
    assert L.rh_build_bundle(path.encode(), vocab, dim, heads, layers, max_seq, wseed, bits, 2) == 0
    h = L.rh_load(path.encode())
    tok_vocab = int(L.rh_tokenizer_vocab(h))
    with open(path, "rb") as f:
        blob = np.frombuffer(f.read(), np.uint8)
    os.remove(path)
    st = np.array([rng_stream(13, STREAM_TESTING)], np.uint64)
    n_seq, plen, n_new = 6, 10, 24
    prompts = prompt_ids(st, n_seq * plen, vocab).reshape(n_seq, plen)
    seeds = np.array([500 + i for i in range(n_seq)], np.uint64)
    cases = [(GREEDY, 0.0, 0, 0.0, 1.3, 4, False), (TOPK, 0.9, 6, 0.0, 1.15, 2, True),
             (TOPP, 0.8, 0, 0.85, 1.0, 0, True), (TOPK, 1.1, 40, 0.0, 1.4, 6, True)]
    out = {"spec": np.array([vocab, dim, heads, layers, max_seq, wseed, bits], np.int64), "prompts": prompts,
           "seeds": seeds, "tokenizer_vocab": np.array([tok_vocab], np.int64),
           "bundle_fnv": np.array([fnv(blob)], np.uint64), "count": np.array([len(cases)], np.int64)}

    def run(strategy, temperature, top_k, top_p, penalty, min_new, stops):
        st_t = np.array([t for q in stops for t in q] or [0], np.uint32)
        st_l = np.array([len(q) for q in stops] or [0], np.uint64)
        toks = np.empty((n_seq, n_new), np.uint32)
        res = np.empty((n_seq, 5), np.uint32)
        sd = seeds if strategy else None
        rc = L.rh_generate_ex(h, prompts.ctypes.data, n_seq, plen, n_new, strategy, temperature, top_k, top_p,
                              sd.ctypes.data if sd is not None else None, penalty, min_new, st_t.ctypes.data,
                              st_l.ctypes.data, len(stops), toks.ctypes.data, res.ctypes.data)
        assert rc == 0, rc
        return toks, res

    # a near-flat draw (top-p 1 at temperature 4): seeds scanned, in order,
    # for a set whose draws include EOS, so that EOS ends some sequences
    base = 600
    while True:
        seeds = np.array([base + i for i in range(n_seq)], np.uint64)
        t, r = run(TOPP, 4.0, 0, 1.0, 1.0, 2, [])
        if r[:, 2].any():
            break
        base += n_seq
    out["eos_seeds"] = seeds.copy()
    cases.append((TOPP, 4.0, 0, 1.0, 1.0, 2, False))
    out["count"] = np.array([len(cases)], np.int64)
    for i, (strategy, temperature, top_k, top_p, penalty, min_new, with_stops) in enumerate(cases):
        seeds = out["eos_seeds"] if i == len(cases) - 1 else out["seeds"]
        out[f"c{i}_seeds"] = seeds
        stops = []
        if with_stops:
            t0, _ = run(strategy, temperature, top_k, top_p, penalty, min_new, [])
            stops = [(int(t0[0, min_new + 3]),), (int(t0[1, min_new + 5]), int(t0[1, min_new + 6]))]
        toks, res = run(strategy, temperature, top_k, top_p, penalty, min_new, stops)
        out[f"c{i}_params"] = np.array([strategy, top_k, min_new], np.int64)
        out[f"c{i}_params_f"] = np.array([temperature, top_p, penalty], np.float32)
        out[f"c{i}_stop_tokens"] = np.array([t for q in stops for t in q], np.uint32)
        out[f"c{i}_stop_lengths"] = np.array([len(q) for q in stops], np.int64)
        out[f"c{i}_tokens"] = toks
        out[f"c{i}_results"] = res
    L.rh_free(h)
    np.savez_compressed(os.path.join(HERE, "controls.npz"), **out)


def gen_arch():
    # the architecture bits (src/include/core/model_types.h:26-36) on the
    # reference's own forward: tied + RoPE + RMSNorm + SwiGLU; GELU; RoPE +
    # RMSNorm with ring eviction (capacity 32, 24 + 24 tokens, positions past
    # max_seq_len); greedy and top-k
    gen_model("arch23", 512, 128, 4, 2, 64, 31, 8, 5, 3, 12, 20, GREEDY, 0.0, 0, 0.0, None, 3, flags=23)
    gen_model("arch8", 512, 128, 4, 2, 64, 32, 4, 6, 3, 12, 20, TOPK, 0.8, 8, 0.0, [80, 81, 82], 3, flags=8)
    gen_model("arch6", 400, 64, 2, 2, 32, 33, 8, 7, 2, 24, 24, TOPK, 0.8, 5, 0.0, [90, 91], 2, flags=6)


class QuantError(ctypes.Structure):
    # quant_error_t (src/include/core/quantize.h:58-80)
    _fields_ = [("count", ctypes.c_size_t), ("max_abs_error", ctypes.c_float), ("rms_error", ctypes.c_double),
                ("rms_relative", ctypes.c_double), ("original_rms", ctypes.c_double),
                ("clipped", ctypes.c_size_t), ("levels_used", ctypes.c_size_t)]


def qdq_inputs():
    """Inputs of the simulated grid: the reference test's fill pattern, and
    Gaussian values with near-zero entries (-0.0 reconstructions) and an
    all-zero group."""
    out = []
    for si, (rows, cols) in enumerate([(3, 5), (8, 32), (64, 48), (1, 100), (17, 1)]):
        out.append(fill_quantize_test(rows * cols, si + 1).reshape(rows, cols))
    st = np.array([rng_stream(77, STREAM_TESTING)], np.uint64)
    g = gaussian(st, 40 * 24, 1.0).reshape(40, 24)
    g[::7, :] *= np.float32(1e-4)
    g[:, 5] = 0.0
    out.append(g)
    return out


def gen_qdq():
    # quantize_dequantize_into (src/core/quantize.c:118-174) of the
    # reference's build: reconstructions (bit patterns) and error fields
    fn = L.quantize_dequantize_into
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p]
    out = {}
    n = 0
    for x in qdq_inputs():
        for gran in (0, 1, 2):
            for bits in (2, 3, 4, 8, 12, 16):
                dst = np.empty_like(x)
                e = QuantError()
                assert fn(x.ctypes.data, dst.ctypes.data, x.shape[0], x.shape[1], bits, gran,
                          ctypes.addressof(e)) == 0
                out[f"q{n}_src"] = x
                out[f"q{n}_args"] = np.array([gran, bits], np.int64)
                out[f"q{n}_dst_bits"] = dst.view(np.uint32)
                out[f"q{n}_counts"] = np.array([e.count, e.clipped, e.levels_used], np.int64)
                out[f"q{n}_stats"] = np.array([e.max_abs_error, e.rms_error, e.rms_relative, e.original_rms],
                                              np.float64)
                n += 1
    out["count"] = np.array([n], np.int64)
    np.savez_compressed(os.path.join(HERE, "qdq.npz"), **out)


def masked_cases(seed):
    """Inputs of the masked full-prefix forward: (ids, padding or None,
    attention or None) per case; T <= 64."""
    rng = np.random.RandomState(seed)
    st = np.array([rng_stream(seed, STREAM_TESTING)], np.uint64)
    cases = []

    def ids(T):
        return prompt_ids(st, T, 512)

    cases.append((ids(20), None, None))                                   # plain causal
    pad = np.ones(24, np.uint8); pad[-5:] = 0
    cases.append((ids(24), pad, None))                                    # right padding
    pad = np.ones(24, np.uint8); pad[:6] = 0
    cases.append((ids(24), pad, None))                                    # left padding
    pad = (rng.rand(32) > 0.25).astype(np.uint8); pad[3] = 1
    cases.append((ids(32), pad, None))                                    # holes
    pad = (rng.rand(32) > 0.25).astype(np.uint8); pad[10] = 1; pad[-1] = 1
    att = (rng.rand(32, 32) > 0.3).astype(np.uint8)
    att[10, :] = 0                                                        # a real query with no key
    cases.append((ids(32), pad, att))                                     # padding + custom mask
    cases.append((ids(64), None, None))                                   # T = max_seq_len
    att = (rng.rand(64, 64) > 0.5).astype(np.uint8)
    att[63, :] = 0                                                        # the last position attends to nothing
    cases.append((ids(64), None, att))                                    # custom mask only
    return cases


def gen_masked():
    # model_forward_masked (src/core/transformer.c:527-576) on the reference's
    # build: the default architecture (INT8) and tied + RoPE + RMSNorm +
    # SwiGLU (INT4), seven mask cases each, plus a padding mask with no real
    # position (rejected)
    out = {}
    for mi, (wseed, bits, flags) in enumerate([(51, 8, 0), (52, 4, 23)]):
        V, d, H, Ly, T = 512, 128, 4, 2, 64
        path = f"/tmp/dz_golden_masked{mi}.bin"
        assert L.rh_build_bundle_arch(path.encode(), V, d, H, Ly, T, wseed, bits, 2, flags) == 0
        h = L.rh_load(path.encode())
        with open(path, "rb") as f:
            blob = np.frombuffer(f.read(), np.uint8)
        os.remove(path)
        out[f"m{mi}_spec"] = np.array([V, d, H, Ly, T, wseed, bits], np.int64)
        out[f"m{mi}_flags"] = np.array([flags], np.int64)
        out[f"m{mi}_bundle_fnv"] = np.array([fnv(blob)], np.uint64)
        cases = masked_cases(60 + mi)
        for ci, (ids, pad, att) in enumerate(cases):
            lg = np.empty(V, np.float32)
            rc = L.rh_forward_masked(h, ids.ctypes.data, ids.size, pad.ctypes.data if pad is not None else None,
                                     att.ctypes.data if att is not None else None, lg.ctypes.data)
            assert rc == 0, rc
            out[f"m{mi}_c{ci}_ids"] = ids
            out[f"m{mi}_c{ci}_pad"] = pad if pad is not None else np.zeros(0, np.uint8)
            out[f"m{mi}_c{ci}_att"] = att if att is not None else np.zeros(0, np.uint8)
            out[f"m{mi}_c{ci}_logits"] = lg
        bad = np.zeros(16, np.uint8)
        lg = np.empty(V, np.float32)
        out[f"m{mi}_rejected_rc"] = np.array([L.rh_forward_masked(h, cases[0][0].ctypes.data, 16, bad.ctypes.data,
                                                                  None, lg.ctypes.data)], np.int64)
        out[f"m{mi}_count"] = np.array([len(cases)], np.int64)
        L.rh_free(h)
    np.savez_compressed(os.path.join(HERE, "masked.npz"), **out)


GENERATORS = {"rng": gen_rng, "quant": gen_quant, "qmm": gen_qmm, "pe": gen_pe, "bundle": gen_bundle_small,
              "c1": gen_c1, "c2": gen_c2, "ring": gen_ring, "controls": gen_controls, "arch": gen_arch,
              "masked": gen_masked, "qdq": gen_qdq,
              "c4": gen_c4}

if __name__ == "__main__":
    # no argument: every fixture except the config-4 sample (minutes of CPU)
    names = sys.argv[1:] or [n for n in GENERATORS if n != "c4"]
    for n in names:
        GENERATORS[n]()
    print("golden fixtures written to", HERE, ":", " ".join(names))
