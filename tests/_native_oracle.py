"""ctypes bindings to the CPU checkers (test infrastructure only).

`Oracle` wraps oracle/liboracle.so (our CPU restatement of the reference);
`RefHarness` wraps oracle/_ref/libdzref.so (the reference's own sources, built
by oracle/Makefile where the reference tree is present). Only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline leg use this module.
"""
import ctypes
import os
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
ORACLE_SO = os.path.join(ORACLE_DIR, "liboracle.so")
REF_SO = os.path.join(ORACLE_DIR, "_ref", "libdzref.so")
BRIDGE_SO = os.path.join(ORACLE_DIR, "_ref", "libdzref_bridge.so")

P = ctypes.c_void_p
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64
U32 = ctypes.c_uint32
F32 = ctypes.c_float
F64 = ctypes.c_double
I32 = ctypes.c_int

STREAM_INIT = 0x9E3779B97F4A7C15
STREAM_DROPOUT = 0xBF58476D1CE4E5B9
STREAM_SAMPLING = 0x94D049BB133111EB
STREAM_TESTING = 0x2545F4914F6CDD1D

GRAN_TENSOR, GRAN_ROW, GRAN_COLUMN = 0, 1, 2
GREEDY, TOPK, TOPP = 0, 1, 2
FLT_MAX = np.float32(3.4028234663852886e38)


def _ptr(a):
    return a.ctypes.data if a is not None else None


def _sig(lib, name, res, *args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = list(args)
    return f


def build_oracle():
    subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)


class Oracle:
    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build_oracle()
        L = ctypes.CDLL(ORACLE_SO)
        self.L = L
        _sig(L, "or_rng_stream", U64, U64, U64)
        _sig(L, "or_rng_next", U64, P)
        _sig(L, "or_rng_unit", F64, P)
        _sig(L, "or_fill_gaussian", None, P, P, SZ, F64)
        _sig(L, "or_prompt_ids", None, P, P, SZ, U32, P, SZ)
        _sig(L, "or_scale_count", SZ, SZ, SZ, I32)
        _sig(L, "or_packed_size", SZ, SZ, I32)
        _sig(L, "or_quantize_pack", I32, P, SZ, SZ, I32, I32, P, P)
        _sig(L, "or_quantize_unpack", I32, P, P, SZ, SZ, I32, I32, P)
        _sig(L, "or_matmul_quantized", I32, P, SZ, SZ, SZ, P, P, I32, I32, P)
        _sig(L, "or_positional_encoding", None, P, SZ, SZ)
        _sig(L, "or_positional_encoding_at", None, P, SZ, SZ)
        _sig(L, "or_model_param_count", SZ, SZ, SZ, SZ)
        _sig(L, "or_model_create", P, SZ, SZ, SZ, SZ, SZ, P)
        _sig(L, "or_model_create_arch", P, SZ, SZ, SZ, SZ, SZ, U32, P)
        _sig(L, "or_model_free", None, P)
        _sig(L, "or_cache_create", P, P, SZ)
        _sig(L, "or_cache_reset", None, P)
        _sig(L, "or_cache_free", None, P)
        _sig(L, "or_forward_token", I32, P, P, U32, P)
        _sig(L, "or_forward_masked", I32, P, P, SZ, P, P, P)
        _sig(L, "or_sample_next_token", U32, P, SZ, I32, F32, SZ, F32, P)
        _sig(L, "or_generate", I32, P, P, P, SZ, SZ, SZ, I32, F32, SZ, F32, P, P, SZ, P, P)
        _sig(L, "or_fnv1a", U64, U64, P, SZ)
        _sig(L, "or_generate_ex", I32, P, P, P, SZ, SZ, SZ, I32, F32, SZ, F32, P, F32, U32, SZ, U32, P, SZ, P, P,
             SZ, P, P, P)

    # --- rng / synthetic inputs
    def rng_stream(self, seed, stream):
        return self.L.or_rng_stream(seed, stream)

    def gaussian(self, state, count, sd):
        """state: 1-element uint64 array, advanced in place."""
        out = np.empty(count, np.float32)
        self.L.or_fill_gaussian(_ptr(state), _ptr(out), count, sd)
        return out

    def prompt_ids(self, state, count, vocab, excluded=(256, 257, 258, 259)):
        out = np.empty(count, np.uint32)
        ex = np.array(excluded, np.uint32)
        self.L.or_prompt_ids(_ptr(state), _ptr(out), count, vocab, _ptr(ex), len(ex))
        return out

    # --- quantization
    def quantize_pack(self, w, bits, gran):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        scales = np.empty(self.L.or_scale_count(rows, cols, gran), np.float32)
        packed = np.empty(self.L.or_packed_size(rows * cols, bits), np.uint8)
        rc = self.L.or_quantize_pack(_ptr(w), rows, cols, bits, gran, _ptr(scales), _ptr(packed))
        if rc != 0:
            raise ValueError("quantize_pack rejected input")
        return scales, packed

    def quantize_unpack(self, scales, packed, rows, cols, bits, gran):
        out = np.empty((rows, cols), np.float32)
        rc = self.L.or_quantize_unpack(_ptr(np.ascontiguousarray(scales, np.float32)),
                                       _ptr(np.ascontiguousarray(packed, np.uint8)),
                                       rows, cols, bits, gran, _ptr(out))
        return rc, out

    def matmul_quantized(self, a, k, n, scales, packed, bits, gran):
        a = np.ascontiguousarray(a, np.float32)
        m = a.size // k
        c = np.empty((m, n), np.float32)
        rc = self.L.or_matmul_quantized(_ptr(a), m, k, n, _ptr(scales), _ptr(packed), bits, gran, _ptr(c))
        assert rc == 0
        return c

    def positional_encoding(self, rows, dim):
        out = np.empty((rows, dim), np.float32)
        self.L.or_positional_encoding(_ptr(out), rows, dim)
        return out

    def fnv1a(self, data, running=0xCBF29CE484222325):
        data = np.ascontiguousarray(data)
        return self.L.or_fnv1a(running, _ptr(data), data.nbytes)

    def sample(self, logits, strategy, temperature, top_k, top_p, state):
        lg = np.array(logits, np.float32)
        return self.L.or_sample_next_token(_ptr(lg), lg.size, strategy, temperature, top_k, top_p,
                                           _ptr(state) if state is not None else None)

    # --- model
    def model(self, spec, params):
        h = self.L.or_model_create_arch(spec.vocab, spec.dim, spec.heads, spec.layers, spec.max_seq,
                                        getattr(spec, "architecture_flags", 0),
                                        _ptr(np.ascontiguousarray(params, np.float32)))
        assert h
        return OracleModel(self, spec, h)


class OracleModel:
    def __init__(self, o, spec, handle):
        self.o, self.spec, self.h = o, spec, handle
        self.cache = o.L.or_cache_create(handle, spec.max_seq)

    def reset(self):
        self.o.L.or_cache_reset(self.cache)

    def forward_token(self, token):
        out = np.empty(self.spec.vocab, np.float32)
        self.o.L.or_forward_token(self.h, self.cache, int(token), _ptr(out))
        return out

    def forward_masked(self, ids, padding=None, attention=None):
        """or_forward_masked: logits of the last real position, or None when
        the input is rejected."""
        ids = np.ascontiguousarray(ids, np.uint32)
        pad = None if padding is None else np.ascontiguousarray(padding, np.uint8)
        att = None if attention is None else np.ascontiguousarray(attention, np.uint8)
        out = np.empty(self.spec.vocab, np.float32)
        rc = self.o.L.or_forward_masked(self.h, _ptr(ids), ids.size, _ptr(pad), _ptr(att), _ptr(out))
        return out if rc == 0 else None

    def generate(self, prompts, n_new, strategy=GREEDY, temperature=0.0, top_k=0, top_p=0.0,
                 seeds=None, masked=(256, 257, 258, 259), want_logits=False):
        prompts = np.ascontiguousarray(prompts, np.uint32)
        n_seq, plen = prompts.shape
        toks = np.empty((n_seq, n_new), np.uint32)
        lg = np.empty((n_seq, n_new, self.spec.vocab), np.float32) if want_logits else None
        sd = np.ascontiguousarray(seeds, np.uint64) if seeds is not None else None
        mk = np.array(masked, np.uint32)
        self.o.L.or_generate(self.h, self.cache, _ptr(prompts), n_seq, plen, n_new, strategy,
                             temperature, top_k, top_p, _ptr(sd), _ptr(mk), len(mk), _ptr(toks), _ptr(lg))
        return toks, lg

    def generate_ex(self, prompts, n_new, controls, strategy=GREEDY, temperature=0.0, top_k=0, top_p=0.0,
                    seeds=None, want_logits=False):
        """generation_decode_with_options with its controls (Controls):
        tokens [n_seq, n_new] (UINT32_MAX after the end), results [n_seq, 5]
        and, when asked, the logits of every draw after penalty and masking."""
        prompts = np.ascontiguousarray(prompts, np.uint32)
        n_seq, plen = prompts.shape
        toks = np.empty((n_seq, n_new), np.uint32)
        res = np.empty((n_seq, 5), np.uint32)
        lg = np.empty((n_seq, n_new, self.spec.vocab), np.float32) if want_logits else None
        sd = np.ascontiguousarray(seeds, np.uint64) if seeds is not None else None
        c = controls
        mk = np.array(c.masked, np.uint32)
        st, sl = c.stop_arrays()
        rc = self.o.L.or_generate_ex(self.h, self.cache, _ptr(prompts), n_seq, plen, n_new, strategy, temperature,
                                     top_k, top_p, _ptr(sd), c.penalty, c.eos_id, c.min_new, c.mask_from,
                                     _ptr(mk), len(mk), _ptr(st), _ptr(sl), len(c.stops), _ptr(toks), _ptr(res),
                                     _ptr(lg))
        assert rc == 0
        return toks, res, lg

    def close(self):
        if self.h:
            self.o.L.or_cache_free(self.cache)
            self.o.L.or_model_free(self.h)
            self.h = None

    __del__ = close


class Controls:
    """The generation loop's controls beyond sample_next_token
    (generation_options_t, src/include/cli/generation.h): repetition
    penalty, EOS id and minimum new tokens, control ids masked and the first
    masked id of the tokenizer's unassigned range, stop sequences."""

    def __init__(self, penalty=1.0, eos_id=259, min_new=0, masked=(256, 257, 258), mask_from=1 << 31,
                 stops=()):
        self.penalty, self.eos_id, self.min_new = float(penalty), int(eos_id), int(min_new)
        self.masked, self.mask_from = tuple(masked), int(mask_from)
        self.stops = [tuple(int(t) for t in s) for s in stops]

    def stop_arrays(self):
        toks = np.array([t for s in self.stops for t in s] or [0], np.uint32)
        lens = np.array([len(s) for s in self.stops] or [0], np.uint64)
        return toks, lens


class RefHarness:
    """The reference's own sources (oracle/_ref/libdzref.so)."""

    def __init__(self, path=REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = ctypes.CDLL(path)
        self.L = L
        if path == BRIDGE_SO:
            # the reference-side binding (oracle/dz_bridge.c)
            _sig(L, "br_attach", I32, P, ctypes.c_char_p, I32)
            _sig(L, "br_attach_next", I32, ctypes.c_char_p, I32)
            # the reference's public API (src/include/dranzer.h)
            _sig(L, "dranzer_bundle_load", I32, ctypes.c_char_p, I32, P, P, P)
            _sig(L, "dranzer_model_free", None, P)
            _sig(L, "dranzer_tokenizer_free", None, P)
            _sig(L, "dranzer_cache_create", I32, P, SZ, P)
            _sig(L, "dranzer_cache_forward", I32, P, U32, P, SZ)
            _sig(L, "dranzer_cache_reset", None, P)
            _sig(L, "dranzer_cache_free", None, P)
            _sig(L, "dranzer_generation_create", I32, P, P, SZ, P)
            _sig(L, "dranzer_generation_reset", I32, P, ctypes.c_char_p, SZ)
            _sig(L, "dranzer_generation_next_greedy", I32, P, P, P, P)
            _sig(L, "dranzer_generation_free", None, P)
            _sig(L, "br_detach", None, P)
            _sig(L, "br_device_forwards", SZ)
        _sig(L, "rh_model", P, P)
        _sig(L, "dranzer_rng_stream", U64, U64, U64)
        _sig(L, "dranzer_rng_next", U64, P)
        _sig(L, "dranzer_rng_unit", F64, P)
        _sig(L, "rh_fill_gaussian", None, P, P, SZ, F64)
        _sig(L, "rh_build_bundle", I32, ctypes.c_char_p, SZ, SZ, SZ, SZ, SZ, U64, I32, I32)
        _sig(L, "rh_build_bundle_arch", I32, ctypes.c_char_p, SZ, SZ, SZ, SZ, SZ, U64, I32, I32, U32)
        _sig(L, "rh_load", P, ctypes.c_char_p)
        _sig(L, "rh_free", None, P)
        _sig(L, "rh_reset", None, P)
        _sig(L, "rh_param_count", SZ, P)
        _sig(L, "rh_params", ctypes.POINTER(F32), P)
        _sig(L, "rh_forward_token", I32, P, U32, P)
        _sig(L, "rh_generate", I32, P, P, SZ, SZ, SZ, I32, F32, SZ, F32, P, P, SZ, P, P)
        _sig(L, "rh_qmat_encode", P, P, SZ, SZ, I32, I32)
        _sig(L, "rh_qmat_scales", ctypes.POINTER(F32), P, ctypes.POINTER(SZ))
        _sig(L, "rh_qmat_packed", ctypes.POINTER(ctypes.c_uint8), P, ctypes.POINTER(SZ))
        _sig(L, "rh_qmat_matmul", I32, P, P, P, SZ)
        _sig(L, "rh_qmat_free", None, P)
        _sig(L, "rh_now", F64)
        _sig(L, "quantize_pack", I32, P, SZ, SZ, I32, I32, P, SZ, P, SZ)
        _sig(L, "quantize_unpack", I32, P, SZ, P, SZ, SZ, SZ, I32, I32, P)
        _sig(L, "sample_next_token", U32, P, SZ, I32, F32, SZ, F32, P)
        _sig(L, "compute_positional_encoding", I32, P, SZ, SZ)
        _sig(L, "rh_generate_ex", I32, P, P, SZ, SZ, SZ, I32, F32, SZ, F32, P, F32, SZ, P, P, SZ, P, P)
        _sig(L, "rh_tokenizer_vocab", SZ, P)
        _sig(L, "rh_forward_masked", I32, P, P, SZ, P, P, P)

    def quantize_pack(self, w, bits, gran):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        ns = 1 if gran == 0 else rows if gran == 1 else cols
        nb = (rows * cols * bits + 7) // 8
        scales = np.empty(ns, np.float32)
        packed = np.empty(nb, np.uint8)
        rc = self.L.quantize_pack(_ptr(w), rows, cols, bits, gran, _ptr(scales), ns, _ptr(packed), nb)
        if rc != 0:
            raise ValueError("quantize_pack rejected input")
        return scales, packed

    def qmat(self, w, bits, gran):
        w = np.ascontiguousarray(w, np.float32)
        h = self.L.rh_qmat_encode(_ptr(w), w.shape[0], w.shape[1], bits, gran)
        assert h
        return h

    def qmat_codes(self, h):
        n = SZ()
        s = self.L.rh_qmat_scales(h, ctypes.byref(n))
        scales = np.ctypeslib.as_array(s, shape=(n.value,)).copy()
        p = self.L.rh_qmat_packed(h, ctypes.byref(n))
        packed = np.ctypeslib.as_array(p, shape=(n.value,)).copy()
        return scales, packed

    def qmat_matmul(self, h, a, n):
        a = np.ascontiguousarray(a, np.float32)
        m = a.shape[0]
        c = np.empty((m, n), np.float32)
        assert self.L.rh_qmat_matmul(h, _ptr(a), _ptr(c), m) == 0
        return c

    def sample(self, logits, strategy, temperature, top_k, top_p, state):
        lg = np.array(logits, np.float32)
        return self.L.sample_next_token(_ptr(lg), lg.size, strategy, temperature, top_k, top_p,
                                        _ptr(state) if state is not None else None)
