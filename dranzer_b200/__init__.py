"""dranzer-b200: DRANZER's quantized-weight inference path on B200.

Python mirror of the reference's interfaces for this path, over the C ABI of
include/dz_host.h and include/dz_cuda.h (dranzer_b200/libdz_cuda.so):

  quantize_pack / quantize_unpack      src/include/core/quantize.h:129-140
  QuantizedWeightMatrix,
  matmul_quantized_weight              src/include/core/quantized_matmul.h:13-42
  Bundle (code-retaining loader),
  save_quantized_bundle                src/include/core/bundle.h:52-85
  Model, KVCache.forward_tokens        model_forward_token, src/core/transformer.c:755
  KVCache.select                       sample_next_token, src/cli/sampling.c:179
  KVCache.generate                     generation_decode_with_options, src/cli/generation.c:198

Functions raise ValueError where the reference returns -1 for invalid
arguments and DzError for device failures. Nothing here falls back to the CPU.
"""
import ctypes

import numpy as np

from ._native import (DzBundleInfo, DzBundleMeta, DzError, DzGenerationControls, DzGenerationResult,
                      DzModelDesc, DzSampling, DzTensorBlob, check, lib)

__all__ = ["GRAN_TENSOR", "GRAN_ROW", "GRAN_COLUMN", "GREEDY", "TOPK", "TOPP", "STREAM_INIT",
           "STREAM_DROPOUT", "STREAM_SAMPLING", "STREAM_TESTING", "DzError", "available",
           "rng_stream", "synth_gaussian", "synth_prompt_ids", "quantized_scale_count",
           "quantized_packed_size", "quantize_pack", "quantize_unpack", "quantized_slice", "positional_encoding", "fnv1a",
           "QuantizedWeightMatrix", "matmul_quantized_weight", "Bundle", "save_quantized_bundle",
           "minimal_tokenizer", "model_tensor_layout", "Sampling", "Controls", "Model", "KVCache"]

GRAN_TENSOR, GRAN_ROW, GRAN_COLUMN = 0, 1, 2
GREEDY, TOPK, TOPP = 0, 1, 2
PREFILL_AUTO, PREFILL_TOKENS, PREFILL_BATCHED = 0, 1, 2
KIND_PROJECTION, KIND_EMBEDDING, KIND_BIAS, KIND_NORM = 0, 1, 2, 3
STREAM_INIT = 0x9E3779B97F4A7C15
STREAM_DROPOUT = 0xBF58476D1CE4E5B9
STREAM_SAMPLING = 0x94D049BB133111EB
STREAM_TESTING = 0x2545F4914F6CDD1D
FNV_OFFSET = 0xCBF29CE484222325


def _p(a):
    return a.ctypes.data if a is not None else None


def available():
    """True when a compute-capability 10.x device is usable."""
    return bool(lib().dz_cuda_available())


# ---------------------------------------------------------------- rng / inputs

def rng_stream(seed, stream):
    return lib().dz_rng_stream(seed, stream)


def synth_gaussian(state, count, sd):
    """N(0, sd) values; `state` is a 1-element uint64 array advanced in place."""
    out = np.empty(count, np.float32)
    lib().dz_synth_gaussian(_p(state), _p(out), count, sd)
    return out


def synth_prompt_ids(state, count, vocab, excluded=(256, 257, 258, 259)):
    out = np.empty(count, np.uint32)
    ex = np.array(excluded, np.uint32)
    lib().dz_synth_prompt_ids(_p(state), _p(out), count, vocab, _p(ex), len(ex))
    return out


def fnv1a(data, running=FNV_OFFSET):
    data = np.ascontiguousarray(data)
    return lib().dz_fnv1a(running, _p(data), data.nbytes)


# --------------------------------------------------------------- quantization

def quantized_scale_count(rows, cols, granularity):
    out = np.zeros(1, np.uint64)
    if lib().dz_quantized_scale_count(rows, cols, granularity, _p(out)) != 0:
        raise ValueError("invalid shape or granularity")
    return int(out[0])


def quantized_packed_size(value_count, bits):
    out = np.zeros(1, np.uint64)
    if lib().dz_quantized_packed_size(value_count, bits, _p(out)) != 0:
        raise ValueError("invalid value count or bit width")
    return int(out[0])


def quantize_pack(values, bits, granularity=GRAN_COLUMN):
    """(scales, packed) of a rows x cols float32 matrix; bit-exact with the reference build."""
    w = np.ascontiguousarray(values, np.float32)
    if w.ndim != 2:
        raise ValueError("values must be 2-D (rows x cols)")
    rows, cols = w.shape
    ns = quantized_scale_count(rows, cols, granularity)
    nb = quantized_packed_size(rows * cols, bits)
    scales = np.empty(ns, np.float32)
    packed = np.empty(nb, np.uint8)
    if lib().dz_quantize_pack(_p(w), rows, cols, bits, granularity, _p(scales), ns, _p(packed), nb) != 0:
        raise ValueError("quantize_pack rejected the input (non-finite value or bad arguments)")
    return scales, packed


def quantized_slice(scales, packed, rows, cols, bits, granularity, axis, start, count):
    """Rows (axis 0) or columns (axis 1) [start, start + count) of a quantized
    matrix as (scales, packed) of its own (dz_quantized_slice)."""
    s = np.ascontiguousarray(scales, np.float32)
    p = np.ascontiguousarray(packed, np.uint8)
    r2, c2 = (count, cols) if axis == 0 else (rows, count)
    so = np.empty(quantized_scale_count(r2, c2, granularity), np.float32)
    po = np.empty(quantized_packed_size(r2 * c2, bits), np.uint8)
    if lib().dz_quantized_slice(_p(s), s.size, _p(p), p.size, rows, cols, bits, granularity, axis, start, count,
                                _p(so), _p(po)) != 0:
        raise ValueError("quantized_slice: bad arguments")
    return so, po


def quantize_unpack(scales, packed, rows, cols, bits, granularity=GRAN_COLUMN):
    s = np.ascontiguousarray(scales, np.float32)
    p = np.ascontiguousarray(packed, np.uint8)
    out = np.empty((rows, cols), np.float32)
    if lib().dz_quantize_unpack(_p(s), s.size, _p(p), p.size, rows, cols, bits, granularity, _p(out)) != 0:
        raise ValueError("quantize_unpack rejected the payload (non-canonical codes or bad scales)")
    return out


def quantize_dequantize(values, bits, granularity=GRAN_COLUMN):
    """quantize_dequantize_into (dz_quantize_dequantize_into): the simulated
    grid of a [rows, cols] float32 matrix; returns (reconstruction, error
    fields as a dict)."""
    from ._native import DzQuantError
    v = np.ascontiguousarray(values, np.float32)
    if v.ndim != 2:
        raise ValueError("quantize_dequantize: a 2-D matrix")
    out = np.empty_like(v)
    e = DzQuantError()
    if lib().dz_quantize_dequantize_into(_p(v), _p(out), v.shape[0], v.shape[1], bits, granularity,
                                         ctypes.addressof(e)) != 0:
        raise ValueError("quantize_dequantize: bad arguments")
    return out, {f: getattr(e, f) for f, _ in DzQuantError._fields_}


def positional_encoding(rows, dim):
    out = np.empty((rows, dim), np.float32)
    check(lib().dz_positional_encoding(_p(out), rows, dim), "positional_encoding")
    return out


def _blob(kind, rows, cols, bits=0, gran=GRAN_COLUMN, scales=None, packed=None, f32=None):
    b = DzTensorBlob()
    b.kind, b.rows, b.cols, b.bits, b.granularity = kind, rows, cols, bits, gran
    if scales is not None:
        b.scales = scales.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        b.scale_count = scales.size
        b.packed = packed.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))
        b.packed_size = packed.size
    if f32 is not None:
        b.f32 = f32.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    return b


class QuantizedWeightMatrix:
    """quantized_weight_matrix_t resident on a device (codes in the strip layout)."""

    def __init__(self, scales, packed, rows, cols, bits, granularity=GRAN_COLUMN, device=0):
        self._scales = np.ascontiguousarray(scales, np.float32)
        self._packed = np.ascontiguousarray(packed, np.uint8)
        self.rows, self.cols, self.bits, self.granularity, self.device = rows, cols, bits, granularity, device
        blob = _blob(KIND_PROJECTION, rows, cols, bits, granularity, self._scales, self._packed)
        h = ctypes.c_void_p()
        check(lib().dz_cuda_qmatrix_create(device, ctypes.byref(blob), ctypes.byref(h)), "qmatrix_create")
        self.handle = h.value

    @classmethod
    def encode(cls, values, bits, granularity=GRAN_COLUMN, device=0):
        """quantized_weight_matrix_encode (src/core/quantized_matmul.c:15-47) then upload."""
        w = np.ascontiguousarray(values, np.float32)
        s, p = quantize_pack(w, bits, granularity)
        return cls(s, p, w.shape[0], w.shape[1], bits, granularity, device)

    @property
    def nbytes(self):
        return lib().dz_cuda_qmatrix_bytes(self.handle)

    def unpack(self):
        out = np.empty((self.rows, self.cols), np.float32)
        check(lib().dz_cuda_qmatrix_unpack(self.handle, _p(out)), "qmatrix_unpack")
        return out

    def codes(self):
        out = np.empty(self._packed.size, np.uint8)
        check(lib().dz_cuda_qmatrix_codes(self.handle, _p(out)), "qmatrix_codes")
        return out

    def matmul(self, A):
        a = np.ascontiguousarray(A, np.float32)
        if a.ndim == 1:
            a = a[None, :]
        m, k = a.shape
        c = np.empty((m, self.cols), np.float32)
        check(lib().dz_cuda_matmul_quantized(_p(a), self.handle, _p(c), m, k), "matmul_quantized")
        return c

    def matmul_async(self, a_ptr, c_ptr, m, stream_ptr=None):
        check(lib().dz_cuda_matmul_quantized_async(a_ptr, self.handle, c_ptr, m, self.rows, stream_ptr),
              "matmul_quantized_async")

    def close(self):
        if getattr(self, "handle", None):
            lib().dz_cuda_qmatrix_free(self.handle)
            self.handle = None

    __del__ = close


def matmul_quantized_weight(A, weights):
    """C = A . deq(W) (matmul_quantized_weight, src/core/quantized_matmul.c:253-295)."""
    return weights.matmul(A)


# -------------------------------------------------------------------- bundles

def model_tensor_layout(desc):
    d = _desc(desc)
    n = lib().dz_model_tensor_layout(ctypes.byref(d), None, 0)
    arr = (DzTensorBlob * n)()
    lib().dz_model_tensor_layout(ctypes.byref(d), arr, n)
    return [(int(t.kind), int(t.rows), int(t.cols)) for t in arr]


def _desc(desc):
    if isinstance(desc, DzModelDesc):
        return desc
    d = DzModelDesc()
    d.vocab_size, d.embedding_dim, d.num_heads, d.num_layers, d.max_seq_len = (
        desc.vocab, desc.dim, desc.heads, desc.layers, desc.max_seq)
    d.architecture_flags = getattr(desc, "architecture_flags", 0)
    return d


def minimal_tokenizer(max_vocab):
    out = np.zeros(32, np.uint8)
    check(lib().dz_tokenizer_minimal(max_vocab, _p(out)), "tokenizer_minimal")
    return out


def save_quantized_bundle(path, desc, params, bits, granularity=GRAN_COLUMN, train_window=None, seed=0,
                          tokenizer=None, input_fingerprint=0, input_bytes=0, training_steps=0, loss_bits=0):
    """model_bundle_save_quantized (src/core/bundle.c:280-501) for a flat float32 parameter vector."""
    d = _desc(desc)
    p = np.ascontiguousarray(params, np.float32)
    meta = DzBundleMeta()
    meta.train_window = train_window if train_window is not None else d.max_seq_len
    meta.seed, meta.input_fingerprint, meta.input_bytes = seed, input_fingerprint, input_bytes
    meta.training_steps, meta.loss_bits = training_steps, loss_bits
    tok = minimal_tokenizer(d.vocab_size) if tokenizer is None else np.ascontiguousarray(tokenizer, np.uint8)
    check(lib().dz_bundle_save_quantized(path.encode(), ctypes.byref(d), _p(p), bits, granularity,
                                         ctypes.byref(meta), _p(tok), tok.size), "bundle_save_quantized")


class Bundle:
    """A v1/v2/v3 bundle opened with codes retained (dz_bundle_open)."""

    def __init__(self, path):
        h = ctypes.c_void_p()
        check(lib().dz_bundle_open(path.encode(), ctypes.byref(h)), f"bundle_open({path})")
        self.handle = h.value
        self.desc = DzModelDesc()
        lib().dz_bundle_desc(self.handle, ctypes.byref(self.desc))
        self.info = DzBundleInfo()
        lib().dz_bundle_info(self.handle, ctypes.byref(self.info))
        n = lib().dz_bundle_tensor_count(self.handle)
        ptr = lib().dz_bundle_tensors(self.handle)
        self.tensors = (DzTensorBlob * n).from_address(ptr)

    def tensor(self, i):
        """(kind, rows, cols, f32 | None, scales | None, packed | None) as numpy views."""
        t = self.tensors[i]
        f32 = scales = packed = None
        if t.f32:
            f32 = np.ctypeslib.as_array(t.f32, shape=(t.rows * t.cols,)).reshape(t.rows, t.cols)
        if t.scales:
            scales = np.ctypeslib.as_array(t.scales, shape=(t.scale_count,))
            packed = np.ctypeslib.as_array(t.packed, shape=(t.packed_size,))
        return int(t.kind), int(t.rows), int(t.cols), f32, scales, packed

    def close(self):
        if getattr(self, "handle", None):
            lib().dz_bundle_close(self.handle)
            self.handle = None

    __del__ = close


# ----------------------------------------------------------------- model path

class Sampling:
    """dz_sampling_t: strategy, temperature, top_k, top_p and the masked ids."""

    def __init__(self, strategy=GREEDY, temperature=0.0, top_k=0, top_p=0.0, masked=(256, 257, 258, 259)):
        self.masked = np.array(masked, np.uint32)
        self.c = DzSampling()
        self.c.strategy, self.c.temperature, self.c.top_k, self.c.top_p = strategy, temperature, top_k, top_p
        self.c.masked_ids = self.masked.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))
        self.c.n_masked = self.masked.size


class Controls:
    """dz_generation_controls_t: the generation loop's controls beyond token
    selection (generation_options_t, src/include/cli/generation.h):
    repetition penalty, EOS id and minimum new tokens, the first masked id of
    the tokenizer's unassigned range, stop sequences (lists of ids)."""

    def __init__(self, penalty=1.0, eos_id=259, min_new=0, mask_from=0xFFFFFFFF, stops=()):
        self.stops = [list(int(t) for t in q) for q in stops]
        self._tok = np.array([t for q in self.stops for t in q] or [0], np.uint32)
        self._len = np.array([len(q) for q in self.stops] or [0], np.uint64)
        self.c = DzGenerationControls()
        self.c.repetition_penalty, self.c.eos_id = penalty, eos_id
        self.c.minimum_new_tokens, self.c.mask_from = min_new, mask_from
        self.c.stop_tokens = self._tok.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))
        self.c.stop_lengths = self._len.ctypes.data_as(ctypes.POINTER(ctypes.c_size_t))
        self.c.n_stops = len(self.stops)


class Model:
    """A bundle's parameters as codes on one device (dz_cuda_model_create)."""

    def __init__(self, desc, blobs, device=0, keepalive=None, tp=None):
        """tp: None, or (rank, world, nccl_id bytes) for one tensor-parallel
        shard (dz_cuda_model_create_tp; collective over the ranks)."""
        self.desc = _desc(desc)
        self.device = device
        self._keep = keepalive
        arr = (DzTensorBlob * len(blobs))(*blobs)
        h = ctypes.c_void_p()
        if tp is None:
            check(lib().dz_cuda_model_create(ctypes.byref(self.desc), arr, len(blobs), device, ctypes.byref(h)),
                  "model_create")
        else:
            rank, world, uid = tp
            idb = (ctypes.c_uint8 * 128).from_buffer_copy(bytes(uid))
            check(lib().dz_cuda_model_create_tp(ctypes.byref(self.desc), arr, len(blobs), device, rank, world, idb,
                                                ctypes.byref(h)), "model_create_tp")
        self.handle = h.value

    @staticmethod
    def tp_unique_id():
        """NCCL unique id (128 bytes) for dz_cuda_model_create_tp, made on one rank."""
        buf = (ctypes.c_uint8 * 128)()
        check(lib().dz_cuda_tp_unique_id(buf), "tp_unique_id")
        return bytes(buf)

    @classmethod
    def from_bundle(cls, bundle, device=0, tp=None):
        return cls(bundle.desc, list(bundle.tensors), device, keepalive=bundle, tp=tp)

    @classmethod
    def from_arrays(cls, desc, tensors, device=0, tp=None):
        """tensors: per tensor (kind, rows, cols, f32 | None, scales | None, packed | None, bits, gran)."""
        keep, blobs = [], []
        for kind, rows, cols, f32, scales, packed, bits, gran in tensors:
            if f32 is not None:
                f32 = np.ascontiguousarray(f32, np.float32)
                keep.append(f32)
                blobs.append(_blob(kind, rows, cols, f32=f32))
            else:
                scales = np.ascontiguousarray(scales, np.float32)
                packed = np.ascontiguousarray(packed, np.uint8)
                keep += [scales, packed]
                blobs.append(_blob(kind, rows, cols, bits, gran, scales, packed))
        return cls(desc, blobs, device, keepalive=keep, tp=tp)

    @property
    def step_bytes(self):
        return lib().dz_cuda_model_step_bytes(self.handle)

    def close(self):
        if getattr(self, "handle", None):
            lib().dz_cuda_model_free(self.handle)
            self.handle = None

    __del__ = close


class KVCache:
    """`batch` independent ring KV caches of `capacity` tokens (dz_cuda_cache_create)."""

    def __init__(self, model, batch, capacity=None):
        self.model = model
        self.batch = batch
        self.capacity = capacity or model.desc.max_seq_len
        self.vocab = model.desc.vocab_size
        h = ctypes.c_void_p()
        check(lib().dz_cuda_cache_create(model.handle, batch, self.capacity, ctypes.byref(h)), "cache_create")
        self.handle = h.value

    PATH_AUTO, PATH_LAYERED, PATH_FUSED = 0, 1, 2

    def set_path(self, path):
        check(lib().dz_cuda_cache_set_path(self.handle, path), "cache_set_path")

    def set_prefill(self, mode):
        """PREFILL_AUTO / PREFILL_TOKENS / PREFILL_BATCHED (dz_cuda_cache_set_prefill)."""
        check(lib().dz_cuda_cache_set_prefill(self.handle, mode), "cache_set_prefill")

    def prefill(self, ids, lens=None, want_logits=True):
        """Batched prefill from empty rings: ids [batch, prompt_len], optional
        per-sequence lengths; returns the last-position logits [batch, V]."""
        ids = np.ascontiguousarray(ids, np.uint32)
        assert ids.ndim == 2 and ids.shape[0] == self.batch
        ln = None if lens is None else np.ascontiguousarray(lens, np.uint32)
        out = np.empty((self.batch, self.vocab), np.float32) if want_logits else None
        check(lib().dz_cuda_prefill(self.handle, _p(ids), _p(ln), ids.shape[1], _p(out)), "prefill")
        return out

    def forward_masked(self, ids, padding=None, attention=None):
        """model_forward_masked for every sequence (dz_cuda_forward_masked):
        ids [batch, seq_len], padding [batch, seq_len] (0 = padding) or None,
        attention [batch, seq_len, seq_len] or None; returns the logits of each
        sequence's last real position [batch, V]. The rings are left empty."""
        ids = np.ascontiguousarray(ids, np.uint32)
        assert ids.ndim == 2 and ids.shape[0] == self.batch
        T = ids.shape[1]
        pad = None if padding is None else np.ascontiguousarray(padding, np.uint8)
        att = None if attention is None else np.ascontiguousarray(attention, np.uint8)
        assert pad is None or pad.shape == (self.batch, T)
        assert att is None or att.shape == (self.batch, T, T)
        out = np.empty((self.batch, self.vocab), np.float32)
        check(lib().dz_cuda_forward_masked(self.handle, _p(ids), T, _p(pad), _p(att), _p(out)), "forward_masked")
        return out

    def uses_fused(self, sampling=None):
        return bool(lib().dz_cuda_cache_uses_fused(self.handle, ctypes.byref(sampling.c) if sampling else None))

    def set_stream(self, stream_ptr):
        check(lib().dz_cuda_cache_set_stream(self.handle, stream_ptr), "cache_set_stream")

    @property
    def stream(self):
        return lib().dz_cuda_cache_stream(self.handle)

    def reset(self, seq_mask=None):
        m = None if seq_mask is None else np.ascontiguousarray(seq_mask, np.uint8)
        check(lib().dz_cuda_cache_reset(self.handle, _p(m)), "cache_reset")

    def forward_tokens(self, token_ids, want_logits=True):
        ids = np.ascontiguousarray(token_ids, np.uint32)
        assert ids.size == self.batch
        out = np.empty((self.batch, self.vocab), np.float32) if want_logits else None
        check(lib().dz_cuda_forward_tokens(self.handle, _p(ids), _p(out)), "forward_tokens")
        return out

    def select(self, sampling=None, rng_states=None):
        ids = np.empty(self.batch, np.uint32)
        st = None if rng_states is None else np.ascontiguousarray(rng_states, np.uint64)
        check(lib().dz_cuda_select(self.handle, ctypes.byref(sampling.c) if sampling else None, _p(st), _p(ids)),
              "select")
        if rng_states is not None:
            rng_states[...] = st
        return ids

    def generate(self, prompts, n_new, sampling=None, seeds=None):
        pr = np.ascontiguousarray(prompts, np.uint32)
        assert pr.shape[0] == self.batch
        sd = None if seeds is None else np.ascontiguousarray(seeds, np.uint64)
        out = np.empty((self.batch, n_new), np.uint32)
        check(lib().dz_cuda_generate(self.handle, _p(pr), pr.shape[1], n_new,
                                     ctypes.byref(sampling.c) if sampling else None, _p(sd), _p(out)),
              "generate")
        return out

    def generate_ex(self, prompts, n_new, sampling=None, controls=None, seeds=None):
        """generation_decode_with_options for every sequence: tokens [batch,
        n_new] (0xffffffff after a sequence's end) and results [batch, 5]
        (new_count, emitted_count, stopped_on_eos, stopped_on_stop_sequence,
        stop_sequence_index)."""
        pr = np.ascontiguousarray(prompts, np.uint32)
        assert pr.shape[0] == self.batch
        sd = None if seeds is None else np.ascontiguousarray(seeds, np.uint64)
        out = np.empty((self.batch, n_new), np.uint32)
        res = (DzGenerationResult * self.batch)()
        check(lib().dz_cuda_generate_ex(self.handle, _p(pr), pr.shape[1], n_new,
                                        ctypes.byref(sampling.c) if sampling else None,
                                        ctypes.byref(controls.c) if controls else None, _p(sd), _p(out), res),
              "generate_ex")
        r = np.array([[x.new_count, x.emitted_count, x.stopped_on_eos, x.stopped_on_stop_sequence,
                       x.stop_sequence_index] for x in res], np.uint32)
        return out, r

    def select_ex(self, sampling=None, controls=None, rng_states=None):
        ids = np.empty(self.batch, np.uint32)
        st = None if rng_states is None else np.ascontiguousarray(rng_states, np.uint64)
        check(lib().dz_cuda_select_ex(self.handle, ctypes.byref(sampling.c) if sampling else None,
                                      ctypes.byref(controls.c) if controls else None, _p(st), _p(ids)),
              "select_ex")
        if rng_states is not None:
            rng_states[...] = st
        return ids

    def generate_async(self, prompts_ptr, prompt_len, n_new, sampling, seeds_ptr, out_ptr):
        check(lib().dz_cuda_generate_async(self.handle, prompts_ptr, prompt_len, n_new,
                                           ctypes.byref(sampling.c) if sampling else None, seeds_ptr, out_ptr),
              "generate_async")

    def generate_launches(self, prompt_len, n_new, sampling=None):
        return lib().dz_cuda_generate_launches(self.handle, prompt_len, n_new,
                                               ctypes.byref(sampling.c) if sampling else None)

    def close(self):
        if getattr(self, "handle", None):
            lib().dz_cuda_cache_free(self.handle)
            self.handle = None

    __del__ = close
