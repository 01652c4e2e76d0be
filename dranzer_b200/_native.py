"""ctypes binding of dranzer_b200/libdz_cuda.so (include/dz_host.h, include/dz_cuda.h).

Loading fails loudly when the library has not been built: there is no Python
or CPU fallback for anything this module exposes.
"""
import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libdz_cuda.so")

P = ctypes.c_void_p
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64
U32 = ctypes.c_uint32
I32 = ctypes.c_int
F32 = ctypes.c_float
F64 = ctypes.c_double
CP = ctypes.c_char_p

DZ_OK = 0
STATUS_NAMES = {0: "DZ_OK", -1: "DZ_E_INVALID", -2: "DZ_E_IO", -3: "DZ_E_FORMAT", -4: "DZ_E_CHECKSUM",
                -5: "DZ_E_NOMEM", -6: "DZ_E_UNSUPPORTED", -7: "DZ_E_DEVICE", -8: "DZ_E_TIMEOUT",
                -9: "DZ_E_NOT_BUNDLE"}


class DzModelDesc(ctypes.Structure):
    _fields_ = [("vocab_size", SZ), ("embedding_dim", SZ), ("num_heads", SZ), ("num_layers", SZ),
                ("max_seq_len", SZ), ("architecture_flags", U32)]


class DzTensorBlob(ctypes.Structure):
    _fields_ = [("kind", U32), ("rows", SZ), ("cols", SZ), ("bits", I32), ("granularity", I32),
                ("scales", ctypes.POINTER(F32)), ("scale_count", SZ),
                ("packed", ctypes.POINTER(ctypes.c_uint8)), ("packed_size", SZ),
                ("f32", ctypes.POINTER(F32))]


class DzBundleInfo(ctypes.Structure):
    _fields_ = [("format_version", U32), ("numeric", U32), ("bits", I32), ("granularity", I32),
                ("policy_flags", U32), ("train_window", U64), ("seed", U64), ("input_fingerprint", U64),
                ("input_bytes", U64), ("training_steps", U32), ("loss_bits", U32),
                ("total_param_count", U64), ("values_quantized", U64), ("scales_stored", U64)]


class DzBundleMeta(ctypes.Structure):
    _fields_ = [("train_window", U64), ("seed", U64), ("input_fingerprint", U64), ("input_bytes", U64),
                ("training_steps", U32), ("loss_bits", U32)]


class DzKernelStat(ctypes.Structure):
    _fields_ = [("kind", U32), ("launches", U32), ("total_ms", F64), ("bytes", F64), ("flops", F64)]


KERNEL_CLASSES = ["step_begin", "qmv", "attention", "layernorm", "select", "seqgen", "split", "allreduce"]
FUSED_PHASES = ["embed", "weight_wait", "qmv", "attention", "layernorm", "select"]


class DzQuantError(ctypes.Structure):
    _fields_ = [("count", ctypes.c_size_t), ("max_abs_error", ctypes.c_float), ("rms_error", ctypes.c_double),
                ("rms_relative", ctypes.c_double), ("original_rms", ctypes.c_double),
                ("clipped", ctypes.c_size_t), ("levels_used", ctypes.c_size_t)]


class DzSampling(ctypes.Structure):
    _fields_ = [("strategy", I32), ("temperature", F32), ("top_k", U32), ("top_p", F32),
                ("masked_ids", ctypes.POINTER(U32)), ("n_masked", SZ)]


class DzGenerationControls(ctypes.Structure):
    _fields_ = [("repetition_penalty", F32), ("eos_id", U32), ("minimum_new_tokens", SZ), ("mask_from", U32),
                ("stop_tokens", ctypes.POINTER(U32)), ("stop_lengths", ctypes.POINTER(SZ)), ("n_stops", SZ)]


class DzGenerationResult(ctypes.Structure):
    _fields_ = [("new_count", U32), ("emitted_count", U32), ("stopped_on_eos", U32),
                ("stopped_on_stop_sequence", U32), ("stop_sequence_index", U32)]


# name -> (restype, argtypes); every exported symbol of include/dz_host.h and include/dz_cuda.h
SIGNATURES = {
    # dz_host.h
    "dz_rng_stream": (U64, [U64, U64]),
    "dz_rng_next": (U64, [P]),
    "dz_rng_unit": (F64, [P]),
    "dz_synth_gaussian": (None, [P, P, SZ, F64]),
    "dz_quantized_slice": (I32, [P, SZ, P, SZ, SZ, SZ, I32, I32, I32, SZ, SZ, P, P]),
    "dz_synth_prompt_ids": (None, [P, P, SZ, U32, P, SZ]),
    "dz_quantized_scale_count": (I32, [SZ, SZ, I32, P]),
    "dz_quantized_packed_size": (I32, [SZ, I32, P]),
    "dz_quantize_pack": (I32, [P, SZ, SZ, I32, I32, P, SZ, P, SZ]),
    "dz_quantize_unpack": (I32, [P, SZ, P, SZ, SZ, SZ, I32, I32, P]),
    "dz_quantize_dequantize_into": (I32, [P, P, SZ, SZ, I32, I32, P]),
    "dz_quantize_dequantize": (I32, [P, SZ, SZ, I32, I32, P]),
    "dz_positional_encoding": (I32, [P, SZ, SZ]),
    "dz_fnv1a": (U64, [U64, P, SZ]),
    "dz_bundle_open": (I32, [CP, P]),
    "dz_bundle_close": (None, [P]),
    "dz_bundle_desc": (I32, [P, P]),
    "dz_bundle_info": (I32, [P, P]),
    "dz_bundle_tensor_count": (SZ, [P]),
    "dz_bundle_tensor": (I32, [P, SZ, P]),
    "dz_bundle_tensors": (P, [P]),
    "dz_bundle_tokenizer": (P, [P, P]),
    "dz_model_tensor_layout": (SZ, [P, P, SZ]),
    "dz_model_param_count": (SZ, [P]),
    "dz_bundle_save_quantized": (I32, [CP, P, P, I32, I32, P, P, SZ]),
    "dz_tokenizer_minimal": (I32, [U64, P]),
    # dz_cuda.h
    "dz_cuda_available": (I32, []),
    "dz_cuda_last_error": (I32, [P, SZ]),
    "dz_cuda_qmatrix_create": (I32, [I32, P, P]),
    "dz_cuda_qmatrix_free": (None, [P]),
    "dz_cuda_qmatrix_bytes": (SZ, [P]),
    "dz_cuda_qmatrix_unpack": (I32, [P, P]),
    "dz_cuda_qmatrix_codes": (I32, [P, P]),
    "dz_cuda_matmul_quantized": (I32, [P, P, P, SZ, SZ]),
    "dz_cuda_matmul_quantized_async": (I32, [P, P, P, SZ, SZ, P]),
    "dz_cuda_matmul_quantized_noalloc": (I32, [P, P, P, SZ, SZ, P]),
    "dz_cuda_model_create": (I32, [P, P, SZ, I32, P]),
    "dz_cuda_model_free": (None, [P]),
    "dz_cuda_model_step_bytes": (SZ, [P]),
    "dz_cuda_cache_create": (I32, [P, SZ, SZ, P]),
    "dz_cuda_cache_free": (None, [P]),
    "dz_cuda_cache_set_stream": (I32, [P, P]),
    "dz_cuda_cache_stream": (P, [P]),
    "dz_cuda_cache_reset": (I32, [P, P]),
    "dz_cuda_forward_tokens": (I32, [P, P, P]),
    "dz_cuda_select": (I32, [P, P, P, P]),
    "dz_cuda_generate": (I32, [P, P, SZ, SZ, P, P, P]),
    "dz_cuda_generate_async": (I32, [P, P, SZ, SZ, P, P, P]),
    "dz_cuda_generate_launches": (SZ, [P, SZ, SZ, P]),
    "dz_cuda_profile_generate": (I32, [P, P, SZ, SZ, P, P, P, P, SZ]),
    "dz_cuda_cache_set_path": (I32, [P, I32]),
    "dz_cuda_cache_set_prefill": (I32, [P, I32]),
    "dz_cuda_tp_unique_id": (I32, [P]),
    "dz_cuda_model_create_tp": (I32, [P, P, SZ, I32, I32, I32, P, P]),
    "dz_cuda_prefill": (I32, [P, P, P, SZ, P]),
    "dz_cuda_forward_masked": (I32, [P, P, SZ, P, P, P]),
    "dz_cuda_cache_uses_fused": (I32, [P, P]),
    "dz_cuda_generate_ex": (I32, [P, P, SZ, SZ, P, P, P, P, P]),
    "dz_cuda_select_ex": (I32, [P, P, P, P, P]),
}

_lib = None


def lib():
    """The loaded library; raises if it is missing (build with dranzer_b200.build)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m dranzer_b200.build` "
                               "(there is no fallback path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class DzError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def last_error():
    buf = ctypes.create_string_buffer(512)
    st = lib().dz_cuda_last_error(buf, 512)
    return st, buf.value.decode(errors="replace")


def check(status, what=""):
    if status != DZ_OK:
        _, msg = last_error()
        raise DzError(status, f"{what}: {msg}" if what else msg)
    return status
