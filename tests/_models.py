"""Model specs and synthetic weights shared by the tests (test infrastructure).

The tensor inventory follows the reference's model_param_tensors()
(src/core/model_params.c:39-103): token_embeddings, output_projection,
output_bias, then per layer W_q, W_k, W_v, W_o, ln_gamma_attn, ln_beta_attn,
W_ff1, b_ff1, W_ff2, b_ff2, ln_gamma_ffn, ln_beta_ffn. Embeddings and
projections are drawn N(0, 0.02) in that order from
rng_stream(seed, TESTING); LayerNorm gamma is 1, beta and biases are 0.
"""
from dataclasses import dataclass

import numpy as np

KIND_PROJECTION, KIND_EMBEDDING, KIND_BIAS, KIND_NORM = 0, 1, 2, 3


@dataclass(frozen=True)
class Spec:
    vocab: int
    dim: int
    heads: int
    layers: int
    max_seq: int
    architecture_flags: int = 0   # src/include/core/model_types.h:26-36

    @property
    def ffn(self):
        return 4 * self.dim


C1 = Spec(512, 128, 4, 4, 64)


TIED, ROPE, RMSNORM, GELU, SWIGLU = 1, 2, 4, 8, 16


def inventory(spec):
    """model_param_tensors (src/core/model_params.c:39-103) for the spec's
    architecture bits: no output projection with tied embeddings, no norm
    betas with RMSNorm, the gate branch after b_ff1 with SwiGLU."""
    d, V, F = spec.dim, spec.vocab, spec.ffn
    f = spec.architecture_flags
    out = [("token_embeddings", V, d, KIND_EMBEDDING)]
    if not f & TIED:
        out.append(("output_projection", d, V, KIND_PROJECTION))
    out.append(("output_bias", 1, V, KIND_BIAS))
    for l in range(spec.layers):
        out += [(f"layer{l}.W_q", d, d, KIND_PROJECTION), (f"layer{l}.W_k", d, d, KIND_PROJECTION),
                (f"layer{l}.W_v", d, d, KIND_PROJECTION), (f"layer{l}.W_o", d, d, KIND_PROJECTION),
                (f"layer{l}.ln_gamma_attn", 1, d, KIND_NORM)]
        if not f & RMSNORM:
            out.append((f"layer{l}.ln_beta_attn", 1, d, KIND_NORM))
        out += [(f"layer{l}.W_ff1", d, F, KIND_PROJECTION), (f"layer{l}.b_ff1", 1, F, KIND_BIAS)]
        if f & SWIGLU:
            out += [(f"layer{l}.W_ff_gate", d, F, KIND_PROJECTION), (f"layer{l}.b_ff_gate", 1, F, KIND_BIAS)]
        out += [(f"layer{l}.W_ff2", F, d, KIND_PROJECTION), (f"layer{l}.b_ff2", 1, d, KIND_BIAS),
                (f"layer{l}.ln_gamma_ffn", 1, d, KIND_NORM)]
        if not f & RMSNORM:
            out.append((f"layer{l}.ln_beta_ffn", 1, d, KIND_NORM))
    return out


def synth_params(oracle, spec, seed):
    """fp32 parameters in the reference's flat layout, as a list of arrays."""
    from _native_oracle import STREAM_TESTING
    state = np.array([oracle.rng_stream(seed, STREAM_TESTING)], np.uint64)
    tensors = []
    for name, r, c, kind in inventory(spec):
        if kind in (KIND_PROJECTION, KIND_EMBEDDING):
            t = oracle.gaussian(state, r * c, 0.02).reshape(r, c)
        elif kind == KIND_NORM and "ln_gamma" in name:
            t = np.ones((r, c), np.float32)
        else:
            t = np.zeros((r, c), np.float32)
        tensors.append(t)
    return tensors


def quantize_params(oracle, spec, tensors, bits, gran=2):
    """Per tensor: (kind, fp32 or None, scales or None, packed or None) and the
    flat dequantized parameter vector the reference's loader would produce."""
    recs, flat = [], []
    for (name, r, c, kind), t in zip(inventory(spec), tensors):
        if kind == KIND_PROJECTION:
            s, p = oracle.quantize_pack(t, bits, gran)
            rc, deq = oracle.quantize_unpack(s, p, r, c, bits, gran)
            assert rc == 0
            recs.append((name, kind, r, c, None, s, p))
            flat.append(deq.ravel())
        else:
            recs.append((name, kind, r, c, t, None, None))
            flat.append(t.ravel())
    return recs, np.concatenate(flat)
