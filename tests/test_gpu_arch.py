"""The architecture bits (src/include/core/model_types.h:26-36) on the
device: tied embeddings, RoPE, RMSNorm, GELU and SwiGLU.

- Against the reference's own forward and generation loop
  (tests/golden/arch23.npz: tied + RoPE + RMSNorm + SwiGLU, greedy;
  arch8.npz: GELU, INT4, top-k; arch6.npz: RoPE + RMSNorm with ring
  eviction, capacity 32, positions past max_seq_len, top-k): the bundle the
  device's writer produces is the reference writer's bytes, the prompt logits
  of every position and the logits of every draw within 1e-3, the token
  streams identical except at documented near-ties (tests/_margins.py).
- Against the oracle at head dimensions 64 and 128 (the specialised
  attention kernels), random norm gains and biases (the reference initialises
  them to 1 and 0, which would leave the bias and gate paths untested), batched
  prefill over 160 rows (tensor-core GEMM for the FFN products) and
  ROW-granularity scales (the SwiGLU gate as its own device matrix).

Logits: max |g - r| / max |r| <= 1e-3 per position."""
import os

import numpy as np
import pytest

from conftest import golden
from _margins import check_streams, stream_margins
from _models import (GELU, KIND_BIAS, KIND_NORM, RMSNORM, ROPE, SWIGLU, TIED, Spec, inventory,
                     quantize_params, synth_params)
from test_gpu_model import _abs_err, _golden_logit_err, _oracle_margins

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
MASKED = [256, 257, 258, 259]


def _rel(a, r):
    a = np.array(a, np.float32, copy=True)
    r = np.array(r, np.float32, copy=True)
    a[..., MASKED] = 0
    r[..., MASKED] = 0
    return np.abs(a - r).max(axis=-1) / np.maximum(np.abs(r).max(axis=-1), 1e-6)


@pytest.fixture(scope="module", params=["arch23", "arch8", "arch6"])
def arch_golden(request, gpu, oracle, tmp_path_factory):
    name = request.param
    g = golden(f"{name}.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    spec = Spec(V, d, H, L, T, int(g["architecture_flags"][0]))
    params = np.concatenate([t.ravel() for t in synth_params(oracle, spec, wseed)])
    path = str(tmp_path_factory.mktemp(name) / f"{name}.bin")
    gpu.save_quantized_bundle(path, spec, params, bits, gpu.GRAN_COLUMN, train_window=T, seed=wseed)
    assert gpu.fnv1a(np.fromfile(path, np.uint8)) == int(g["bundle_fnv"][0])
    bundle = gpu.Bundle(path)
    assert bundle.desc.architecture_flags == spec.architecture_flags
    model = gpu.Model.from_bundle(bundle)
    yield name, g, spec, model
    model.close()
    bundle.close()


def test_arch_prompt_and_draw_logits(gpu, arch_golden):
    """Every prompt position of sequence 0 through the step API, and the
    logits of each stored draw (the reference's tokens fed back), against the
    reference's."""
    name, g, spec, model = arch_golden
    cache = gpu.KVCache(model, 1)
    pl = np.stack([cache.forward_tokens(np.array([t], np.uint32))[0] for t in g["prompts"][0]])
    err_p = _rel(pl, g["prompt_logits"])
    cache.close()
    lg = g["logits"]
    n = lg.shape[0]
    cache = gpu.KVCache(model, n)
    for t in range(g["prompts"].shape[1]):
        out = cache.forward_tokens(g["prompts"][:n, t])
    dec = [out]
    for i in range(1, lg.shape[1]):
        dec.append(cache.forward_tokens(g["tokens"][:n, i - 1]))
    err_d = _rel(np.stack(dec, 1), lg)
    cache.close()
    print(f"{name}: max-rel prompt {err_p.max():.2e} draws {err_d.max():.2e}")
    assert err_p.max() <= LOGIT_TOL, err_p
    assert err_d.max() <= LOGIT_TOL, err_d


def test_arch_batched_prefill_logits(gpu, arch_golden):
    """The batched prefill's last-position logits against the reference's
    logits of the first draw."""
    name, g, spec, model = arch_golden
    lg = g["logits"]
    n = lg.shape[0]
    cache = gpu.KVCache(model, n)
    cache.set_prefill(gpu.PREFILL_BATCHED)
    err = _rel(cache.prefill(g["prompts"][:n]), lg[:, 0])
    cache.close()
    assert err.max() <= LOGIT_TOL, err


@pytest.mark.parametrize("mode", ["tokens", "batched"])
def test_arch_generation_stream(gpu, arch_golden, mode):
    """dz_cuda_generate with the golden's sampling and seeds (layered path:
    the fused kernel runs the default architecture only)."""
    name, g, spec, model = arch_golden
    strategy, top_k = (int(x) for x in g["sampling"])
    temperature, top_p = (float(x) for x in g["sampling_f"])
    seeds = g["seeds"] if g["seeds"].size else None
    samp = gpu.Sampling(strategy, temperature, top_k, top_p)
    B, n_new = g["tokens"].shape
    cache = gpu.KVCache(model, B)
    cache.set_prefill({"tokens": gpu.PREFILL_TOKENS, "batched": gpu.PREFILL_BATCHED}[mode])
    assert not cache.uses_fused(samp)
    toks = cache.generate(g["prompts"], n_new, samp, seeds=seeds)
    cache.close()
    err = _golden_logit_err(gpu, model, g)
    bad = check_streams(toks, g["tokens"], g["margins"], err)
    print(f"{name} ({mode}): observed logit error {err:.3g}, near-tie divergences {bad}")


# ------------------------------------------------------- against the oracle

def _perturbed(oracle, spec, seed):
    """Synthetic weights with random norm gains (1 + N(0, 0.1)), betas and
    biases (N(0, 0.05))."""
    tensors = synth_params(oracle, spec, seed)
    rng = np.random.RandomState(seed)
    for i, (name, r, c, kind) in enumerate(inventory(spec)):
        if kind == KIND_NORM and "gamma" in name:
            tensors[i] = (1.0 + 0.1 * rng.randn(r, c)).astype(np.float32)
        elif kind in (KIND_NORM, KIND_BIAS):
            tensors[i] = (0.05 * rng.randn(r, c)).astype(np.float32)
    return tensors


CASES = [
    # (dim, heads, flags, bits, granularity)
    (256, 4, TIED | ROPE | RMSNORM | SWIGLU, 8, 2),
    (512, 4, TIED | ROPE | RMSNORM | SWIGLU, 4, 2),
    (512, 4, ROPE | SWIGLU, 8, 1),
    (256, 4, GELU | RMSNORM, 4, 2),
    (512, 4, TIED | GELU, 8, 2),
]


@pytest.mark.parametrize("dim,heads,flags,bits,gran", CASES)
@pytest.mark.parametrize("mode", ["tokens", "batched"])
def test_arch_against_oracle(gpu, oracle, dim, heads, flags, bits, gran, mode):
    """Four sequences of 40 prompt tokens (160 prefill rows), then 6 fed
    tokens, every position's logits against the oracle's forward; then a greedy
    generation against the oracle's loop."""
    spec = Spec(1000, dim, heads, 2, 64, flags)
    recs, flat = quantize_params(oracle, spec, _perturbed(oracle, spec, 41 + flags), bits, gran)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, gran) for (_, k, r, c, f, s, p) in recs])
    om = oracle.model(spec, flat)
    B, T, extra = 4, 40, 6
    rng = np.random.RandomState(flags)
    prompts = rng.randint(0, 1000, size=(B, T)).astype(np.uint32)
    nxt = rng.randint(0, 1000, size=(extra, B)).astype(np.uint32)
    ref = np.zeros((B, extra + 1, 1000), np.float32)
    for b in range(B):
        om.reset()
        for t in range(T):
            r = om.forward_token(prompts[b, t])
        ref[b, 0] = r
        for i in range(extra):
            ref[b, i + 1] = om.forward_token(nxt[i, b])
    cache = gpu.KVCache(model, B)
    if mode == "batched":
        cache.set_prefill(gpu.PREFILL_BATCHED)
        got = [cache.prefill(prompts)]
    else:
        cache.set_prefill(gpu.PREFILL_TOKENS)
        for t in range(T):
            first = cache.forward_tokens(prompts[:, t])
        got = [first]
    got += [cache.forward_tokens(nxt[i]) for i in range(extra)]
    got = np.stack(got, 1)
    rel = _rel(got, ref)
    print(f"flags {flags} d {dim} INT{bits} gran {gran} ({mode}): max-rel {rel.max():.2e}")
    assert rel.max() <= LOGIT_TOL, rel.max(axis=0)
    gtok, glg, margins = _oracle_margins(oracle, om, prompts, 8)
    toks = cache.generate(prompts, 8, gpu.Sampling(gpu.GREEDY))
    check_streams(toks, gtok, margins, _abs_err(got, ref))
    cache.close()
    om.close()
    model.close()
