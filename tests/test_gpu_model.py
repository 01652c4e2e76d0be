"""The decode path on the device against the reference's golden logits and
token streams (tests/golden/{c1,c2,ring}.npz) and against the oracle.

Logit parity metric (the normalized form of src/tests/core/
test_quantized_matmul.c:79): max_i |g_i - r_i| / max(max_i |r_i|, 1e-6),
target <= 1e-3 per position. Token streams: identical; a divergence is
accepted only at a documented near-tie (the reference's own top-2 gap or
sampling boundary margin within 10x the observed logit error, tests/_margins.py),
after which the sequence is not compared further."""
import os

import numpy as np
import pytest

from conftest import golden
from _margins import check_streams, stream_margins, unit_draws
from _models import Spec, quantize_params, synth_params
from _native_oracle import STREAM_SAMPLING

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def _model_from_golden(gpu, oracle, name, tmp_path):
    g = golden(f"{name}.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    spec = Spec(V, d, H, L, T)
    params = np.concatenate([t.ravel() for t in synth_params(oracle, spec, wseed)])
    path = str(tmp_path / f"{name}.bin")
    gpu.save_quantized_bundle(path, spec, params, bits, gpu.GRAN_COLUMN, train_window=T, seed=wseed)
    b = gpu.Bundle(path)
    return g, spec, gpu.Model.from_bundle(b)


def _rel(a, r):
    return np.abs(a - r).max(axis=-1) / np.maximum(np.abs(r).max(axis=-1), 1e-6)


def test_c1_logits_every_position(gpu, oracle, tmp_path):
    g, spec, model = _model_from_golden(gpu, oracle, "c1", tmp_path)
    cache = gpu.KVCache(model, 1)
    prompt, toks = g["prompts"][0], g["tokens"][0]
    out = [cache.forward_tokens(np.array([t], np.uint32))[0] for t in prompt]
    err_p = _rel(np.stack(out), g["prompt_logits"])
    assert err_p.max() <= LOGIT_TOL, err_p.max()
    # decode positions: the logits each greedy draw was taken from
    dec = [out[-1]]
    for t in toks[:-1]:
        dec.append(cache.forward_tokens(np.array([t], np.uint32))[0])
    ref = g["logits"][0].copy()
    ref[:, [256, 257, 258, 259]] = np.float32(0)
    got = np.stack(dec)
    got[:, [256, 257, 258, 259]] = 0
    err_d = _rel(got, ref)
    assert err_d.max() <= LOGIT_TOL, err_d.max()
    print(f"c1 max-rel logits: prompt {err_p.max():.2e} decode {err_d.max():.2e}")
    cache.close(); model.close()


MASKED = [256, 257, 258, 259]


def _abs_err(got, ref):
    """Max absolute logit error, masked ids excluded (the reference holds
    -FLT_MAX there, the device the raw logit)."""
    g = np.array(got, np.float32, copy=True)
    r = np.array(ref, np.float32, copy=True)
    g[..., MASKED] = 0
    r[..., MASKED] = 0
    return float(np.abs(g - r).max())


def _golden_logit_err(gpu, model, g, capacity=None):
    """The device's observed logit error on the golden sequences whose
    reference logits are stored: their prompts and reference tokens fed
    through the step API, logits compared at every draw."""
    lg = g["logits"]
    n = lg.shape[0]
    cache = gpu.KVCache(model, n, capacity)
    prompts, toks = g["prompts"][:n], g["tokens"][:n]
    for t in range(prompts.shape[1]):
        out = cache.forward_tokens(prompts[:, t])
    err = _abs_err(out, lg[:, 0])
    for i in range(1, lg.shape[1]):
        out = cache.forward_tokens(toks[:, i - 1])
        err = max(err, _abs_err(out, lg[:, i]))
    cache.close()
    return err


def _oracle_margins(oracle, om, prompts, n_new, strategy=0, temperature=0.0, top_k=0, top_p=0.0, seeds=None):
    """The oracle's tokens, logits and decision margins for a generation."""
    toks, lg = om.generate(prompts, n_new, strategy, temperature, top_k, top_p, seeds, want_logits=True)
    units = None
    if seeds is not None:
        units = unit_draws(oracle.rng_stream, lambda st: oracle.L.or_rng_unit(st.ctypes.data), seeds, n_new,
                           STREAM_SAMPLING)
    return toks, lg, stream_margins(lg, toks, strategy, temperature, top_k, top_p, units)


PATHS = {"layered": 1, "fused": 2}


def _cache(gpu, model, batch, path, sampling, capacity=None):
    cache = gpu.KVCache(model, batch, capacity)
    cache.set_path(PATHS[path])
    assert cache.uses_fused(sampling) == (path == "fused")
    return cache


@pytest.mark.parametrize("path", ["layered", "fused"])
def test_c1_greedy_stream(gpu, oracle, tmp_path, path):
    g, spec, model = _model_from_golden(gpu, oracle, "c1", tmp_path)
    samp = gpu.Sampling(gpu.GREEDY)
    cache = _cache(gpu, model, 1, path, samp)
    toks = cache.generate(g["prompts"], 48, samp)
    check_streams(toks, g["tokens"], g["margins"], _golden_logit_err(gpu, model, g))
    cache.close(); model.close()


@pytest.mark.parametrize("path", ["layered", "fused"])
def test_c2_top_p_streams(gpu, oracle, tmp_path, path):
    """64 sequences x (32 prompt + 32 top-p 0.9 draws at T=0.8), per-sequence seeds."""
    g, spec, model = _model_from_golden(gpu, oracle, "c2", tmp_path)
    samp = gpu.Sampling(gpu.TOPP, 0.8, 0, 0.9)
    cache = _cache(gpu, model, 64, path, samp)
    toks = cache.generate(g["prompts"], 32, samp, seeds=g["seeds"])
    err = _golden_logit_err(gpu, model, g)
    bad = check_streams(toks, g["tokens"], g["margins"], err)
    print(f"c2 {path}: observed logit error {err:.3g}, near-tie divergences {bad}")
    # repeated launches of the cached graph give the same streams
    np.testing.assert_array_equal(cache.generate(g["prompts"], 32, samp, seeds=g["seeds"]), toks)
    cache.close(); model.close()


@pytest.mark.parametrize("path", ["layered", "fused"])
def test_ring_eviction_top_k(gpu, oracle, tmp_path, path):
    """Capacity 32 with 24 + 40 tokens: ring eviction and positions past max_seq_len."""
    g, spec, model = _model_from_golden(gpu, oracle, "ring", tmp_path)
    samp = gpu.Sampling(gpu.TOPK, 0.8, 5, 0.0)
    cache = _cache(gpu, model, 2, path, samp)
    toks = cache.generate(g["prompts"], 40, samp, seeds=g["seeds"])
    check_streams(toks, g["tokens"], g["margins"], _golden_logit_err(gpu, model, g))
    cache.close(); model.close()


def test_step_api_matches_generate(gpu, oracle, tmp_path):
    """forward_tokens + select per step reproduces the on-device generation loop."""
    g, spec, model = _model_from_golden(gpu, oracle, "c2", tmp_path)
    B = 8
    cache = gpu.KVCache(model, B)
    samp = gpu.Sampling(gpu.TOPP, 0.8, 0, 0.9)
    prompts, seeds = g["prompts"][:B], g["seeds"][:B]
    cache.reset()
    for t in range(prompts.shape[1]):
        cache.forward_tokens(prompts[:, t], want_logits=False)
    st = np.array([gpu.rng_stream(int(s), gpu.STREAM_SAMPLING) for s in seeds], np.uint64)
    out = []
    for i in range(32):
        ids = cache.select(samp, st)
        out.append(ids)
        if i + 1 < 32:
            cache.forward_tokens(ids, want_logits=False)
    np.testing.assert_array_equal(np.stack(out, 1), g["tokens"][:B])
    cache.close(); model.close()


def test_batched_against_oracle_with_reset_mask(gpu, oracle):
    spec = Spec(700, 96, 3, 2, 40)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, 21), 8)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, 8, 2) for (_, k, r, c, f, s, p) in recs])
    om = oracle.model(spec, flat)
    B = 5
    cache = gpu.KVCache(model, B, 40)
    rng = np.random.RandomState(0)
    seqs = rng.randint(0, 700, size=(B, 12)).astype(np.uint32)
    for t in range(12):
        got = cache.forward_tokens(seqs[:, t])
    # reset only sequence 2 and feed it again from the start
    mask = np.zeros(B, np.uint8); mask[2] = 1
    cache.reset(mask)
    for t in range(5):
        got = cache.forward_tokens(seqs[:, t] if t == 0 else np.where(np.arange(B) == 2, seqs[:, t], 0))
    om.reset()
    for t in range(5):
        r = om.forward_token(seqs[2, t])
    assert _rel(got[2], r) <= 1e-4
    cache.close(); model.close()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("shape", [(700, 80, 5, 3, 48, 9), (600, 128, 2, 2, 40, 30), (500, 128, 1, 2, 70, 12),
                                   (400, 128, 16, 1, 64, 50)])
def test_fused_matches_layered_random_model(gpu, oracle, bits, shape):
    """Both paths on models off the golden shapes: d=80 with 5 heads of 16
    (F=320, V=700, L=3), d=128 with 2 heads of 64, 1 head of 128 and 16 heads
    of 8 (one warp per head over 2 chunks of keys, the ring wrapping); batch 7,
    greedy and top-k: identical token streams, equal to the oracle's."""
    spec = Spec(*shape[:5])
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, 33), bits)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs])
    rng = np.random.RandomState(bits)
    prompts = rng.randint(0, min(256, shape[0]), size=(7, shape[5])).astype(np.uint32)
    assert gpu.KVCache(model, 7).uses_fused(gpu.Sampling(gpu.GREEDY))
    seeds = np.arange(7, dtype=np.uint64) + 100
    om = oracle.model(spec, flat)
    for samp, sd, strat in ((gpu.Sampling(gpu.GREEDY), None, 0), (gpu.Sampling(gpu.TOPK, 0.7, 12, 0.0), seeds, 1)):
        outs = []
        for path in ("layered", "fused"):
            cache = _cache(gpu, model, 7, path, samp)
            outs.append(cache.generate(prompts, 20, samp, seeds=sd))
            cache.close()
        np.testing.assert_array_equal(outs[0], outs[1])
        ref, _ = om.generate(prompts, 20, strat, samp.c.temperature, samp.c.top_k, 0.0, sd)
        np.testing.assert_array_equal(outs[1], ref)
    model.close()


def test_fused_not_eligible_falls_back(gpu, oracle):
    """A d=256 INT8 model (W1 is 256 KB in the device layout) runs layered under AUTO."""
    spec = Spec(300, 256, 4, 1, 16)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, 4), 8)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, 8, 2) for (_, k, r, c, f, s, p) in recs])
    cache = gpu.KVCache(model, 2)
    samp = gpu.Sampling(gpu.GREEDY)
    assert not cache.uses_fused(samp)
    with pytest.raises(gpu.DzError):
        cache.set_path(2)
    prompts = np.array([[1, 2, 3], [4, 5, 6]], np.uint32)
    toks = cache.generate(prompts, 5, samp)
    om = oracle.model(spec, flat)
    ref, _ = om.generate(prompts, 5, 0, 0.0, 0, 0.0, None)
    np.testing.assert_array_equal(toks, ref)
    cache.close(); model.close()


@pytest.mark.parametrize("bits", [8, 4])
def test_large_batch_tensor_core_path(gpu, oracle, bits):
    """A d=1024 model at batch 24: every projection is large enough for the
    tensor-core GEMM (integer limbs, tcgen05). Logits of every step of two
    sequences within tolerance, and identical greedy streams for all."""
    spec = Spec(1200, 1024, 8, 2, 48)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, 44), bits)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs])
    B = 24
    rng = np.random.RandomState(bits + 5)
    prompts = rng.randint(0, 256, size=(B, 10)).astype(np.uint32)
    cache = gpu.KVCache(model, B, 48)
    assert not cache.uses_fused(gpu.Sampling(gpu.GREEDY))
    om = oracle.model(spec, flat)
    for t in range(10):
        got = cache.forward_tokens(prompts[:, t])
    err = 0.0
    for b in (0, 17):
        om.reset()
        for t in range(10):
            r = om.forward_token(prompts[b, t])
        assert _rel(got[b], r) <= LOGIT_TOL, (b, _rel(got[b], r))
        err = max(err, _abs_err(got[b], r))
    cache.reset()
    toks = cache.generate(prompts, 8, gpu.Sampling(gpu.GREEDY))
    ref, _, margins = _oracle_margins(oracle, om, prompts, 8)
    check_streams(toks, ref, margins, err)
    cache.close(); model.close()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("hd", [32, 64, 128])
def test_batched_prefill_matches_token_prefill(gpu, oracle, bits, hd):
    """dz_cuda_prefill (all prompt positions per layer pass, causal attention
    over each prompt) against the per-token prefill and the oracle: last-position
    logits within tolerance for full and ragged prompts, and generation through
    both prefill policies giving the oracle's greedy streams."""
    H = 512 // hd
    spec = Spec(900, 512, H, 2, 64)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, 50 + hd), bits)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs])
    B, T = 5, 21
    rng = np.random.RandomState(hd + bits)
    prompts = rng.randint(0, 256, size=(B, T)).astype(np.uint32)
    lens = np.array([21, 7, 13, 1, 20], np.uint32)
    om = oracle.model(spec, flat)
    ref = []
    for b in range(B):
        om.reset()
        for t in range(int(lens[b])):
            r = om.forward_token(prompts[b, t])
        ref.append(r)
    cache = gpu.KVCache(model, B, 64)
    got = cache.prefill(prompts, lens)
    err = 0.0
    for b in range(B):
        assert _rel(got[b], ref[b]) <= LOGIT_TOL, (b, _rel(got[b], ref[b]))
        err = max(err, _abs_err(got[b], ref[b]))
    # the rings hold each prompt: one decode step continues every sequence
    nxt = rng.randint(0, 256, size=B).astype(np.uint32)
    step = cache.forward_tokens(nxt)
    for b in range(B):
        om.reset()
        for t in range(int(lens[b])):
            om.forward_token(prompts[b, t])
        r = om.forward_token(nxt[b])
        assert _rel(step[b], r) <= LOGIT_TOL, (b, _rel(step[b], r))
        err = max(err, _abs_err(step[b], r))
    samp = gpu.Sampling(gpu.GREEDY)
    outs = []
    for mode in (gpu.PREFILL_TOKENS, gpu.PREFILL_BATCHED):
        cache.set_prefill(mode)
        outs.append(cache.generate(prompts, 6, samp))
    gref, _, margins = _oracle_margins(oracle, om, prompts, 6)
    for o in outs:
        check_streams(o, gref, margins, err)
    cache.close(); model.close()


def test_batched_prefill_rejects_bad_lengths(gpu, oracle):
    spec = Spec(300, 256, 4, 1, 16)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, 4), 8)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, 8, 2) for (_, k, r, c, f, s, p) in recs])
    cache = gpu.KVCache(model, 2, 16)
    with pytest.raises(gpu.DzError):
        cache.prefill(np.zeros((2, 5), np.uint32), np.array([0, 5], np.uint32))
    with pytest.raises(gpu.DzError):
        cache.prefill(np.zeros((2, 20), np.uint32))
    cache.close(); model.close()
