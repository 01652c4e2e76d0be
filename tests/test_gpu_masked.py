"""The masked full-prefix forward on the device (dz_cuda_forward_masked,
model_forward_masked of src/core/transformer.c:527-576).

- Against the reference's own build (tests/golden/masked.npz): plain
  causal, right / left / scattered padding, a custom attention mask with a
  real query that attends to nothing, T = max_seq_len; the default
  architecture (INT8) and tied + RoPE + RMSNorm + SwiGLU (INT4).
- Against the oracle (or_forward_masked, pinned to the same vectors) for four
  sequences of 100 positions at head dimensions 64 and 128, each with its own
  padding and attention mask, random norm gains and biases.
- Properties: without masks the result is the batched prefill's, bit for bit;
  the rings are empty afterwards; invalid inputs are refused.

Logits: max |g - r| / max |r| <= 1e-3."""
import numpy as np
import pytest

from conftest import golden
from _models import RMSNORM, ROPE, SWIGLU, TIED, Spec, quantize_params, synth_params
from test_gpu_arch import _perturbed
from test_oracle_golden import masked_golden_cases

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3


def _rel(a, r):
    return float(np.abs(a - r).max() / max(np.abs(r).max(), 1e-6))


@pytest.mark.parametrize("mi", [0, 1])
def test_masked_forward_matches_reference(gpu, oracle, mi):
    g = golden("masked.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g[f"m{mi}_spec"])
    spec = Spec(V, d, H, L, T, int(g[f"m{mi}_flags"][0]))
    recs, _ = quantize_params(oracle, spec, synth_params(oracle, spec, wseed), bits)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs])
    cache = gpu.KVCache(model, 1)
    errs = []
    for ci, (ids, pad, att, ref) in enumerate(masked_golden_cases(g, mi)):
        got = cache.forward_masked(ids[None], None if pad is None else pad[None],
                                   None if att is None else att[None])[0]
        errs.append(_rel(got, ref))
    print(f"model {mi}: max-rel per case {np.array(errs)}")
    assert max(errs) <= LOGIT_TOL, errs
    with pytest.raises(gpu.DzError):   # a padding mask without a real position
        cache.forward_masked(g[f"m{mi}_c0_ids"][None, :16], np.zeros((1, 16), np.uint8))
    cache.close()
    model.close()


def _masks(rng, B, T):
    pad = np.ones((B, T), np.uint8)
    pad[0, -17:] = 0                                   # right padding
    pad[1, :23] = 0                                    # left padding
    pad[2] = (rng.rand(T) > 0.3).astype(np.uint8)      # holes
    pad[2, 5] = 1
    att = (rng.rand(B, T, T) > 0.35).astype(np.uint8)
    att[3, 40, :] = 0                                  # a real query with no key
    att[1, -1, :] = 0                                  # sequence 1's last position attends to nothing
    return pad, att


@pytest.mark.parametrize("dim,flags,bits", [(256, 0, 8), (512, 0, 4), (256, TIED | ROPE | RMSNORM | SWIGLU, 4),
                                            (512, TIED | ROPE | RMSNORM | SWIGLU, 8)])
def test_masked_forward_batched_matches_oracle(gpu, oracle, dim, flags, bits):
    spec = Spec(1000, dim, 4, 2, 128, flags)
    recs, flat = quantize_params(oracle, spec, _perturbed(oracle, spec, 70 + flags), bits)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs])
    om = oracle.model(spec, flat)
    B, T = 4, 100
    rng = np.random.RandomState(dim + flags)
    ids = rng.randint(0, 1000, size=(B, T)).astype(np.uint32)
    pad, att = _masks(rng, B, T)
    cache = gpu.KVCache(model, B)
    for p, a in ((pad, None), (None, att), (pad, att)):
        got = cache.forward_masked(ids, p, a)
        for b in range(B):
            ref = om.forward_masked(ids[b], None if p is None else p[b], None if a is None else a[b])
            err = _rel(got[b], ref)
            assert err <= LOGIT_TOL, (b, err, p is not None, a is not None)
    cache.close()
    om.close()
    model.close()


def test_masked_forward_properties(gpu, oracle):
    spec = Spec(900, 512, 4, 2, 96)
    recs, _ = quantize_params(oracle, spec, _perturbed(oracle, spec, 5), 8)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, 8, 2) for (_, k, r, c, f, s, p) in recs])
    B, T = 3, 80
    ids = np.random.RandomState(9).randint(0, 900, size=(B, T)).astype(np.uint32)
    cache = gpu.KVCache(model, B)
    cache.set_prefill(gpu.PREFILL_BATCHED)
    want = cache.prefill(ids)
    # no masks: the batched prefill's arithmetic, bit for bit; all-ones masks
    # (the masked attention kernel) within fp32 noise of it
    np.testing.assert_array_equal(cache.forward_masked(ids), want)
    for p, a in ((np.ones((B, T), np.uint8), None), (None, np.ones((B, T, T), np.uint8))):
        got = cache.forward_masked(ids, p, a)
        assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    # the rings are left empty: the next step is position 0
    first = cache.forward_tokens(ids[:, 0])
    fresh = gpu.KVCache(model, B)
    np.testing.assert_array_equal(first, fresh.forward_tokens(ids[:, 0]))
    fresh.close()
    for bad in (lambda: cache.forward_masked(ids[:, :0]),                                  # seq_len 0
                lambda: cache.forward_masked(np.zeros((B, 97), np.uint32)),                # above max_seq_len
                lambda: cache.forward_masked(ids, np.zeros((B, T), np.uint8))):            # no real position
        with pytest.raises((gpu.DzError, AssertionError, ValueError)):
            bad()
    cache.close()
    model.close()
