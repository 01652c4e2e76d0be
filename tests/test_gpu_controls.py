"""The generation loop's controls on the device (dz_cuda_generate_ex,
dz_cuda_select_ex) against the reference's own generation_decode_with_options
(src/cli/generation.c:198-308, tests/golden/controls.npz): repetition
penalty over prompt and generated ids, the tokenizer's unassigned ids masked,
EOS under a minimum length, stop sequences, and the per-sequence results.
Tokens: identical, or a first divergence where the reference's decision
margin is below 10x the observed logit error (tests/_margins.py); results
are compared for every sequence that did not diverge."""
import numpy as np
import pytest

from conftest import golden
from _margins import check_streams, stream_margins, unit_draws
from _models import Spec, quantize_params, synth_params
from _native_oracle import STREAM_SAMPLING, Controls as OracleControls

pytestmark = pytest.mark.gpu

CTRL_IDS = (256, 257, 258)   # PAD, UNK, BOS


def _cases(g):
    for i in range(int(g["count"][0])):
        strategy, top_k, min_new = (int(x) for x in g[f"c{i}_params"])
        temperature, top_p, penalty = (float(x) for x in g[f"c{i}_params_f"])
        st, sl = g[f"c{i}_stop_tokens"], g[f"c{i}_stop_lengths"]
        stops, off = [], 0
        for n in sl:
            stops.append([int(t) for t in st[off:off + n]])
            off += n
        yield i, strategy, top_k, min_new, temperature, top_p, penalty, stops, g[f"c{i}_seeds"]


@pytest.fixture(scope="module")
def ctl_model(gpu, oracle):
    g = golden("controls.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    spec = Spec(V, d, H, L, T)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, wseed), bits)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs])
    om = oracle.model(spec, flat)
    # the device's observed logit error on these prompts: the step API against
    # the oracle's forward, last prompt position of four sequences
    cache = gpu.KVCache(model, g["prompts"].shape[0])
    for t in range(g["prompts"].shape[1]):
        got = cache.forward_tokens(g["prompts"][:, t])
    cache.close()
    err = 0.0
    for b in range(4):
        om.reset()
        for t in range(g["prompts"].shape[1]):
            r = om.forward_token(g["prompts"][b, t])
        err = max(err, float(np.abs(got[b] - r).max()))
    yield g, spec, model, om, err
    om.close()
    model.close()


def _oracle_run(oracle, om, g, strategy, top_k, min_new, temperature, top_p, penalty, stops, seeds, n_new):
    """The oracle's run of the same case with its logits and margins (the
    oracle equals the reference on these cases, test_oracle_golden.py)."""
    c = OracleControls(penalty=penalty, min_new=min_new, mask_from=int(g["tokenizer_vocab"][0]), stops=stops)
    toks, res, lg = om.generate_ex(g["prompts"], n_new, c, strategy, temperature, top_k, top_p,
                                   seeds if strategy else None, want_logits=True)
    units = None
    if strategy:
        units = unit_draws(oracle.rng_stream, lambda st: oracle.L.or_rng_unit(st.ctypes.data), seeds, n_new,
                           STREAM_SAMPLING)
    ended = toks == 0xFFFFFFFF
    margins = stream_margins(lg, np.where(ended, 0, toks), strategy, temperature, top_k, top_p, units)
    margins[ended] = np.inf
    return toks, res, margins


def test_generate_ex_matches_reference_loop(gpu, oracle, ctl_model):
    g, spec, model, om, err = ctl_model
    B = g["prompts"].shape[0]
    cache = gpu.KVCache(model, B)
    samp_masked = CTRL_IDS
    for i, strategy, top_k, min_new, temperature, top_p, penalty, stops, seeds in _cases(g):
        n_new = g[f"c{i}_tokens"].shape[1]
        samp = gpu.Sampling(strategy, temperature, top_k, top_p, samp_masked)
        ctl = gpu.Controls(penalty=penalty, eos_id=259, min_new=min_new, mask_from=int(g["tokenizer_vocab"][0]),
                           stops=stops)
        toks, res = cache.generate_ex(g["prompts"], n_new, samp, ctl, seeds=seeds if strategy else None)
        ref_t, ref_r = g[f"c{i}_tokens"], g[f"c{i}_results"]
        _, _, margins = _oracle_run(oracle, om, g, strategy, top_k, min_new, temperature, top_p, penalty, stops,
                                    seeds, n_new)
        bad = check_streams(toks, ref_t, margins, err)
        diverged = {q for q, _ in bad}
        for q in range(B):
            if q not in diverged:
                np.testing.assert_array_equal(res[q], ref_r[q], err_msg=f"case {i} sequence {q}")
        print(f"case {i}: results {res[:, :4].tolist()} near-ties {bad}")
    cache.close()


def test_select_ex_in_the_host_loop(gpu, oracle, ctl_model):
    """The reference's loop run on the host over the step API: forward the
    prompt, then per draw dz_cuda_select_ex (penalty over the fed tokens and
    the unassigned-id mask; EOS masked by the caller under the minimum
    length), stop matching on the host, forward the drawn token."""
    g, spec, model, om, err = ctl_model
    B, plen = g["prompts"].shape
    tv = int(g["tokenizer_vocab"][0])
    for i, strategy, top_k, min_new, temperature, top_p, penalty, stops, seeds in _cases(g):
        if i not in (1, 3):   # a penalty and stops, top-k
            continue
        n_new = g[f"c{i}_tokens"].shape[1]
        cache = gpu.KVCache(model, B)
        cache.reset()
        for t in range(plen):
            cache.forward_tokens(g["prompts"][:, t], want_logits=False)
        st = np.array([gpu.rng_stream(int(s), gpu.STREAM_SAMPLING) for s in seeds], np.uint64)
        ctl = gpu.Controls(penalty=penalty, mask_from=tv)
        out = np.full((B, n_new), 0xFFFFFFFF, np.uint32)
        done = np.zeros(B, bool)
        for k in range(n_new):
            masked = CTRL_IDS + ((259,) if k < min_new else ())
            ids = cache.select_ex(gpu.Sampling(strategy, temperature, top_k, top_p, masked), ctl, st)
            for q in range(B):
                if done[q]:
                    continue
                out[q, k] = ids[q]
                gen = list(out[q, :k + 1])
                if ids[q] == 259:
                    done[q] = True
                for s in stops:
                    n = len(s)
                    if n <= k + 1 and k + 1 - n >= min_new and gen[k + 1 - n:] == s:
                        done[q] = True
            if k + 1 < n_new:
                cache.forward_tokens(np.where(done, 0, ids).astype(np.uint32), want_logits=False)
        _, _, margins = _oracle_run(oracle, om, g, strategy, top_k, min_new, temperature, top_p, penalty, stops,
                                    seeds, n_new)
        check_streams(out, g[f"c{i}_tokens"], margins, err)
        cache.close()


def test_controls_with_batched_prefill_match_oracle(gpu, oracle):
    # observed logit error bound: 2e-4 (the d=512 tests of test_gpu_model.py
    # measure a few 1e-5 on these shapes)
    """A d=512 model (batched prefill under AUTO, prompt ids recorded in the
    token history by the prefill): penalty 1.3, a stop sequence and a minimum
    length, greedy and top-k, against the oracle's loop."""
    spec = Spec(900, 512, 8, 2, 64)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, 71), 8)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, 8, 2) for (_, k, r, c, f, s, p) in recs])
    om = oracle.model(spec, flat)
    B, T, n_new = 4, 12, 16
    rng = np.random.RandomState(71)
    prompts = rng.randint(0, 256, size=(B, T)).astype(np.uint32)
    prompts[:, 3] = prompts[:, 0]   # repeated prompt ids
    seeds = np.arange(B, dtype=np.uint64) + 900
    cache = gpu.KVCache(model, B, 64)
    for strategy, temperature, top_k in ((0, 0.0, 0), (1, 0.9, 12)):
        # stops taken from a run without them
        c0 = OracleControls(penalty=1.3, min_new=2, mask_from=260)
        t0, _, _ = om.generate_ex(prompts, n_new, c0, strategy, temperature, top_k, 0.0,
                                  seeds if strategy else None)
        stops = [[int(t0[0, 6])], [int(t0[2, 4]), int(t0[2, 5])]]
        oc = OracleControls(penalty=1.3, min_new=2, mask_from=260, stops=stops)
        ref_t, ref_r, lg = om.generate_ex(prompts, n_new, oc, strategy, temperature, top_k, 0.0,
                                          seeds if strategy else None, want_logits=True)
        samp = gpu.Sampling(strategy, temperature, top_k, 0.0, CTRL_IDS)
        ctl = gpu.Controls(penalty=1.3, eos_id=259, min_new=2, mask_from=260, stops=stops)
        toks, res = cache.generate_ex(prompts, n_new, samp, ctl, seeds=seeds if strategy else None)
        units = None
        if strategy:
            units = unit_draws(oracle.rng_stream, lambda st: oracle.L.or_rng_unit(st.ctypes.data), seeds, n_new,
                               STREAM_SAMPLING)
        ended = ref_t == 0xFFFFFFFF
        margins = stream_margins(lg, np.where(ended, 0, ref_t), strategy, temperature, top_k, 0.0, units)
        margins[ended] = np.inf
        bad = check_streams(toks, ref_t, margins, 2e-4)
        for q in set(range(B)) - {q for q, _ in bad}:
            np.testing.assert_array_equal(res[q], ref_r[q])
    cache.close()
    om.close()
    model.close()


def test_select_ex_penalty_after_fused_generation_is_refused(gpu, ctl_model):
    g, spec, model, om, err = ctl_model
    cache = gpu.KVCache(model, 2)
    samp = gpu.Sampling(gpu.GREEDY)
    assert cache.uses_fused(samp)
    cache.generate(g["prompts"][:2], 4, samp)
    with pytest.raises(gpu.DzError):
        cache.select_ex(samp, gpu.Controls(penalty=1.2))
    cache.reset()
    cache.forward_tokens(g["prompts"][:2, 0], want_logits=False)
    cache.select_ex(samp, gpu.Controls(penalty=1.2))
    cache.close()
