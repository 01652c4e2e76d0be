"""The oracle pinned against vectors produced by the reference's own sources
(tests/golden/, made by tests/golden/make_golden.py) and the RNG literals of the
reference's src/tests/core/test_rng.c."""
import numpy as np
import pytest

from conftest import golden
from _native_oracle import (GREEDY, STREAM_DROPOUT, STREAM_INIT, STREAM_SAMPLING, STREAM_TESTING)
from _models import Spec, quantize_params, synth_params


def test_rng_literals_of_reference_test(oracle):
    # src/tests/core/test_rng.c:44-58 (seed 42) and :116-119 (unit draws, seed 7 TESTING)
    pinned = {
        STREAM_INIT: (0x7C247ADEFCC8B7D8, [0x74E6E38914990A99, 0xE691ECCDAFF973E7, 0xCDBCCD2D9CE51561,
                                           0x2312AC28B968814A, 0xCC25BD84D515B7C8, 0x6E3591667D837B0F]),
        STREAM_DROPOUT: (0x16A27C5E3E3F3C94, [0x4A129E81ABCFD69D, 0xF862E617FC394C6F, 0x781752B023792B70,
                                              0x0E406FCEFDBCBB04, 0xEBF205EBB93362B0, 0xF14F0245AA6151D6]),
        STREAM_SAMPLING: (0xAA80027AC7B32959, [0xF3FBD30AEAE63199, 0x6C467EA74180E1A3, 0x0009017CCD079354,
                                               0x33875B26D07B1E58, 0x9EDE1A0789C7AF2F, 0x4823040D5887BF4A]),
    }
    for stream, (init, draws) in pinned.items():
        st = np.array([oracle.rng_stream(42, stream)], np.uint64)
        assert int(st[0]) == init
        for d in draws:
            assert oracle.L.or_rng_next(st.ctypes.data) == d
    st = np.array([oracle.rng_stream(7, STREAM_TESTING)], np.uint64)
    bits = [0x3FE54B94A5BC9DA3, 0x3FC9AC8DCE2DCC4C, 0x3FB4F41D979BD588, 0x3FCAC3BA2B5730E8]
    for b in bits:
        u = oracle.L.or_rng_unit(st.ctypes.data)
        assert np.array([u], np.float64).view(np.uint64)[0] == b


def test_rng_golden(oracle):
    g = golden("rng.npz")
    for a, seed in enumerate(g["seeds"]):
        for b, stream in enumerate(g["streams"]):
            st = np.array([oracle.rng_stream(int(seed), int(stream))], np.uint64)
            assert st[0] == g["init"][a, b]
            for k in range(8):
                assert oracle.L.or_rng_next(st.ctypes.data) == g["draws"][a, b, k]
            for k in range(4):
                assert oracle.L.or_rng_unit(st.ctypes.data) == g["units"][a, b, k]
    st = np.array([oracle.rng_stream(0, STREAM_TESTING)], np.uint64)
    np.testing.assert_array_equal(oracle.gaussian(st, 4096, 0.02), g["gaussian_seed0"])


def _quant_cases():
    g = golden("quant.npz")
    for n in range(int(g["count"])):
        r, c, bits, gran = (int(x) for x in g[f"c{n}_meta"])
        w = g[f"c{n}_w"] if f"c{n}_w" in g.files else g["adv_w"]
        yield w.reshape(r, c), bits, gran, g[f"c{n}_s"], g[f"c{n}_p"]


def test_quantize_pack_bit_exact(oracle):
    count = 0
    for w, bits, gran, s_ref, p_ref in _quant_cases():
        s, p = oracle.quantize_pack(w, bits, gran)
        np.testing.assert_array_equal(s.view(np.uint32), s_ref.view(np.uint32))
        np.testing.assert_array_equal(p, p_ref)
        rc, deq = oracle.quantize_unpack(s, p, w.shape[0], w.shape[1], bits, gran)
        assert rc == 0
        count += 1
    assert count >= 120


def test_unpack_rejects_noncanonical(oracle):
    # src/tests/core/test_quantize.c:332-349: the unused all-ones code and
    # non-zero padding bits are rejected
    w = np.arange(15, dtype=np.float32).reshape(3, 5) - 7
    for bits in (3, 4, 5, 8):
        s, p = oracle.quantize_pack(w, bits, 2)
        ones = (1 << bits) - 1
        bad = p.copy()
        bad[0] = np.uint8((int(bad[0]) & ~ones & 0xFF) | ones)
        assert oracle.quantize_unpack(s, bad, 3, 5, bits, 2)[0] == -1
        if (15 * bits) % 8:
            pad = p.copy()
            pad[-1] = np.uint8(int(pad[-1]) | 0x80)
            assert oracle.quantize_unpack(s, pad, 3, 5, bits, 2)[0] == -1
        neg = s.copy()
        neg[0] = -1.0
        assert oracle.quantize_unpack(neg, p, 3, 5, bits, 2)[0] == -1
        assert oracle.quantize_unpack(s, p, 3, 5, bits, 2)[0] == 0


def test_c3_weights_bit_exact_4096(oracle):
    g = golden("quant.npz")
    st = np.array([oracle.rng_stream(3, STREAM_TESTING)], np.uint64)
    oracle.gaussian(st, 512 * 4096, 1.0)
    w = oracle.gaussian(st, 4096 * 4096, 0.02).reshape(4096, 4096)
    for N, bits, hs, hp in g["c3_hashes"]:
        if N != 4096:
            continue
        s, p = oracle.quantize_pack(w, int(bits), 2)
        assert oracle.fnv1a(s) == hs and oracle.fnv1a(p) == hp


def test_matmul_quantized_golden(oracle):
    g = golden("qmm.npz")
    for n in range(int(g["count"])):
        m, k, nn, bits, gran = (int(x) for x in g[f"t{n}_meta"])
        s, p = oracle.quantize_pack(g[f"t{n}_b"], bits, gran)
        c = oracle.matmul_quantized(g[f"t{n}_a"], k, nn, s, p, bits, gran)
        ref = g[f"t{n}_c"]
        # src/tests/core/test_quantized_matmul.c:79
        assert np.abs(c - ref).max() <= 1e-4 * (1 + np.abs(ref).max())


def test_positional_encoding_golden(oracle):
    pe = oracle.positional_encoding(64, 128)
    ref = golden("pe.npz")["pe_64x128"]
    # within 1 ulp of the reference build (its sinf/cosf are vectorised)
    assert np.abs(pe - ref).max() <= 1.2e-7


@pytest.mark.parametrize("name", ["c1", "c2", "ring", "arch23", "arch8", "arch6"])
def test_model_generation_golden(oracle, name):
    """The oracle's forward and generation loop against the reference's
    (archNN: the architecture bits NN, src/include/core/model_types.h:26-36)."""
    g = golden(f"{name}.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    flags = int(g["architecture_flags"][0]) if "architecture_flags" in g.files else 0
    spec = Spec(V, d, H, L, T, flags)
    recs, flat = quantize_params(oracle, spec, synth_params(oracle, spec, wseed), bits)
    m = oracle.model(spec, flat)
    strategy, top_k = (int(x) for x in g["sampling"])
    temperature, top_p = (float(x) for x in g["sampling_f"])
    seeds = g["seeds"] if g["seeds"].size else None
    toks, lg = m.generate(g["prompts"], g["tokens"].shape[1], strategy, temperature, top_k, top_p, seeds,
                          want_logits=True)
    ref_lg = g["logits"]
    nl = ref_lg.shape[0]
    err = np.abs(lg[:nl] - ref_lg).max(axis=-1) / np.maximum(np.abs(ref_lg).max(axis=-1), 1e-6)
    assert err.max() <= 1e-4, err.max()
    # token streams identical (the oracle is the reference's arithmetic in strict IEEE)
    np.testing.assert_array_equal(toks, g["tokens"])
    m.reset()
    pl = np.stack([m.forward_token(t) for t in g["prompts"][0]])
    ref_pl = g["prompt_logits"]
    assert (np.abs(pl - ref_pl).max(axis=-1) / np.abs(ref_pl).max(axis=-1)).max() <= 1e-4


def test_generation_controls_match_reference(oracle):
    """or_generate_ex against the reference's own generation loop
    (generation_decode_with_options, tests/golden/controls.npz): repetition
    penalty, minimum length, EOS, stop sequences and the tokenizer's masking
    give identical tokens and identical result fields."""
    from _native_oracle import Controls
    g = golden("controls.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    spec = Spec(V, d, H, L, T)
    _, flat = quantize_params(oracle, spec, synth_params(oracle, spec, wseed), bits)
    om = oracle.model(spec, flat)
    for i in range(int(g["count"][0])):
        strategy, top_k, min_new = (int(x) for x in g[f"c{i}_params"])
        temperature, top_p, penalty = (float(x) for x in g[f"c{i}_params_f"])
        st, sl = g[f"c{i}_stop_tokens"], g[f"c{i}_stop_lengths"]
        stops, off = [], 0
        for n in sl:
            stops.append(tuple(st[off:off + n]))
            off += n
        c = Controls(penalty=penalty, min_new=min_new, mask_from=int(g["tokenizer_vocab"][0]), stops=stops)
        toks, res, _ = om.generate_ex(g["prompts"], g[f"c{i}_tokens"].shape[1], c, strategy, temperature, top_k,
                                      top_p, g[f"c{i}_seeds"] if strategy else None)
        np.testing.assert_array_equal(toks, g[f"c{i}_tokens"], err_msg=f"case {i}")
        np.testing.assert_array_equal(res, g[f"c{i}_results"], err_msg=f"case {i}")
    om.close()


def masked_golden_cases(g, mi):
    """(ids, padding or None, attention or None, reference logits) of model mi
    in tests/golden/masked.npz."""
    for ci in range(int(g[f"m{mi}_count"][0])):
        ids = g[f"m{mi}_c{ci}_ids"]
        pad, att = g[f"m{mi}_c{ci}_pad"], g[f"m{mi}_c{ci}_att"]
        T = ids.size
        yield (ids, pad if pad.size else None, att.reshape(T, T) if att.size else None,
               g[f"m{mi}_c{ci}_logits"])


@pytest.mark.parametrize("mi", [0, 1])
def test_masked_forward_matches_reference(oracle, mi):
    """or_forward_masked against model_forward_masked of the reference's build
    (tests/golden/masked.npz): plain causal, right / left / scattered
    padding, a custom attention mask with a real query that attends to
    nothing, T = max_seq_len; the default architecture (INT8) and tied + RoPE +
    RMSNorm + SwiGLU (INT4). A padding mask without a real position is
    rejected by both."""
    g = golden("masked.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g[f"m{mi}_spec"])
    spec = Spec(V, d, H, L, T, int(g[f"m{mi}_flags"][0]))
    _, flat = quantize_params(oracle, spec, synth_params(oracle, spec, wseed), bits)
    m = oracle.model(spec, flat)
    for ci, (ids, pad, att, ref) in enumerate(masked_golden_cases(g, mi)):
        got = m.forward_masked(ids, pad, att)
        err = np.abs(got - ref).max() / np.abs(ref).max()
        assert err <= 1e-4, (ci, err)
    assert int(g[f"m{mi}_rejected_rc"][0]) != 0
    assert m.forward_masked(g[f"m{mi}_c0_ids"][:16], np.zeros(16, np.uint8)) is None
    m.close()
