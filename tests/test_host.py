"""The product's host library (include/dz_host.h) against the reference's own
outputs: quantizer bit-exactness, bundle writer byte-identity, the
code-retaining loader, and canonical-payload / corruption rejection
(src/tests/core/test_quantize.c, test_model_bundle.c:270-358)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden
from _models import C1, Spec, inventory, quantize_params, synth_params


def test_quantize_pack_bit_exact(dz):
    g = golden("quant.npz")
    for n in range(int(g["count"])):
        r, c, bits, gran = (int(x) for x in g[f"c{n}_meta"])
        w = (g[f"c{n}_w"] if f"c{n}_w" in g.files else g["adv_w"]).reshape(r, c)
        s, p = dz.quantize_pack(w, bits, gran)
        np.testing.assert_array_equal(s.view(np.uint32), g[f"c{n}_s"].view(np.uint32))
        np.testing.assert_array_equal(p, g[f"c{n}_p"])
        deq = dz.quantize_unpack(s, p, r, c, bits, gran)
        assert deq.shape == (r, c)


def test_quantize_dequantize_bit_exact(dz):
    """dz_quantize_dequantize_into against quantize_dequantize_into of the
    reference's build (tests/golden/qdq.npz): every reconstruction bit pattern
    (signed zeros included), the counts exact, the double statistics to 1e-12
    (test_quantize.c:124-140 allows that much between its two call forms)."""
    g = golden("qdq.npz")
    for n in range(int(g["count"][0])):
        gran, bits = (int(x) for x in g[f"q{n}_args"])
        out, e = dz.quantize_dequantize(g[f"q{n}_src"], bits, gran)
        np.testing.assert_array_equal(out.view(np.uint32), g[f"q{n}_dst_bits"], err_msg=f"case {n}")
        assert [e["count"], e["clipped"], e["levels_used"]] == g[f"q{n}_counts"].tolist(), n
        ref = g[f"q{n}_stats"]
        assert np.float32(e["max_abs_error"]) == np.float32(ref[0]), n
        np.testing.assert_allclose([e["rms_error"], e["rms_relative"], e["original_rms"]], ref[1:], rtol=1e-12,
                                   atol=0)
    # the reconstruction is what unpacking the packed codes gives, up to the sign of zero
    x = g["q7_src"]
    for gran in (0, 1, 2):
        for bits in (4, 8):
            out, _ = dz.quantize_dequantize(x, bits, gran)
            s, p = dz.quantize_pack(x, bits, gran)
            np.testing.assert_array_equal(out + np.float32(0), dz.quantize_unpack(s, p, *x.shape, bits, gran))
    with pytest.raises(ValueError):
        dz.quantize_dequantize(x, 1, 2)
    with pytest.raises(ValueError):
        dz.quantize_dequantize(x, 8, 3)


@pytest.mark.parametrize("N", [4096, 11008, 32000])
def test_c3_weights_bit_exact(dz, N):
    """Full-size C3 matrices (K=4096), generator and quantizer of the product."""
    g = golden("quant.npz")
    st = np.array([dz.rng_stream(3, dz.STREAM_TESTING)], np.uint64)
    dz.synth_gaussian(st, 512 * 4096, 1.0)
    w = dz.synth_gaussian(st, 4096 * N, 0.02).reshape(4096, N)
    for n_, bits, hs, hp in g["c3_hashes"]:
        if int(n_) != N:
            continue
        s, p = dz.quantize_pack(w, int(bits), dz.GRAN_COLUMN)
        assert dz.fnv1a(s) == hs and dz.fnv1a(p) == hp


def test_unpack_matches_oracle_and_rejects(dz, oracle):
    rng = np.random.RandomState(5)
    for bits in (2, 3, 4, 5, 8, 12, 16):
        for gran in (0, 1, 2):
            w = (rng.randn(13, 29) * 0.3).astype(np.float32)
            s, p = dz.quantize_pack(w, bits, gran)
            a = dz.quantize_unpack(s, p, 13, 29, bits, gran)
            rc, b = oracle.quantize_unpack(s, p, 13, 29, bits, gran)
            assert rc == 0
            np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
            ones = (1 << min(bits, 8)) - 1
            bad = p.copy()
            if bits <= 8:
                bad[0] = np.uint8((int(bad[0]) & ~ones & 0xFF) | ones)
                with pytest.raises(ValueError):
                    dz.quantize_unpack(s, bad, 13, 29, bits, gran)
            if (13 * 29 * bits) % 8:
                pad = p.copy()
                pad[-1] = np.uint8(int(pad[-1]) | 0x80)
                with pytest.raises(ValueError):
                    dz.quantize_unpack(s, pad, 13, 29, bits, gran)


def test_quantize_rejects_bad_arguments(dz):
    w = np.ones((3, 5), np.float32)
    with pytest.raises(ValueError):
        dz.quantize_pack(w, 1, 2)
    with pytest.raises(ValueError):
        dz.quantize_pack(w, 17, 2)
    with pytest.raises(ValueError):
        dz.quantize_pack(w, 8, 3)
    w[1, 1] = np.inf
    with pytest.raises(ValueError):
        dz.quantize_pack(w, 8, 2)
    with pytest.raises(ValueError):
        dz.quantized_scale_count(0, 5, 2)


def test_positional_encoding_matches_reference(dz):
    pe = dz.positional_encoding(64, 128)
    assert np.abs(pe - golden("pe.npz")["pe_64x128"]).max() <= 1.2e-7


def _flat_params(oracle, spec, seed):
    return np.concatenate([t.ravel() for t in synth_params(oracle, spec, seed)])


@pytest.mark.parametrize("name", ["c1", "c2", "ring", "arch23", "arch8", "arch6"])
def test_bundle_writer_byte_identical(dz, oracle, tmp_path, name):
    """dz_bundle_save_quantized writes the reference writer's exact bytes (v2,
    and v3 with the architecture bits for archNN)."""
    g = golden(f"{name}.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    flags = int(g["architecture_flags"][0]) if "architecture_flags" in g.files else 0
    spec = Spec(V, d, H, L, T, flags)
    params = _flat_params(oracle, spec, wseed)
    path = str(tmp_path / "b.bin")
    dz.save_quantized_bundle(path, spec, params, bits, dz.GRAN_COLUMN, train_window=T, seed=wseed)
    blob = np.fromfile(path, np.uint8)
    assert blob.size == int(g["bundle_size"][0])
    assert dz.fnv1a(blob) == int(g["bundle_fnv"][0])


@pytest.mark.parametrize("bits", [4, 8])
def test_loader_retains_reference_codes(dz, oracle, bits):
    """A reference-written bundle opens with its codes and scales retained; they
    equal the oracle's quantization of the same synthetic weights."""
    path = os.path.join(GOLDEN, f"bundle_small_int{bits}.bin")
    b = dz.Bundle(path)
    spec = Spec(300, 16, 2, 2, 8)
    assert (b.desc.vocab_size, b.desc.embedding_dim, b.desc.num_heads, b.desc.num_layers,
            b.desc.max_seq_len) == (300, 16, 2, 2, 8)
    assert b.info.format_version == 2 and b.info.bits == bits and b.info.granularity == 2
    tensors = synth_params(oracle, spec, 9)
    for i, ((name, r, c, kind), t) in enumerate(zip(inventory(spec), tensors)):
        k, rr, cc, f32, scales, packed = b.tensor(i)
        assert (k, rr, cc) == (kind, r, c)
        if kind == 0:
            s_ref, p_ref = oracle.quantize_pack(t, bits, 2)
            np.testing.assert_array_equal(scales.view(np.uint32), s_ref.view(np.uint32))
            np.testing.assert_array_equal(packed, p_ref)
        else:
            np.testing.assert_array_equal(f32, t)
    b.close()


def test_loader_rejects_corruption(dz, tmp_path):
    """Checksum, truncation, trailing-byte and forged-shape rejection
    (src/tests/core/test_model_bundle.c:338-358)."""
    src = np.fromfile(os.path.join(GOLDEN, "bundle_small_int4.bin"), np.uint8)

    def opened(blob):
        p = str(tmp_path / "x.bin")
        blob.tofile(p)
        try:
            dz.Bundle(p).close()
            return 0
        except dz.DzError as e:
            return e.status

    assert opened(src) == 0
    flip = src.copy(); flip[300] ^= 1                  # weight payload bit
    assert opened(flip) == -4
    hdr = src.copy(); hdr[30] ^= 1                     # header field (vocab)
    assert opened(hdr) == -4
    tok = src.copy(); tok[-20] ^= 1                    # tokenizer payload
    assert opened(tok) == -4
    assert opened(src[:-1]) == -3                      # truncated
    assert opened(np.concatenate([src, np.zeros(1, np.uint8)])) == -3
    magic = src.copy(); magic[0] = ord("X")
    assert opened(magic) == -9
    code = src.copy()                                   # a non-canonical code (15) with a valid checksum
    code[184 + 32 + 300 * 4 + 0] |= 0x0F               # first packed byte of output_projection... re-sum
    assert opened(code) in (-3, -4)


@pytest.mark.parametrize("flags", [0, 1, 4, 16, 23, 8, 22])
def test_model_layout_matches_reference_inventory(dz, flags):
    spec = Spec(512, 128, 4, 4, 64, flags)
    lay = dz.model_tensor_layout(spec)
    assert lay == [(k, r, c) for (_, r, c, k) in inventory(spec)]


def test_layout_rejects_unsupported_architectures(dz):
    # unknown bits, and GELU with SwiGLU (src/core/bundle.c:142-144)
    for flags in (32, 8 | 16):
        assert dz.model_tensor_layout(Spec(512, 128, 4, 1, 64, flags)) == []


@pytest.mark.parametrize("bits", [8, 4, 3])
@pytest.mark.parametrize("gran", [0, 1, 2])
def test_quantized_slice_equals_quantizing_the_slice(dz, bits, gran):
    """A column slice of a COLUMN-quantized matrix (row slice of ROW-quantized)
    is bit-identical to quantizing that slice of the float matrix; every slice
    unpacks to the same values as the whole; odd INT4 counts keep a zero pad."""
    rng = np.random.RandomState(bits * 3 + gran)
    rows, cols = 37, 53
    w = (rng.randn(rows, cols) * 0.05).astype(np.float32)
    s, p = dz.quantize_pack(w, bits, gran)
    full = dz.quantize_unpack(s, p, rows, cols, bits, gran)
    for axis, start, count in ((1, 10, 17), (0, 5, 31), (1, 0, cols), (0, 36, 1), (1, 52, 1)):
        so, po = dz.quantized_slice(s, p, rows, cols, bits, gran, axis, start, count)
        r2, c2 = (count, cols) if axis == 0 else (rows, count)
        part = dz.quantize_unpack(so, po, r2, c2, bits, gran)
        ref = full[start:start + count] if axis == 0 else full[:, start:start + count]
        np.testing.assert_array_equal(part, ref)
        if (gran == 2 and axis == 1) or (gran == 1 and axis == 0):
            ws = w[start:start + count] if axis == 0 else w[:, start:start + count]
            s2, p2 = dz.quantize_pack(np.ascontiguousarray(ws), bits, gran)
            np.testing.assert_array_equal(so.view(np.uint32), s2.view(np.uint32))
            np.testing.assert_array_equal(po, p2)
    with pytest.raises(ValueError):
        dz.quantized_slice(s, p, rows, cols, bits, gran, 1, 50, 10)


def test_synth_gaussian_in_parallel_pieces_is_one_sequential_pass(dz, oracle):
    """dz_synth_gaussian cuts long fills into pieces started from jumped RNG
    states; values and final state equal the oracle's sequential pass and a
    fill split across two calls."""
    from _native_oracle import STREAM_TESTING
    n = 3 * (1 << 22) + 77
    s1 = np.array([oracle.rng_stream(9, STREAM_TESTING)], np.uint64)
    s2, s3 = s1.copy(), s1.copy()
    a = oracle.gaussian(s1, n, 0.02)
    b = dz.synth_gaussian(s2, n, 0.02)
    c = np.concatenate([dz.synth_gaussian(s3, 10, 0.02), dz.synth_gaussian(s3, n - 10, 0.02)])
    assert np.array_equal(a, b) and np.array_equal(a, c)
    assert s1[0] == s2[0] == s3[0]
