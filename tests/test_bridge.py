"""The reference-side binding of the device path (oracle/dz_bridge.c): the
reference's own generation loop (generation_decode_with_options,
src/cli/generation.c:198-308, unchanged objects) linked with the early branch
of model_forward_token that the integration guide adds, through -Wl,--wrap.

- CPU: with no model attached the wrapped calls reach the reference's code,
  so the bridge library reproduces the reference's golden outputs bit for bit.
- GPU: with the model attached, every decode step of the reference's loop
  runs through dz_cuda_forward_tokens; logits within 1e-3 of the reference's
  and token streams and result fields the reference's (a divergence only at
  a documented near-tie, tests/_margins.py)."""
import os

import numpy as np
import pytest

from conftest import golden
from _margins import check_streams

MASKED = np.array([256, 257, 258, 259], np.uint32)


def _load(bridge, g, tmp_path, name):
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    path = str(tmp_path / f"{name}.bin")
    assert bridge.L.rh_build_bundle(path.encode(), V, d, H, L, T, wseed, bits, 2) == 0
    h = bridge.L.rh_load(path.encode())
    assert h
    return h, path


def _generate(bridge, h, g, with_logits=True):
    prompts = np.ascontiguousarray(g["prompts"], np.uint32)
    n_seq, plen = prompts.shape
    n_new = g["tokens"].shape[1]
    strategy, top_k = (int(x) for x in g["sampling"])
    temperature, top_p = (float(x) for x in g["sampling_f"])
    seeds = np.ascontiguousarray(g["seeds"], np.uint64) if g["seeds"].size else None
    toks = np.empty((n_seq, n_new), np.uint32)
    lg = np.empty((n_seq, n_new, int(g["spec"][0])), np.float32)
    rc = bridge.L.rh_generate(h, prompts.ctypes.data, n_seq, plen, n_new, strategy, temperature, top_k, top_p,
                              seeds.ctypes.data if seeds is not None else None, MASKED.ctypes.data, 4,
                              toks.ctypes.data, lg.ctypes.data)
    assert rc == 0
    return toks, lg


@pytest.mark.parametrize("name", ["c1", "ring"])
def test_bridge_passes_through_without_a_device_model(bridge, tmp_path, name):
    g = golden(f"{name}.npz")
    h, _ = _load(bridge, g, tmp_path, name)
    before = bridge.L.br_device_forwards()
    toks, lg = _generate(bridge, h, g)
    bridge.L.rh_free(h)
    np.testing.assert_array_equal(toks, g["tokens"])
    n = g["logits"].shape[0]
    np.testing.assert_array_equal(lg[:n].view(np.uint32), g["logits"].view(np.uint32))
    assert bridge.L.br_device_forwards() == before


def _masked_rel(a, r):
    a = np.array(a, np.float32, copy=True)
    r = np.array(r, np.float32, copy=True)
    a[..., MASKED] = 0
    r[..., MASKED] = 0
    return np.abs(a - r).max(axis=-1) / np.maximum(np.abs(r).max(axis=-1), 1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["c1", "c2", "ring"])
def test_bridge_runs_the_reference_loop_on_the_device(gpu, bridge, tmp_path, name):
    g = golden(f"{name}.npz")
    h, path = _load(bridge, g, tmp_path, name)
    model = bridge.L.rh_model(h)
    assert bridge.L.br_attach(model, path.encode(), 0) == 0
    before = bridge.L.br_device_forwards()
    toks, lg = _generate(bridge, h, g)
    served = bridge.L.br_device_forwards() - before
    bridge.L.br_detach(model)
    bridge.L.rh_free(h)
    n_seq, n_new = g["tokens"].shape
    plen = g["prompts"].shape[1]
    # every step of every sequence ran on the device (the loop feeds the
    # prompt, then each draw but the last)
    assert served == n_seq * (plen + n_new - 1), served
    n = g["logits"].shape[0]
    # compared up to each sequence's first divergence from the reference
    rel = _masked_rel(lg[:n], g["logits"])
    ok = np.cumprod(toks[:n] == g["tokens"][:n], axis=1).astype(bool)
    ok = np.concatenate([np.ones((n, 1), bool), ok[:, :-1]], axis=1)
    assert rel[ok].max() <= 1e-3, rel[ok].max()
    err = float(np.abs(np.where(ok[..., None], lg[:n] - g["logits"], 0))[..., [i for i in range(lg.shape[-1])
                                                                            if i not in MASKED]].max())
    bad = check_streams(toks, g["tokens"], g["margins"], max(err, 1e-6))
    print(f"{name}: bridged reference loop, {served} device steps, max-rel {rel[ok].max():.2e}, near-ties {bad}")


# ------------------------------------------------ the reference's public API

PROMPT = b"the quick brown fox jumps over"
API_MASKED = [256, 257, 258]   # PAD, UNK, BOS (dranzer_generation_next_greedy, src/api/dranzer.c:374-384)


def _api_load(bridge, path):
    import ctypes
    m, t = ctypes.c_void_p(), ctypes.c_void_p()
    assert bridge.L.dranzer_bundle_load(path.encode(), 0, ctypes.byref(m), ctypes.byref(t), None) == 0
    return m, t


def _api_cache_logits(bridge, m, ids, V):
    import ctypes
    c = ctypes.c_void_p()
    assert bridge.L.dranzer_cache_create(m, 0, ctypes.byref(c)) == 0
    out = np.empty((len(ids), V), np.float32)
    for i, t in enumerate(ids):
        assert bridge.L.dranzer_cache_forward(c, int(t), out[i].ctypes.data, V) == 0
    bridge.L.dranzer_cache_free(c)
    return out


def _api_greedy(bridge, m, t, n):
    import ctypes
    gen = ctypes.c_void_p()
    assert bridge.L.dranzer_generation_create(m, t, 0, ctypes.byref(gen)) == 0
    assert bridge.L.dranzer_generation_reset(gen, PROMPT, len(PROMPT)) == 0
    toks = []
    piece = ctypes.create_string_buffer(64)
    for _ in range(n):
        tid, size = ctypes.c_uint32(), ctypes.c_size_t(64)
        rc = bridge.L.dranzer_generation_next_greedy(gen, ctypes.byref(tid), piece, ctypes.byref(size))
        assert rc in (0, 9), rc   # DRANZER_OK, DRANZER_FINISHED
        toks.append(tid.value)
        if rc == 9:
            break
    bridge.L.dranzer_generation_free(gen)
    return np.array(toks, np.uint32)


def test_bridge_public_api_passes_through(bridge, tmp_path):
    """dranzer_cache_forward over the c1 prompt through the bridge library,
    no device model: the reference's prompt logits bit for bit."""
    g = golden("c1.npz")
    _, path = _load(bridge, g, tmp_path, "c1api")
    m, t = _api_load(bridge, path)
    lg = _api_cache_logits(bridge, m, g["prompts"][0], int(g["spec"][0]))
    np.testing.assert_array_equal(lg.view(np.uint32), g["prompt_logits"].view(np.uint32))
    bridge.L.dranzer_tokenizer_free(t)
    bridge.L.dranzer_model_free(m)


@pytest.mark.gpu
def test_bridge_public_api_on_the_device(gpu, bridge, tmp_path):
    """The public API (src/api/dranzer.c:228-414) on a device-attached model:
    dranzer_cache_forward logits within 1e-3 of the same calls on the CPU,
    and dranzer_generation_reset / _next_greedy giving the CPU's tokens (a
    divergence only where the CPU's top-2 gap is below 10x the observed
    logit error)."""
    g = golden("c1.npz")
    V = int(g["spec"][0])
    _, path = _load(bridge, g, tmp_path, "c1api")
    m, t = _api_load(bridge, path)
    ids = np.concatenate([g["prompts"][0], g["tokens"][0][:16]])
    cpu_lg = _api_cache_logits(bridge, m, ids, V)
    cpu_toks = _api_greedy(bridge, m, t, 24)
    # the CPU's greedy margins along its own stream (BOS, the prompt's bytes,
    # the draws), masked as the API masks
    feed = np.concatenate([[258], np.frombuffer(PROMPT, np.uint8).astype(np.uint32), cpu_toks[:-1]])
    lg = _api_cache_logits(bridge, m, feed, V)[len(PROMPT):]   # the logits each draw was taken from
    lg[:, API_MASKED] = -np.finfo(np.float32).max
    lg[:, 260:] = -np.finfo(np.float32).max                  # ids past the tokenizer's 260
    top2 = np.sort(lg, axis=-1)[:, -2:]
    margins = top2[:, 1] - top2[:, 0]
    assert bridge.L.br_attach_next(path.encode(), 0) == 0
    before = bridge.L.br_device_forwards()
    dev_lg = _api_cache_logits(bridge, m, ids, V)
    assert bridge.L.br_device_forwards() - before == len(ids)
    rel = np.abs(dev_lg - cpu_lg).max(axis=-1) / np.abs(cpu_lg).max(axis=-1)
    assert rel.max() <= 1e-3, rel.max()
    err = float(np.abs(dev_lg - cpu_lg).max())
    dev_toks = _api_greedy(bridge, m, t, 24)
    assert bridge.L.br_device_forwards() - before > len(ids) + len(PROMPT)
    n = min(len(cpu_toks), len(dev_toks))
    diff = np.nonzero(cpu_toks[:n] != dev_toks[:n])[0]
    if diff.size:
        i = int(diff[0])
        assert margins[i] < 10 * err, (i, margins[i], err)
    else:
        assert len(cpu_toks) == len(dev_toks)
    print(f"public API on the device: max-rel {rel.max():.2e}, tokens {dev_toks.tolist()}")
    bridge.L.dranzer_tokenizer_free(t)
    bridge.L.dranzer_model_free(m)
