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
