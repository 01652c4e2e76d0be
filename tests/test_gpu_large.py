"""Parity at the sizes the path is measured on.

- The config-4 model itself (24 layers, d 2048, 16 heads, F 8192, V 32000,
  INT8, weights seed 4): the first two of its 512-token prompts through the
  batched prefill, then 8 greedy steps, against logits and tokens of the
  reference's own build (tests/golden/c4s.npz, from
  src/core/transformer.c:755-858 via model_forward_token and
  src/cli/sampling.c:38-53). W_ff2 has K = 8192.
- One layer at the config-5 width (d 6144, 48 heads of 128, F 24576, INT4,
  weights seed 5), against the oracle's layer math (the reference's decode
  step restated, oracle/dz_oracle.c): the full-model config 5 does not fit the
  host oracle, so it is pinned per layer. W_ff2 has K = 24576. On two GPUs the
  same layer also runs tensor-parallel (heads and FFN columns split, NCCL
  all-reduce after attention-out and FFN-down).

Logits: max |g - r| / max |r| <= 1e-3 at every compared position. Tokens:
identical, or a first divergence where the reference's decision margin is
below 10x the observed logit error (tests/_margins.py)."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import golden
from _margins import check_streams, stream_margins
from _models import Spec, quantize_params, synth_params

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-3
MASKED = [256, 257, 258, 259]


def _unmask(x):
    x = np.array(x, np.float32, copy=True)
    x[..., MASKED] = 0
    return x


def _rel(a, r):
    a, r = _unmask(a), _unmask(r)
    return np.abs(a - r).max(axis=-1) / np.maximum(np.abs(r).max(axis=-1), 1e-6)


def _abs(a, r):
    return float(np.abs(_unmask(a) - _unmask(r)).max())


# ------------------------------------------------------------------ config 4

@pytest.fixture(scope="module")
def c4(gpu, tmp_path_factory):
    from dranzer_b200 import workloads as W
    g = golden("c4s.npz")
    V, d, H, L, T, wseed, bits = (int(x) for x in g["spec"])
    spec = W.Spec(V, d, H, L, T)
    path = str(tmp_path_factory.mktemp("c4") / "c4.bin")
    gpu.save_quantized_bundle(path, spec, W.model_params(spec, wseed), bits, gpu.GRAN_COLUMN, train_window=T,
                              seed=wseed)
    # the same bytes the reference's writer produced: same weights, codes and scales
    assert os.path.getsize(path) == int(g["bundle_size"][0])
    assert gpu.fnv1a(np.fromfile(path, np.uint8)) == int(g["bundle_fnv"][0])
    bundle = gpu.Bundle(path)
    model = gpu.Model.from_bundle(bundle)
    yield g, model
    model.close()
    bundle.close()


def test_c4_sample_logits_and_greedy_stream(gpu, c4):
    """Two 512-token prompts of the config-4 workload: the last prompt
    position's logits from the batched prefill and the logits of each of the
    next 7 positions (fed the reference's tokens) within 1e-3 of the
    reference's; the greedy streams of dz_cuda_generate equal the reference's
    except at documented near-ties."""
    g, model = c4
    prompts, ref_tok, ref_lg = g["prompts"], g["tokens"], g["logits"]
    B, n_new = ref_tok.shape
    cache = gpu.KVCache(model, B, 640)
    rel, err = [], 0.0
    out = cache.prefill(prompts)
    for i in range(n_new):
        if i:
            out = cache.forward_tokens(ref_tok[:, i - 1])
        rel.append(_rel(out, ref_lg[:, i]).max())
        err = max(err, _abs(out, ref_lg[:, i]))
    print(f"c4 sample: max-rel per position {np.array(rel)}; max abs {err:.3g}")
    assert max(rel) <= LOGIT_TOL, rel
    toks = cache.generate(prompts, n_new, gpu.Sampling(gpu.GREEDY))
    check_streams(toks, ref_tok, g["margins"], err)
    cache.close()


# ------------------------------------------------------------- config-5 width

C5W = Spec(1024, 6144, 48, 1, 64)
C5W_BITS = 4


@pytest.fixture(scope="module")
def c5w(oracle):
    tensors = synth_params(oracle, C5W, 5)
    recs, flat = quantize_params(oracle, C5W, tensors, C5W_BITS)
    om = oracle.model(C5W, flat)
    rng = np.random.RandomState(5)
    prompts = rng.randint(0, 1024, size=(2, 6)).astype(np.uint32)
    nxt = rng.randint(0, 256, size=(3, 2)).astype(np.uint32)
    # oracle logits: last prompt position, then three fed tokens
    ref = np.zeros((2, 4, C5W.vocab), np.float32)
    for b in range(2):
        om.reset()
        for t in range(prompts.shape[1]):
            r = om.forward_token(prompts[b, t])
        ref[b, 0] = r
        for i in range(3):
            ref[b, i + 1] = om.forward_token(nxt[i, b])
    gtok, glg = om.generate(prompts, 4, want_logits=True)
    margins = stream_margins(glg, gtok, 0)
    params = np.concatenate([t.ravel() for t in tensors])
    yield recs, params, prompts, nxt, ref, gtok, margins
    om.close()


def _c5w_run(gpu, model, prompts, nxt, mode):
    cache = gpu.KVCache(model, 2, 64)
    cache.set_prefill(mode)
    if mode == gpu.PREFILL_BATCHED:
        first = cache.prefill(prompts)
    else:
        for t in range(prompts.shape[1]):
            first = cache.forward_tokens(prompts[:, t])
    out = [first] + [cache.forward_tokens(nxt[i]) for i in range(nxt.shape[0])]
    toks = cache.generate(prompts, 4, gpu.Sampling(gpu.GREEDY))
    cache.close()
    return np.stack(out, 1), toks


@pytest.mark.parametrize("mode", ["tokens", "batched"])
def test_c5_width_layer_matches_oracle(gpu, c5w, mode):
    """d 6144, 48 heads, F 24576 (W_ff2 K = 24576), INT4: the decode step
    and the batched prefill against the oracle's layer math on one GPU."""
    recs, params, prompts, nxt, ref, gtok, margins = c5w
    model = gpu.Model.from_arrays(C5W, [(k, r, c, f, s, p, C5W_BITS, 2) for (_, k, r, c, f, s, p) in recs])
    m = {"tokens": gpu.PREFILL_TOKENS, "batched": gpu.PREFILL_BATCHED}[mode]
    got, toks = _c5w_run(gpu, model, prompts, nxt, m)
    model.close()
    rel = _rel(got, ref)
    print(f"c5 width ({mode} prefill): max-rel per position {rel.max(axis=0)}")
    assert rel.max() <= LOGIT_TOL, rel
    check_streams(toks, gtok, margins, _abs(got, ref))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_rank(rank, world, port, td):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    import dranzer_b200 as dz
    uid = [dz.Model.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    bundle = dz.Bundle(os.path.join(td, "c5w.bin"))
    model = dz.Model.from_bundle(bundle, device=rank, tp=(rank, world, uid[0]))
    data = np.load(os.path.join(td, "inputs.npz"))
    got, toks = _c5w_run(dz, model, data["prompts"], data["nxt"], dz.PREFILL_BATCHED)
    np.savez(os.path.join(td, f"r{rank}.npz"), logits=got, tokens=toks)
    model.close()
    bundle.close()
    dist.barrier()
    dist.destroy_process_group()


def test_c5_width_layer_tp2_matches_oracle(gpu, c5w):
    """The same layer tensor-parallel over two GPUs (24 heads and 12288 FFN
    columns per rank): every rank's logits within 1e-3 of the oracle's and its
    greedy stream the oracle's."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    recs, params, prompts, nxt, ref, gtok, margins = c5w
    with tempfile.TemporaryDirectory() as td:
        gpu.save_quantized_bundle(os.path.join(td, "c5w.bin"), C5W, params, C5W_BITS, gpu.GRAN_COLUMN, seed=5)
        np.savez(os.path.join(td, "inputs.npz"), prompts=prompts, nxt=nxt)
        mp.spawn(_tp_rank, args=(2, _free_port(), td), nprocs=2, join=True)
        for r in range(2):
            d = np.load(os.path.join(td, f"r{r}.npz"))
            rel = _rel(d["logits"], ref)
            assert rel.max() <= LOGIT_TOL, (r, rel)
            check_streams(d["tokens"], gtok, margins, _abs(d["logits"], ref))
