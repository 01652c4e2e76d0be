"""Tensor parallelism: the shard layout (host logic, two gloo ranks on CPU)
and, where two B200s are present, TP=2 generation against one GPU."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from _models import Spec, quantize_params, synth_params


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _shard(dz, rec, rank, world, spec):
    """This rank's piece of one projection record, as the device model cuts it
    (Q/K/V and W1 by columns, W_o and W2 by rows)."""
    name, kind, rows, cols, f32, scales, packed = rec
    D, F = spec.dim, 4 * spec.dim
    if name.endswith(("W_q", "W_k", "W_v")):
        axis, start, count = 1, rank * D // world, D // world
    elif name.endswith("W_ff1"):
        axis, start, count = 1, rank * F // world, F // world
    elif name.endswith("W_o"):
        axis, start, count = 0, rank * D // world, D // world
    elif name.endswith("W_ff2"):
        axis, start, count = 0, rank * F // world, F // world
    else:
        return None
    return axis, dz.quantized_slice(scales, packed, rows, cols, 4, 2, axis, start, count)


def _gloo_rank(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import dranzer_b200 as dz
    from _native_oracle import Oracle
    spec = Spec(300, 64, 4, 2, 16)
    o = Oracle()
    recs, _ = quantize_params(o, spec, synth_params(o, spec, 7), 4)
    ok, checked = True, 0
    for rec in recs:
        name, kind, rows, cols, f32, scales, packed = rec
        sh = _shard(dz, rec, rank, world, spec)
        if sh is None:
            continue
        axis, (s, p) = sh
        r2, c2 = (rows // world, cols) if axis == 0 else (rows, cols // world)
        mine = torch.from_numpy(dz.quantize_unpack(s, p, r2, c2, 4, 2))
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        whole = torch.cat(parts, dim=axis).numpy()
        ok &= bool(np.array_equal(whole, dz.quantize_unpack(scales, packed, rows, cols, 4, 2)))
        checked += 1
    if rank == 0:
        with open(out, "w") as f:
            f.write("ok" if ok and checked == 6 * spec.layers else f"mismatch ({checked} checked)")
    dist.barrier()
    dist.destroy_process_group()


def test_tp_shards_reassemble_on_two_gloo_ranks():
    """Every rank's Q/K/V/W1 columns and W_o/W2 rows, gathered over two gloo
    ranks, are the whole quantized matrices again (INT4, odd shapes per rank)."""
    port = _free_port()
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "r")
        mp.spawn(_gloo_rank, args=(2, port, out), nprocs=2, join=True)
        assert open(out).read() == "ok"


def _gpu_rank(rank, world, port, td, bits):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    import dranzer_b200 as dz
    from _native_oracle import Oracle
    spec = Spec(900, 512, 8, 2, 64)
    o = Oracle()
    recs, _ = quantize_params(o, spec, synth_params(o, spec, 61), bits)
    arrays = [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs]
    uid = [dz.Model.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    model = dz.Model.from_arrays(spec, arrays, device=rank, tp=(rank, world, uid[0]))
    B, T = 6, 20
    prompts = np.random.RandomState(bits).randint(0, 256, size=(B, T)).astype(np.uint32)
    samp = dz.Sampling(dz.GREEDY)
    cache = dz.KVCache(model, B, 64)
    logits = cache.prefill(prompts)
    cache.set_prefill(dz.PREFILL_BATCHED)
    toks = cache.generate(prompts, 10, samp)
    cache.set_prefill(dz.PREFILL_TOKENS)
    toks_t = cache.generate(prompts, 10, samp)
    np.save(os.path.join(td, f"r{rank}.npy"), np.concatenate([logits.ravel(), toks.ravel().astype(np.float32),
                                                              toks_t.ravel().astype(np.float32)]))
    cache.close()
    model.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [8, 4])
def test_tp2_matches_one_gpu(gpu, bits):
    """TP=2 over two B200s (NCCL all-reduce after attention-out and FFN-down)
    gives both ranks the same logits and tokens as the one-GPU model:
    last-prompt logits within 1e-5 relative, identical greedy streams."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from _native_oracle import Oracle
    spec = Spec(900, 512, 8, 2, 64)
    o = Oracle()
    recs, _ = quantize_params(o, spec, synth_params(o, spec, 61), bits)
    model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, bits, 2) for (_, k, r, c, f, s, p) in recs])
    B, T = 6, 20
    prompts = np.random.RandomState(bits).randint(0, 256, size=(B, T)).astype(np.uint32)
    cache = gpu.KVCache(model, B, 64)
    ref_logits = cache.prefill(prompts)
    cache.set_prefill(gpu.PREFILL_BATCHED)
    ref = cache.generate(prompts, 10, gpu.Sampling(gpu.GREEDY))
    cache.close(); model.close()
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_gpu_rank, args=(2, _free_port(), td, bits), nprocs=2, join=True)
        n = ref_logits.size
        for r in range(2):
            a = np.load(os.path.join(td, f"r{r}.npy"))
            lg = a[:n].reshape(ref_logits.shape)
            rel = np.abs(lg - ref_logits).max() / np.abs(ref_logits).max()
            assert rel <= 1e-5, (r, rel)
            np.testing.assert_array_equal(a[n:n + ref.size].reshape(ref.shape), ref.astype(np.float32))
            np.testing.assert_array_equal(a[n + ref.size:].reshape(ref.shape), ref.astype(np.float32))
