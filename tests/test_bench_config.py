"""bench.py's reference arm carries its own copy of the workload table (it
loads nothing of dranzer_b200); it must describe the same jobs as
dranzer_b200/workloads.py, which the device arm uses."""
import importlib.util
import os

from conftest import ROOT


def _bench():
    spec = importlib.util.spec_from_file_location("dz_bench", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_reference_table_matches_workloads(dz):
    from dranzer_b200 import workloads as W
    b = _bench()
    assert set(b.REF_WORKLOADS) == set(W.WORKLOADS)
    for key, wl in W.WORKLOADS.items():
        r = b.REF_WORKLOADS[key]
        s = wl.spec
        assert (r["name"], r["vocab"], r["dim"], r["heads"], r["layers"], r["max_seq"]) == \
            (wl.name, s.vocab, s.dim, s.heads, s.layers, s.max_seq), key
        assert (r["bits"], r["weight_seed"], r["prompt_seed"], r["batch"], r["prompt_len"], r["n_new"]) == \
            (wl.bits, wl.weight_seed, wl.prompt_seed, wl.batch, wl.prompt_len, wl.n_new), key
        assert (r["strategy"], r["temperature"], r["top_k"], r["top_p"], r["seed_base"]) == \
            (wl.strategy, wl.temperature, wl.top_k, wl.top_p, wl.seed_base), key
        assert r["cpu_sample"] == wl.cpu_sample, key
    assert b.MASKED == W.MASKED


def test_shards_cover_the_job_once():
    b = _bench()
    for n in (1, 7, 64, 256):
        for world in (1, 2, 3, 4, 8):
            parts = [b.shard(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1


def test_reference_prompts_are_the_device_prompts(dz, ref):
    """The reference arm draws its prompts with the reference build's RNG;
    they are the ids the device arm's workload generator draws."""
    from dranzer_b200 import workloads as W
    b = _bench()
    for key in ("c2", "c4"):
        w = b.REF_WORKLOADS[key]
        got = b.ref_prompts(w, 3, w["prompt_len"])
        assert (got == W.prompts(W.WORKLOADS[key], 0, 3)).all(), key
