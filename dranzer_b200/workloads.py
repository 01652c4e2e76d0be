"""The synthetic workloads the path is measured on, and their inputs.

Weights: N(0, 0.02) for embeddings and projections drawn in the
model_param_tensors() order (src/core/model_params.c:39-103) from
dz_rng_stream(weight_seed, TESTING), one value per two unit draws through
Box-Muller; LayerNorm gamma 1, beta 0, biases 0. Prompt ids are uniform over
[0, V) minus {256, 257, 258, 259} (rng_next % V with rejection) from
dz_rng_stream(prompt_seed, TESTING). No BOS is prepended. Control ids
256-258 and EOS 259 are masked before every draw (EOS through a minimum
length equal to the decode length), so every sequence decodes exactly n_new
tokens. The reference names no dataset; these synthetic inputs are the whole
workload.
"""
from dataclasses import dataclass, field

import numpy as np

import dranzer_b200 as dz

MASKED = (256, 257, 258, 259)


@dataclass(frozen=True)
class Spec:
    vocab: int
    dim: int
    heads: int
    layers: int
    max_seq: int
    architecture_flags: int = 0


@dataclass(frozen=True)
class Workload:
    name: str
    spec: Spec
    bits: int
    weight_seed: int
    prompt_seed: int
    batch: int             # sequences of the whole job (split over the GPUs)
    prompt_len: int
    n_new: int
    strategy: int = dz.GREEDY
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 0.0
    seed_base: int = 0     # per-sequence sampling seed = seed_base + global sequence index
    capacity: int = 0      # KV ring capacity per sequence (0: the model's max_seq)
    # CPU baseline sample: (sequences, prompt_len, n_new, all_threads_in_one_session); None = the whole job
    cpu_sample: tuple = None
    notes: str = field(default="", compare=False)

    def sampling(self):
        return dz.Sampling(self.strategy, self.temperature, self.top_k, self.top_p, MASKED)


# config 1: INT8 greedy, batch 1, 16-token prompt + 48 decode
C1 = Workload("c1-int8-greedy-b1-16+48", Spec(512, 128, 4, 4, 64), 8, 0, 1, 1, 16, 48)
# config 2: INT4, 64 prompts x (32 + 32), top-p 0.9 at temperature 0.8 (the
# CLI default, src/cli/cli.c:70), per-sequence seed 2*1000 + i
C2 = Workload("c2-int4-topp0.9-64x(32+32)", Spec(512, 128, 4, 4, 64), 4, 0, 2, 64, 32, 32,
              dz.TOPP, 0.8, 0, 0.9, 2000)
# config 4: the scaled architecture (24 layers, d 2048, 16 heads, F 8192, V
# 32000, context 2048), INT8, weights seed 4; 256 prompts of 512 tokens
# (seed 4) prefilled, then 128 greedy steps; the ring holds the 640 tokens a
# sequence uses. The CPU baseline times one sequence of 16 + 4 tokens (the
# job's 4:1 prompt-to-decode ratio) with every host thread in the
# reference's OpenMP matmul.
C4 = Workload("c4-int8-greedy-256x(512+128)", Spec(32000, 2048, 16, 24, 2048), 8, 4, 4, 256, 512, 128,
              capacity=640, cpu_sample=(1, 16, 4, True))
WORKLOADS = {"c1": C1, "c2": C2, "c4": C4}


def model_params(spec, seed):
    """Flat float32 parameters in the reference's layout (src/core/model.c:38-67,213-228)."""
    state = np.array([dz.rng_stream(seed, dz.STREAM_TESTING)], np.uint64)
    parts = []
    for kind, rows, cols in dz.model_tensor_layout(spec):
        if kind in (dz.KIND_PROJECTION, dz.KIND_EMBEDDING):
            parts.append(dz.synth_gaussian(state, rows * cols, 0.02))
        else:
            parts.append(np.zeros(rows * cols, np.float32))
    # LayerNorm gammas: the first of each NORM pair in every layer
    flat = np.concatenate(parts)
    off = 0
    norm_seen = 0
    for kind, rows, cols in dz.model_tensor_layout(spec):
        if kind == dz.KIND_NORM:
            if norm_seen % 2 == 0:
                flat[off:off + rows * cols] = 1.0
            norm_seen += 1
        off += rows * cols
    return flat


def prompts(wl, lo=0, hi=None):
    """[hi - lo, prompt_len] ids of the job's sequences lo..hi-1 (sequence i
    takes ids [i * prompt_len, (i + 1) * prompt_len) of one stream)."""
    hi = wl.batch if hi is None else hi
    state = np.array([dz.rng_stream(wl.prompt_seed, dz.STREAM_TESTING)], np.uint64)
    ids = dz.synth_prompt_ids(state, hi * wl.prompt_len, wl.spec.vocab, MASKED)
    return ids[lo * wl.prompt_len:].reshape(hi - lo, wl.prompt_len)


def seeds(wl, lo=0, hi=None):
    """Per-sequence sampling seeds of the job's sequences lo..hi-1."""
    hi = wl.batch if hi is None else hi
    return np.array([wl.seed_base + i for i in range(lo, hi)], np.uint64)


def shard(n_items, rank, world):
    """Contiguous share of n_items for `rank` of `world` (balanced, no gaps)."""
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def write_bundle(wl, path):
    dz.save_quantized_bundle(path, wl.spec, model_params(wl.spec, wl.weight_seed), wl.bits,
                             dz.GRAN_COLUMN, train_window=wl.spec.max_seq, seed=wl.weight_seed)
    return path
