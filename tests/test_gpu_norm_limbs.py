"""The norm fused with the next product's activation split
(dz_layernorm_limbs_kernel): with it (the default) and without it
(DZ_NORM_LIMBS=0) a batched prefill and three greedy decode steps give the
same logits bit for bit. The norm's output, the limbs and the row shifts are
the same numbers; only who writes the limbs differs.

Each setting runs in a fresh process (the switch is read once per process).
The model is wide enough (d 1024, V 1100) and the batch large enough
(24 sequences, 40 prompt tokens) that the QKV, W_ff1 and head products run on
the tensor-core GEMM in the prefill and in the decode steps."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))

SCRIPT = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[2])
import dranzer_b200 as gpu
from _models import Spec, quantize_params
from _native_oracle import Oracle
from test_gpu_arch import _perturbed
oracle = Oracle()
spec = Spec(1100, 1024, 8, 2, 96)
recs, _ = quantize_params(oracle, spec, _perturbed(oracle, spec, 41), 8)
model = gpu.Model.from_arrays(spec, [(k, r, c, f, s, p, 8, 2) for (_, k, r, c, f, s, p) in recs])
B, T = 24, 40
ids = np.random.RandomState(2).randint(0, 1100, size=(B, T)).astype(np.uint32)
cache = gpu.KVCache(model, B)
cache.set_prefill(gpu.PREFILL_BATCHED)
outs = [cache.prefill(ids)]
tok = outs[0].argmax(axis=1).astype(np.uint32)
for _ in range(3):
    lg = cache.forward_tokens(tok)
    outs.append(lg)
    tok = lg.argmax(axis=1).astype(np.uint32)
np.save(sys.argv[3], np.stack(outs))
cache.close()
model.close()
"""


def _run(tmp_path, name, fused):
    env = dict(os.environ)
    if fused:
        env.pop("DZ_NORM_LIMBS", None)
    else:
        env["DZ_NORM_LIMBS"] = "0"
    out = str(tmp_path / f"{name}.npy")
    subprocess.run([sys.executable, "-c", SCRIPT, HERE, os.path.dirname(HERE), out], env=env, check=True,
                   timeout=600)
    return np.load(out)


def test_norm_limbs_bit_identical(gpu, tmp_path):
    fused = _run(tmp_path, "fused", True)
    plain = _run(tmp_path, "plain", False)
    assert fused.shape == (4, 24, 1100) and np.isfinite(fused).all()
    np.testing.assert_array_equal(fused, plain)
