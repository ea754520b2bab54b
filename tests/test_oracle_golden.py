"""Pins the oracle's full forward against transformers fp32 golden fixtures.

The fixtures (tests/golden/*.npz, made by tests/golden/make_golden.py) hold a
causal transformers forward of the same seeded bf16 weights.  The oracle
runs the prompt token by token, as the reference's prefill loop does
(src/generator.zig:243-251), and must agree layer by layer.
"""

import hashlib
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from make_golden import fixture_configs  # noqa: E402

# fp32 vs fp32 with different summation orders and libm vs torch transcendentals.
REL_L2_TOL = 2e-5
LOGIT_ABS_TOL = 2e-5


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", sorted(fixture_configs()))
def test_oracle_matches_transformers(oracle, name):
    cfg, seed = fixture_configs()[name]
    fx = np.load(os.path.join(HERE, "golden", f"{name}.npz"))
    blob = oracle.synthetic_blob(cfg, seed=int(fx["seed"]))
    assert hashlib.sha256(blob.tobytes()).digest() == fx["blob_sha256"].tobytes(), "generator changed"
    r = oracle.RefRunner(cfg, blob=blob, max_seq=64, threads=2)
    for pos, tok in enumerate(fx["tokens"]):
        logits = r.forward_token(int(tok), pos)
        for layer in range(cfg.num_hidden_layers):
            err = rel_l2(r.hidden(layer), fx["hidden"][layer, pos])
            assert err < REL_L2_TOL, (pos, layer, err)
        assert np.max(np.abs(logits - fx["logits"][pos])) < LOGIT_ABS_TOL, pos
        assert oracle.argmax(logits) == int(np.argmax(fx["logits"][pos]))


def test_oracle_without_rope_scaling_differs_from_llama3_fixture(oracle):
    # The llama fixture really exercises the llama3 frequency rule.
    cfg, seed = fixture_configs()["llama3_tiny_rs"]
    fx = np.load(os.path.join(HERE, "golden", "llama3_tiny_rs.npz"))
    cfg.rope_scaling_type = 0
    r = oracle.RefRunner(cfg, blob=oracle.synthetic_blob(cfg, seed=int(fx["seed"])), max_seq=64)
    worst = 0.0
    for pos, tok in enumerate(fx["tokens"][:8]):
        logits = r.forward_token(int(tok), pos)
        worst = max(worst, float(np.max(np.abs(logits - fx["logits"][pos]))))
    assert worst > 1e-4
