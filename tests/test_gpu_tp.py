"""Tensor-parallel parity on 2+ GPUs: every rank runs its shard through the C ABI.

Ranks are child processes (spawn), one per GPU, sharing an NCCL id made by the
parent.  q/k/v and gate/up are split by heads / rows, o_proj and down_proj
by columns with an NCCL all-reduce after each, the LM head by vocabulary
with a gathered argmax.  Rank 0's logits and greedy stream must match the
oracle like the single-GPU path does.
"""

import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

pytestmark = pytest.mark.gpu


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank_main(rank, world, nccl_id, cfg, blob, prompt, n_new, q):
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        os.environ.setdefault("VVLI_NCCL_TIMEOUT_S", "60")
        import vvli_b200
        r = vvli_b200.Runner(cfg, max_seq=128, device=rank, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
        r.load_weights(blob)
        logits = [r.forward_token(t, p) for p, t in enumerate(prompt)]
        r.reset()
        tokens, _ = r.generate_greedy(prompt, n_new)
        r.close()
        q.put((rank, "ok", np.stack(logits), tokens))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), None, None))


def run_tp(cfg, blob, prompt, n_new, world):
    import vvli_b200
    nccl_id = vvli_b200.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, nccl_id, cfg, blob, prompt, n_new, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, logits, tokens = q.get(timeout=300)
        results[rank] = (status, logits, tokens)
    for p in procs:
        p.join(timeout=60)
    for rank, (status, _, _) in results.items():
        assert status == "ok", (rank, status)
    return results


@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["qwen2_tiny", "llama3_tiny_rs"])
def test_tp2_matches_oracle(oracle, name):
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()[name]
    blob = oracle.synthetic_blob(cfg, seed=seed)
    prompt = [5, 17, 99, 201, 3, 64]
    ref = oracle.RefRunner(cfg, blob=blob, max_seq=128)
    ref_logits = np.stack([ref.forward_token(t, p) for p, t in enumerate(prompt)])
    ref.reset()
    ref_tokens = ref.generate_greedy(prompt, 24)
    res = run_tp(cfg, blob, prompt, 24, 2)
    for rank in range(2):
        _, logits, tokens = res[rank]
        assert np.max(np.abs(logits - ref_logits)) < 1e-4, rank
        assert tokens == ref_tokens, rank


@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
def test_tp2_llama3_2_1b_architecture(oracle):
    from vvli_b200 import config as C
    cfg = C.llama3_2_1b()
    ref = oracle.RefRunner(cfg, synthetic_seed=0, max_seq=128)
    blob = np.array(ref.blob_view())
    prompt = [11, 2222, 33333, 4444, 55]
    ref_logits = np.stack([ref.forward_token(t, p) for p, t in enumerate(prompt)])
    ref.reset()
    ref_tokens = ref.generate_greedy(prompt, 16)
    res = run_tp(cfg, blob, prompt, 16, 2)
    _, logits, tokens = res[0]
    assert np.max(np.abs(logits - ref_logits)) < 2e-2
    assert tokens == ref_tokens
