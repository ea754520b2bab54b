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
import types

import numpy as np
import pytest

from vvli_b200 import sampler as S

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

pytestmark = pytest.mark.gpu

SAMPLE_OPTS = types.SimpleNamespace(temperature=0.8, top_p=0.95, top_k=40, repeat_penalty=1.1, repeat_last_n=64,
                                    seed=None)


def gpu_count():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank_main(rank, world, nccl_id, cfg, blob, prompt, n_new, mega, q):
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        os.environ.setdefault("VVLI_NCCL_TIMEOUT_S", "60")
        os.environ["VVLI_MEGAKERNEL"] = "1" if mega else "0"
        import time
        import vvli_b200
        import vvli_b200._abi
        t0 = time.time()

        def note(what):
            print(f"[rank {rank} +{time.time() - t0:.1f}s] {what}", file=sys.stderr, flush=True)

        r = vvli_b200.Runner(cfg, max_seq=128, device=rank, tp_rank=rank, tp_size=world, nccl_id=nccl_id, max_batch=3)
        r.load_weights(blob)
        used_mega = r.query("megakernel") == 1
        note(f"created, megakernel={used_mega} ({vvli_b200._abi.lib().vvli_cuda_last_error().decode()})")
        logits = [r.forward_token(t, p) for p, t in enumerate(prompt)]
        note("forward_token done")
        # Sampler.next on the last token's logits (gathered from every rank)
        state = np.array([11, 22, 33, 44], dtype=np.uint64)
        stok = r.sample(SAMPLE_OPTS, list(prompt), state)
        note("sample done")
        r.reset()
        tokens, _ = r.generate_greedy(prompt, n_new)
        note("generate done")
        # decode batch under tensor parallelism: three sequences' first tokens
        blogits, bam = r.forward_batch(prompt[:3], [0, 0, 0])
        note("forward_batch done")
        r.close()
        q.put((rank, "ok", np.stack(logits), tokens, used_mega, blogits, bam, (stok, state)))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), None, None, None, None, None, None))


def run_tp(cfg, blob, prompt, n_new, world, mega=True):
    """Runs every rank; with mega, the decode steps are the tensor-parallel megakernel
    (partial sums exchanged over NVLink inside the kernel), else the per-kernel step with NCCL."""
    import vvli_b200
    nccl_id = vvli_b200.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, nccl_id, cfg, blob, prompt, n_new, mega, q), daemon=True)
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, logits, tokens, used_mega, blogits, bam, sampled = q.get(timeout=120)
            results[rank] = (status, logits, tokens, used_mega, blogits, bam, sampled)
    finally:
        for p in procs:  # the ranks this test started, and only those
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    for rank, (status, _, _, used_mega, _, _, _) in results.items():
        assert status == "ok", (rank, status)
        assert used_mega == mega, (rank, used_mega)
    return results


@pytest.mark.skipif(gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mega", [True, False], ids=["megakernel", "per_kernel"])
@pytest.mark.parametrize("name", ["qwen2_tiny", "llama3_tiny_rs"])
def test_tp2_matches_oracle(oracle, name, mega):
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()[name]
    blob = oracle.synthetic_blob(cfg, seed=seed)
    prompt = [5, 17, 99, 201, 3, 64]
    ref = oracle.RefRunner(cfg, blob=blob, max_seq=128)
    ref_logits = np.stack([ref.forward_token(t, p) for p, t in enumerate(prompt)])
    ref.reset()
    ref_tokens = ref.generate_greedy(prompt, 24)
    res = run_tp(cfg, blob, prompt, 24, 2, mega)
    for rank in range(2):
        _, logits, tokens, _, blogits, bam, (stok, state) = res[rank]
        assert np.max(np.abs(logits - ref_logits)) < 1e-4, rank
        assert tokens == ref_tokens, rank
        # the sampled token and the advanced state: as the oracle's Sampler.next
        # on the same (gathered) logits with the same draw
        x = S.Xoshiro256(0)
        x.s = [11, 22, 33, 44]
        u = x.float32()
        assert stok == oracle.sampler_next(logits[-1], prompt, [], SAMPLE_OPTS, u), rank
        assert [int(v) for v in state] == x.s, rank
        assert (stok, list(state)) == (res[0][6][0], list(res[0][6][1])), rank
        # batch rows b: token prompt[b] at position 0 of its own sequence
        for b in range(3):
            ref.reset()
            want = ref.forward_token(prompt[b], 0)
            assert np.max(np.abs(blogits[b] - want)) < 2e-3, (rank, b)
            assert bam[b] == oracle.argmax(want), (rank, b)


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
    _, logits, tokens, _, _, _, _ = res[0]
    assert np.max(np.abs(logits - ref_logits)) < 2e-2
    assert tokens == ref_tokens
