"""Tensor-parallel decomposition on CPU: 2 gloo ranks, no GPU.

Each rank slices the host weight blob with the runtime's own shard plan
(vvli_cuda_tp_plan: the same code that fills each GPU's weights), runs a
numpy forward of its shard -- local q/k/v heads and gate/up rows, column
partials of o_proj and down_proj summed with a gloo all_reduce, a vocabulary
shard of the LM head gathered with all_gather -- and rank 0 compares the
logits with the single-process oracle.
"""

import ctypes
import os
import socket
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))


def tp_plan(cfg, rank, world):
    from vvli_b200 import _abi
    c = cfg.to_c()
    n = ctypes.c_uint64(0)
    assert _abi.lib().vvli_cuda_tp_plan(ctypes.byref(c), rank, world, None, 0, ctypes.byref(n)) == 0
    out = np.zeros((n.value, 9), dtype=np.uint64)
    assert _abi.lib().vvli_cuda_tp_plan(ctypes.byref(c), rank, world,
                                        out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), n.value,
                                        ctypes.byref(n)) == 0
    return out


def shards(cfg, blob, plan):
    """{tensor_id: [pieces as float32 arrays]} sliced from the blob by the plan."""
    from vvli_b200.weights import bf16_to_f32
    got = {}
    for dst, tid, src, rows, cols, ld, r0, c0, kind in (tuple(int(v) for v in row) for row in plan):
        full = blob[src: src + (r0 + rows) * ld].reshape(-1, ld) if rows > 1 else blob[src: src + c0 + cols][None]
        piece = full[r0: r0 + rows, c0: c0 + cols] if rows > 1 else full[:, c0: c0 + cols]
        got.setdefault(tid, []).append(bf16_to_f32(np.ascontiguousarray(piece)).reshape(rows, cols))
    return got


def rms(x, w, eps):
    ss = np.float32(np.sum(x.astype(np.float32) ** 2, dtype=np.float32))
    return x * w * np.float32(1.0 / np.sqrt(ss / np.float32(x.size) + np.float32(eps)))


def rank_forward(rank, world, port, cfg, seed, prompt, q):
    import torch
    import torch.distributed as dist
    import oracle
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        blob = oracle.synthetic_blob(cfg, seed=seed)
        W = shards(cfg, blob, tp_plan(cfg, rank, world))
        L, h, d = cfg.num_hidden_layers, cfg.hidden_size, cfg.head_dim()
        nq_l, nkv_l = cfg.num_attention_heads // world, cfg.num_key_value_heads // world
        group = cfg.kv_group_size()
        emb = W[0][0]
        lm = W[2 + 12 * L][0] if not cfg.tie_word_embeddings else (emb if world == 1 else W[0][1])
        keys = [[] for _ in range(L)]
        vals = [[] for _ in range(L)]
        all_logits = []
        for pos, tok in enumerate(prompt):
            x = emb[tok].copy()
            for l in range(L):
                b = 1 + 12 * l
                xn = rms(x, W[b][0][0], cfg.rms_norm_eps)
                qv = W[b + 1][0] @ xn + (W[b + 2][0][0] if cfg.qkv_bias else 0)
                kv = W[b + 3][0] @ xn + (W[b + 4][0][0] if cfg.qkv_bias else 0)
                vv = W[b + 5][0] @ xn + (W[b + 6][0][0] if cfg.qkv_bias else 0)
                qv = oracle.apply_rope(qv, nq_l, d, pos, cfg)
                kv = oracle.apply_rope(kv, nkv_l, d, pos, cfg)
                keys[l].append(kv.reshape(nkv_l, d))
                vals[l].append(vv.reshape(nkv_l, d))
                K = np.stack(keys[l])
                V = np.stack(vals[l])
                attn = np.zeros(nq_l * d, np.float32)
                for hq in range(nq_l):
                    g = hq // group
                    s = (K[:, g, :] @ qv[hq * d:(hq + 1) * d]) / np.float32(np.sqrt(d))
                    p = np.exp(s - s.max())
                    p /= p.sum()
                    attn[hq * d:(hq + 1) * d] = p @ V[:, g, :]
                part = torch.from_numpy((W[b + 7][0] @ attn).astype(np.float32))
                dist.all_reduce(part)
                x = x + part.numpy()
                xn = rms(x, W[b + 8][0][0], cfg.rms_norm_eps)
                gate = W[b + 9][0] @ xn
                up = W[b + 10][0] @ xn
                ff = (gate / (1 + np.exp(-gate))) * up
                part = torch.from_numpy((W[b + 11][0] @ ff).astype(np.float32))
                dist.all_reduce(part)
                x = x + part.numpy()
            xn = rms(x, W[1 + 12 * L][0][0], cfg.rms_norm_eps)
            local = torch.from_numpy((lm @ xn).astype(np.float32))
            gathered = [torch.zeros_like(local) for _ in range(world)]
            dist.all_gather(gathered, local)
            all_logits.append(torch.cat(gathered).numpy()[: cfg.vocab_size])
        dist.destroy_process_group()
        q.put((rank, "ok", np.stack(all_logits)))
    except Exception as e:
        q.put((rank, repr(e), None))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("name", ["qwen2_tiny", "llama3_tiny_rs"])
def test_tp2_gloo_forward_matches_oracle(oracle, name):
    import multiprocessing as mp
    from make_golden import fixture_configs
    cfg, seed = fixture_configs()[name]
    prompt = [5, 17, 99, 201, 3]
    ref = oracle.RefRunner(cfg, blob=oracle.synthetic_blob(cfg, seed=seed), max_seq=64)
    ref_logits = np.stack([ref.forward_token(t, p) for p, t in enumerate(prompt)])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=rank_forward, args=(r, 2, port, cfg, seed, prompt, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, status, logits = q.get(timeout=240)
        res[rank] = (status, logits)
    for p in procs:
        p.join(timeout=30)
    for rank in range(2):
        assert res[rank][0] == "ok", res[rank][0]
        assert np.max(np.abs(res[rank][1] - ref_logits)) < 1e-4


def test_tp_plan_covers_every_tensor_once():
    from make_golden import fixture_configs
    from vvli_b200 import config as C
    for cfg in (fixture_configs()["qwen2_tiny"][0], C.llama3_8b()):
        for world in (1, 2, 4, 8) if cfg.num_key_value_heads % 8 == 0 else (1, 2):
            covered = {}
            for rank in range(world):
                for dst, tid, src, rows, cols, ld, r0, c0, kind in tp_plan(cfg, rank, world).tolist():
                    covered.setdefault(tid, 0)
                    covered[tid] += rows * cols
            import oracle
            table = {int(t): int(n) for _, n, t in oracle.tensor_table(cfg).tolist()}
            for tid, n in table.items():
                replicated = tid == 0 or tid % 12 in (1, 9) or tid == 1 + 12 * cfg.num_hidden_layers
                if tid == 0:  # embedding replicated; tied LM head adds one vocab shard per rank
                    extra = n if (cfg.tie_word_embeddings and world > 1) else 0
                    assert covered[tid] == world * n + extra, (tid, world)
                elif replicated:
                    assert covered[tid] == world * n, (tid, world)
                else:
                    assert covered[tid] == n, (tid, world)
