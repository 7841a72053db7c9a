"""Tensor-parallel partition math on CPU with two gloo ranks (no GPU).

Each rank takes its shard of a layer (q4b.shard_layer, the slicing the GPU model uses), computes
its partial projections, and the ranks combine them the way the native step does: column-split
outputs concatenate in head order, row-split partials sum (all_reduce), and the vocab-split greedy
head keeps the largest value with the lowest index across ranks. Every combination must equal the
unsharded computation (scripts/llm/llama_q4.py:149-153, 216-239)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CFG = dict(hidden_size=64, num_attention_heads=8, num_key_value_heads=2, head_dim=16, intermediate_size=96,
           vocab_size=50)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    g = torch.Generator().manual_seed(0)
    D, H, Hkv, hd, I = 64, 8, 2, 16, 96
    shapes = {"self_attn.q_proj.weight": (H * hd, D), "self_attn.k_proj.weight": (Hkv * hd, D),
              "self_attn.v_proj.weight": (Hkv * hd, D), "self_attn.o_proj.weight": (D, H * hd),
              "mlp.gate_proj.weight": (I, D), "mlp.up_proj.weight": (I, D), "mlp.down_proj.weight": (D, I)}
    return {k: torch.randn(s, generator=g, dtype=torch.float64) for k, s in shapes.items()}


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from q4b.llama import shard_layer
        W = _weights()
        D, H, Hkv, hd, I = 64, 8, 2, 16, 96
        x = torch.randn(3, D, generator=torch.Generator().manual_seed(1), dtype=torch.float64)
        sh = shard_layer(CFG, lambda n: W[n], rank, world)
        # q|k|v column split: gather the shards' outputs and put them back in head order
        part = x @ sh["wqkv"].T
        parts = [torch.zeros_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        hq, hk = H // world * hd, Hkv // world * hd
        q_full = torch.cat([p[:, :hq] for p in parts], 1)
        k_full = torch.cat([p[:, hq:hq + hk] for p in parts], 1)
        v_full = torch.cat([p[:, hq + hk:] for p in parts], 1)
        ref = torch.cat([x @ W["self_attn.q_proj.weight"].T, x @ W["self_attn.k_proj.weight"].T,
                         x @ W["self_attn.v_proj.weight"].T], 1)
        assert torch.allclose(torch.cat([q_full, k_full, v_full], 1), ref)
        # attention output columns of this rank's heads -> o_proj row split: partials sum
        o = torch.randn(3, H * hd, generator=torch.Generator().manual_seed(2), dtype=torch.float64)
        o_shard = o[:, rank * hq:(rank + 1) * hq]
        y = o_shard @ sh["wo"].T
        dist.all_reduce(y)
        assert torch.allclose(y, o @ W["self_attn.o_proj.weight"].T)
        # gate|up column split -> SwiGLU per rank -> down row split
        gu = x @ sh["wgu"].T
        a = torch.nn.functional.silu(gu[:, :I // world]) * gu[:, I // world:]
        yd = a @ sh["wdown"].T
        dist.all_reduce(yd)
        gu_full = x @ torch.cat([W["mlp.gate_proj.weight"], W["mlp.up_proj.weight"]], 0).T
        a_full = torch.nn.functional.silu(gu_full[:, :I]) * gu_full[:, I:]
        assert torch.allclose(yd, a_full @ W["mlp.down_proj.weight"].T)
        # vocab-split greedy head: largest value, lowest index on ties (torch.argmax semantics)
        logits = torch.randn(50, generator=torch.Generator().manual_seed(3), dtype=torch.float64)
        logits[7] = logits[31] = logits.max() + 1.0  # a tie across the two ranks' halves
        V = 50 // world
        loc = logits[rank * V:(rank + 1) * V]
        i = int(torch.argmax(loc))
        key = torch.tensor([float(loc[i]), float(rank * V + i)], dtype=torch.float64)
        keys = [torch.zeros_like(key) for _ in range(world)]
        dist.all_gather(keys, key)
        best = max(keys, key=lambda k: (float(k[0]), -float(k[1])))
        assert int(best[1]) == int(torch.argmax(logits)) == 7
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tp2_partition_math_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def test_shard_rejects_indivisible():
    from q4b.llama import shard_layer
    W = _weights()
    with pytest.raises(ValueError):
        shard_layer(CFG, lambda n: W[n], 0, 3)
