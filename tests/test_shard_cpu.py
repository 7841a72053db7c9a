"""Shards of one packed int4 linear over two gloo ranks (no GPU): the column split's outputs
concatenate and the row split's partial outputs sum to the unsharded QLinear result
(scripts/llm/llama_q4.py:48-51, 69-72 restated by the oracle)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    rng = np.random.default_rng(3)
    n, k, g = 96, 512, 128
    qw = rng.integers(-2**31, 2**31 - 1, size=(n, k // 8), dtype=np.int64).astype(np.int32)
    sc = (np.abs(rng.standard_normal((n, k // g))) * 0.02).astype(np.float16)
    x = rng.standard_normal((3, k)).astype(np.float32)
    return qw, sc, x, g


def _worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from oracle import q4_oracle as O
        from q4b.shard import shard_q4, shard_x
        qw, sc, x, g = _case()
        ref = x @ O.dequantize_q4(qw, sc, g).T
        out = {}
        for split in ("col", "row"):
            qr, sr = shard_q4(torch.from_numpy(qw), torch.from_numpy(sc), g, rank, world, split)
            xr = shard_x(torch.from_numpy(x), rank, world, split)
            y = torch.from_numpy(xr.numpy() @ O.dequantize_q4(qr.numpy(), sr.numpy(), g).T)
            if split == "col":
                parts = [torch.zeros_like(y) for _ in range(world)]
                dist.all_gather(parts, y)
                y = torch.cat(parts, 1)
            else:
                dist.all_reduce(y)
            out[split] = float(np.abs(y.numpy() - ref).max() / np.abs(ref).max())
        q.put((rank, out))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


def test_shards_combine_to_the_unsharded_linear():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(res[r], dict), res[r]
        assert res[r]["col"] < 1e-6 and res[r]["row"] < 1e-6, res[r]


def test_shard_rules():
    from q4b.shard import shard_ok, shard_q4
    assert shard_ok(5120, 3072, 128, 8, "col") and shard_ok(5120, 3072, 128, 8, "row")
    assert not shard_ok(5120, 3072, 128, 16, "row")  # 192 k per rank is not whole groups
    with pytest.raises(ValueError):
        shard_q4(torch.zeros(10, 4, dtype=torch.int32), torch.zeros(10, 1, dtype=torch.float16), 32, 0, 3, "col")
