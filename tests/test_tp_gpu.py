"""Tensor-parallel GPU parity: the reference's tiny KAT model sharded over 2 GPUs (NCCL) gives the
reference's greedy tokens under both schedules, with graphs on/off and the synchronous protocol.
Needs >= 2 GPUs (skipped otherwise)."""

import json
import pathlib
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

HERE = pathlib.Path(__file__).resolve().parent
pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_tiny_ref_tokens():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr",
           "127.0.0.1", "--master-port", str(_port()), str(HERE / "tp_gpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600,
                       env={**__import__("os").environ, "NCCL_NVLS_ENABLE": "0"})
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("TP_RESULT ")]
    assert r.returncode == 0 and line, r.stderr[-3000:]
    out = json.loads(line[0][len("TP_RESULT "):])
    z = np.load(HERE / "golden" / "model_tiny_ref.npz")
    for key, toks in out.items():
        schedule = key.split("_")[0]
        assert toks == z[f"{schedule}_tokens"].tolist(), key
