"""GPU tests of the export contract: a model written by q4b.export and loaded back generates the
reference's tokens; the entry points named like export_llama.py's, driven by run_host.py's loop
(scripts/llm/run_host.py:40-54), do too; the runner CLI runs an export directory with its meta.json
prompt; the pack cache quantises once and serves the same model afterwards."""

import json
import pathlib
import subprocess
import sys

import numpy as np
import pytest
import torch

import golden_inputs as gi
from conftest import ROOT, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_export(tmp_path_factory):
    import q4b
    from q4b import export
    z = load_golden("model_tiny_ref")
    spec = gi.MODEL_SPECS["tiny_ref"]
    model = q4b.LlamaQ4.from_packed(spec["cfg"], z, spec["max_ctx"], vocab_chunk=spec["vocab_chunk"],
                                    max_chunk=spec["chunk"])
    out = tmp_path_factory.mktemp("export") / "tiny_ref"
    export.export(model, out, spec["chunk"], spec["buckets"], prompt=z["prompt"], ref_tokens=z["bucketed_tokens"])
    return out, z, spec


def test_loaded_export_generates_reference_tokens(tiny_export):
    import q4b
    from q4b import export
    out, z, spec = tiny_export
    model = export.load(out)
    r = q4b.Runner(model, spec["chunk"], spec["buckets"], "bucketed")
    toks, _ = r.generate(z["prompt"].tolist(), spec["max_new"])
    assert toks == z["bucketed_tokens"].tolist()


def test_entry_points_by_name(tiny_export):
    """run_host.py's schedule over the named functions: prefill_c{C}_l{bucket(s + C)} per chunk,
    then decode_l{bucket(pos + 1)} per token; decode_logits_l{L0} returns the logits row."""
    from q4b import export
    out, z, spec = tiny_export
    model = export.load(out)
    meta = json.loads((out / "meta.json").read_text())
    fns = export.entry_points(model, meta["chunk"], meta["buckets"])
    assert list(fns) == meta["entry_points"]
    C, buckets, prompt = meta["chunk"], meta["buckets"], meta["prompt"]
    caches = model.new_caches()

    def bucket(n):
        return next(L for L in buckets if L >= n)

    i32 = lambda *v: torch.tensor(v, dtype=torch.int32)  # noqa: E731
    n = len(prompt)
    for s in range(0, n, C):
        m = min(C, n - s)
        chunk = torch.zeros(1, C, dtype=torch.int32)
        chunk[0, :m] = torch.tensor(prompt[s:s + m])
        nxt = int(fns[f"prefill_c{C}_l{bucket(s + C)}"](chunk, i32(s), i32(m - 1), *caches))
    toks = [nxt]
    for i in range(1, len(meta["ref_tokens"])):
        pos = n + i - 1
        nxt = int(fns[f"decode_l{bucket(pos + 1)}"](i32(nxt).reshape(1, 1), i32(pos), i32(0), *caches))
        toks.append(nxt)
    assert toks == meta["ref_tokens"]
    lg = fns[f"decode_logits_l{buckets[0]}"](i32(toks[0]).reshape(1, 1), i32(3), i32(0), *model.new_caches())
    assert tuple(lg.shape) == (1, meta["vocab"]) and lg.dtype == torch.float32


def test_runner_cli_on_an_export(tiny_export):
    """python -m q4b.runner --model-dir <export>: the prompt comes from meta.json; the JSON report
    holds the reference's tokens."""
    out, z, spec = tiny_export
    env = dict(__import__("os").environ, PYTHONPATH=str(ROOT / "iree-adreno-genai-tuner_b200"))
    p = subprocess.run([sys.executable, "-m", "q4b.runner", "--model-dir", str(out), "--chunk", str(spec["chunk"]),
                        "--buckets", ",".join(map(str, spec["buckets"])), "--max_new_tokens", str(spec["max_new"]),
                        "--max_ctx", str(spec["max_ctx"])], capture_output=True, text=True, env=env, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    rep = json.loads(p.stdout.strip().splitlines()[-1])
    assert rep["tokens"] == z["bucketed_tokens"].tolist()
    assert rep["schedule"] == "bucketed" and rep["chunk"] == spec["chunk"]


def test_pack_cache(tmp_path):
    import q4b
    from q4b import export
    cfg = q4b.SYNTHETIC["tiny"]
    built = []

    def build():
        built.append(1)
        return q4b.LlamaQ4(None, group=128, max_ctx=256, sd=q4b.SyntheticStateDict(cfg, seed=3), cfg=cfg,
                           max_chunk=32, per_linear_group=True)

    m1, hit1 = export.cached(tmp_path, build, cfg, "synthetic:3", 128, 256, per_linear_group=True, chunk=32,
                             buckets=[128, 256])
    m2, hit2 = export.cached(tmp_path, build, cfg, "synthetic:3", 128, 256, per_linear_group=True, chunk=32,
                             buckets=[128, 256])
    assert (hit1, hit2) == (False, True) and len(built) == 1
    prompt = np.random.default_rng(0).integers(0, cfg["vocab_size"], 40).tolist()
    t1, _ = q4b.Runner(m1, 32, [128, 256]).generate(prompt, 12)
    t2, _ = q4b.Runner(m2, 32, [128, 256]).generate(prompt, 12)
    assert t1 == t2
    for a, b in zip(m1.layers, m2.layers):
        assert torch.equal(a.wgu.qweight, b.wgu.qweight) and torch.equal(a.wdown.scales, b.wdown.scales)
