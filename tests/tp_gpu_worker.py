"""One rank of the tensor-parallel GPU parity checks (launched by tests/test_tp_gpu.py under
torch.distributed.run). Default: builds the reference's tiny KAT model (HF random init, seed 0)
sharded over the ranks, runs the llm_runner.c schedule, and rank 0 prints the tokens as JSON.
Q4B_TP_MODE=persistent: the persistent decode step sharded over the ranks (see persistent_main);
collectives: the standalone TP collectives; ref3b: the 3B shape against the reference's stream."""

import json
import os
import pathlib
import sys
from datetime import timedelta

HERE = pathlib.Path(__file__).resolve().parent
for p in (HERE.parent / "iree-adreno-genai-tuner_b200", HERE.parent, HERE / "golden"):
    sys.path.insert(0, str(p))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


# the persistent decode step's smallest shape (head_dim 128, D a multiple of 1024); the o / down
# shards of 2 ranks (K 512 and 1024) cover a partial 1024-k unit and the padded scale rows
PCFG = dict(hidden_size=1024, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2, head_dim=128,
            intermediate_size=2048, vocab_size=4096, rms_norm_eps=1e-5, rope_theta=500000.0,
            max_position_embeddings=4096, tie_word_embeddings=True, hidden_act="silu", attention_bias=False,
            initializer_range=0.2)
PROMPT, STEPS = 40, 12
# Q4B_TP_CFG=3b2: two layers of the Llama-3.2-3B shape (24 heads, 8 KV heads: one KV head per rank
# at 8 ranks; o / down shard scale rows of 12, 6 and 3 groups at 2, 4 and 8 ranks)
CFGS = {"small": PCFG}


def _cfg():
    name = os.environ.get("Q4B_TP_CFG", "small")
    if name == "3b2":
        import q4b
        return dict(q4b.SYNTHETIC["3b"], num_hidden_layers=2)
    return CFGS[name]


def _persistent_decode(model, persistent, gather):
    """Prefill (per-projection path), then STEPS decode steps: (tokens, full-vocab logits per step)."""
    os.environ["Q4B_PERSISTENT"] = "1" if persistent else "0"
    caches = model.new_caches()
    p = np.random.default_rng(7).integers(0, model.vocab, PROMPT).astype(np.int32)
    dev = caches[0].device
    nxt, _ = model.step(torch.from_numpy(p).reshape(1, -1), torch.tensor([0]), torch.tensor([PROMPT - 1]), caches, 64)
    toks, logits = [int(nxt)], []
    for i in range(STEPS):
        pos = PROMPT + i
        L = 64 if pos < 64 else 128
        nxt, lg = model.step(nxt.reshape(1, 1), torch.tensor([pos]), torch.tensor([0]), caches, L)
        toks.append(int(nxt))
        logits.append(gather(lg.to(dev)).cpu().numpy()[0])
    return toks, np.stack(logits)


def persistent_main(rank, world, dev):
    """tp=world persistent decode (peer-memory partial sums, one launch per token) against the
    per-projection tp path (NCCL) and, on rank 0, the single-GPU model: tokens equal, logits within
    1e-3 of max|logit|; the runner's graphs give the same tokens with the persistent step on / off."""
    import q4b
    from q4b import _lib

    def gather(lg):
        parts = [torch.empty_like(lg) for _ in range(world)]
        dist.all_gather(parts, lg.contiguous())
        return torch.cat(parts, dim=1)

    cfg = _cfg()
    sd = q4b.SyntheticStateDict(cfg, seed=5, device=dev)
    model = q4b.LlamaQ4(None, group=128, max_ctx=1024, vocab_chunk=cfg["vocab_size"], sd=sd, cfg=cfg,
                        max_chunk=64, tp_rank=rank, tp_size=world, device=dev)
    model.attach_tp()
    t_on, l_on = _persistent_decode(model, True, gather)
    kernels = _one_step_kernels(model)
    t_off, l_off = _persistent_decode(model, False, gather)
    status = int(_lib.lib().q4b_device_status(1))
    prompt = np.random.default_rng(7).integers(0, cfg["vocab_size"], PROMPT).tolist()
    graphs = {}
    for on in (True, False):
        os.environ["Q4B_PERSISTENT"] = "1" if on else "0"
        r = q4b.Runner(model, 16, [64, 128, 256], "bucketed", graphs=True)
        graphs[on], _ = r.generate(prompt, 24)
        del r
    out = dict(tokens_on=t_on, tokens_off=t_off, graphs_on=graphs[True], graphs_off=graphs[False],
               diff_on_off=float(np.abs(l_on - l_off).max()), scale=float(max(1.0, np.abs(l_off).max())),
               status=status, kernels=sorted(kernels))
    if rank == 0:
        single = q4b.LlamaQ4(None, group=128, max_ctx=1024, vocab_chunk=cfg["vocab_size"], sd=sd, cfg=cfg,
                             max_chunk=64, device=dev)
        t1, l1 = _persistent_decode(single, True, lambda x: x)
        out.update(tokens_single=t1, diff_single=float(np.abs(l_on - l1).max()))
    return out


def collectives_main(rank, world, dev):
    """The standalone collectives of the C ABI across the ranks: fp32 / fp16 all-reduce sums and the
    vocabulary-split argmax gather (every rank holds shard r of one global logits row)."""
    import ctypes

    import q4b
    from q4b import _lib
    L = q4b.lib()
    uid = (ctypes.c_ubyte * 128)()
    if rank == 0:
        _lib.check(L.q4b_tp_unique_id(uid, 128), "tp_unique_id")
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
    tp = ctypes.c_void_p()
    _lib.check(L.q4b_tp_init(rank, world, uid, 128, ctypes.byref(tp)), "tp_init")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator().manual_seed(11)
    parts = [torch.randn(4096, generator=g) for _ in range(world)]
    x = parts[rank].to(dev)
    _lib.check(L.q4b_tp_allreduce_f32(tp, x.data_ptr(), 4096, st), "allreduce f32")
    h = parts[rank].half().to(dev)
    _lib.check(L.q4b_tp_allreduce_f16(tp, h.data_ptr(), 4096, st), "allreduce f16")
    V = 16032 * world
    logits = torch.randn(V, generator=g)
    shard = logits[rank * 16032:(rank + 1) * 16032].contiguous().to(dev)
    ws = torch.zeros(L.q4b_tp_argmax_workspace(tp) // 8, dtype=torch.int64, device=dev)
    tok = torch.empty(1, dtype=torch.int32, device=dev)
    _lib.check(L.q4b_tp_argmax_gather(tp, shard.data_ptr(), 16032, rank * 16032, tok.data_ptr(), ws.data_ptr(),
                                      ws.numel() * 8, st), "argmax_gather")
    torch.cuda.synchronize()
    want = torch.stack(parts).sum(0)
    out = dict(f32_err=float((x.cpu() - want).abs().max()), f16_err=float((h.float().cpu() - want).abs().max()),
               token=int(tok), want_token=int(torch.argmax(logits)))
    L.q4b_tp_destroy(tp)
    return out


def ref3b_main(rank, world, dev):
    """BASELINE config 4 at full depth over the ranks: the 3B-shape model (SyntheticStateDict seed 0,
    the weights tests/golden/model_3b_ref.npz was made from) sharded over the ranks, the bench's
    request through the runner (persistent decode step on every rank); rank 0 reports the tokens."""
    import q4b
    z = np.load(HERE / "golden" / "model_3b_ref.npz")
    cfg = q4b.SYNTHETIC["3b"]
    model = q4b.LlamaQ4(None, group=128, max_ctx=4096, vocab_chunk=32064,
                        sd=q4b.SyntheticStateDict(cfg, seed=0, device=dev), cfg=cfg, max_chunk=128,
                        tp_rank=rank, tp_size=world, device=dev)
    model.attach_tp()
    r = q4b.Runner(model, 128, [256, 512, 1024, 2048, 4096], "bucketed", graphs=True)
    toks, rep = r.generate(z["prompt"].tolist(), len(z["tokens"]))
    out = dict(tokens=toks, chunks=[c[0] for c in rep["chunks"]],
               decode_path=int(q4b.lib().q4b_model_decode_path(model.native())),
               status=int(q4b.lib().q4b_device_status(1)))
    del r  # graphs holding NCCL calls go before the process group
    return out


def _one_step_kernels(model):
    from torch.profiler import ProfilerActivity, profile
    os.environ["Q4B_PERSISTENT"] = "1"
    caches = model.new_caches()
    model.step(torch.tensor([[3]], dtype=torch.int32), torch.tensor([5]), torch.tensor([0]), caches, 64)
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        model.step(torch.tensor([[3]], dtype=torch.int32), torch.tensor([6]), torch.tensor([0]), caches, 64)
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type.name == "CUDA"}


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    mode = os.environ.get("Q4B_TP_MODE")
    if mode in ("persistent", "collectives", "ref3b"):
        out = {"persistent": persistent_main, "collectives": collectives_main, "ref3b": ref3b_main}[mode](rank, world, dev)
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            print("TP_RESULT " + json.dumps(out), flush=True)
        dist.destroy_process_group()
        return
    import golden_inputs as gi
    import q4b
    from transformers import LlamaConfig, LlamaForCausalLM
    name = os.environ.get("Q4B_TP_MODEL", "tiny_ref")
    spec = gi.MODEL_SPECS[name]
    z = np.load(HERE / "golden" / f"model_{name}.npz")
    torch.manual_seed(spec["seed"])
    hf = LlamaForCausalLM(LlamaConfig(**spec["cfg"], attn_implementation="eager")).eval()
    sd = {k: v.clone() for k, v in hf.state_dict().items()}
    model = q4b.LlamaQ4(None, group=spec["group"], max_ctx=spec["max_ctx"], vocab_chunk=spec["vocab_chunk"], sd=sd,
                        cfg=spec["cfg"], per_linear_group=True, max_chunk=spec["chunk"], tp_rank=rank,
                        tp_size=world, device=dev)
    model.attach_tp()
    out = {}
    for schedule in ("bucketed", "max"):
        for graphs, sync in ((True, False), (False, False), (True, True)):
            r = q4b.Runner(model, spec["chunk"], spec["buckets"], schedule, graphs=graphs, sync_every_step=sync)
            toks, _ = r.generate(z["prompt"].tolist(), spec["max_new"])
            out[f"{schedule}_{int(graphs)}{int(sync)}"] = toks
            del r  # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    dist.barrier()
    if rank == 0:
        print("TP_RESULT " + json.dumps(out), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
