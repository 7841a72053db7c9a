"""One rank of the tensor-parallel GPU parity check (launched by tests/test_tp_gpu.py under
torch.distributed.run): builds the reference's tiny KAT model (HF random init, seed 0) sharded
over the ranks, runs the llm_runner.c schedule, and rank 0 prints the tokens as JSON."""

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


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
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
