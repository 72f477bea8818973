"""One rank of the tensor-parallel parity check (launched by tests/test_gpu_tp.py).

    python -m torch.distributed.run --nproc-per-node T --master-addr 127.0.0.1 \
        --master-port P tests/tp_worker.py --out result.json

Every rank builds the same seeded weights, keeps its shard (init_model_tp) and
runs the same steps.  Rank 0 compares the gathered logits with the oracle and
with a single-GPU model of the same weights, and every rank's greedy and
sampled tokens with rank 0's.  The verdict goes to --out (rank 0).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "oracle"):
    sys.path.insert(0, str(p))

LOGIT_RTOL = 2e-4
LOGIT_ATOL = 1e-5


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    ap.add_argument("--kv-heads", type=int, default=1)
    ap.add_argument("--heads", type=int, default=4)
    ap.add_argument("--head-dim", type=int, default=64)
    ap.add_argument("--steps", type=int, default=12)
    ap.add_argument("--hidden", type=int, default=256)
    ap.add_argument("--intermediate", type=int, default=512)
    ap.add_argument("--bf16", action="store_true", help="bf16 weights (the kernels that split row groups)")
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    from mogemma_b200 import _core, synth

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    d = synth.tiny(hidden=args.hidden, heads=args.heads, kv_heads=args.kv_heads, head_dim=args.head_dim,
                   intermediate=args.intermediate, vocab=4096)
    w = synth.make_weights(d, seed=11, bf16=args.bf16)
    meta = synth.metadata_of(w)
    wd = "bf16" if args.bf16 else "f32"
    llm = _core.init_model_tp(meta, device=rank, capacity=64, seed=7, weight_dtype=wd)
    toks = [int(t) for t in synth.prompt_ids(args.steps, d.vocab, seed=5)]
    result: dict = {"world": world, "kv_heads": args.kv_heads, "heads": args.heads, "head_dim": args.head_dim}

    def run(model: dict) -> tuple[list, list, list]:
        # teacher-forced logits (the reference step(): full-vocabulary fp32 logits),
        # then a prefill and greedy / top-k streams drawn on the device
        logits = [_core.step(model, t, 0.0, 0, 1.0) for t in toks]
        _core.prefill(model, toks[:-1])
        greedy = list(_core.generate(model, toks[-1], 10, 0.0, 0, 1.0))
        sampled = list(_core.generate(model, greedy[-1], 10, 0.8, 40, 1.0))
        return logits, greedy, sampled

    tp_logits, greedy, sampled = run(llm)
    streams = torch.tensor(np.asarray(greedy + sampled, dtype=np.int64), device="cuda")
    gathered = [torch.zeros_like(streams) for _ in range(world)]
    dist.all_gather(gathered, streams)
    result["streams_equal_across_ranks"] = all(bool(torch.equal(g, gathered[0])) for g in gathered)

    if rank == 0:
        import oracle

        ref = oracle.RefModel(w, max_seq_len=64)
        errs = []
        for t, lg in zip(toks, tp_logits):
            r = ref.step(t)
            errs.append(float(np.max(np.abs(lg - r))) / (LOGIT_ATOL + LOGIT_RTOL * float(np.max(np.abs(r)))))
        result["oracle_err_over_tol"] = max(errs)
        single = _core.init_model(meta, device=0, capacity=64, seed=7, weight_dtype=wd)
        one_logits, one_greedy, _ = run(single)
        result["single_gpu_max_abs_diff"] = max(float(np.max(np.abs(a - b))) for a, b in zip(one_logits, tp_logits))
        result["greedy_equal_single_gpu"] = one_greedy == greedy
        single["_handle"].close()
        result["ok"] = bool(result["oracle_err_over_tol"] <= 1.0 and result["streams_equal_across_ranks"]
                            and result["greedy_equal_single_gpu"])
        Path(args.out).write_text(json.dumps(result))
    _core.close_tp(llm)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
