"""One rank of the tensor-parallel GPU check (launched by tests/test_gpu_tp.py through
torch.distributed.run, one process per GPU). Every rank opens a TP handle of each blob and a
single-GPU handle, runs the same prefills on both and reports, as one JSON file per rank
($MMFREE_TP_OUT/rank<r>.json):
  * FixedQ510: bit equality of the last-position logits and of the first ids of a batched
    prefill (serve_begin), TP against one GPU; with the configuration-4 fixture, against the
    reference's own logits;
  * Float: the largest logit difference over the logit range.
"""
from __future__ import annotations

import datetime
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import torch
    import torch.distributed as dist

    from matmulfreellmcpu_b200 import api, tp
    from matmulfreellmcpu_b200 import blob as B

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    cache = os.environ.get("MMFREE_BLOB_CACHE", "/tmp/mmfree_blobs")
    names = sys.argv[1:] or ["370M"]
    out = {"rank": rank, "world": world}
    for name in names:
        if rank == 0:
            path = B.cached_blob(name, 0, cache)
        dist.barrier()
        path = B.cached_blob(name, 0, cache)
        V = B.CONFIGS[name]["vocab_size"]
        fix = None
        if name == "2.7B":
            with np.load(os.path.join(ROOT, "tests", "golden", "config4_prefill_2.7B.npz")) as z:
                fix = {k: z[k] for k in z.files}
            ids = fix["ids"]
        else:
            ids = B.seeded_ids(40, 9, V)
        prompts = [B.seeded_ids(24, 50 + k, V) for k in range(3)]
        for mode in ("fixed", "float"):
            m = tp.open_model(path, mode, rank, world, local)
            lg = m.forward_last(ids)
            first = m.serve_begin(prompts)
            m.serve_end()
            m.close()
            with api.Model(path, mode, device=local) as one:
                lg1 = one.forward_last(ids)
                first1 = one.serve_begin(prompts)
                one.serve_end()
            r = {}
            if mode == "fixed":
                r["logits_bits_equal_1gpu"] = bool(np.array_equal(lg.view(np.uint32), lg1.view(np.uint32)))
                r["first_ids_equal_1gpu"] = bool(np.array_equal(first, first1))
                if fix is not None:
                    r["logits_bits_equal_reference"] = bool(
                        np.array_equal(lg.view(np.uint32), fix["fixed_logits"].view(np.uint32)))
            else:
                span = float(lg1.max() - lg1.min())
                r["max_abs_over_range_1gpu"] = float(np.abs(lg - lg1).max()) / span
                if fix is not None:
                    ref = fix["float_logits"]
                    r["max_abs_over_range_reference"] = float(np.abs(lg - ref).max()) / float(ref.max() - ref.min())
            out[f"{name}/{mode}"] = r
    dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(os.environ["MMFREE_TP_OUT"], f"rank{rank}.json"), "w") as f:
        json.dump(out, f)


if __name__ == "__main__":
    main()
