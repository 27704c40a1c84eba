#!/usr/bin/env python3
"""Record torch's CUDA topk on tie-heavy inputs (needs a CUDA device).

torch.topk's order among equal values is not specified; the reference's eager
router (model.py:214) runs it on the GPU, so the router kernel and the oracle
follow what torch's CUDA topk does. This script stores inputs whose values are
small integers (ties at every boundary) and torch.topk's indices for 8, 16 and
32 columns and k = 1..8, fp32, as tests/golden/topk_cuda_ties.npz:

    python tests/golden/make_topk_ties.py
"""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    rng = np.random.default_rng(2026)
    out = {}
    for nb in (8, 16, 32):
        for k in range(1, 9):
            for hi in (2, 3, 6):
                v = rng.integers(1, hi + 1, size=(96, nb)).astype(np.float32)
                _, idx = torch.topk(torch.from_numpy(v).cuda(), k, dim=-1)
                out[f"v_{nb}_{k}_{hi}"] = v.astype(np.int8)
                out[f"i_{nb}_{k}_{hi}"] = idx.cpu().numpy().astype(np.int8)
    out["torch_version"] = np.array(torch.__version__)
    out["device"] = np.array(torch.cuda.get_device_name(0))
    path = os.path.join(HERE, "topk_cuda_ties.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    main()
