"""Generate the golden fixtures: outputs of the reference fp64-emu itself.

Runs on a CUDA machine with the reference build in oracle/_ref
(python oracle/build_ref.py).  Inputs are rebuilt from numpy seeds
(tests/helpers.make), so only the case list and the reference's outputs are
stored: tests/golden/reference_outputs.npz (float64 arrays, keyed by case id)
and tests/golden/cases.json.

    python tests/golden/make_golden.py [--out DIR]
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))

from helpers import make  # noqa: E402

# id: (op, batch, M, K, N, dist, seed, kwargs)
CASES = {
    "mm_nt_randn_64x512x48": ("mm_nt", 1, 64, 512, 48, "randn", 1, {}),
    "mm_nt_randn_64x4096x40": ("mm_nt", 1, 64, 4096, 40, "randn", 2, {}),
    "mm_nt_randn_odd_33x1000x29": ("mm_nt", 1, 33, 1000, 29, "randn", 3, {}),
    "mm_nt_wide8_48x600x40": ("mm_nt", 1, 48, 600, 40, "wide8", 4, {}),
    "mm_nt_wide16_48x512x40": ("mm_nt", 1, 48, 512, 40, "wide16", 5, {}),
    "mm_nt_illcond_48x512x40": ("mm_nt", 1, 48, 512, 40, "illcond", 6, {}),
    "mm_nt_illcond40_48x512x40": ("mm_nt", 1, 48, 512, 40, "illcond40", 7, {}),
    "mm_nt_spike_48x512x40": ("mm_nt", 1, 48, 512, 40, "spike", 8, {}),
    "mm_nt_wide30_40x300x36": ("mm_nt", 1, 40, 300, 36, "wide30", 9, {}),
    "mm_randn_reduced_48x1000x40": ("mm", 1, 48, 1000, 40, "randn", 10, {"nprimes": 13, "corr": False}),
    "mm_randn_fast_recombine_48x300x50": ("mm", 1, 48, 300, 50, "randn", 11, {"exact": False}),
    "mm_randn_bits40_40x700x44": ("mm", 1, 40, 700, 44, "randn", 12, {"bits": 40}),
    "mm_randn_bits20_40x200x30": ("mm", 1, 40, 200, 30, "randn", 13, {"bits": 20}),
    "mm_int20_default_48x512x40": ("mm", 1, 48, 512, 40, "int20", 14, {}),
    "mm_int20_reduced_48x512x40": ("mm", 1, 48, 512, 40, "int20", 15, {"nprimes": 13, "corr": False}),
    "mm_randn_p20_32x256x24": ("mm", 1, 32, 256, 24, "randn", 16, {"nprimes": 20}),
    "mm_randn_p7_32x256x24": ("mm", 1, 32, 256, 24, "randn", 17, {"nprimes": 7}),
    "mm_tiny_1x1x1": ("mm", 1, 1, 1, 1, "randn", 18, {}),
    "bmm_randn_3x40x200x30": ("bmm", 3, 40, 200, 30, "randn", 19, {}),
    "bmm_nt_unif_4x33x100x27": ("bmm_nt", 4, 33, 100, 27, "unif", 20, {}),
    "mm_deepk_randn_8x140000x6": ("mm", 1, 8, 140000, 6, "randn", 21, {}),
    "mm_nt_k70000_16x70000x12": ("mm_nt", 1, 16, 70000, 12, "randn", 22, {}),
}


def inputs(case):
    op, batch, M, K, N, dist, seed, kw = case
    nt = op.endswith("_nt")
    if batch == 1:
        return make(dist, M, K, N, seed=seed, nt=nt)
    pairs = [make(dist, M, K, N, seed=seed * 100 + b, nt=nt) for b in range(batch)]
    return np.stack([p[0] for p in pairs]), np.stack([p[1] for p in pairs])


def main():
    import argparse
    import torch
    import fp64_emu_ref as R
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    out_dir = ap.parse_args().out
    os.makedirs(out_dir, exist_ok=True)
    outs = {}
    for cid, case in CASES.items():
        A, B = inputs(case)
        op, kw = case[0], case[7]
        C = getattr(R, op)(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), **kw)
        outs[cid] = C.cpu().numpy()
        print(cid, outs[cid].shape, flush=True)
    np.savez_compressed(os.path.join(out_dir, "reference_outputs.npz"), **outs)
    with open(os.path.join(out_dir, "cases.json"), "w") as f:
        json.dump({k: list(v[:7]) + [v[7]] for k, v in CASES.items()}, f, indent=1)
    print("reference:", torch.cuda.get_device_name(0), "cases:", len(outs))


if __name__ == "__main__":
    main()
