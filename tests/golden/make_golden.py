"""Records golden vectors from the reference's own CUDA kernels.

Run on a B200 with the reference extension built by oracle/build_ref.py
(oracle/_ref/_tma_dwconv_ref_C*.so):

    python tests/golden/make_golden.py tests/golden/ref_kernels.npz

For each case, x ~ N(0,1) and w ~ N(0,1/9) are drawn on the CPU from
torch.manual_seed(1000 + i), converted to fp16, and passed to the reference's
dwconv_ws (n_stage 2, 3 and 4, which must agree) and dwconv_v0.  The file
stores x, w, pad and both outputs as raw fp16 bits.  tests/test_oracle.py
checks the CPU oracle against these vectors bit for bit.
"""
import glob
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

CASES = [  # N, H, W, C, pad
    (2, 16, 16, 64, 0),
    (2, 16, 16, 64, 1),
    (2, 16, 16, 64, 2),
    (2, 16, 16, 64, 3),
    (1, 8, 8, 64, 1),
    (2, 7, 45, 64, 1),
    (1, 5, 33, 64, 2),
    (1, 9, 34, 128, 1),
]


def load_reference():
    paths = glob.glob(os.path.join(REPO, "oracle", "_ref", "_tma_dwconv_ref_C*.so"))
    if not paths:
        raise SystemExit("reference extension not built (python oracle/build_ref.py)")
    spec = importlib.util.spec_from_file_location("_tma_dwconv_ref_C", paths[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(out_path: str) -> None:
    ref = load_reference()
    arrays = {}
    for i, (N, H, W, C, pad) in enumerate(CASES):
        torch.manual_seed(1000 + i)
        x = torch.randn(N, H, W, C).half()
        w = (torch.randn(3, 3, C) / 3).half()
        xd, wd = x.cuda(), w.cuda()
        ws = [ref.dwconv_ws(xd, wd, pad, s).cpu() for s in (2, 3, 4)]
        assert all(torch.equal(ws[0].view(torch.int16), o.view(torch.int16)) for o in ws[1:])
        v0 = ref.dwconv_v0(xd, wd, pad).cpu()
        arrays[f"c{i}_shape"] = np.array([N, H, W, C, pad], dtype=np.int64)
        arrays[f"c{i}_x"] = x.numpy().view(np.uint16)
        arrays[f"c{i}_w"] = w.numpy().view(np.uint16)
        arrays[f"c{i}_ws"] = ws[0].numpy().view(np.uint16)
        arrays[f"c{i}_v0"] = v0.numpy().view(np.uint16)
        same = np.array_equal(arrays[f"c{i}_ws"], arrays[f"c{i}_v0"])
        print(f"case {i} {(N, H, W, C, pad)}: ws(2,3,4) agree; v0 == ws: {same}")
    np.savez_compressed(out_path, **arrays)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ref_kernels.npz"))
