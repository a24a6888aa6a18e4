"""Engram tensors of a merged safetensors folder -> a .pt with local names
(reference: extract_engram.py:1-23).

    python -m micro_engram.tools.extract MODEL_DIR [micro_engram.pt]
"""
import glob
import os
import sys

import torch


def extract(src):
    """{local name: tensor} of every '.micro_engram.' key in the folder's safetensors."""
    from safetensors import safe_open

    sd = {}
    for fn in sorted(glob.glob(os.path.join(src, "*.safetensors"))):
        with safe_open(fn, "pt") as fh:
            for k in fh.keys():
                if ".micro_engram." in k:
                    sd[k.split(".micro_engram.", 1)[1]] = fh.get_tensor(k)
    return sd


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if not argv:
        raise SystemExit("usage: extract MODEL_DIR [OUT.pt]")
    out = argv[1] if len(argv) > 1 else "micro_engram.pt"
    sd = extract(argv[0])
    if not sd:
        raise SystemExit("no micro_engram keys found")
    torch.save(sd, out)
    print(f"saved {len(sd)} tensors to {out}: " + ", ".join(sorted(sd)[:4]) + ", ...")


if __name__ == "__main__":
    main()
