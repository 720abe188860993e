"""Write a checkpoint of the unmodified reference optimizer for the interop test.

    python tests/golden/make_ref_checkpoint.py --reference /path/to/LUMA/src

Imports ``luma_optimizer`` from that tree (or from ``baseline/_ref`` when the
reference was installed there), trains three small fp32 tensors in two param
groups for three steps with ``LUMA(backend="pytorch")`` on CPU, exactly as a
user would (the reference's own RNG, nothing patched), and saves
``tests/golden/ref_checkpoint.pt``: the reference's ``state_dict()``, the
params after those steps, the group hyper-parameters and the grads of three
further steps.  ``tests/test_gpu_interop.py`` loads it into ``luma_b200.LUMA``
and continues training.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

SHAPES = [(300,), (17, 33), (5000,)]
GROUPS = [dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01),
          dict(lr=3e-4, betas=(0.8, 0.99), eps=1e-6, weight_decay=0.0)]
GROUP_OF = [0, 1, 0]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.path.join(ROOT, "baseline", "_ref"),
                    help="directory holding the luma_optimizer package")
    ap.add_argument("--out", default=os.path.join(HERE, "ref_checkpoint.pt"))
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from luma_optimizer import LUMA

    torch.manual_seed(2024)
    params = [torch.nn.Parameter(torch.randn(s) * 0.02) for s in SHAPES]
    groups = [dict(params=[p for p, gi in zip(params, GROUP_OF) if gi == k], **hp)
              for k, hp in enumerate(GROUPS)]
    opt = LUMA(groups, backend="pytorch")
    gen = torch.Generator().manual_seed(7)
    for _ in range(3):
        for p in params:
            p.grad = torch.randn(p.shape, generator=gen) * 1e-2
        opt.step()
    later = [[torch.randn(p.shape, generator=gen) * 1e-2 for p in params] for _ in range(3)]
    torch.save({"state_dict": opt.state_dict(),
                "params": [p.detach().clone() for p in params],
                "group_of": GROUP_OF, "groups": GROUPS, "grads": later,
                "reference": "luma_optimizer.LUMA(backend='pytorch'), CPU, 3 steps"}, args.out)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
