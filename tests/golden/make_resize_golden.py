"""Golden vectors of the input path's resize from an independent
implementation: PyTorch's CPU uint8 antialiased bilinear interpolation
(torch.nn.functional.interpolate(..., mode="bilinear", antialias=True) on a
channels-last uint8 tensor), the kernel the reference's aa_resize
(image.c:209-339) restates. Inputs are regenerated from the seeded
generator (include/sam3_synth.h); small outputs are stored whole, outputs at
the encoder's 1008 x 1008 as SHA-256 digests.

    python tests/golden/make_resize_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import binding as ob  # noqa: E402

SEED = 20261202
# (name, input h, input w, output side): down- and upscaling on each axis
CASES = [("resize_small_down", 61, 47, 23), ("resize_small_up", 13, 19, 40),
         ("resize_small_mixed", 29, 90, 45)]
BIG = [("resize_big_down", 1500, 2100, 1008), ("resize_big_up", 700, 640, 1008),
       ("resize_big_near", 1010, 1003, 1008)]


def image(i, h, w):
    return ob.u8(SEED, 9500 + i, (h, w, 3))


def torch_resize(img, side):
    import torch
    import torch.nn.functional as F
    t = torch.from_numpy(img).permute(2, 0, 1)[None].contiguous(memory_format=torch.channels_last)
    out = F.interpolate(t, size=(side, side), mode="bilinear", antialias=True,
                        align_corners=False)
    return out[0].permute(1, 2, 0).contiguous().numpy()


def main():
    for i, (name, h, w, side) in enumerate(CASES):
        np.savez_compressed(os.path.join(HERE, name + ".npz"),
                            out=torch_resize(image(i, h, w), side))
        print(name)
    with open(os.path.join(HERE, "resize_big.sha256"), "w") as f:
        for j, (name, h, w, side) in enumerate(BIG):
            d = hashlib.sha256(torch_resize(image(100 + j, h, w), side).tobytes()).hexdigest()
            f.write(f"{name} {h} {w} {side} {d}\n")
            print(name, d)


if __name__ == "__main__":
    main()
