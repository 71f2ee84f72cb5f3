"""Golden output of the full PE backbone (config 4) from the oracle.

One 1008 x 1008 x 3 uint8 tile ~ U{0..255} (generator stream
SAM3_IMAGE_STREAM_TILE(0)), random-init weights N(0, 0.02) with zero
biases, LayerNorm gamma 1 / beta 0, 2D axial RoPE (theta 10000), global
blocks 7/15/23/31, run through the oracle's restatement of
sam_encode_trunk (sam3_model.c:1112-1144) in fp32. The full output is
5184 x 1024 floats; the fixture keeps every 97th token row plus whole-tensor
statistics, which is enough for a cosine / max-abs check of the GPU
encoder without running the 5 TFLOP oracle on the test machine.

    python tests/golden/make_backbone_golden.py      (about 2 CPU-minutes)
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import binding as ob  # noqa: E402

SEED = 1
ROW_STEP = 97


def image_stream(tile):
    return 3 * 1000003 + tile  # SAM3_IMAGE_STREAM_TILE


def main():
    t0 = time.time()
    w = ob.TrunkWeights(SEED)
    img = ob.u8(SEED, image_stream(0), (1008, 1008, 3))
    x = ob.encode_trunk(w, ob.image_input(img))
    rows = np.arange(0, x.shape[0], ROW_STEP)
    np.savez_compressed(os.path.join(HERE, "backbone_c4.npz"), rows=rows, x=x[rows],
                        mean=np.float64(x.mean()), std=np.float64(x.std()),
                        absmax=np.float64(np.abs(x).max()), seed=SEED)
    print("backbone golden", x.shape, x.std(), f"{time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
