"""The input path's resize (aa_resize, image.c:209-339) in the oracle against
golden vectors from PyTorch's uint8 antialiased bilinear interpolation
(tests/golden/make_resize_golden.py), and the float normalisation of
image_encoder_input (image.c:346-371). CPU only; the GPU path is checked
against the oracle in tests/test_gpu_input.py."""
import hashlib
import os

import numpy as np

from tests.golden.make_resize_golden import BIG, CASES, image

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_resize_small_cases_match_torch_golden(ob):
    for i, (name, h, w, side) in enumerate(CASES):
        want = np.load(os.path.join(GOLDEN, name + ".npz"))["out"]
        assert np.array_equal(ob.aa_resize(image(i, h, w), side, side), want), name


def test_resize_encoder_size_matches_torch_digest(ob):
    digests = {}
    with open(os.path.join(GOLDEN, "resize_big.sha256")) as f:
        for line in f:
            name, h, w, side, d = line.split()
            digests[name] = (int(h), int(w), int(side), d)
    for j, (name, h, w, side) in enumerate(BIG):
        assert digests[name][:3] == (h, w, side)
        got = ob.aa_resize(image(100 + j, h, w), side, side)
        assert hashlib.sha256(got.tobytes()).hexdigest() == digests[name][3], name


def test_image_encoder_input_crop_and_normalisation(ob):
    img = image(7, 300, 400)
    # a crop already at the output size is copied, not resampled
    out = ob.image_encoder_input(img, 50, 20, 64, 64, side=64)
    crop = img[20:84, 50:114]
    want = (crop.transpose(2, 0, 1).astype(np.float32) / np.float32(255) - np.float32(0.5)) \
        / np.float32(0.5)
    assert np.array_equal(out, want)
    # otherwise the crop is resized first
    out = ob.image_encoder_input(img, 10, 30, 200, 150, side=64)
    rs = ob.aa_resize(np.ascontiguousarray(img[30:180, 10:210]), 64, 64)
    want = (rs.transpose(2, 0, 1).astype(np.float32) / np.float32(255) - np.float32(0.5)) \
        / np.float32(0.5)
    assert np.array_equal(out, want)
