"""GPU input path (cb_image_encoder_input: crop, uint8 antialiased resize,
normalisation) against the oracle's restatement of image_encoder_input
(image.c:346-371). Integer resize: bit-exact; the float normalisation is the
same IEEE operations: bit-exact."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from tests.golden.make_resize_golden import image  # noqa: E402


@pytest.mark.parametrize("rows,cols,x0,y0,w,h", [
    (1600, 2200, 37, 91, 1500, 1400),    # downscale both axes
    (900, 1200, 100, 50, 700, 640),      # upscale both axes
    (1100, 1100, 3, 5, 1010, 1003),      # near the output size
    (1200, 1300, 120, 77, 1008, 1008),   # already the output size: copied
    (500, 3000, 0, 0, 3000, 500),        # extreme aspect ratio
])
def test_image_encoder_input_vs_oracle(cb, sb, ob, rows, cols, x0, y0, w, h):
    img = image(200 + rows % 97, rows, cols)
    dimg = cb.upload(img, sb.U8)
    tiles = cb.alloc(2 * 1008 * 1008 * 3, sb.U8)
    chw = cb.alloc(3 * 1008 * 1008 * 4, sb.F32)
    cb.image_encoder_input(dimg, cols, rows, x0, y0, w, h, 1008, tiles=tiles, tile=1, chw=chw)
    got_t = np.empty((2, 1008, 1008, 3), np.uint8)
    got_f = np.empty((3, 1008, 1008), np.float32)
    cb.read(tiles, got_t)
    cb.read(chw, got_f)
    crop = np.ascontiguousarray(img[y0:y0 + h, x0:x0 + w])
    want_t = crop if (w, h) == (1008, 1008) else ob.aa_resize(crop, 1008, 1008)
    assert np.array_equal(got_t[1], want_t)
    assert np.array_equal(got_f, ob.image_encoder_input(img, x0, y0, w, h))


def test_image_encoder_input_rejects_out_of_image_crop(cb, sb):
    dimg = cb.alloc(100 * 100 * 3, sb.U8)
    tiles = cb.alloc(1008 * 1008 * 3, sb.U8)
    with pytest.raises(sb.CBError):
        cb.image_encoder_input(dimg, 100, 100, 50, 50, 60, 10, 1008, tiles=tiles)


def test_resized_tile_feeds_encoder(cb, sb, ob):
    """The device tile is cb_encode_tiles' input: encoding it equals encoding
    the same tile uploaded from the host."""
    img = image(300, 1300, 1700)
    dimg = cb.upload(img, sb.U8)
    tiles = cb.alloc(1008 * 1008 * 3, sb.U8)
    cb.image_encoder_input(dimg, 1700, 1300, 0, 0, 1700, 1300, 1008, tiles=tiles)
    enc = sb.Encoder(cb, max_tiles=1, depth=1, global_blocks=(0,))
    enc.init_random(9)
    out_a = cb.alloc(5184 * 1024 * 4, sb.F32)
    enc.encode_tiles(tiles, 1, out_a)
    host_tile = ob.aa_resize(img, 1008, 1008)
    out_b = cb.alloc(5184 * 1024 * 4, sb.F32)
    enc.encode_tiles(cb.upload(host_tile, sb.U8), 1, out_b)
    a = np.empty((5184, 1024), np.float32)
    b = np.empty_like(a)
    cb.read(out_a, a)
    cb.read(out_b, b)
    assert np.array_equal(a, b)
    enc.close()
