"""GPU parity of the point-prompt mask decoder (sam_decode, sam3_model.c:
1239-1399) and of its upscaling kernels against the oracle's restatement,
same seeded weights, image features and points.

Tolerances: convt_scatter without activation is bit-exact (same fp32
operations); with GELU it differs only by the erf of the CUDA math library
against glibc's (rtol 1e-6, atol 1e-6). mask_logits sums 32 products in another order
(rtol 1e-5). The whole decode runs its Linears on bf16 tensor-core GEMMs
against the oracle's fp32: low-resolution logits cosine >= 0.999 and max
error <= 5% of the logits' range, IoU predictions within 0.01."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def cos_sim(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.mark.parametrize("P,H,W,Co,act,with_add", [(2, 5, 3, 8, 0, True),
                                                    (3, 4, 4, 4, 1, True),
                                                    (1, 72, 72, 64, 0, True),
                                                    (1, 3, 6, 12, 2, False)])
def test_convt_scatter_vs_oracle(cb, sb, ob, P, H, W, Co, act, with_add):
    G = ob.normal(31, 1, (P * H * W, Co * 4))
    bias = ob.normal(31, 2, (Co,))
    add = ob.normal(31, 3, (4 * H * W * Co,)) if with_add else None
    want = ob.convt_scatter(G, bias, add, P, H, W, Co, act)
    mG, mb = cb.upload(G, sb.F32), cb.upload(bias, sb.F32)
    ma = cb.upload(add, sb.F32) if with_add else None
    out = cb.alloc(want.nbytes, sb.F32)
    cb.convt_scatter(mG, out, mb, ma, P, H, W, Co, act)
    got = np.empty_like(want)
    cb.read(out, got)
    if act == 1:
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
    else:
        assert np.array_equal(got, want)


@pytest.mark.parametrize("P,npix", [(3, 77), (2, 288 * 288)])
def test_mask_logits_vs_oracle(cb, sb, ob, P, npix):
    U = ob.normal(32, 1, (P, npix, 32))
    hyper = ob.normal(32, 2, (P, 96))
    want = ob.mask_logits(U, hyper, P, npix)
    out = cb.alloc(want.nbytes, sb.F32)
    cb.mask_logits(cb.upload(U, sb.F32), cb.upload(hyper, sb.F32), out, P, npix)
    got = np.empty_like(want)
    cb.read(out, got)
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def _decoder(cb, sb, ob, seed, batch, std):
    dec = sb.Decoder(cb, batch)
    dec.init_random(seed, std)
    emb, s0, s1 = ob.decoder_image(seed)
    dec.set_image(cb.upload(emb, sb.F32), cb.upload(s0, sb.F32), cb.upload(s1, sb.F32))
    return dec, (emb, s0, s1)


def _check(got_iou, got_low, want_iou, want_low):
    c = cos_sim(got_low, want_low)
    assert c >= 0.999, c
    span = float(want_low.max() - want_low.min())
    assert np.abs(got_low - want_low).max() <= 0.05 * span
    assert np.abs(got_iou - want_iou).max() <= 0.01


@pytest.mark.parametrize("points", [[[100.5, 200.25], [800.0, 30.0]],
                                    [[0.0, 0.0], [1007.0, 1007.0], [503.5, 499.0]]])
def test_decoder_vs_oracle(cb, sb, ob, points):
    seed, std = 41, 0.05
    pts = np.array(points, np.float32)
    P = len(pts)
    dec, img = _decoder(cb, sb, ob, seed, 4, std)
    low = cb.alloc(P * 3 * 288 * 288 * 4, sb.F32)
    iou = dec.decode(pts, low)
    got = np.empty((P, 3, 288, 288), np.float32)
    cb.read(low, got)
    w = ob.DecoderWeights(seed, std)
    want_iou, want_low = ob.sam_decode(w, *img, pts)
    _check(iou, got, want_iou, want_low)
    dec.close()


def test_decoder_set_weight_equals_init_random(cb, sb, ob):
    """Loading every tensor from host fp32 data (a checkpoint loader's path)
    gives, bit for bit, the decode of the device-side random init."""
    seed, std = 43, 0.05
    pts = np.array([[300.0, 700.0], [12.0, 900.0]], np.float32)
    dec_a, img = _decoder(cb, sb, ob, seed, 2, std)
    low_a = cb.alloc(2 * 3 * 288 * 288 * 4, sb.F32)
    iou_a = dec_a.decode(pts, low_a)
    w = ob.DecoderWeights(seed, std)
    dec_b = sb.Decoder(cb, 2)
    for i, t in enumerate(w.t):
        dec_b.set_weight(i, t)
    dec_b.set_image(*[cb.upload(a, sb.F32) for a in img])
    low_b = cb.alloc(2 * 3 * 288 * 288 * 4, sb.F32)
    iou_b = dec_b.decode(pts, low_b)
    a = np.empty((2, 3, 288, 288), np.float32)
    b = np.empty_like(a)
    cb.read(low_a, a)
    cb.read(low_b, b)
    assert np.array_equal(a, b)
    assert np.array_equal(iou_a, iou_b)
    dec_a.close()
    dec_b.close()


def test_decoder_prompt_independent_of_batch(cb, sb, ob):
    """A prompt's outputs do not depend on the other prompts of its batch.
    The token->image attention splits its keys over a number of CTAs that
    depends on the batch size, so its fp32 sums round differently; a changed
    last bit can flip a later bf16 rounding of a GEMM operand, hence a bound
    of 0.1% of the logits' range rather than bitwise equality."""
    seed = 44
    dec, _ = _decoder(cb, sb, ob, seed, 3, 0.05)
    pts = np.array([[64.0, 64.0], [900.0, 100.0], [500.0, 600.0]], np.float32)
    low3 = cb.alloc(3 * 3 * 288 * 288 * 4, sb.F32)
    iou3 = dec.decode(pts, low3)
    low1 = cb.alloc(3 * 288 * 288 * 4, sb.F32)
    iou1 = dec.decode(pts[1:2], low1)
    a = np.empty((3, 3, 288, 288), np.float32)
    b = np.empty((1, 3, 288, 288), np.float32)
    cb.read(low3, a)
    cb.read(low1, b)
    span = float(a[1].max() - a[1].min())
    assert np.abs(b[0] - a[1]).max() <= 1e-3 * span
    assert np.abs(iou1[0] - iou3[1]).max() <= 1e-3
    dec.close()


def test_decoder_rejects_bad_arguments(cb, sb):
    dec = sb.Decoder(cb, 2)
    dec.init_random(1)
    low = cb.alloc(3 * 3 * 288 * 288 * 4, sb.F32)
    with pytest.raises(sb.CBError):
        dec.decode(np.zeros((1, 2), np.float32), low)  # no image set
    dec.close()
