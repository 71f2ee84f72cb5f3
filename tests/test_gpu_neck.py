"""GPU parity of the SimpleFPN neck (point_neck, sam3_model.c:1098-1110)
against the oracle's restatement, same seeded weights and trunk output.

Every convolution runs on the bf16 tensor-core GEMM (fp32 accumulation)
against the oracle's fp32, through up to four chained convolutions:
each output (image embedding, feat_s0, feat_s1) cosine >= 0.999 and
relative L2 error <= 3e-2."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def cos_sim(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _run(cb, sb, neck, x, ntile, grid):
    T = grid * grid
    outs = [cb.alloc(ntile * T * 256 * 4, sb.F32), cb.alloc(ntile * 16 * T * 32 * 4, sb.F32),
            cb.alloc(ntile * 4 * T * 64 * 4, sb.F32)]
    neck.run(x, ntile, *outs)
    shapes = [(ntile, T, 256), (ntile, 16 * T, 32), (ntile, 4 * T, 64)]
    res = []
    for m, shp in zip(outs, shapes):
        a = np.empty(shp, np.float32)
        cb.read(m, a)
        res.append(a)
    return res


@pytest.mark.parametrize("grid", [13, 24, 72])
def test_neck_vs_oracle(cb, sb, ob, grid):
    seed = 51
    neck = sb.Neck(cb, grid=grid, embed=1024, max_tiles=1)
    neck.init_random(seed, 0.02)
    x = ob.normal(seed, 9300, (grid * grid, 1024))
    got = _run(cb, sb, neck, cb.upload(x, sb.F32), 1, grid)
    want = ob.point_neck(ob.NeckWeights(seed, 0.02), x, grid)
    for g, w, name in zip(got, want, ("emb", "feat_s0", "feat_s1")):
        c, e = cos_sim(g[0], w), rel_l2(g[0], w)
        assert c >= 0.999 and e <= 3e-2, (name, c, e)
    neck.close()


@pytest.mark.parametrize("grid,ntile", [(24, 2), (72, 3)])
def test_neck_batch_equals_single_tiles(cb, sb, ob, grid, ntile):
    """Tiles batched into one call give, bit for bit, the per-tile results
    (at grid 72 the 3x3 convolutions of levels 0 and 1 run on CTA pairs)."""
    seed = 52
    neck = sb.Neck(cb, grid=grid, embed=1024, max_tiles=ntile)
    neck.init_random(seed, 0.02)
    xs = ob.normal(seed, 9301, (ntile, grid * grid, 1024))
    both = _run(cb, sb, neck, cb.upload(xs, sb.F32), ntile, grid)
    for t in range(ntile):
        one = _run(cb, sb, neck, cb.upload(xs[t], sb.F32), 1, grid)
        for a, b in zip(one, both):
            assert np.array_equal(a[0], b[t])
    neck.close()


def test_neck_set_weight_equals_init_random(cb, sb, ob):
    """Loading every tensor from host fp32 data (a checkpoint loader's path)
    gives the random init's outputs bit for bit."""
    seed, grid = 53, 24
    a = sb.Neck(cb, grid=grid, embed=1024)
    a.init_random(seed, 0.02)
    b = sb.Neck(cb, grid=grid, embed=1024)
    w = ob.NeckWeights(seed, 0.02)
    for i, t in enumerate(w.t):
        if ob.neck_tensor_info(i)[0]:
            b.set_weight(i, t)
    x = cb.upload(ob.normal(seed, 9302, (grid * grid, 1024)), sb.F32)
    for p, q in zip(_run(cb, sb, a, x, 1, grid), _run(cb, sb, b, x, 1, grid)):
        assert np.array_equal(p, q)
    a.close()
    b.close()


def test_neck_feeds_decoder(cb, sb, ob):
    """The neck's outputs are the decoder's image inputs: trunk output ->
    cb_neck_run -> cb_decoder_set_image -> cb_decode runs and gives the
    oracle's decode of the oracle's neck outputs."""
    seed, grid = 54, 72
    neck = sb.Neck(cb, grid=grid, embed=1024)
    neck.init_random(seed, 0.02)
    x = ob.normal(seed, 9303, (grid * grid, 1024))
    T = grid * grid
    emb, s0, s1 = (cb.alloc(T * 256 * 4, sb.F32), cb.alloc(16 * T * 32 * 4, sb.F32),
                   cb.alloc(4 * T * 64 * 4, sb.F32))
    neck.run(cb.upload(x, sb.F32), 1, emb, s0, s1)
    dec = sb.Decoder(cb, 2)
    dec.init_random(seed, 0.05)
    dec.set_image(emb, s0, s1)
    pts = np.array([[250.0, 300.0], [900.0, 850.0]], np.float32)
    low = cb.alloc(2 * 3 * 288 * 288 * 4, sb.F32)
    iou = dec.decode(pts, low)
    got = np.empty((2, 3, 288, 288), np.float32)
    cb.read(low, got)
    want_iou, want_low = ob.sam_decode(ob.DecoderWeights(seed, 0.05),
                                       *ob.point_neck(ob.NeckWeights(seed, 0.02), x, grid), pts)
    assert cos_sim(got, want_low) >= 0.999
    assert np.abs(iou - want_iou).max() <= 0.01
    dec.close()
    neck.close()
