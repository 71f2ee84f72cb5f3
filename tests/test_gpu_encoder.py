"""GPU parity of the PE backbone (the encoder of the C-ABI) against the
oracle's restatement of sam_encode_trunk / vit_block, same seeded weights
and tiles. embeddings cosine >= 0.999 vs fp32."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "backbone_c4.npz")


def cos_sim(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def image_stream(tile):
    return 3 * 1000003 + tile


def test_encoder_two_blocks_vs_oracle(cb, sb, ob):
    """Prologue + one windowed and one global block, full 72 x 72 grid."""
    seed = 5
    enc = sb.Encoder(cb, max_tiles=1, depth=2, global_blocks=(1,))
    enc.init_random(seed)
    img = ob.u8(seed, image_stream(0), (1008, 1008, 3))
    tiles = cb.upload(img, sb.U8)
    out = cb.alloc(5184 * 1024 * 4, sb.F32)
    enc.encode_tiles(tiles, 1, out)
    got = np.empty((5184, 1024), np.float32)
    cb.read(out, got)
    cb.sync()
    w = ob.TrunkWeights(seed, depth=2, global_blocks=(1,))
    want = ob.encode_trunk(w, ob.image_input(img))
    c = cos_sim(got, want)
    assert c >= 0.999, c
    assert np.abs(got - want).max() < 0.1 * np.abs(want).max()
    enc.close()


def test_encoder_batch_equals_single_tiles(cb, sb, ob):
    """Batching tiles into one GEMM M dimension does not change results."""
    seed = 6
    enc = sb.Encoder(cb, max_tiles=2, depth=2, global_blocks=(0,))
    enc.init_random(seed)
    imgs = np.stack([ob.u8(seed, image_stream(t), (1008, 1008, 3)) for t in range(2)])
    tiles = cb.upload(imgs, sb.U8)
    out2 = cb.alloc(2 * 5184 * 1024 * 4, sb.F32)
    enc.encode_tiles(tiles, 2, out2)
    both = np.empty((2, 5184, 1024), np.float32)
    cb.read(out2, both)
    for t in range(2):
        one = cb.upload(imgs[t], sb.U8)
        out1 = cb.alloc(5184 * 1024 * 4, sb.F32)
        enc.encode_tiles(one, 1, out1)
        single = np.empty((5184, 1024), np.float32)
        cb.read(out1, single)
        assert np.array_equal(single, both[t])
    enc.close()


@pytest.mark.parametrize("ntile", [3, 8, 11, 16, 21])
def test_encode_tiles_host_pipeline_equals_device_path(cb, sb, ob, ntile):
    """The host-buffer entry point (chunks of about a quarter of the tiles,
    at least 4, with copies in and out overlapping the encode: 3 tiles = one
    chunk, 8 = 2 x 4 as one GPU of eight gets, 11 = 4 + 4 + 3, 16 = 4 x 4,
    21 = 6 + 6 + 5 + a final 4) returns,
    bit for bit, what the device-buffer path returns for the same tiles, and
    a second call reuses its staging buffers."""
    seed = 8
    enc = sb.Encoder(cb, max_tiles=ntile, depth=1, global_blocks=(0,))
    enc.init_random(seed)
    imgs = np.stack([ob.u8(seed, image_stream(t), (1008, 1008, 3)) for t in range(ntile)])
    tiles = cb.upload(imgs, sb.U8)
    out = cb.alloc(ntile * 5184 * 1024 * 4, sb.F32)
    enc.encode_tiles(tiles, ntile, out)
    want = np.empty((ntile, 5184, 1024), np.float32)
    cb.read(out, want)
    cb.sync()
    host_in = torch.from_numpy(imgs).pin_memory()
    host_out = torch.empty(ntile, 5184, 1024, dtype=torch.float32).pin_memory()
    for _ in range(2):
        host_out.zero_()
        enc.encode_tiles_host(host_in, host_out)
        assert np.array_equal(host_out.numpy(), want)
    enc.close()


def test_encode_blocks_matches_oracle_vit_block(cb, sb, ob):
    """cb_encode_blocks on raster tokens == oracle vit_block, per block kind."""
    seed = 7
    enc = sb.Encoder(cb, max_tiles=1, depth=2, global_blocks=(1,))
    enc.init_random(seed)
    w = ob.TrunkWeights(seed, depth=2, global_blocks=(1,))
    x0 = ob.normal(seed, 99, (5184, 1024))
    for blk in (0, 1):
        mx = cb.upload(x0, sb.F32)
        enc.encode_blocks(mx, 1, blk, blk + 1)
        got = np.empty_like(x0)
        cb.read(mx, got)
        want = x0.copy()
        ob.encode_trunk(w, None, blk, blk + 1, x=want)
        assert cos_sim(got - x0, want - x0) >= 0.999
    enc.close()


def test_encoder_full_backbone_vs_golden(cb, sb):
    """Config 4: the whole 32-block trunk on one tile vs the oracle's output
    (tests/golden/make_backbone_golden.py)."""
    if not os.path.exists(GOLDEN):
        pytest.skip("backbone golden fixture missing")
    g = np.load(GOLDEN)
    seed = int(g["seed"])
    enc = sb.Encoder(cb, max_tiles=1)
    enc.init_random(seed)
    from oracle import binding as ob
    img = ob.u8(seed, image_stream(0), (1008, 1008, 3))
    tiles = cb.upload(img, sb.U8)
    out = cb.alloc(5184 * 1024 * 4, sb.F32)
    enc.encode_tiles(tiles, 1, out)
    got = np.empty((5184, 1024), np.float32)
    cb.read(out, got)
    cb.sync()
    rows = g["rows"]
    c = cos_sim(got[rows], g["x"])
    assert c >= 0.999, c
    assert abs(float(got.std()) - float(g["std"])) < 0.01 * float(g["std"])
    enc.close()


def _load_checkpoint(enc, w):
    """Push every tensor of oracle TrunkWeights through cb_encoder_set_weight
    in the checkpoint's shapes, as a loader following load_encoder
    (sam3_model.c:473-581) would."""
    E, p = w.E, w.patch
    enc.set_weight("PATCH_W", 0, w.pe_w.reshape(E, 3, p, p))
    enc.set_weight("POS", 0, w.pos)  # [grid^2, E], raster order
    enc.set_weight("LN_PRE_W", 0, w.lnpw)
    enc.set_weight("LN_PRE_B", 0, w.lnpb)
    enc.set_weight("ROPE_WIN", 0, w.rope_win.reshape(w.window * w.window, w.hd // 2, 2))
    enc.set_weight("ROPE_GLOB", 0, w.rope_glob.reshape(w.grid * w.grid, w.hd // 2, 2))
    for i, b in enumerate(w.blocks):
        for name, key in (("N1_W", "n1w"), ("N1_B", "n1b"), ("QKV_W", "qkvw"),
                          ("QKV_B", "qkvb"), ("PROJ_W", "projw"), ("PROJ_B", "projb"),
                          ("N2_W", "n2w"), ("N2_B", "n2b"), ("FC1_W", "l1w"),
                          ("FC1_B", "l1b"), ("FC2_W", "l2w"), ("FC2_B", "l2b")):
            enc.set_weight(name, i, b[key])


def test_encoder_set_weight_equals_init_random(cb, sb, ob):
    """Loading every tensor from host fp32 data in checkpoint shapes (the
    loader's path: patch weight padded to the GEMM's K, pos_embed permuted
    to window-major rows, RoPE tables, every block tensor) gives, bit for
    bit, the encode of the device-side random init."""
    seed = 17
    img = ob.u8(seed, image_stream(0), (1008, 1008, 3))
    tiles = cb.upload(img, sb.U8)
    outs = []
    for loaded in (False, True):
        enc = sb.Encoder(cb, max_tiles=1, depth=2, global_blocks=(1,))
        if loaded:
            _load_checkpoint(enc, ob.TrunkWeights(seed, depth=2, global_blocks=(1,)))
        else:
            enc.init_random(seed)
        out = cb.alloc(5184 * 1024 * 4, sb.F32)
        enc.encode_tiles(tiles, 1, out)
        got = np.empty((5184, 1024), np.float32)
        cb.read(out, got)
        cb.sync()
        outs.append(got)
        enc.close()
    assert np.array_equal(outs[0], outs[1])


def test_encoder_pos_embed_tiled_from_pretrain_grid_vs_oracle(cb, sb, ob):
    """A pos_embed with visible structure: a 24 x 24 pretraining grid (plus
    the class token that SAM 3 drops) tiled over the 72 x 72 grid as
    tile_abs_pos does (sam3_model.c:492-498), loaded through set_weight and
    compared with the oracle, which adds it in raster order. A wrong
    raster -> window-major permutation of POS fails this test, whereas the
    init_random comparison above would not see it (both paths permute)."""
    seed = 18
    w = ob.TrunkWeights(seed, depth=2, global_blocks=(1,))
    pt = 24
    pe = ob.normal(seed, 77, (1 + pt * pt, w.E), 0.0, 0.5)
    i = np.arange(w.grid * w.grid)
    y, x = i // w.grid % pt, i % w.grid % pt
    w.pos = np.ascontiguousarray(pe[1 + y * pt + x])
    enc = sb.Encoder(cb, max_tiles=1, depth=2, global_blocks=(1,))
    _load_checkpoint(enc, w)
    img = ob.u8(seed, image_stream(0), (1008, 1008, 3))
    tiles = cb.upload(img, sb.U8)
    out = cb.alloc(5184 * 1024 * 4, sb.F32)
    enc.encode_tiles(tiles, 1, out)
    got = np.empty((5184, 1024), np.float32)
    cb.read(out, got)
    cb.sync()
    want = ob.encode_trunk(w, ob.image_input(img))
    c = cos_sim(got, want)
    assert c >= 0.999, c
    assert np.abs(got - want).max() < 0.1 * np.abs(want).max()
    enc.close()


def test_encoder_set_weight_rejects_wrong_shapes(cb, sb):
    enc = sb.Encoder(cb, max_tiles=1, depth=2, global_blocks=(1,))
    for which, block, n in (("PATCH_W", 0, 1024 * 588 - 1), ("POS", 0, 5184 * 1024 + 1),
                            ("ROPE_WIN", 0, 576 * 32), ("QKV_W", 0, 10), ("FC1_B", 1, 1024),
                            ("N1_W", 2, 1024)):
        with pytest.raises(sb.CBError):
            enc.set_weight(which, block, np.zeros(n, np.float32))
    enc.close()
