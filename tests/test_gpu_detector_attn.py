"""GPU parity of the detector's attention (cb_attend, the attend of
sam3_text.c:305-343 with softmax_ext, sam3_kernels.cl:889-921) against the
oracle's restatement: fp32 CUDA-core path (causal mask, box relative
position bias, few or many keys) max-abs <= 1e-4 relative to the output
scale; tensor-core paths (fusion-encoder self-attention; queries over the
image with or without the box bias; bf16 operands, heads zero-padded to 64)
cosine >= 0.9999, max-abs <= 1e-2 (relative to the output scale where a
bias makes rows peaked)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _run(cb, sb, Q, K, V, heads, hd, causal=0, dy=None, dx=None, W=0, mode=0):
    Nq, Nk = Q.shape[0], K.shape[0]
    O = cb.alloc(Nq * heads * hd * 4, sb.F32)
    up = lambda a: cb.upload(np.ascontiguousarray(a, np.float32), sb.F32)  # noqa: E731
    cb.attend(Nq, Nk, heads, hd, up(Q), Q.shape[1], up(K), K.shape[1], up(V), V.shape[1], O,
              heads * hd, causal, up(dy) if dy is not None else None,
              up(dx) if dx is not None else None, W, mode)
    out = np.empty((Nq, heads * hd), np.float32)
    cb.read(O, out)
    return out


@pytest.mark.parametrize("Nq,Nk,heads,hd,causal,rpb", [
    (201, 5184, 8, 32, 0, True),    # decoder queries over the image, box bias
    (201, 201, 8, 32, 0, False),    # decoder self-attention
    (201, 33, 8, 32, 0, False),     # queries over the prompt tokens
    (32, 32, 16, 64, 1, False),     # causal text encoder
    (300, 700, 4, 64, 0, True),     # bias on another key grid
])
def test_attend_fp32_vs_oracle(cb, sb, ob, Nq, Nk, heads, hd, causal, rpb):
    E = heads * hd
    Q = ob.normal(61, 1, (Nq, E))
    K = ob.normal(61, 2, (Nk, E))
    V = ob.normal(61, 3, (Nk, E))
    dy = dx = None
    W = 0
    if rpb:
        W = 72 if Nk == 5184 else 28
        dy = ob.normal(61, 4, (Nq * (Nk // W) * heads,), 0.0, 2.0)
        dx = ob.normal(61, 5, (Nq * W * heads,), 0.0, 2.0)
    got = _run(cb, sb, Q, K, V, heads, hd, causal, dy, dx, W, mode=1)
    want = ob.attend(Q, K, V, heads, hd, causal, dy, dx, W)
    assert np.abs(got - want).max() <= 1e-4 * max(1.0, float(np.abs(want).max()))


@pytest.mark.parametrize("N", [1500, 5184])
def test_attend_tensor_core_fusion_encoder_vs_oracle(cb, sb, ob, N):
    heads, hd = 8, 32
    E = heads * hd
    Q = ob.normal(62, 1, (N, E))
    K = ob.normal(62, 2, (N, E))
    V = ob.normal(62, 3, (N, E))
    got = _run(cb, sb, Q, K, V, heads, hd, mode=0)
    want = ob.attend(Q, K, V, heads, hd)
    a, b = got.astype(np.float64).ravel(), want.astype(np.float64).ravel()
    assert a @ b / (np.linalg.norm(a) * np.linalg.norm(b)) >= 0.9999
    assert np.abs(got - want).max() <= 1e-2


@pytest.mark.parametrize("Nq,Nk,heads,hd,rpb", [
    (201, 5184, 8, 32, True),    # the detector decoder's queries over the image, box bias
    (300, 1500, 4, 64, False),   # ragged query and key tiles, no bias
    (77, 1100, 2, 32, True),     # one query tile, keys split many ways, bias on a 44-wide grid
])
def test_attend_tensor_core_cross_vs_oracle(cb, sb, ob, Nq, Nk, heads, hd, rpb):
    """Queries over many keys on the tcgen05 kernel (k_attn_tc_cross): heads
    padded to 64 in bf16, the box bias as a dense per-score term, the keys
    split over CTAs and merged when the query tiles are few. Bound of the
    other tensor-core attention tests, max-abs relative to the output scale
    (the bias of std 2 makes some rows peaked)."""
    E = heads * hd
    Q = ob.normal(63, 1, (Nq, E))
    K = ob.normal(63, 2, (Nk, E))
    V = ob.normal(63, 3, (Nk, E))
    dy = dx = None
    W = 0
    if rpb:
        W = 72 if Nk == 5184 else 44
        dy = ob.normal(63, 4, (Nq * (Nk // W) * heads,), 0.0, 2.0)
        dx = ob.normal(63, 5, (Nq * W * heads,), 0.0, 2.0)
    got = _run(cb, sb, Q, K, V, heads, hd, 0, dy, dx, W, mode=0)
    want = ob.attend(Q, K, V, heads, hd, 0, dy, dx, W)
    a, b = got.astype(np.float64).ravel(), want.astype(np.float64).ravel()
    assert np.isfinite(got).all()
    assert a @ b / (np.linalg.norm(a) * np.linalg.norm(b)) >= 0.9999
    assert np.abs(got - want).max() <= 1e-2 * max(1.0, float(np.abs(want).max()))


@pytest.mark.parametrize("Nq,Nk,hd", [(1500, 1500, 32), (300, 1500, 32), (150, 2000, 64)])
def test_attend_tensor_core_strided_output_vs_oracle(cb, sb, ob, Nq, Nk, hd):
    """Row strides wider than the heads (inputs and output): the tensor-core
    kernel writes each head's hd real columns straight into the caller's
    rows and leaves the columns past the heads untouched."""
    heads = 4
    E = heads * hd
    lq, lk, lo = E + 4, E + 8, E + 12
    Q = ob.normal(64, 1, (Nq, lq))
    K = ob.normal(64, 2, (Nk, lk))
    V = ob.normal(64, 3, (Nk, lk))
    up = lambda a: cb.upload(np.ascontiguousarray(a, np.float32), sb.F32)  # noqa: E731
    O = up(np.full((Nq, lo), 7.0, np.float32))
    cb.attend(Nq, Nk, heads, hd, up(Q), lq, up(K), lk, up(V), lk, O, lo, 0, None, None, 0, 0)
    got = np.empty((Nq, lo), np.float32)
    cb.read(O, got)
    want = ob.attend(Q[:, :E], K[:, :E], V[:, :E], heads, hd)
    assert (got[:, E:] == 7.0).all()
    a, b = got[:, :E].astype(np.float64).ravel(), want.astype(np.float64).ravel()
    assert a @ b / (np.linalg.norm(a) * np.linalg.norm(b)) >= 0.9999
    assert np.abs(got[:, :E] - want).max() <= 1e-2


def test_attend_rejects_bad_shapes(cb, sb):
    m = cb.alloc(64 * 64 * 4, sb.F32)
    with pytest.raises(sb.CBError):
        cb.attend(8, 8, 2, 48, m, 96, m, 96, m, 96, m, 96)  # hd 48 unsupported
