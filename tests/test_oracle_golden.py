"""The oracle (C restatement) against golden vectors produced by the
reference's own kernels (tests/golden/make_golden.py), and, where the
compiled reference is present, against it live on fresh seeded inputs."""
import os

import numpy as np
import pytest

from tests.golden.make_golden import cases

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
# Bit-exact cases: the restatement keeps the reference's order of operations
# exactly. The others differ only in the order of a work-group reduction
# (256-way tree in the reference, serial in the oracle).
REDUCTION_ORDER = {"layernorm_1024", "layernorm_256_gelu", "softmax_576",
                   "softmax_100", "attention_win6", "attention_win5_odd",
                   "softmax_ext_rpb", "softmax_ext_causal"}


@pytest.mark.parametrize("name,run", cases(), ids=[c[0] for c in cases()])
def test_oracle_matches_reference_golden(name, run):
    golden = np.load(os.path.join(GOLDEN, name + ".npz"))
    got = run(False)
    for k in golden.files:
        g, o = golden[k], got[k]
        assert g.shape == o.shape
        if name in REDUCTION_ORDER:
            np.testing.assert_allclose(o, g, rtol=2e-6, atol=2e-6)
        else:
            assert np.array_equal(o, g), f"{name}/{k} not bit-exact"


def test_oracle_vs_live_reference_random(ob):
    if not ob.have_ref():
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(7)
    for (M, N, K, tb) in [(19, 23, 41, 1), (50, 9, 8, 0), (2, 4, 9, 1)]:
        A = rng.standard_normal((M, K)).astype(np.float32)
        B = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
        c1 = np.zeros((M, N), np.float32)
        c2 = np.zeros((M, N), np.float32)
        ob.gemm(M, N, K, A, B, tb, c1, alpha=0.25, act=1)
        ob.ref_gemm(M, N, K, A, B, tb, c2, alpha=0.25, act=1)
        assert np.array_equal(c1, c2)
    X = rng.standard_normal((5, 300)).astype(np.float32)
    g = np.ones(300, np.float32)
    b = np.zeros(300, np.float32)
    assert np.array_equal(ob.layernorm(X, g, b), ob.ref_layernorm(X, g, b, local=1))
    S = rng.standard_normal((7, 333)).astype(np.float32)
    assert np.array_equal(ob.softmax_rows(S), ob.ref_softmax_rows(S, local=1))


def test_generator_is_deterministic_and_normal(ob):
    a = ob.normal(1, 2, (200000,))
    b = ob.normal(1, 2, (200000,))
    c = ob.normal(1, 3, (200000,))
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    assert np.abs(a).max() < 6.0
    u = ob.u8(5, 6, (100000,))
    assert u.min() == 0 and u.max() == 255 and abs(u.mean() - 127.5) < 1.0


def test_rope_table_layout(ob):
    cs = ob.rope_axial(4, 64, 10000.0)
    # position p = y * 4 + x; pairs j < 16 rotate by x * f_j, j >= 16 by y
    p = 2 * 4 + 3
    f0 = 1.0
    assert np.isclose(cs[p, 0, 0], np.cos(3 * f0)) and np.isclose(cs[p, 0, 1], np.sin(3 * f0))
    assert np.isclose(cs[p, 16, 0], np.cos(2 * f0))
    f5 = 10000.0 ** (-4 * 5 / 64)
    assert np.isclose(cs[p, 5, 1], np.sin(3 * f5), atol=1e-6)
