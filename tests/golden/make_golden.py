"""Generate the golden vectors in tests/golden/ from the REFERENCE kernels.

The reference ships no kernel-level golden vectors or known-answer tests
(its tests need GRASS, an OpenCL device and the gated checkpoint). These
fixtures are outputs of the reference's own sam3_kernels.cl, compiled
unmodified as host C++ by oracle/Makefile (oracle/_ref/libsam3ref.so), on
inputs drawn from the seeded generator (include/sam3_synth.h). Only the
outputs are stored; tests regenerate the inputs from the seeds.

    make -C oracle ref REF=<reference tree> && python tests/golden/make_golden.py [case names]

Launch geometry is the reference host code's: layernorm with 256-item
work-groups for rows of >= 1024 channels (sam3_model.c:320), softmax_rows
with 256 (sam3_model.c:336), gemm_cpu_t / gemm_cpu_n (profile=cpu,
sam3_model.c:289-296), run1d kernels in groups of 256.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import binding as ob  # noqa: E402

SEED = 20261201


def cases():
    """(name, builder) pairs; builder(use_ref) -> dict of output arrays."""
    out = []

    def gemm_case(name, M, N, K, transb, act, with_bias, with_r, alpha, stream):
        def run(use_ref):
            A = ob.normal(SEED, stream, (M, K))
            B = ob.normal(SEED, stream + 1, (N, K) if transb else (K, N))
            bias = ob.normal(SEED, stream + 2, (N,)) if with_bias else None
            R0 = ob.normal(SEED, stream + 3, (M, N))
            Cm = R0.copy()
            f = ob.ref_gemm if use_ref else ob.gemm
            f(M, N, K, A, B, transb, Cm, bias=bias, R=Cm if with_r else None,
              alpha=alpha, act=act)
            return {"C": Cm}
        out.append((name, run))

    gemm_case("gemm_t_odd", 37, 29, 70, 1, 1, True, True, 0.5, 100)
    gemm_case("gemm_t_qk", 64, 64, 64, 1, 0, False, False, 0.125, 110)
    gemm_case("gemm_n_pv", 45, 64, 45, 0, 0, False, False, 1.0, 120)
    gemm_case("gemm_n_relu", 33, 20, 17, 0, 2, True, True, 1.0, 130)

    def ln_case(name, rows, Cn, act, stream):
        def run(use_ref):
            X = ob.normal(SEED, stream, (rows, Cn), 0.5, 2.0)
            g = ob.normal(SEED, stream + 1, (Cn,), 1.0, 0.1)
            b = ob.normal(SEED, stream + 2, (Cn,), 0.0, 0.1)
            if use_ref:
                return {"Y": ob.ref_layernorm(X, g, b, 1e-5, act,
                                              256 if Cn >= 1024 else 64)}
            return {"Y": ob.layernorm(X, g, b, 1e-5, act)}
        out.append((name, run))

    ln_case("layernorm_1024", 24, 1024, 0, 200)
    ln_case("layernorm_256_gelu", 16, 256, 1, 210)

    def softmax_case(name, rows, L, stream):
        def run(use_ref):
            S = ob.normal(SEED, stream, (rows, L), 0.0, 3.0)
            return {"P": ob.ref_softmax_rows(S, 256 if L >= 256 else 64)
                    if use_ref else ob.softmax_rows(S)}
        out.append((name, run))

    softmax_case("softmax_576", 12, 576, 300)
    softmax_case("softmax_100", 10, 100, 310)

    def rope_case(name, side, nwin, E, stream):
        def run(use_ref):
            N = side * side
            qkv = ob.normal(SEED, stream, (nwin * N, 3 * E))
            cs = ob.rope_axial(side, 64)
            return {"qkv": ob.rope_apply(qkv, E, 64, N, cs, use_ref=use_ref)}
        out.append((name, run))

    rope_case("rope_win6", 6, 2, 128, 400)

    def attn_case(name, side, nseq, E, stream):
        def run(use_ref):
            N = side * side
            qkv = ob.normal(SEED, stream, (nseq * N, 3 * E))
            cs = ob.rope_axial(side, 64)
            qkv = ob.rope_apply(qkv, E, 64, N, cs, use_ref=use_ref)
            f = ob.ref_attention if use_ref else ob.attention
            return {"O": f(qkv, nseq, N, E, E // 64, 64, 0.125)}
        out.append((name, run))

    attn_case("attention_win6", 6, 3, 128, 500)
    attn_case("attention_win5_odd", 5, 2, 128, 510)

    def window_case(name, H, Cn, ws, stream):
        def run(use_ref):
            nwx = (H + ws - 1) // ws
            X = ob.normal(SEED, stream, (H * H, Cn))
            Wd = ob.normal(SEED, stream + 1, (nwx * nwx * ws * ws, Cn))
            part = np.empty((nwx * nwx * ws * ws, Cn), np.float32)
            X2 = X.copy()
            if use_ref:
                ob.ref().ref_window_partition(X, part, H, Cn, ws, nwx)
                ob.ref().ref_window_unpartition_add(X2, Wd, H, Cn, ws, nwx)
            else:
                ob.lib().or_window_partition(X, part, H, Cn, ws, nwx)
                ob.lib().or_window_unpartition_add(X2, Wd, H, Cn, ws, nwx)
            return {"part": part, "unpart": X2}
        out.append((name, run))

    window_case("window_pad", 10, 8, 4, 600)

    def im2col_case(name, grid, ps, stream):
        def run(use_ref):
            side = grid * ps + 3
            img = ob.normal(SEED, stream, (3, side, side))
            col = np.empty((grid * grid, 3 * ps * ps), np.float32)
            (ob.ref().ref_patch_im2col if use_ref else ob.lib().or_patch_im2col)(
                img, col, side, grid, ps)
            return {"col": col}
        out.append((name, run))

    im2col_case("patch_im2col", 4, 5, 700)

    def add_case(name, n, bmod, stream):
        def run(use_ref):
            a = ob.normal(SEED, stream, (n,))
            b = ob.normal(SEED, stream + 1, (bmod,))
            o = np.empty(n, np.float32)
            (ob.ref().ref_add_bcast if use_ref else ob.lib().or_add_bcast)(o, a, b, n, bmod)
            return {"out": o}
        out.append((name, run))

    add_case("add_bcast", 1000, 48, 800)

    def mha_case(name, P, Nq, Nk, dint, shared_kv, stream):
        def run(use_ref):
            q = ob.normal(SEED, stream, (P * Nq, dint))
            kvp = 1 if shared_kv else P
            k = ob.normal(SEED, stream + 1, (kvp * Nk, dint))
            v = ob.normal(SEED, stream + 2, (kvp * Nk, dint))
            sk = 0 if shared_kv else Nk * dint
            return {"O": ob.mha(P, Nq, Nk, dint, q, Nq * dint, k, sk, v, sk,
                                use_ref=use_ref)}
        out.append((name, run))

    mha_case("mha_self", 3, 8, 8, 256, False, 900)
    mha_case("mha_t2i_many", 2, 8, 300, 128, False, 910)
    mha_case("mha_t2i_shared", 2, 7, 1000, 128, True, 920)
    mha_case("mha_i2t_few", 2, 40, 7, 128, False, 930)

    def convt_case(name, P, H, W, Co, act, with_add, stream):
        def run(use_ref):
            G = ob.normal(SEED, stream, (P * H * W, Co * 4))
            bias = ob.normal(SEED, stream + 1, (Co,))
            add = ob.normal(SEED, stream + 2, (4 * H * W * Co,)) if with_add else None
            return {"out": ob.convt_scatter(G, bias, add, P, H, W, Co, act, use_ref=use_ref)}
        out.append((name, run))

    convt_case("convt_scatter_add", 2, 5, 3, 8, 0, True, 1000)
    convt_case("convt_scatter_gelu", 3, 4, 4, 4, 1, True, 1010)
    convt_case("convt_scatter_relu_noadd", 1, 3, 6, 12, 2, False, 1020)

    def logits_case(name, P, npix, stream):
        def run(use_ref):
            U = ob.normal(SEED, stream, (P, npix, 32))
            hyper = ob.normal(SEED, stream + 1, (P, 96))
            return {"out": ob.mask_logits(U, hyper, P, npix, use_ref=use_ref)}
        out.append((name, run))

    logits_case("mask_logits", 3, 77, 1100)

    def im2col_case(name, H, W, Cn, t0, n, stream):
        def run(use_ref):
            X = ob.normal(SEED, stream, (H * W, Cn))
            return {"col": ob.im2col3x3(X, H, W, Cn, t0, n, use_ref=use_ref)}
        out.append((name, run))

    im2col_case("im2col3x3_band", 7, 5, 6, 9, 20, 1200)

    def softmax_ext_case(name, Nq, L, heads, h0, causal, W, stream):
        def run(use_ref):
            S = ob.normal(SEED, stream, (heads * Nq, L), 0.0, 3.0)
            dy = dx = None
            if W:
                dy = ob.normal(SEED, stream + 1, (Nq * (L // W) * 8,), 0.0, 2.0)
                dx = ob.normal(SEED, stream + 2, (Nq * W * 8,), 0.0, 2.0)
            return {"P": ob.softmax_ext(S, Nq, h0, causal, dy, dx, W, 8, use_ref=use_ref)}
        out.append((name, run))

    softmax_ext_case("softmax_ext_rpb", 5, 48, 2, 3, 0, 8, 1300)
    softmax_ext_case("softmax_ext_causal", 12, 12, 3, 0, 1, 0, 1310)
    return out


def main(only=None):
    """Write every case's fixture (or only the named ones)."""
    if not ob.have_ref():
        sys.exit("oracle/_ref/libsam3ref.so missing: run make -C oracle "
                 "where the reference tree is present")
    for name, run in cases():
        if only and name not in only:
            continue
        res = run(True)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **res)
        print(name, {k: v.shape for k, v in res.items()})


if __name__ == "__main__":
    main(sys.argv[1:] or None)
