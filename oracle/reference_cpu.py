"""The reference's CPU path of the backbone, for the timed CPU baseline
(test infrastructure only).

vit_block (sam3_model.c:981-1028) and the sam_encode_trunk prologue
(sam3_model.c:1112-1135) orchestrated in Python over the REFERENCE kernels
themselves (oracle/_ref: sam3_kernels.cl compiled as host C++), with the
profile=cpu GEMM kernels gemm_cpu_t / gemm_cpu_n (sam3_model.c:249-296) on
OpenMP threads. The work-group reductions (layernorm, softmax_rows) run
with one work-item per group: on a CPU device PoCL turns a 256-item group
into loops, and one-item groups are the loop form the executor can run at
that speed (the 256-item form needs one fiber per work-item).
"""
import numpy as np

from . import binding as ob


class RefTrunk:
    def __init__(self, seed, depth=2, global_blocks=(1,), **kw):
        self.w = ob.TrunkWeights(seed, depth=depth, global_blocks=global_blocks, **kw)
        self.r = ob.ref()

    def prologue(self, rgb):
        w = self.w
        T, E, K = w.grid * w.grid, w.E, 3 * w.patch * w.patch
        img = ob.image_input(rgb)
        col = np.empty((T, K), np.float32)
        self.r.ref_patch_im2col(img, col, w.img, w.grid, w.patch)
        x = np.zeros((T, E), np.float32)
        ob.ref_gemm(T, E, K, col, w.pe_w, 1, x)
        self.r.ref_add_bcast(x, x, w.pos.reshape(-1), T * E, T * E)
        x2 = np.empty_like(x)
        self.r.ref_layernorm(x, x2, w.lnpw, w.lnpb, T, E, 1e-5, 0, 1)
        return x2

    def block(self, x, i):
        w = self.w
        b = w.blocks[i]
        G, E, hd = w.grid, w.E, w.hd
        T = G * G
        s = b["window"] or G
        nwx = (G + s - 1) // s
        nwin, N = nwx * nwx, s * s
        rows = nwin * N
        xn = np.empty_like(x)
        self.r.ref_layernorm(x, xn, b["n1w"], b["n1b"], T, E, 1e-5, 0, 1)
        A = xn
        if b["window"]:
            A = np.empty((rows, E), np.float32)
            self.r.ref_window_partition(xn, A, G, E, s, nwx)
        qkv = np.empty((rows, 3 * E), np.float32)
        ob.ref_gemm(rows, 3 * E, E, A, b["qkvw"], 1, qkv, bias=b["qkvb"])
        cs = w.rope_win if b["window"] else w.rope_glob
        self.r.ref_rope_apply(qkv, rows, E, hd, N, np.ascontiguousarray(cs.reshape(-1)))
        hc = max(1, min(E // hd, (512 << 20) // 4 // (nwin * N * N)))
        attn = ob.ref_attention(qkv, nwin, N, E, E // hd, hd, 1.0 / np.sqrt(hd),
                                head_chunk=hc, softmax_local=1)
        if b["window"]:
            tmp = np.empty((rows, E), np.float32)
            ob.ref_gemm(rows, E, E, attn, b["projw"], 1, tmp, bias=b["projb"])
            self.r.ref_window_unpartition_add(x, tmp, G, E, s, nwx)
        else:
            ob.ref_gemm(T, E, E, attn, b["projw"], 1, x, bias=b["projb"], R=x)
        self.r.ref_layernorm(x, xn, b["n2w"], b["n2b"], T, E, 1e-5, 0, 1)
        h = np.empty((T, w.mlp), np.float32)
        ob.ref_gemm(T, w.mlp, E, xn, b["l1w"], 1, h, bias=b["l1b"], act=1)
        ob.ref_gemm(T, E, w.mlp, h, b["l2w"], 1, x, bias=b["l2b"], R=x)
        return x
