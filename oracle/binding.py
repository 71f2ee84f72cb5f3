"""ctypes bindings of the oracle libraries (test infrastructure only).

numpy in, numpy out. Each function names the reference code it restates;
``ref_*`` functions run the reference's own kernels (oracle/_ref).
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_lib = None
_ref = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


class GemmArgs(C.Structure):
    """or_gemm_args / ref_gemm_args: sam3_kernels.cl:57-77 argument list."""
    _fields_ = [("M", C.c_int), ("N", C.c_int), ("K", C.c_int),
                ("A", C.c_void_p), ("aoff", C.c_long), ("lda", C.c_int),
                ("sa0", C.c_long), ("sa1", C.c_long),
                ("B", C.c_void_p), ("boff", C.c_long), ("ldb", C.c_int),
                ("sb0", C.c_long), ("sb1", C.c_long), ("transb", C.c_int),
                ("C", C.c_void_p), ("coff", C.c_long), ("ldc", C.c_int),
                ("sc0", C.c_long), ("sc1", C.c_long), ("nb1", C.c_int),
                ("bias", C.c_void_p), ("R", C.c_void_p), ("roff", C.c_long),
                ("alpha", C.c_float), ("act", C.c_int)]


class Block(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in
                ("n1w", "n1b", "qkvw", "qkvb", "projw", "projb", "n2w", "n2b",
                 "l1w", "l1b", "l2w", "l2b")] + [("window", C.c_int)]


class Trunk(C.Structure):
    _fields_ = [(n, C.c_int) for n in
                ("E", "heads", "hd", "mlp", "depth", "grid", "patch", "img")] + \
               [(n, C.c_void_p) for n in ("pe_w", "pos", "lnpw", "lnpb")] + \
               [("blocks", C.POINTER(Block)), ("rope_win", C.c_void_p),
                ("rope_glob", C.c_void_p)]


def build():
    """Compile liboracle.so (and oracle/_ref when the reference is present)."""
    subprocess.check_call(["make", "-s", "-C", HERE])


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _lib = C.CDLL(path)
        L = _lib
        L.or_gemm.argtypes = [C.POINTER(GemmArgs), C.c_int]
        L.or_layernorm.argtypes = [f32p, f32p, f32p, f32p, C.c_long, C.c_int,
                                   C.c_float, C.c_int]
        L.or_softmax_rows.argtypes = [f32p, C.c_long, C.c_int]
        L.or_rope_apply.argtypes = [f32p, C.c_long, C.c_int, C.c_int, C.c_int,
                                    f32p]
        L.or_add_bcast.argtypes = [f32p, f32p, f32p, C.c_long, C.c_long]
        L.or_window_partition.argtypes = [f32p, f32p] + [C.c_int] * 4
        L.or_window_unpartition_add.argtypes = [f32p, f32p] + [C.c_int] * 4
        L.or_patch_im2col.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_int]
        L.or_image_input.argtypes = [u8p, C.c_int, f32p]
        L.or_mha.argtypes = [C.c_int] * 4 + [f32p, C.c_long, f32p, C.c_long,
                                             f32p, C.c_long, f32p]
        L.or_attention.argtypes = [f32p] + [C.c_int] * 5 + [C.c_float, f32p]
        L.or_encode_trunk.argtypes = [C.POINTER(Trunk), C.c_void_p, f32p,
                                      C.c_int, C.c_int]
        L.or_num_threads.restype = C.c_int
        L.or_convt_scatter.argtypes = [f32p, f32p, f32p, C.c_void_p] + [C.c_int] * 5
        L.or_mask_logits.argtypes = [f32p, f32p, f32p, C.c_int, C.c_long]
        L.or_pe_encode.argtypes = [f32p, C.c_float, C.c_float, f32p]
        L.or_dec_tensor.argtypes = [C.c_int] + [C.POINTER(C.c_int)] * 3
        L.or_sam_decode.argtypes = [C.POINTER(C.c_void_p), f32p, f32p, f32p, C.c_int,
                                    f32p, f32p, f32p]
        L.or_im2col3x3.argtypes = [f32p, f32p] + [C.c_int] * 4 + [C.c_long]
        L.or_aa_resize.argtypes = [u8p] + [C.c_int] * 5 + [u8p]
        L.or_softmax_ext.argtypes = [f32p, C.c_long] + [C.c_int] * 4 + [C.c_void_p,
                                                                       C.c_void_p,
                                                                       C.c_int, C.c_int]
        L.or_attend.argtypes = [C.c_int] * 4 + [f32p, C.c_int, f32p, C.c_int, f32p, C.c_int,
                                                f32p, C.c_int, C.c_int, C.c_void_p,
                                                C.c_void_p, C.c_int]
        L.or_image_encoder_input.argtypes = [u8p] + [C.c_int] * 6 + [f32p]
        L.or_neck_tensor.argtypes = [C.c_int, C.c_int] + [C.POINTER(C.c_int)] * 3
        L.or_point_neck.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.c_int, f32p, f32p,
                                    f32p, f32p]
        L.sam3_synth_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_size_t,
                                        C.c_float, C.c_float, f32p]
        L.sam3_synth_u8.argtypes = [C.c_uint64, C.c_uint64, C.c_size_t, u8p]
        L.sam3_synth_rope_axial.argtypes = [C.c_int, C.c_int, C.c_double, f32p]
    return _lib


def have_ref():
    return os.path.exists(os.path.join(HERE, "_ref", "libsam3ref.so"))


def ref():
    global _ref
    if _ref is None:
        path = os.path.join(HERE, "_ref", "libsam3ref.so")
        _ref = C.CDLL(path)
        R = _ref
        R.ref_gemm.argtypes = [C.POINTER(GemmArgs), C.c_int, C.c_int]
        R.ref_layernorm.argtypes = [f32p, f32p, f32p, f32p, C.c_long, C.c_int,
                                    C.c_float, C.c_int, C.c_int]
        R.ref_softmax_rows.argtypes = [f32p, C.c_long, C.c_int, C.c_int]
        R.ref_rope_apply.argtypes = [f32p, C.c_long, C.c_int, C.c_int, C.c_int,
                                     f32p]
        R.ref_add_bcast.argtypes = [f32p, f32p, f32p, C.c_long, C.c_long]
        R.ref_window_partition.argtypes = [f32p, f32p] + [C.c_int] * 4
        R.ref_window_unpartition_add.argtypes = [f32p, f32p] + [C.c_int] * 4
        R.ref_patch_im2col.argtypes = [f32p, f32p, C.c_int, C.c_int, C.c_int]
        R.ref_mha.argtypes = [C.c_int] * 4 + [f32p, C.c_long, f32p, C.c_long,
                                              f32p, C.c_long, f32p]
        R.ref_mha.restype = C.c_int
        R.ref_num_threads.restype = C.c_int
        R.ref_convt_scatter.argtypes = [f32p, f32p, f32p, C.c_void_p] + [C.c_int] * 5
        R.ref_mask_logits.argtypes = [f32p, f32p, f32p, C.c_int, C.c_long]
        R.ref_im2col3x3.argtypes = [f32p, f32p] + [C.c_int] * 4 + [C.c_long]
        R.ref_softmax_ext.argtypes = [f32p, C.c_long] + [C.c_int] * 4 + [C.c_void_p,
                                                                        C.c_void_p,
                                                                        C.c_int, C.c_int,
                                                                        C.c_int]
    return _ref


# ---------------------------------------------------------------- generator
def normal(seed, stream, shape, mean=0.0, std=1.0):
    out = np.empty(int(np.prod(shape)), np.float32)
    lib().sam3_synth_normal(seed, stream, out.size, mean, std, out)
    return out.reshape(shape)


def u8(seed, stream, shape):
    out = np.empty(int(np.prod(shape)), np.uint8)
    lib().sam3_synth_u8(seed, stream, out.size, out)
    return out.reshape(shape)


def rope_axial(side, hd=64, theta=10000.0):
    out = np.empty(side * side * hd, np.float32)
    lib().sam3_synth_rope_axial(side, hd, theta, out)
    return out.reshape(side * side, hd // 2, 2)


# ---------------------------------------------------------------- kernels
def _gemm_args(M, N, K, A, B, transb, Cm, aoff=0, lda=None, sa=(0, 0),
               boff=0, ldb=None, sb=(0, 0), coff=0, ldc=None, sc=(0, 0), nb1=1,
               bias=None, R=None, roff=0, alpha=1.0, act=0):
    a = GemmArgs()
    a.M, a.N, a.K = M, N, K
    a.A, a.aoff, a.lda = A.ctypes.data, aoff, K if lda is None else lda
    a.sa0, a.sa1 = sa
    a.B, a.boff = B.ctypes.data, boff
    a.ldb = (K if transb else N) if ldb is None else ldb
    a.sb0, a.sb1 = sb
    a.transb = transb
    a.C, a.coff, a.ldc = Cm.ctypes.data, coff, N if ldc is None else ldc
    a.sc0, a.sc1 = sc
    a.nb1 = nb1
    a.bias = None if bias is None else bias.ctypes.data
    a.R = None if R is None else R.ctypes.data
    a.roff, a.alpha, a.act = roff, alpha, act
    return a


def gemm(M, N, K, A, B, transb, Cm, nb=1, **kw):
    """or_gemm: gemm_cpu_t / gemm_cpu_n arithmetic (sam3_kernels.cl:334-448)."""
    a = _gemm_args(M, N, K, A, B, transb, Cm, **kw)
    lib().or_gemm(C.byref(a), nb)
    return Cm


def ref_gemm(M, N, K, A, B, transb, Cm, nb=1, profile=0, **kw):
    a = _gemm_args(M, N, K, A, B, transb, Cm, **kw)
    ref().ref_gemm(C.byref(a), nb, profile)
    return Cm


def layernorm(X, g, b, eps=1e-5, act=0, Y=None):
    rows, Cn = X.shape
    Y = np.empty_like(X) if Y is None else Y
    lib().or_layernorm(X, Y, g, b, rows, Cn, eps, act)
    return Y


def ref_layernorm(X, g, b, eps=1e-5, act=0, local=256):
    rows, Cn = X.shape
    Y = np.empty_like(X)
    ref().ref_layernorm(X, Y, g, b, rows, Cn, eps, act, local)
    return Y


def softmax_rows(S):
    S = np.ascontiguousarray(S, np.float32).copy()
    lib().or_softmax_rows(S, S.shape[0], S.shape[1])
    return S


def ref_softmax_rows(S, local=256):
    S = np.ascontiguousarray(S, np.float32).copy()
    ref().ref_softmax_rows(S, S.shape[0], S.shape[1], local)
    return S


def rope_apply(qkv, E, hd, npos, cs, use_ref=False):
    q = np.ascontiguousarray(qkv, np.float32).copy()
    f = ref().ref_rope_apply if use_ref else lib().or_rope_apply
    f(q, q.shape[0], E, hd, npos, np.ascontiguousarray(cs, np.float32))
    return q


def attention(qkv, nseq, N, E, heads, hd, alpha):
    """vit_block attention core (sam3_model.c:1000-1013) on roped qkv."""
    out = np.empty((nseq * N, E), np.float32)
    lib().or_attention(np.ascontiguousarray(qkv, np.float32), nseq, N, E,
                       heads, hd, alpha, out)
    return out


def ref_attention(qkv, nseq, N, E, heads, hd, alpha, head_chunk=None,
                  softmax_local=None):
    """The reference's attention launches (sam3_model.c:1000-1013): QK^T
    gemm_cpu_t, softmax_rows (work-group 256 as sam3_model.c:336 picks, or
    softmax_local items), P.V gemm_cpu_n, heads chunked like head_chunk()
    (sam3_model.c:793-798)."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    out = np.zeros((nseq * N, E), np.float32)
    hc = heads if head_chunk is None else head_chunk
    plane = N * N
    tstride = N * 3 * E
    for h0 in range(0, heads, hc):
        hcc = min(hc, heads - h0)
        S = np.empty(nseq * hcc * plane, np.float32)
        ref_gemm(N, N, hd, qkv, qkv, 1, S, nb=nseq * hcc, aoff=h0 * hd,
                 lda=3 * E, sa=(tstride, hd), boff=E + h0 * hd, ldb=3 * E,
                 sb=(tstride, hd), ldc=N, sc=(hcc * plane, plane), nb1=hcc,
                 alpha=alpha)
        ref().ref_softmax_rows(S, nseq * hcc * N, N, softmax_local or
                               (256 if N >= 256 else 64))
        ref_gemm(N, hd, N, S, qkv, 0, out, nb=nseq * hcc, lda=N,
                 sa=(hcc * plane, plane), boff=2 * E + h0 * hd, ldb=3 * E,
                 sb=(tstride, hd), coff=h0 * hd, ldc=E, sc=(N * E, hd),
                 nb1=hcc)
    return out


def mha(P, Nq, Nk, dint, qp, sq, kp, sk, vp, sv, use_ref=False):
    o = np.zeros((P * Nq, dint), np.float32)
    f = ref().ref_mha if use_ref else lib().or_mha
    rc = f(P, Nq, Nk, dint, qp, sq, kp, sk, vp, sv, o)
    if rc != 0:
        raise ValueError("mha: unsupported shape")
    return o


def image_input(rgb):
    side = rgb.shape[0]
    out = np.empty((3, side, side), np.float32)
    lib().or_image_input(np.ascontiguousarray(rgb), side, out)
    return out


def num_threads():
    return lib().or_num_threads()


# ---------------------------------------------------------------- backbone
class TrunkWeights:
    """fp32 random-init weights of the PE backbone, drawn from the same
    streams as the GPU path (include/sam3_synth.h)."""

    def __init__(self, seed, depth=32, E=1024, heads=16, mlp=4096, grid=72,
                 patch=14, window=24, global_blocks=(7, 15, 23, 31), std=0.02):
        S = 1024  # SAM3_STREAM_BLOCK0
        self.E, self.heads, self.hd, self.mlp = E, heads, E // heads, mlp
        self.depth, self.grid, self.patch = depth, grid, patch
        self.img = grid * patch
        self.window = window
        self.globals = set(global_blocks)
        T = grid * grid
        self.pe_w = normal(seed, 1, (E, 3 * patch * patch), 0.0, std)
        self.pos = normal(seed, 2, (T, E), 0.0, std)
        self.lnpw = np.ones(E, np.float32)
        self.lnpb = np.zeros(E, np.float32)
        self.blocks = []
        for i in range(depth):
            b = dict(
                n1w=np.ones(E, np.float32), n1b=np.zeros(E, np.float32),
                n2w=np.ones(E, np.float32), n2b=np.zeros(E, np.float32),
                qkvw=normal(seed, S + 16 * i + 0, (3 * E, E), 0.0, std),
                qkvb=np.zeros(3 * E, np.float32),
                projw=normal(seed, S + 16 * i + 1, (E, E), 0.0, std),
                projb=np.zeros(E, np.float32),
                l1w=normal(seed, S + 16 * i + 2, (mlp, E), 0.0, std),
                l1b=np.zeros(mlp, np.float32),
                l2w=normal(seed, S + 16 * i + 3, (E, mlp), 0.0, std),
                l2b=np.zeros(E, np.float32),
                window=0 if i in self.globals else window)
            self.blocks.append(b)
        self.rope_win = rope_axial(window, self.hd)
        self.rope_glob = rope_axial(grid, self.hd)

    def ctypes(self):
        blocks = (Block * self.depth)()
        for i, b in enumerate(self.blocks):
            for k in ("n1w", "n1b", "qkvw", "qkvb", "projw", "projb", "n2w",
                      "n2b", "l1w", "l1b", "l2w", "l2b"):
                setattr(blocks[i], k, b[k].ctypes.data)
            blocks[i].window = b["window"]
        t = Trunk()
        t.E, t.heads, t.hd, t.mlp = self.E, self.heads, self.hd, self.mlp
        t.depth, t.grid, t.patch, t.img = self.depth, self.grid, self.patch, self.img
        t.pe_w, t.pos = self.pe_w.ctypes.data, self.pos.ctypes.data
        t.lnpw, t.lnpb = self.lnpw.ctypes.data, self.lnpb.ctypes.data
        t.blocks = blocks
        t.rope_win, t.rope_glob = self.rope_win.ctypes.data, self.rope_glob.ctypes.data
        self._keep = blocks
        return t


def encode_trunk(w, img_chw, first=0, last=None, x=None):
    """sam_encode_trunk (sam3_model.c:1112-1144); returns x [T, E]. With
    img_chw None the prologue is skipped and x is block `first`'s input."""
    T = w.grid * w.grid
    x = np.zeros((T, w.E), np.float32) if x is None else x
    t = w.ctypes()
    img = None if img_chw is None else np.ascontiguousarray(img_chw, np.float32)
    lib().or_encode_trunk(C.byref(t), None if img is None else img.ctypes.data, x, first,
                          w.depth if last is None else last)
    return x


# ---------------------------------------------------------------- mask decoder
def convt_scatter(G, bias, add, P, H, W, Co, act=0, use_ref=False):
    """convt_scatter (sam3_kernels.cl:766-781): G [P*H*W, Co*4] -> [P, 2H, 2W, Co]."""
    G = np.ascontiguousarray(G, np.float32)
    out = np.empty((P, 2 * H, 2 * W, Co), np.float32)
    addp = None
    if add is not None:
        add = np.ascontiguousarray(add, np.float32)
        addp = add.ctypes.data
    fn = ref().ref_convt_scatter if use_ref else lib().or_convt_scatter
    fn(G, out, np.ascontiguousarray(bias, np.float32), addp, P, H, W, Co, act)
    return out


def mask_logits(U, hyper, P, npix, use_ref=False):
    """mask_logits (sam3_kernels.cl:789-807): U [P, npix, 32], hyper [P, 96]."""
    out = np.empty((P, 3, npix), np.float32)
    fn = ref().ref_mask_logits if use_ref else lib().or_mask_logits
    fn(np.ascontiguousarray(U, np.float32), np.ascontiguousarray(hyper, np.float32), out,
       npix, P * npix)
    return out


def pe_encode(gauss, x, y):
    out = np.empty(256, np.float32)
    lib().or_pe_encode(np.ascontiguousarray(gauss, np.float32), x, y, out)
    return out


DEC_TENSORS = 128
DEC_STREAM = 8192
DEC_IMG_STREAM = 9216


def dec_tensor_info(i):
    r, c, k = C.c_int(), C.c_int(), C.c_int()
    lib().or_dec_tensor(i, C.byref(r), C.byref(c), C.byref(k))
    return r.value, c.value, k.value


class DecoderWeights:
    """The decoder's random-init tensors (include/sam3_synth.h: tensor i
    draws stream 8192 + i; W and B kinds N(0, std), LayerNorm weights
    N(1, 0.1), LayerNorm biases N(0, 0.1), embeddings N(0, 1)), fp32 in the
    checkpoint layout."""

    def __init__(self, seed, std=0.02):
        self.t = []
        for i in range(DEC_TENSORS):
            r, c, k = dec_tensor_info(i)
            mean = 1.0 if k == 2 else 0.0
            sd = 1.0 if k == 4 else (0.1 if k in (2, 3) else std)
            self.t.append(normal(seed, DEC_STREAM + i, (r, c), mean, sd))

    def ctypes(self):
        arr = (C.c_void_p * DEC_TENSORS)(*[a.ctypes.data for a in self.t])
        return arr


def decoder_image(seed):
    """Synthetic image-side decoder inputs: emb [5184, 256], feat_s0
    [82944, 32], feat_s1 [20736, 64], N(0, 1)."""
    return (normal(seed, DEC_IMG_STREAM + 0, (5184, 256)),
            normal(seed, DEC_IMG_STREAM + 1, (16 * 5184, 32)),
            normal(seed, DEC_IMG_STREAM + 2, (4 * 5184, 64)))


def sam_decode(w, emb, s0, s1, points):
    """Decoder caches + sam_decode (sam3_model.c:1153-1170, 1239-1399) for the
    prompts points [P, 2]; returns (iou [P, 3], lowres [P, 3, 288, 288])."""
    pts = np.ascontiguousarray(points, np.float32).reshape(-1, 2)
    P = pts.shape[0]
    iou = np.empty((P, 3), np.float32)
    low = np.empty((P, 3, 288, 288), np.float32)
    lib().or_sam_decode(w.ctypes(), np.ascontiguousarray(emb, np.float32),
                        np.ascontiguousarray(s0, np.float32),
                        np.ascontiguousarray(s1, np.float32), P, pts, iou, low)
    return iou, low


# ---------------------------------------------------------------- neck
NECK_TENSORS = 29
NECK_STREAM = 10240


def im2col3x3(X, H, W, Cn, t0, n, use_ref=False):
    """im2col3x3 (sam3_kernels.cl:746-760): tokens t0 .. t0 + n of X [H*W, C]."""
    out = np.empty((n, 9 * Cn), np.float32)
    fn = ref().ref_im2col3x3 if use_ref else lib().or_im2col3x3
    fn(np.ascontiguousarray(X, np.float32), out, H, W, Cn, t0, n * 9 * Cn)
    return out


def neck_tensor_info(i, E=1024):
    r, c, k = C.c_int(), C.c_int(), C.c_int()
    lib().or_neck_tensor(i, E, C.byref(r), C.byref(c), C.byref(k))
    return r.value, c.value, k.value


class NeckWeights:
    """The neck's random-init tensors (include/sam3_synth.h: tensor i draws
    stream 10240 + i, N(0, std)); empty arrays for tensors a level lacks."""

    def __init__(self, seed, std=0.02, E=1024):
        self.E = E
        self.t = []
        for i in range(NECK_TENSORS):
            r, c, _ = neck_tensor_info(i, E)
            self.t.append(normal(seed, NECK_STREAM + i, (r, c), 0.0, std) if r
                          else np.zeros((1,), np.float32))

    def ctypes(self):
        return (C.c_void_p * NECK_TENSORS)(*[a.ctypes.data for a in self.t])


def point_neck(w, x, grid):
    """point_neck (sam3_model.c:1098-1110) on x [grid^2, E]; returns
    (emb [grid^2, 256], feat_s0 [16 grid^2, 32], feat_s1 [4 grid^2, 64])."""
    T = grid * grid
    emb = np.empty((T, 256), np.float32)
    s0 = np.empty((16 * T, 32), np.float32)
    s1 = np.empty((4 * T, 64), np.float32)
    lib().or_point_neck(w.ctypes(), grid, w.E, np.ascontiguousarray(x, np.float32), emb, s0, s1)
    return emb, s0, s1


# ---------------------------------------------------------------- input path
def aa_resize(rgb, nw, nh):
    """aa_resize (image.c:284-339) of an HWC uint8 image to nh x nw."""
    rgb = np.ascontiguousarray(rgb, np.uint8)
    h, w = rgb.shape[:2]
    out = np.empty((nh, nw, 3), np.uint8)
    lib().or_aa_resize(rgb, w, h, w, nw, nh, out)
    return out


def image_encoder_input(rgb, x0, y0, w, h, side=1008):
    """image_encoder_input (image.c:346-371): float CHW [3, side, side]."""
    rgb = np.ascontiguousarray(rgb, np.uint8)
    out = np.empty((3, side, side), np.float32)
    lib().or_image_encoder_input(rgb, rgb.shape[1], x0, y0, w, h, side, out)
    return out


# ---------------------------------------------------------------- detector attention
def _ptr(a):
    return None if a is None else np.ascontiguousarray(a, np.float32).ctypes.data


def softmax_ext(S, Nq, h0=0, causal=0, dy=None, dx=None, W=0, nh=8, use_ref=False, local=64):
    """softmax_ext (sam3_kernels.cl:889-921) on S [rows, L] in place (a copy)."""
    S = np.array(S, np.float32, copy=True, order="C")
    dy = None if dy is None else np.ascontiguousarray(dy, np.float32)
    dx = None if dx is None else np.ascontiguousarray(dx, np.float32)
    args = (S, S.shape[0], S.shape[1], Nq, h0, causal, _ptr(dy), _ptr(dx), W, nh)
    if use_ref:
        ref().ref_softmax_ext(*args, local)
    else:
        lib().or_softmax_ext(*args)
    return S


def attend(Q, K, V, heads, hd, causal=0, dy=None, dx=None, W=0):
    """attend (sam3_text.c:305-343): Q [Nq, heads*hd], K, V [Nk, heads*hd]."""
    Q = np.ascontiguousarray(Q, np.float32)
    K = np.ascontiguousarray(K, np.float32)
    V = np.ascontiguousarray(V, np.float32)
    dy = None if dy is None else np.ascontiguousarray(dy, np.float32)
    dx = None if dx is None else np.ascontiguousarray(dx, np.float32)
    O = np.zeros((Q.shape[0], heads * hd), np.float32)
    lib().or_attend(Q.shape[0], K.shape[0], heads, hd, Q, Q.shape[1], K, K.shape[1], V,
                    V.shape[1], O, heads * hd, causal, _ptr(dy), _ptr(dx), W)
    return O
