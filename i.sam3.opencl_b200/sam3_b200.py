"""Python host mirror of the C-ABI (include/sam3_cuda.h) through ctypes.

The library is the product; this module only loads it and exposes the
reference operator API (sam3_ops.h: gemm, linear, layernorm, add_bcast,
plus attention / mha and the encoder) with the same names and argument
meaning, so tests and the benchmark read like the reference's call sites.
Device memory may come from torch (``Backend.wrap(tensor)``) or from
``Backend.alloc``. There is no CPU path: loading fails loudly without the
built library, and calls fail with the backend's status text.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsam3cuda.so")

F32, BF16, F16, U8 = 0, 1, 2, 3
ACT_NONE, ACT_GELU, ACT_RELU = 0, 1, 2
ATTN_TC, ATTN_F32 = 0, 1

STATUS = {0: "CB_OK", 1: "CB_ENODEV", 2: "CB_EALLOC", 3: "CB_EARG",
          4: "CB_ECUDA", 5: "CB_ETIMEOUT", 6: "CB_EDTYPE"}

# Functions the header declares; tests check the library exports each one.
EXPORTS = [
    "cb_init", "cb_free", "cb_errstr", "cb_last_error", "cb_device", "cb_num_sms",
    "cb_alloc", "cb_wrap", "cb_upload", "cb_upload_weight", "cb_write", "cb_read",
    "cb_release", "cb_ptr", "cb_bytes", "cb_dtype", "cb_sync", "cb_set_stream",
    "cb_stream", "cb_device_error", "cb_clear_error", "cb_profile",
    "cb_profile_entry", "cb_mat", "cb_bmat",
    "cb_gemm", "cb_linear", "cb_layernorm", "cb_add_bcast", "cb_softmax_rows",
    "cb_rope_apply", "cb_window_partition", "cb_window_unpartition_add",
    "cb_patch_im2col", "cb_attention", "cb_attention_noalloc", "cb_mha",
    "cb_encoder_default_config",
    "cb_encoder_create", "cb_encoder_free", "cb_encoder_init_random",
    "cb_encoder_set_weight", "cb_encode_tiles", "cb_encode_blocks",
    "cb_encode_tiles_host", "cb_synth_normal", "cb_diag_exp2", "cb_diag_wait_timeout",
    "cb_convt_scatter", "cb_mask_logits", "cb_decoder_create", "cb_decoder_free",
    "cb_decoder_init_random", "cb_decoder_set_weight", "cb_decoder_set_image",
    "cb_decode", "cb_neck_create", "cb_neck_free", "cb_neck_init_random",
    "cb_neck_set_weight", "cb_neck_run", "cb_image_encoder_input",
    "cb_attend",
    "sam3_synth_normal", "sam3_synth_u8", "sam3_synth_rope_axial",
]

W = dict(PATCH_W=0, POS=1, LN_PRE_W=2, LN_PRE_B=3, ROPE_WIN=4, ROPE_GLOB=5,
         N1_W=10, N1_B=11, QKV_W=12, QKV_B=13, PROJ_W=14, PROJ_B=15, N2_W=16,
         N2_B=17, FC1_W=18, FC1_B=19, FC2_W=20, FC2_B=21)


# ---------------------------------------------------------------- tile sharding
def tile_shard(total, world, rank):
    """This rank's contiguous block of the crop loop, as (start, count).

    The reference encodes its crops one after another (amg.c:702-709); crops
    are independent through the backbone, so with one process per GPU each
    rank takes a contiguous block and no collective is needed in the data
    path. Counts differ by at most one (lower ranks take the extra crops)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError(f"tile_shard: total={total} world={world} rank={rank}")
    base, extra = divmod(total, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


def max_over_ranks(value, pg=None, device=None):
    """The largest of a per-rank float over the process group (a step takes
    as long as its slowest rank). pg: torch.distributed or None (one rank);
    device: where the reduction tensor lives ("cuda" for NCCL, None for
    gloo)."""
    if pg is None:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


class Opnd(C.Structure):
    """struct cb_opnd (sam3_ops.h:19-24 with cl_mem -> cb_mem)."""
    _fields_ = [("buf", C.c_void_p), ("off", C.c_int64), ("ld", C.c_int32),
                ("s0", C.c_int64), ("s1", C.c_int64)]


class EncoderConfig(C.Structure):
    _fields_ = [("embed", C.c_int), ("depth", C.c_int), ("heads", C.c_int),
                ("mlp", C.c_int), ("grid", C.c_int), ("patch", C.c_int),
                ("window", C.c_int), ("max_tiles", C.c_int),
                ("global_mask", C.c_uint64)]


class CBError(RuntimeError):
    def __init__(self, status, detail):
        super().__init__(f"{STATUS.get(status, status)}: {detail}")
        self.status = status


_lib = None


def lib():
    """Load libsam3cuda.so (built by build.py); fails if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built: run i.sam3.opencl_b200/build.py")
    L = C.CDLL(LIB_PATH)
    vp, i32, i64, f32, sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
    sig = {
        "cb_init": (i32, [C.POINTER(vp), i32]),
        "cb_free": (None, [vp]),
        "cb_errstr": (C.c_char_p, [i32]),
        "cb_last_error": (C.c_char_p, [vp]),
        "cb_device": (i32, [vp]),
        "cb_num_sms": (i32, [vp]),
        "cb_alloc": (i32, [vp, sz, i32, C.POINTER(vp)]),
        "cb_wrap": (i32, [vp, vp, sz, i32, C.POINTER(vp)]),
        "cb_upload": (i32, [vp, vp, sz, i32, C.POINTER(vp)]),
        "cb_upload_weight": (i32, [vp, vp, sz, i32, C.POINTER(vp)]),
        "cb_write": (i32, [vp, vp, sz, vp, sz]),
        "cb_read": (i32, [vp, vp, sz, vp, sz]),
        "cb_release": (i32, [C.POINTER(vp)]),
        "cb_ptr": (vp, [vp]),
        "cb_bytes": (sz, [vp]),
        "cb_dtype": (i32, [vp]),
        "cb_sync": (i32, [vp]),
        "cb_set_stream": (i32, [vp, vp]),
        "cb_stream": (vp, [vp]),
        "cb_device_error": (i32, [vp]),
        "cb_clear_error": (i32, [vp]),
        "cb_profile": (i32, [vp, i32]),
        "cb_profile_entry": (i32, [vp, i32, C.POINTER(C.c_char_p), C.POINTER(C.c_long),
                                   C.POINTER(C.c_double), C.POINTER(C.c_double),
                                   C.POINTER(C.c_double)]),
        "cb_mat": (Opnd, [vp, i64, C.c_int32]),
        "cb_bmat": (Opnd, [vp, i64, C.c_int32, i64, i64]),
        "cb_gemm": (i32, [vp, i32, i32, i32, Opnd, Opnd, i32, Opnd, i32, i32, vp, vp,
                          i64, f32, i32]),
        "cb_linear": (i32, [vp, i32, i32, i32, vp, i64, vp, vp, vp, i64, i32, i32]),
        "cb_layernorm": (i32, [vp, i64, i32, vp, vp, vp, vp, f32, i32]),
        "cb_add_bcast": (i32, [vp, vp, vp, vp, i64, i64]),
        "cb_softmax_rows": (i32, [vp, vp, i64, i32]),
        "cb_rope_apply": (i32, [vp, vp, i64, i32, i32, i32, vp]),
        "cb_window_partition": (i32, [vp, vp, vp, i32, i32, i32, i32]),
        "cb_window_unpartition_add": (i32, [vp, vp, vp, i32, i32, i32, i32]),
        "cb_patch_im2col": (i32, [vp, vp, vp, i32, i32, i32]),
        "cb_attention": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, i32, f32, i32, vp]),
        "cb_attention_noalloc": (i32, [vp, i32, i32, i32, i32, vp, i32, f32, vp, vp, vp]),
        "cb_mha": (i32, [vp, i32, i32, i32, i32, vp, i64, vp, i64, vp, i64, vp]),
        "cb_encoder_default_config": (None, [C.POINTER(EncoderConfig)]),
        "cb_encoder_create": (i32, [vp, C.POINTER(EncoderConfig), C.POINTER(vp)]),
        "cb_encoder_free": (None, [vp]),
        "cb_encoder_init_random": (i32, [vp, C.c_uint64, f32, C.c_double]),
        "cb_encoder_set_weight": (i32, [vp, i32, i32, vp, sz]),
        "cb_encode_tiles": (i32, [vp, vp, i32, vp]),
        "cb_encode_blocks": (i32, [vp, vp, i32, i32, i32]),
        "cb_encode_tiles_host": (i32, [vp, vp, i32, vp]),
        "cb_synth_normal": (i32, [vp, C.c_uint64, C.c_uint64, f32, f32, vp, sz]),
        "cb_diag_exp2": (i32, [vp, vp, vp, i32, vp]),
        "cb_diag_wait_timeout": (i32, [vp, vp, i32, vp]),
        "cb_convt_scatter": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32]),
        "cb_mask_logits": (i32, [vp, vp, vp, vp, i32, i32]),
        "cb_decoder_create": (i32, [vp, i32, C.POINTER(vp)]),
        "cb_decoder_free": (None, [vp]),
        "cb_decoder_init_random": (i32, [vp, C.c_uint64, f32]),
        "cb_decoder_set_weight": (i32, [vp, i32, vp, sz]),
        "cb_decoder_set_image": (i32, [vp, vp, vp, vp]),
        "cb_decode": (i32, [vp, i32, vp, vp, vp]),
        "cb_neck_create": (i32, [vp, i32, i32, i32, C.POINTER(vp)]),
        "cb_neck_free": (None, [vp]),
        "cb_neck_init_random": (i32, [vp, C.c_uint64, f32]),
        "cb_neck_set_weight": (i32, [vp, i32, vp, sz]),
        "cb_neck_run": (i32, [vp, vp, i32, vp, vp, vp]),
        "cb_image_encoder_input": (i32, [vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, i32,
                                         vp]),
        "cb_attend": (i32, [vp, i32, i32, i32, i32, vp, i32, vp, i32, vp, i32, vp, i32, i32,
                            vp, vp, i32, i32]),
        "sam3_synth_normal": (None, [C.c_uint64, C.c_uint64, sz, f32, f32, vp]),
        "sam3_synth_u8": (None, [C.c_uint64, C.c_uint64, sz, vp]),
        "sam3_synth_rope_axial": (None, [i32, i32, C.c_double, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


class Mem:
    """A cb_mem handle. Owns the device buffer unless created by wrap()."""

    def __init__(self, backend, handle, keep=None):
        self.backend = backend
        self.h = C.c_void_p(handle)
        self._keep = keep  # e.g. the torch tensor whose memory is borrowed

    @property
    def ptr(self):
        return lib().cb_ptr(self.h)

    @property
    def nbytes(self):
        return lib().cb_bytes(self.h)

    @property
    def dtype(self):
        return lib().cb_dtype(self.h)

    def release(self):
        if self.h:
            lib().cb_release(C.byref(self.h))
            self.h = C.c_void_p(None)

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class Backend:
    """cb_backend: one CUDA device and stream (ocl_init / ocl_backend)."""

    def __init__(self, device=0):
        h = C.c_void_p()
        rc = lib().cb_init(C.byref(h), device)
        if rc != 0:
            raise CBError(rc, lib().cb_errstr(rc).decode())
        self.h = h

    def check(self, rc):
        if rc != 0:
            raise CBError(rc, lib().cb_last_error(self.h).decode())

    def close(self):
        if self.h:
            lib().cb_free(self.h)
            self.h = C.c_void_p(None)

    @property
    def num_sms(self):
        return lib().cb_num_sms(self.h)

    @property
    def stream(self):
        return lib().cb_stream(self.h)

    def set_stream(self, stream_ptr):
        self.check(lib().cb_set_stream(self.h, stream_ptr))

    def sync(self):
        self.check(lib().cb_sync(self.h))

    def device_error(self):
        return lib().cb_device_error(self.h)

    def profile(self, on):
        """Per-kernel CUDA-event profile (I_SAM3_OPENCL_PROFILE counterpart)."""
        self.check(lib().cb_profile(self.h, 1 if on else 0))

    def profile_table(self):
        """{name: dict(calls, ms, flops, bytes)} of the profile so far."""
        out = {}
        i = 0
        while True:
            name, calls = C.c_char_p(), C.c_long()
            ms, fl, by = C.c_double(), C.c_double(), C.c_double()
            rc = lib().cb_profile_entry(self.h, i, C.byref(name), C.byref(calls),
                                        C.byref(ms), C.byref(fl), C.byref(by))
            if rc != 0:
                break
            out[name.value.decode()] = dict(calls=calls.value, ms=ms.value,
                                            flops=fl.value, bytes=by.value)
            i += 1
        return out

    # ---- buffers
    def alloc(self, nbytes, dtype):
        m = C.c_void_p()
        self.check(lib().cb_alloc(self.h, nbytes, dtype, C.byref(m)))
        return Mem(self, m.value)

    def wrap(self, tensor, dtype=None):
        """Borrow a torch CUDA tensor's memory (kept alive by the handle)."""
        import torch
        dt = dtype if dtype is not None else {
            torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16,
            torch.uint8: U8}[tensor.dtype]
        m = C.c_void_p()
        self.check(lib().cb_wrap(self.h, C.c_void_p(tensor.data_ptr()),
                                 tensor.numel() * tensor.element_size(), dt,
                                 C.byref(m)))
        return Mem(self, m.value, keep=tensor)

    def upload(self, array, dtype):
        import numpy as np
        a = np.ascontiguousarray(array)
        m = C.c_void_p()
        self.check(lib().cb_upload(self.h, a.ctypes.data, a.nbytes, dtype, C.byref(m)))
        return Mem(self, m.value)

    def upload_weight(self, array, dtype=BF16):
        import numpy as np
        a = np.ascontiguousarray(array, dtype=np.float32)
        m = C.c_void_p()
        self.check(lib().cb_upload_weight(self.h, a.ctypes.data, a.size, dtype,
                                          C.byref(m)))
        return Mem(self, m.value)

    def read(self, mem, out):
        """Blocking device -> host copy into numpy array `out`."""
        self.check(lib().cb_read(self.h, mem.h, 0, out.ctypes.data, out.nbytes))
        return out

    def write(self, mem, array, off=0):
        import numpy as np
        a = np.ascontiguousarray(array)
        self.check(lib().cb_write(self.h, mem.h, off, a.ctypes.data, a.nbytes))

    # ---- operators (sam3_ops.h names)
    def gemm(self, M, N, K, A, B, transb, Cm, nb=1, nb1=1, bias=None, R=None,
             roff=0, alpha=1.0, act=ACT_NONE):
        """A, B, Cm: (Mem, off, ld, s0, s1) tuples like bmat()."""
        def op(t):
            m, off, ld, s0, s1 = (tuple(t) + (0, 0))[:5]
            return Opnd(m.h.value, off, ld, s0, s1)
        self.check(lib().cb_gemm(self.h, M, N, K, op(A), op(B), transb, op(Cm), nb,
                                 nb1, bias.h if bias else None,
                                 R.h if R else None, roff, alpha, act))

    def linear(self, rows, n_in, n_out, X, xoff, Wt, b, Y, yoff, act=ACT_NONE,
               residual=0):
        self.check(lib().cb_linear(self.h, rows, n_in, n_out, X.h, xoff, Wt.h,
                                   b.h if b else None, Y.h, yoff, act, residual))

    def layernorm(self, rows, Cn, X, Y, g, b, eps=1e-5, act=ACT_NONE):
        self.check(lib().cb_layernorm(self.h, rows, Cn, X.h, Y.h, g.h, b.h, eps, act))

    def add_bcast(self, out, a, b, n, bmod):
        self.check(lib().cb_add_bcast(self.h, out.h, a.h, b.h, n, bmod))

    def softmax_rows(self, S, rows, L):
        self.check(lib().cb_softmax_rows(self.h, S.h, rows, L))

    def rope_apply(self, qkv, rows, E, hd, npos, cs):
        self.check(lib().cb_rope_apply(self.h, qkv.h, rows, E, hd, npos, cs.h))

    def window_partition(self, X, out, H, Cn, ws, nwx):
        self.check(lib().cb_window_partition(self.h, X.h, out.h, H, Cn, ws, nwx))

    def window_unpartition_add(self, X, Wd, H, Cn, ws, nwx):
        self.check(lib().cb_window_unpartition_add(self.h, X.h, Wd.h, H, Cn, ws, nwx))

    def patch_im2col(self, img, out, side, grid, ps):
        self.check(lib().cb_patch_im2col(self.h, img.h, out.h, side, grid, ps))

    def attention(self, qkv, nseq, N, E, heads, hd, cs, npos, scale, mode, out):
        self.check(lib().cb_attention(self.h, qkv.h, nseq, N, E, heads, hd,
                                      cs.h if cs else None, npos, scale, mode, out.h))

    def mha(self, P, Nq, Nk, dint, qp, sq, kp, sk, vp, sv, o):
        self.check(lib().cb_mha(self.h, P, Nq, Nk, dint, qp.h, sq, kp.h, sk, vp.h,
                                sv, o.h))

    def synth_normal(self, seed, stream, mean, std, out, count):
        self.check(lib().cb_synth_normal(self.h, seed, stream, mean, std, out.h, count))

    def convt_scatter(self, G, out, bias, add, P, H, W, Co, act=ACT_NONE):
        self.check(lib().cb_convt_scatter(self.h, G.h, out.h, bias.h,
                                          add.h if add else None, P, H, W, Co, act))

    def image_encoder_input(self, img, cols, rows, x0, y0, w, h, side=1008, tiles=None,
                            tile=0, chw=None):
        self.check(lib().cb_image_encoder_input(self.h, img.h, cols, rows, x0, y0, w, h, side,
                                                tiles.h if tiles else None, tile,
                                                chw.h if chw else None))

    def attend(self, Nq, Nk, heads, hd, Q, ldq, K, ldk, V, ldv, O, ldo, causal=0, dy=None,
               dx=None, W=0, mode=0):
        self.check(lib().cb_attend(self.h, Nq, Nk, heads, hd, Q.h, ldq, K.h, ldk, V.h, ldv,
                                   O.h, ldo, causal, dy.h if dy else None,
                                   dx.h if dx else None, W, mode))

    def mask_logits(self, U, hyper, out, P, npix):
        self.check(lib().cb_mask_logits(self.h, U.h, hyper.h, out.h, P, npix))


class Encoder:
    """cb_encoder: the PE trunk (sam_encode_trunk) over batches of tiles."""

    def __init__(self, backend, max_tiles=1, depth=None, global_blocks=None,
                 **overrides):
        cfg = EncoderConfig()
        lib().cb_encoder_default_config(C.byref(cfg))
        cfg.max_tiles = max_tiles
        if depth is not None:
            cfg.depth = depth
        for k, v in overrides.items():
            setattr(cfg, k, v)
        if global_blocks is not None:
            mask = 0
            for i in global_blocks:
                mask |= 1 << i
            cfg.global_mask = mask
        self.cfg = cfg
        self.backend = backend
        h = C.c_void_p()
        backend.check(lib().cb_encoder_create(backend.h, C.byref(cfg), C.byref(h)))
        self.h = h

    def init_random(self, seed, std=0.02, theta=10000.0):
        self.backend.check(lib().cb_encoder_init_random(self.h, seed, std, theta))

    def set_weight(self, which, block, array):
        import numpy as np
        a = np.ascontiguousarray(array, dtype=np.float32)
        self.backend.check(lib().cb_encoder_set_weight(
            self.h, W[which] if isinstance(which, str) else which, block,
            a.ctypes.data, a.size))

    def encode_tiles(self, tiles, ntile, out):
        self.backend.check(lib().cb_encode_tiles(self.h, tiles.h, ntile, out.h))

    def encode_blocks(self, x, ntile, first, last):
        self.backend.check(lib().cb_encode_blocks(self.h, x.h, ntile, first, last))

    def encode_tiles_host(self, tiles_u8, out_f32):
        ntile = tiles_u8.shape[0]
        self.backend.check(lib().cb_encode_tiles_host(
            self.h, C.c_void_p(tiles_u8.ctypes.data if hasattr(tiles_u8, "ctypes")
                               else tiles_u8.data_ptr()), ntile,
            C.c_void_p(out_f32.ctypes.data if hasattr(out_f32, "ctypes")
                       else out_f32.data_ptr())))

    def close(self):
        if self.h:
            lib().cb_encoder_free(self.h)
            self.h = C.c_void_p(None)


# Decoder tensor indices (include/sam3_synth.h, SAM3_DT_*).
DEC_TENSORS = 128
DT = dict(ATTN=0, LAYER=56, NF_W=80, NF_B=81, UP0_W=82, UP0_B=83, UP1_W=84, UP1_B=85,
          UP3_W=86, UP3_B=87, HYPER=88, IOU=112, GAUSS=118, POINT_EMB=119,
          NOT_A_POINT=123, NO_MASK=124, OBJ_TOKEN=125, IOU_TOKEN=126, MASK_TOKENS=127)
LOWRES = 288


class Decoder:
    """cb_decoder: the point-prompt mask decoder (sam_decode) for batches of
    up to `batch` prompts on one image."""

    def __init__(self, backend, batch):
        self.backend = backend
        self.batch = batch
        h = C.c_void_p()
        backend.check(lib().cb_decoder_create(backend.h, batch, C.byref(h)))
        self.h = h

    def init_random(self, seed, std=0.02):
        self.backend.check(lib().cb_decoder_init_random(self.h, seed, std))

    def set_weight(self, which, array):
        import numpy as np
        a = np.ascontiguousarray(array, dtype=np.float32)
        self.backend.check(lib().cb_decoder_set_weight(self.h, which, a.ctypes.data, a.size))

    def set_image(self, emb, feat_s0, feat_s1):
        self.backend.check(lib().cb_decoder_set_image(self.h, emb.h, feat_s0.h, feat_s1.h))

    def decode(self, points, lowres):
        """points: float32 [P, 2] (x, y) in input pixels; lowres: F32 Mem of
        at least P * 3 * 288 * 288 values. Returns the IoU predictions [P, 3]."""
        import numpy as np
        pts = np.ascontiguousarray(points, dtype=np.float32).reshape(-1, 2)
        iou = np.empty((pts.shape[0], 3), np.float32)
        self.backend.check(lib().cb_decode(self.h, pts.shape[0], pts.ctypes.data,
                                           iou.ctypes.data, lowres.h))
        return iou

    def close(self):
        if self.h:
            lib().cb_decoder_free(self.h)
            self.h = C.c_void_p(None)


NECK_TENSORS = 29


class Neck:
    """cb_neck: the SimpleFPN neck (point_neck) over batches of tiles."""

    def __init__(self, backend, grid=72, embed=1024, max_tiles=1):
        self.backend = backend
        self.grid, self.embed = grid, embed
        h = C.c_void_p()
        backend.check(lib().cb_neck_create(backend.h, grid, embed, max_tiles, C.byref(h)))
        self.h = h

    def init_random(self, seed, std=0.02):
        self.backend.check(lib().cb_neck_init_random(self.h, seed, std))

    def set_weight(self, which, array):
        import numpy as np
        a = np.ascontiguousarray(array, dtype=np.float32)
        self.backend.check(lib().cb_neck_set_weight(self.h, which, a.ctypes.data, a.size))

    def run(self, x, ntile, emb, feat_s0, feat_s1):
        self.backend.check(lib().cb_neck_run(self.h, x.h, ntile, emb.h, feat_s0.h, feat_s1.h))

    def close(self):
        if self.h:
            lib().cb_neck_free(self.h)
            self.h = C.c_void_p(None)
