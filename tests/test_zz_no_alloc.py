"""cb_attention_noalloc, the allocation-free attention entry point, against
cb_attention (the existing entry point that stages its bf16 copy of qkv in
a cudaMalloc'd scratch buffer), called through the C-ABI.

Callers that own all device memory through their own pool, or that cannot
afford cudaMalloc's synchronisation on their latency path, use the
no-alloc variant; it must give the results of the allocating one. Two calls
in a row with different inputs also check that the shared static scratch
array carries nothing over from the previous call. Tolerance: the attention
bound used throughout the tests (max-abs <= 1e-2, cosine >= 0.9999).

This file is collected last (test_zz_*) so that a run stopping at the first
failure has already run every other test; it also passes on its own in a
fresh process.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def cos_sim(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _inputs(seed, nseq, side, E):
    g = torch.Generator().manual_seed(seed)
    N = side * side
    qkv = torch.randn(nseq * N, 3 * E, generator=g).cuda()
    cs = torch.empty(N * 64, dtype=torch.float32)
    return N, qkv, cs


def test_noalloc_attention_matches_allocating_entry_point(cb, sb):
    lib = sb.lib()
    E, heads, side, nseq = 1024, 16, 24, 9  # config 1: 9 windows of 24 x 24
    for call, seed in enumerate((101, 202)):
        N, qkv, cs = _inputs(seed, nseq, side, E)
        lib.sam3_synth_rope_axial(side, 64, 10000.0, cs.data_ptr())
        cs = cs.cuda()
        ref_qkv = qkv.clone()
        out_ref = torch.empty(nseq * N, E, device="cuda")
        out = torch.full((nseq * N, E), float("nan"), device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        cb.attention(cb.wrap(ref_qkv), nseq, N, E, heads, 64, cb.wrap(cs), N, 0.125,
                     sb.ATTN_TC, cb.wrap(out_ref))
        rc = lib.cb_attention_noalloc(C.c_void_p(qkv.data_ptr()), nseq, N, E, heads,
                                      C.c_void_p(cs.data_ptr()), N, 0.125,
                                      C.c_void_p(out.data_ptr()),
                                      C.c_void_p(err.data_ptr()), C.c_void_p(cb.stream))
        assert rc == 0, lib.cb_errstr(rc)
        cb.sync()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got, want = out.cpu().numpy(), out_ref.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: output not fully written"
        assert np.abs(got - want).max() <= 1e-2, call
        assert cos_sim(got, want) >= 0.9999, call


def test_noalloc_attention_without_rope_or_error_word(cb, sb):
    """The other two branches: no RoPE table (plain bf16 cast into the
    static array) and err == NULL (the library's own error word, cleared by
    the call itself), two calls in a row."""
    lib = sb.lib()
    E, heads, side, nseq = 1024, 16, 24, 2
    for call, seed in enumerate((303, 404)):
        N, qkv, _ = _inputs(seed, nseq, side, E)
        ref_qkv = qkv.clone()
        out_ref = torch.empty(nseq * N, E, device="cuda")
        out = torch.full((nseq * N, E), float("nan"), device="cuda")
        torch.cuda.synchronize()
        cb.attention(cb.wrap(ref_qkv), nseq, N, E, heads, 64, None, N, 0.125,
                     sb.ATTN_TC, cb.wrap(out_ref))
        rc = lib.cb_attention_noalloc(C.c_void_p(qkv.data_ptr()), nseq, N, E, heads, None, 0,
                                      0.125, C.c_void_p(out.data_ptr()), None,
                                      C.c_void_p(cb.stream))
        assert rc == 0, lib.cb_errstr(rc)
        cb.sync()
        torch.cuda.synchronize()
        got, want = out.cpu().numpy(), out_ref.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: output not fully written"
        assert np.abs(got - want).max() <= 1e-2, call
        assert cos_sim(got, want) >= 0.9999, call


def test_noalloc_attention_rejects_oversized_input(cb, sb):
    lib = sb.lib()
    E, heads = 1024, 16
    rows = 5462  # one row more than the 32 MiB bf16 staging array holds at E = 1024
    qkv = torch.zeros(rows, 3 * E, device="cuda")
    out = torch.zeros(rows, E, device="cuda")
    rc = lib.cb_attention_noalloc(C.c_void_p(qkv.data_ptr()), 1, rows, E, heads, None, 0,
                                  0.125, C.c_void_p(out.data_ptr()), None,
                                  C.c_void_p(cb.stream))
    assert rc == 3  # CB_EARG, before any work is queued
