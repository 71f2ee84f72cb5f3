/* The reference's own OpenCL kernels (sam3_kernels.cl), compiled unmodified
 * as host C++ through ocl_shim.hpp, behind a small NDRange executor.
 *
 * TEST INFRASTRUCTURE ONLY. The build recipe (oracle/Makefile) compiles the
 * kernel file where it lies in the reference tree and writes the library to
 * oracle/_ref/libsam3ref.so. It pins the C restatement in oracle.c: the CPU
 * tests compare the two on seeded inputs.
 *
 * Launch geometry follows the reference host code:
 *  - ref_gemm: sam3_model.c:230-302 (profile=cpu: gemm_cpu_t / gemm_cpu_n
 *    with global (ceil(N/4), ceil(M/2), nb) or (ceil(N/8), ceil(M/4), nb);
 *    GPU profile: gemm / gemm_big, 16x16 work-groups);
 *  - layernorm / softmax_rows: sam3_model.c:314-341 (work-group 256 for wide
 *    rows, else 64; any power of two is accepted by the kernels, and 1 turns
 *    the work-group reductions into plain serial sums);
 *  - run1d kernels: 256-item groups, sam3_model.c:209-214;
 *  - mha: sam3_model.c:419-451.
 *
 * Work-groups run in parallel on OpenMP threads; inside a group, kernels
 * with barriers run as one ucontext fiber per work-item. */
#include "ocl_shim.hpp"

#include <cstdlib>
#include <cstring>
#include <omp.h>
#include <ucontext.h>

namespace oclshim {

thread_local WorkItem *cur_wi;

namespace {

struct Fiber {
    ucontext_t ctx;
    WorkItem wi;
    int done;
};

thread_local ucontext_t sched_ctx;
thread_local Fiber *cur_fiber;
thread_local int fiber_mode;
thread_local void (*tl_fn)(void *);
thread_local void *tl_arg;
thread_local char *tl_stacks;
thread_local size_t tl_nstacks;

const size_t kStack = 128 * 1024;

void trampoline()
{
    tl_fn(tl_arg);
    cur_fiber->done = 1;
    swapcontext(&cur_fiber->ctx, &sched_ctx);
}

} // namespace

void wg_barrier()
{
    if (!fiber_mode)
        return;
    swapcontext(&cur_fiber->ctx, &sched_ctx);
}

/* Runs fn(arg) for every work-item of the NDRange (dims <= 3). */
static void run_ndrange(unsigned dims, const size_t *gsz_in,
                        const size_t *lsz_in, int barriers,
                        void (*fn)(void *), void *arg)
{
    size_t gsz[3] = {1, 1, 1}, lsz[3] = {1, 1, 1}, ngrp[3];
    for (unsigned d = 0; d < dims; d++) {
        gsz[d] = gsz_in[d];
        lsz[d] = lsz_in ? lsz_in[d] : 1;
    }
    for (int d = 0; d < 3; d++)
        ngrp[d] = (gsz[d] + lsz[d] - 1) / lsz[d];
    const long total_groups = (long)(ngrp[0] * ngrp[1] * ngrp[2]);
    const size_t litems = lsz[0] * lsz[1] * lsz[2];
    const int use_fibers = barriers && litems > 1;

#pragma omp parallel
    {
        WorkItem wi;
        Fiber *fibers = nullptr;
        memset(&wi, 0, sizeof(wi));
        wi.dims = dims;
        for (int d = 0; d < 3; d++) {
            wi.gsz[d] = gsz[d];
            wi.lsz[d] = lsz[d];
            wi.ngrp[d] = ngrp[d];
        }
        tl_fn = fn;
        tl_arg = arg;
        if (use_fibers) {
            if (tl_nstacks < litems) {
                free(tl_stacks);
                tl_stacks = (char *)malloc(kStack * litems);
                tl_nstacks = litems;
            }
            fibers = (Fiber *)calloc(litems, sizeof(Fiber));
        }
#pragma omp for schedule(dynamic, 4)
        for (long g = 0; g < total_groups; g++) {
            size_t grp[3] = {(size_t)g % ngrp[0], ((size_t)g / ngrp[0]) % ngrp[1],
                             (size_t)g / (ngrp[0] * ngrp[1])};
            if (!use_fibers) {
                fiber_mode = 0;
                for (size_t l2 = 0; l2 < lsz[2]; l2++)
                    for (size_t l1 = 0; l1 < lsz[1]; l1++)
                        for (size_t l0 = 0; l0 < lsz[0]; l0++) {
                            size_t lid[3] = {l0, l1, l2};
                            int inside = 1;
                            for (int d = 0; d < 3; d++) {
                                wi.grp[d] = grp[d];
                                wi.lid[d] = lid[d];
                                wi.gid[d] = grp[d] * lsz[d] + lid[d];
                                if (wi.gid[d] >= gsz[d])
                                    inside = 0;
                            }
                            if (!inside)
                                continue;
                            cur_wi = &wi;
                            fn(arg);
                        }
                continue;
            }
            /* One fiber per work-item; run rounds until all are done. */
            fiber_mode = 1;
            size_t n = 0;
            for (size_t l2 = 0; l2 < lsz[2]; l2++)
                for (size_t l1 = 0; l1 < lsz[1]; l1++)
                    for (size_t l0 = 0; l0 < lsz[0]; l0++, n++) {
                        Fiber *f = &fibers[n];
                        size_t lid[3] = {l0, l1, l2};
                        f->wi = wi;
                        for (int d = 0; d < 3; d++) {
                            f->wi.grp[d] = grp[d];
                            f->wi.lid[d] = lid[d];
                            f->wi.gid[d] = grp[d] * lsz[d] + lid[d];
                        }
                        f->done = 0;
                        getcontext(&f->ctx);
                        f->ctx.uc_stack.ss_sp = tl_stacks + n * kStack;
                        f->ctx.uc_stack.ss_size = kStack;
                        f->ctx.uc_link = nullptr;
                        makecontext(&f->ctx, trampoline, 0);
                    }
            size_t left = n;
            while (left) {
                left = 0;
                for (size_t i = 0; i < n; i++) {
                    Fiber *f = &fibers[i];
                    if (f->done)
                        continue;
                    cur_fiber = f;
                    cur_wi = &f->wi;
                    swapcontext(&sched_ctx, &f->ctx);
                    if (!f->done)
                        left++;
                }
            }
            fiber_mode = 0;
        }
        free(fibers);
    }
}

} // namespace oclshim

#define s0 sv_(0)
#define s1 sv_(1)
#define s2 sv_(2)
#define s3 sv_(3)
#define s4 sv_(4)
#define s5 sv_(5)
#define s6 sv_(6)
#define s7 sv_(7)
#define s8 sv_(8)
#define s9 sv_(9)
#define sa sv_(10)
#define sb sv_(11)
#define sc sv_(12)
#define sd sv_(13)
#define se sv_(14)
#define sf sv_(15)
namespace ocl {
#include SAM3_KERNELS_CL
} // namespace ocl
#undef s0
#undef s1
#undef s2
#undef s3
#undef s4
#undef s5
#undef s6
#undef s7
#undef s8
#undef s9
#undef sa
#undef sb
#undef sc
#undef sd
#undef se
#undef sf

using oclshim::run_ndrange;

extern "C" {

/* ---- GEMM: sam3_kernels.cl:70-448, host side sam3_model.c:230-302 ---- */
struct ref_gemm_args {
    int M, N, K;
    const float *A;
    long aoff;
    int lda;
    long sa0, sa1;
    const float *B;
    long boff;
    int ldb;
    long sb0, sb1;
    int transb;
    float *C;
    long coff;
    int ldc;
    long sc0, sc1;
    int nb1;
    const float *bias, *R;
    long roff;
    float alpha;
    int act;
};

#define GEMM_CALL(k)                                                           \
    ocl::k(a->M, a->N, a->K, a->A, a->aoff, a->lda, a->sa0, a->sa1, a->B,     \
           a->boff, a->ldb, a->sb0, a->sb1, a->transb, a->C, a->coff, a->ldc,  \
           a->sc0, a->sc1, a->nb1, a->bias, a->R, a->roff, a->alpha, a->act)

static void k_gemm_cpu_t(void *p) { ref_gemm_args *a = (ref_gemm_args *)p; GEMM_CALL(gemm_cpu_t); }
static void k_gemm_cpu_n(void *p) { ref_gemm_args *a = (ref_gemm_args *)p; GEMM_CALL(gemm_cpu_n); }
static void k_gemm(void *p) { ref_gemm_args *a = (ref_gemm_args *)p; GEMM_CALL(gemm); }
static void k_gemm_big(void *p) { ref_gemm_args *a = (ref_gemm_args *)p; GEMM_CALL(gemm_big); }

/* profile: 0 = cpu (gemm_cpu_t/_n), 1 = GPU kernels with the reference's
 * own choice between gemm and gemm_big (sam3_model.c:240-243). */
void ref_gemm(const ref_gemm_args *args, int nb, int profile)
{
    ref_gemm_args a = *args;
    size_t g[3], l[3] = {16, 16, 1};
    if (profile == 0) {
        g[0] = a.transb ? (size_t)(a.N + 3) / 4 : (size_t)(a.N + 7) / 8;
        g[1] = a.transb ? (size_t)(a.M + 1) / 2 : (size_t)(a.M + 3) / 4;
        g[2] = nb;
        run_ndrange(3, g, nullptr, 0, a.transb ? k_gemm_cpu_t : k_gemm_cpu_n, &a);
        return;
    }
    int big = a.M >= 128 && a.N >= 64 && a.K % 4 == 0 && a.lda % 4 == 0 &&
              a.aoff % 4 == 0 && a.sa0 % 4 == 0 && a.sa1 % 4 == 0 &&
              a.ldb % 4 == 0 && a.boff % 4 == 0 && a.sb0 % 4 == 0 &&
              a.sb1 % 4 == 0;
    int tile = big ? 128 : 64;
    g[0] = (size_t)((a.N + tile - 1) / tile) * 16;
    g[1] = (size_t)((a.M + tile - 1) / tile) * 16;
    g[2] = nb;
    run_ndrange(3, g, l, 1, big ? k_gemm_big : k_gemm, &a);
}

/* ---- layernorm: sam3_kernels.cl:489-514 ---- */
struct ln_args {
    const float *X;
    float *Y;
    const float *g, *b;
    int C;
    float eps;
    int act;
};
static void k_ln(void *p) { ln_args *a = (ln_args *)p; ocl::layernorm(a->X, a->Y, a->g, a->b, a->C, a->eps, a->act); }

void ref_layernorm(const float *X, float *Y, const float *g, const float *b,
                   long rows, int C, float eps, int act, int local)
{
    ln_args a = {X, Y, g, b, C, eps, act};
    size_t ls = local, gs = rows * ls;
    run_ndrange(1, &gs, &ls, 1, k_ln, &a);
}

/* ---- softmax_rows: sam3_kernels.cl:637-656 ---- */
struct sm_args {
    float *S;
    int L;
};
static void k_sm(void *p) { sm_args *a = (sm_args *)p; ocl::softmax_rows(a->S, a->L); }

void ref_softmax_rows(float *S, long rows, int L, int local)
{
    sm_args a = {S, L};
    size_t ls = local, gs = rows * ls;
    run_ndrange(1, &gs, &ls, 1, k_sm, &a);
}

static void run1d(void (*fn)(void *), void *a, size_t n)
{
    size_t l = 256, g = (n + l - 1) / l * l;
    run_ndrange(1, &g, &l, 0, fn, a);
}

/* ---- rope_apply: sam3_kernels.cl:679-698, host sam3_model.c:965-978 ---- */
struct rope_args {
    float *qkv;
    int E, hd, npos;
    const ocl::float2 *cs;
    int total;
};
static void k_rope(void *p) { rope_args *a = (rope_args *)p; ocl::rope_apply(a->qkv, a->E, a->hd, a->npos, a->cs, a->total); }

void ref_rope_apply(float *qkv, long rows, int E, int hd, int npos,
                    const float *cs)
{
    rope_args a = {qkv, E, hd, npos, (const ocl::float2 *)cs, (int)(rows * E)};
    run1d(k_rope, &a, (size_t)rows * E);
}

/* ---- add_bcast: sam3_kernels.cl:701-708 ---- */
struct add_args {
    float *out;
    const float *a, *b;
    int n, bmod;
};
static void k_add(void *p) { add_args *a = (add_args *)p; ocl::add_bcast(a->out, a->a, a->b, a->n, a->bmod); }

void ref_add_bcast(float *out, const float *a, const float *b, long n,
                   long bmod)
{
    add_args x = {out, a, b, (int)n, (int)bmod};
    run1d(k_add, &x, n);
}

/* ---- window_partition / window_unpartition_add: sam3_kernels.cl:712-741,
 * host sam3_model.c:360-392 ---- */
struct wp_args {
    const float *X;
    float *out;
    int H, W, C, ws, nwx, total;
};
static void k_wp(void *p) { wp_args *a = (wp_args *)p; ocl::window_partition(a->X, a->out, a->H, a->W, a->C, a->ws, a->nwx, a->total); }

void ref_window_partition(const float *X, float *out, int H, int C, int ws,
                          int nwx)
{
    int total = nwx * nwx * ws * ws * C;
    wp_args a = {X, out, H, H, C, ws, nwx, total};
    run1d(k_wp, &a, total);
}

struct wu_args {
    float *X;
    const float *Wd;
    int H, W, C, ws, nwx;
};
static void k_wu(void *p) { wu_args *a = (wu_args *)p; ocl::window_unpartition_add(a->X, a->Wd, a->H, a->W, a->C, a->ws, a->nwx); }

void ref_window_unpartition_add(float *X, const float *Wd, int H, int C,
                                int ws, int nwx)
{
    wu_args a = {X, Wd, H, H, C, ws, nwx};
    run1d(k_wu, &a, (size_t)H * H * C);
}

/* ---- patch_im2col: sam3_kernels.cl:661-672, host sam3_model.c:1120-1130 */
struct pi_args {
    const float *img;
    float *out;
    int side, grid, ps;
};
static void k_pi(void *p) { pi_args *a = (pi_args *)p; ocl::patch_im2col(a->img, a->out, a->side, a->grid, a->ps); }

void ref_patch_im2col(const float *img, float *out, int side, int grid, int ps)
{
    pi_args a = {img, out, side, grid, ps};
    run1d(k_pi, &a, (size_t)grid * grid * 3 * ps * ps);
}

/* ---- decoder attention: sam3_kernels.cl:527-633, host sam3_model.c:419-451 */
struct mha_args {
    const float *Q;
    int sq;
    const float *K;
    int sk;
    const float *V;
    int sv;
    float *O;
    int Nq, Nk, dint, c;
    float scale;
    int total;
};
static void k_few(void *p) { mha_args *a = (mha_args *)p; ocl::attn_fewkeys(a->Q, a->sq, a->K, a->sk, a->V, a->sv, a->O, a->Nq, a->Nk, a->dint, a->c, a->scale, a->total); }
static void k_many(void *p) { mha_args *a = (mha_args *)p; ocl::attn_manykeys(a->Q, a->sq, a->K, a->sk, a->V, a->sv, a->O, a->Nq, a->Nk, a->dint, a->c, a->scale, a->total); }

/* Returns -1 on the shape the reference rejects (sam3_model.c:429-430). */
int ref_mha(int P, int Nq, int Nk, int dint, const float *qp, long sq,
            const float *kp, long sk, const float *vp, long sv, float *o)
{
    const int heads = 8;
    int c = dint / heads;
    int many = Nk > 64;
    mha_args a = {qp, (int)sq, kp, (int)sk, vp, (int)sv, o, Nq, Nk, dint, c,
                  1.0f / sqrtf((float)c), P * heads * Nq};
    if (many && c != 16)
        return -1;
    if (many) {
        size_t gs = (size_t)a.total * 256, ls = 256;
        run_ndrange(1, &gs, &ls, 1, k_many, &a);
    }
    else
        run1d(k_few, &a, a.total);
    return 0;
}

/* ---- convt_scatter: sam3_kernels.cl:766-781, host sam3_model.c:394-410 */
struct ct_args {
    const float *G;
    float *out;
    const float *bias, *add;
    int H, W, Co, total, act;
};
static void k_ct(void *p) { ct_args *a = (ct_args *)p; ocl::convt_scatter(a->G, a->out, a->bias, a->add, a->H, a->W, a->Co, a->total, a->act); }

void ref_convt_scatter(const float *G, float *out, const float *bias,
                       const float *add, int P, int H, int W, int Co, int act)
{
    ct_args a = {G, out, bias, add, H, W, Co, P * 4 * H * W * Co, act};
    run1d(k_ct, &a, (size_t)a.total);
}

/* ---- mask_logits: sam3_kernels.cl:789-807, host sam3_model.c:1387-1399 */
struct ml_args {
    const float *U, *hyper;
    float *out;
    int npix, total;
};
static void k_ml(void *p) { ml_args *a = (ml_args *)p; ocl::mask_logits(a->U, a->hyper, a->out, a->npix, a->total); }

void ref_mask_logits(const float *U, const float *hyper, float *out, int npix,
                     long total)
{
    ml_args a = {U, hyper, out, npix, (int)total};
    run1d(k_ml, &a, (size_t)total);
}

/* ---- im2col3x3: sam3_kernels.cl:746-760, host sam3_model.c:1032-1054 */
struct ic_args {
    const float *X;
    float *out;
    int H, W, C, t0, total;
};
static void k_ic(void *p) { ic_args *a = (ic_args *)p; ocl::im2col3x3(a->X, a->out, a->H, a->W, a->C, a->t0, a->total); }

void ref_im2col3x3(const float *X, float *out, int H, int W, int C, int t0, long total)
{
    ic_args a = {X, out, H, W, C, t0, (int)total};
    run1d(k_ic, &a, (size_t)total);
}

/* ---- softmax_ext: sam3_kernels.cl:889-921, host sam3_text.c:319-337 */
struct sx_args {
    float *S;
    int L, Nq, h0, causal;
    const float *dy, *dx;
    int W, nh;
};
static void k_sx(void *p) { sx_args *a = (sx_args *)p; ocl::softmax_ext(a->S, a->L, a->Nq, a->h0, a->causal, a->dy, a->dx, a->W, a->nh); }

void ref_softmax_ext(float *S, long rows, int L, int Nq, int h0, int causal, const float *dy,
                     const float *dx, int W, int nh, int local)
{
    sx_args a = {S, L, Nq, h0, causal, dy, dx, W, nh};
    size_t ls = local, gs = rows * ls;
    run_ndrange(1, &gs, &ls, 1, k_sx, &a);
}

int ref_num_threads(void) { return omp_get_max_threads(); }

} // extern "C"
