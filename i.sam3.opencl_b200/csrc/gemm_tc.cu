// SPDX-License-Identifier: Unlicense
// Persistent tcgen05 GEMM for the backbone's linear layers (QKV, proj, fc1,
// fc2, patch embedding): C = epi(alpha * A . B^T) with bf16 operands, fp32
// accumulation in tensor memory and the reference GEMM's fused epilogue
// (bias, GELU/ReLU, residual; sam3_kernels.cl:57-69, 147-153), plus an
// optional RoPE rotation of the q/k columns (rope_apply,
// sam3_kernels.cl:679-698) so the QKV output feeds attention directly.
//
// One CTA per SM, 6 warps:
//   warp 0  TMA producer: A/B k-blocks of 64 into a 4-stage smem ring;
//   warp 1  tensor-memory owner and MMA issuer (one elected thread):
//           128 x BN x 16 tcgen05.mma into one of two TMEM accumulators;
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//           lanes 32*(w%4)...), epilogue math, global stores, then release
//           the accumulator so the MMA of the next tile overlaps.
// Tiles are visited m-major (all n-tiles of a row block back to back) so a
// row block of A is read from HBM once and re-read from L2.
#include "kernels.h"
#include "tc_ptx.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>

namespace sam3 {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int kThreads = 192;

struct GemmEpi {
    int M, N, K;
    void *C;
    long ldc;
    const float *bias;
    const float *R;
    long ldr;
    int rmod;  // R row = m % rmod (0: R row = m)
    float alpha;
    int act;
    k_rope rope;
    int *err;
};

template <int BN>
struct GemmSmem {
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
    // full[S], empty[S], tfull[2], tempty[2], drain, then tmem base + abort
    static constexpr int BYTES = BAR_OFF + (2 * STAGES + 5) * 8 + 16 + 1024;
};

__device__ __forceinline__ float gelu_erf(float x)
{
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ float act_fn(float v, int act)
{
    if (act == K_ACT_GELU)
        return gelu_erf(v);
    if (act == K_ACT_RELU)
        return fmaxf(v, 0.0f);
    return v;
}

// Table row of the RoPE rotation for output row m.
__device__ __forceinline__ int rope_row(const k_rope &r, int m)
{
    if (r.mode == 1)
        return m % r.npos;
    const int T = r.grid * r.grid, w2 = r.ws * r.ws;
    const int t = m % T, w = t / w2, i = t % w2;
    const int y = (w / r.nwx) * r.ws + i / r.ws, x = (w % r.nwx) * r.ws + i % r.ws;
    return y * r.grid + x;
}

// Applies the epilogue to 32 consecutive accumulator columns of row m,
// starting at column n, and stores them.
template <bool OUT_BF16>
__device__ __forceinline__ void epilogue_chunk(const GemmEpi &p, int m, int n, uint32_t (&r)[32],
                                               int rrow)
{
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; j++)
        v[j] = p.alpha * __uint_as_float(r[j]);
    const int nvalid = min(32, p.N - n);
    if (p.bias) {
#pragma unroll
        for (int j = 0; j < 32; j++)
            if (j < nvalid)
                v[j] += __ldg(p.bias + n + j);
    }
    if (p.act != K_ACT_NONE) {
#pragma unroll
        for (int j = 0; j < 32; j++)
            v[j] = act_fn(v[j], p.act);
    }
    if (p.R) {
        const float *rp = p.R + (long)(p.rmod ? m % p.rmod : m) * p.ldr + n;
        if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(rp) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 q = *reinterpret_cast<const float4 *>(rp + j);
                v[j] += q.x;
                v[j + 1] += q.y;
                v[j + 2] += q.z;
                v[j + 3] += q.w;
            }
        }
        else {
            for (int j = 0; j < nvalid; j++)
                v[j] += rp[j];
        }
    }
    if (p.rope.mode && n < 2 * p.rope.E) {
        // 32-column chunks never straddle the q/k boundary (E % 64 == 0).
        const float2 *cs = reinterpret_cast<const float2 *>(p.rope.cs) +
                           (long)rrow * (p.rope.hd / 2) + ((n % p.rope.hd) >> 1);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            const float2 rot = __ldg(cs + (j >> 1));
            const float a = v[j], b = v[j + 1];
            v[j] = a * rot.x - b * rot.y;
            v[j + 1] = a * rot.y + b * rot.x;
        }
    }
    if (OUT_BF16) {
        __nv_bfloat16 *cp = reinterpret_cast<__nv_bfloat16 *>(p.C) + (long)m * p.ldc + n;
        if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint4 q;
                q.x = pack_bf16x2(v[j], v[j + 1]);
                q.y = pack_bf16x2(v[j + 2], v[j + 3]);
                q.z = pack_bf16x2(v[j + 4], v[j + 5]);
                q.w = pack_bf16x2(v[j + 6], v[j + 7]);
                *reinterpret_cast<uint4 *>(cp + j) = q;
            }
        }
        else {
            for (int j = 0; j < nvalid; j++)
                cp[j] = __float2bfloat16_rn(v[j]);
        }
    }
    else {
        float *cp = reinterpret_cast<float *>(p.C) + (long)m * p.ldc + n;
        if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4 *>(cp + j) =
                    make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
        else {
            for (int j = 0; j < nvalid; j++)
                cp[j] = v[j];
        }
    }
}

template <int BN, bool OUT_BF16>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmEpi p)
{
    using L = GemmSmem<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
    uint64_t *empty = full + STAGES;
    uint64_t *tfull = empty + STAGES;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int num_m = (p.M + BM - 1) / BM;
    const int num_n = (p.N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int kblocks = (p.K + BK - 1) / BK;

    if (warp == 0) {
        if (elect_one()) {
            prefetch_tmap(&tmA);
            prefetch_tmap(&tmB);
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, last_parity = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                const int m0 = (t / num_n) * BM, n0 = (t % num_n) * BN;
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, p.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sa = smem + stage * L::STAGE_BYTES;
                    mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
                    tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
                    tma_load_2d(sa + L::A_BYTES, &tmB, &full[stage], kb * BK, n0);
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Let every copy this thread issued land before the CTA exits.
            for (int s = 0; s < STAGES; s++)
                if (issued_mask & (1u << s)) {
                    volatile int no_abort = 0;
                    mbar_wait(&full[s], (last_parity >> s) & 1, p.err, &no_abort);
                }
        }
    }
    else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, 0, 0);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err, abort_flag))
                    break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(&full[stage], phase, p.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_addr(smem + stage * L::STAGE_BYTES);
                    const uint32_t sb = sa + L::A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        tc_mma(d, sw128_desc(sa + k * 32, 16, 1024),
                               sw128_desc(sb + k * 32, 16, 1024), idesc, (kb | k) != 0);
                    tc_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok)
                    break;
                tc_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0)
                    acc_phase ^= 1;
            }
            // Drain: wait until every MMA issued above has completed, so
            // tensor memory is idle before it is freed.
            tc_commit(drain);
            volatile int no_abort = 0;
            mbar_wait(drain, 0, p.err, &no_abort);
        }
    }
    else {
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            const bool ok = mbar_wait(&tfull[acc], acc_phase, p.err, abort_flag);
            if (!__all_sync(0xffffffffu, ok))
                break;
            tc_fence_after();
            const int m0 = (t / num_n) * BM, n0 = (t % num_n) * BN;
            const int m = m0 + row_in_tile;
            const int rrow = (p.rope.mode && m < p.M) ? rope_row(p.rope, m) : 0;
            const uint32_t tbase =
                tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                uint32_t r[32];
                tmem_ld32(tbase + c * 32, r);
                tmem_wait_ld();
                const int n = n0 + c * 32;
                if (m < p.M && n < p.N)
                    epilogue_chunk<OUT_BF16>(p, m, n, r, rrow);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0)
                acc_phase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * BN);
    }
}

template <int BN, bool OUT_BF16>
int launch(const CUtensorMap &ta, const CUtensorMap &tb, const GemmEpi &p, int num_sms,
           cudaStream_t s)
{
    using L = GemmSmem<BN>;
    auto kern = gemm_bf16_tc_kernel<BN, OUT_BF16>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    if (e != cudaSuccess)
        return (int)e;
    const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    kern<<<grid, kThreads, L::BYTES, s>>>(ta, tb, p);
    return (int)cudaGetLastError();
}

}  // namespace
}  // namespace sam3

extern "C" int k_gemm_bf16_tc(int M, int N, int K, const void *A, int lda, const void *B,
                              int ldb, void *C, int ldc, int c_bf16, const float *bias,
                              const float *R, int ldr, int rmod, float alpha, int act,
                              const struct k_rope *rope, int *err, int num_sms, k_stream s)
{
    using namespace sam3;
    if (M <= 0 || N <= 0 || K <= 0 || (lda & 7) || (ldb & 7) || lda < K || ldb < K)
        return K_EARG;
    if (rope && rope->mode && (rope->hd != 64 || (rope->E & 63) || 2 * rope->E > N))
        return K_EARG;
    const int BN = N <= 128 ? 128 : 256;
    CUtensorMap ta, tb;
    if (!make_tmap_bf16(&ta, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM) ||
        !make_tmap_bf16(&tb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, (uint32_t)BN))
        return K_ETMAP;
    GemmEpi p;
    p.M = M;
    p.N = N;
    p.K = K;
    p.C = C;
    p.ldc = ldc;
    p.bias = bias;
    p.R = R;
    p.ldr = ldr;
    p.rmod = rmod;
    p.alpha = alpha;
    p.act = act;
    if (rope)
        p.rope = *rope;
    else
        p.rope = k_rope{nullptr, 0, 0, 0, 0, 0, 0, 0};
    p.err = err;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    if (BN == 128)
        return c_bf16 ? launch<128, true>(ta, tb, p, num_sms, st)
                      : launch<128, false>(ta, tb, p, num_sms, st);
    return c_bf16 ? launch<256, true>(ta, tb, p, num_sms, st)
                  : launch<256, false>(ta, tb, p, num_sms, st);
}
