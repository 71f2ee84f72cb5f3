/* OpenCL C 1.2 subset for compiling the reference's kernel source
 * (sam3_kernels.cl) unmodified as host C++.
 *
 * TEST INFRASTRUCTURE ONLY: this shim and the library built with it
 * (oracle/_ref/) are the parity checker. Nothing in the product links it.
 *
 * What it provides:
 *  - the vector types float2/4/8/16 with the member names the kernels use
 *    (.x .y .z .w, .lo .hi; the read-only components .s0 ... .sf are
 *    macros for a member call, defined only around the kernel source),
 *    arithmetic operators, splat construction "(float4)(s)" (a C++
 *    functional cast);
 *  - vloadN / vstoreN, mad, dot, fmax, exp, erf, rsqrt, the int atomics;
 *  - work-item functions backed by a thread-local work-item record that the
 *    NDRange executor (ref_kernels.cpp) fills in;
 *  - barrier(): a fiber switch. Every work-group runs as one fiber per
 *    work-item on one OS thread; "__local" variables become
 *    "static thread_local", i.e. shared by the fibers of the group being run.
 *
 * The kernels' two helpers that take a __local pointer parameter
 * (wg_sum/wg_max, sam3_kernels.cl:454,470) are renamed by macro so that the
 * qualifier can be dropped from the parameter list by token pasting; all
 * their call sites pass the array named "scratch".
 *
 * Arithmetic conventions (shared with the C restatement in oracle.c, so
 * both give identical bits): mad() is a fused multiply-add (fmaf); dot() of
 * float4 is fmaf(w, w', fmaf(z, z', fmaf(y, y', x * x'))); exp/erf/sqrt are
 * the C library's float functions; rsqrt(x) = 1 / sqrtf(x). */
#pragma once

#include <cmath>
#include <cstddef>
#include <cstdint>

namespace oclshim {

struct WorkItem {
    size_t gid[3], lid[3], grp[3], gsz[3], lsz[3], ngrp[3];
    unsigned dims;
};

/* Current work-item of this OS thread (set by the executor). */
extern thread_local WorkItem *cur_wi;
/* Barrier: yields to the work-group scheduler (no-op for 1-item groups). */
void wg_barrier();

} // namespace oclshim

namespace ocl {

typedef unsigned char uchar;
typedef unsigned int uint;
typedef unsigned long ulong;

#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2

inline size_t get_global_id(uint d) { return oclshim::cur_wi->gid[d]; }
inline size_t get_local_id(uint d) { return oclshim::cur_wi->lid[d]; }
inline size_t get_group_id(uint d) { return oclshim::cur_wi->grp[d]; }
inline size_t get_global_size(uint d) { return oclshim::cur_wi->gsz[d]; }
inline size_t get_local_size(uint d) { return oclshim::cur_wi->lsz[d]; }
inline size_t get_num_groups(uint d) { return oclshim::cur_wi->ngrp[d]; }
inline void barrier(int) { oclshim::wg_barrier(); }

struct float2 {
    float x, y;
    float2() = default;
    float2(float s) : x(s), y(s) {}
};

struct float4 {
    float x, y, z, w;
    float4() = default;
    float4(float s) : x(s), y(s), z(s), w(s) {}
    float4(float a, float b, float c, float d) : x(a), y(b), z(c), w(d) {}
    float &operator[](int i) { return i == 0 ? x : i == 1 ? y : i == 2 ? z : w; }
    float operator[](int i) const { return i == 0 ? x : i == 1 ? y : i == 2 ? z : w; }
    float sv_(int i) const { return (*this)[i]; }
};

/* .s0 ... .sf are read through sv_(k): ref_kernels.cpp defines the
 * component names as macros around the kernel source. */
struct float8 {
    float4 lo, hi;
    float8() = default;
    float8(float s) : lo(s), hi(s) {}
    float &operator[](int i) { return i < 4 ? lo[i] : hi[i - 4]; }
    float operator[](int i) const { return i < 4 ? lo[i] : hi[i - 4]; }
    float sv_(int i) const { return (*this)[i]; }
};

struct float16 {
    float8 lo, hi;
    float16() = default;
    float16(float s) : lo(s), hi(s) {}
    float &operator[](int i) { return i < 8 ? lo[i] : hi[i - 8]; }
    float operator[](int i) const { return i < 8 ? lo[i] : hi[i - 8]; }
    float sv_(int i) const { return (*this)[i]; }
};

template <class V> struct vlen;
template <> struct vlen<float4> { static const int n = 4; };
template <> struct vlen<float8> { static const int n = 8; };
template <> struct vlen<float16> { static const int n = 16; };

#define OCLSHIM_VOPS(V)                                                        \
    inline V operator+(const V &a, const V &b) { V r; for (int i = 0; i < vlen<V>::n; i++) r[i] = a[i] + b[i]; return r; } \
    inline V operator-(const V &a, const V &b) { V r; for (int i = 0; i < vlen<V>::n; i++) r[i] = a[i] - b[i]; return r; } \
    inline V operator*(const V &a, const V &b) { V r; for (int i = 0; i < vlen<V>::n; i++) r[i] = a[i] * b[i]; return r; } \
    inline V operator*(const V &a, float s) { V r; for (int i = 0; i < vlen<V>::n; i++) r[i] = a[i] * s; return r; } \
    inline V operator*(float s, const V &a) { V r; for (int i = 0; i < vlen<V>::n; i++) r[i] = s * a[i]; return r; } \
    inline V operator/(const V &a, float s) { V r; for (int i = 0; i < vlen<V>::n; i++) r[i] = a[i] / s; return r; } \
    inline V &operator*=(V &a, float s) { for (int i = 0; i < vlen<V>::n; i++) a[i] *= s; return a; } \
    inline V &operator+=(V &a, const V &b) { for (int i = 0; i < vlen<V>::n; i++) a[i] += b[i]; return a; } \
    inline V mad(const V &a, const V &b, const V &c) { V r; for (int i = 0; i < vlen<V>::n; i++) r[i] = fmaf(a[i], b[i], c[i]); return r; }

OCLSHIM_VOPS(float4)
OCLSHIM_VOPS(float8)
OCLSHIM_VOPS(float16)
#undef OCLSHIM_VOPS

inline float mad(float a, float b, float c) { return fmaf(a, b, c); }
inline float dot(const float4 &a, const float4 &b)
{
    return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, a.x * b.x)));
}
inline float fmax(float a, float b) { return fmaxf(a, b); }
inline float exp(float x) { return expf(x); }
inline float erf(float x) { return erff(x); }
inline float sqrt(float x) { return sqrtf(x); }
inline float rsqrt(float x) { return 1.0f / sqrtf(x); }

template <class T> inline float4 vload4(size_t o, const T *p) { p += o * 4; return float4(p[0], p[1], p[2], p[3]); }
template <class T> inline float8 vload8(size_t o, const T *p) { float8 r; p += o * 8; for (int i = 0; i < 8; i++) r[i] = p[i]; return r; }
template <class T> inline float16 vload16(size_t o, const T *p) { float16 r; p += o * 16; for (int i = 0; i < 16; i++) r[i] = p[i]; return r; }
inline void vstore4(const float4 &v, size_t o, float *p) { p += o * 4; for (int i = 0; i < 4; i++) p[i] = v[i]; }
inline void vstore8(const float8 &v, size_t o, float *p) { p += o * 8; for (int i = 0; i < 8; i++) p[i] = v[i]; }
inline void vstore16(const float16 &v, size_t o, float *p) { p += o * 16; for (int i = 0; i < 16; i++) p[i] = v[i]; }

/* Integer atomics. Work-items of a group run as fibers on one OS thread, so
 * __local atomics need no hardware atomics; global ones use GCC builtins. */
inline int atomic_inc(int *p) { return __atomic_fetch_add(p, 1, __ATOMIC_RELAXED); }
inline int atomic_add(int *p, int v) { return __atomic_fetch_add(p, v, __ATOMIC_RELAXED); }
inline int atomic_min(int *p, int v)
{
    int o = __atomic_load_n(p, __ATOMIC_RELAXED);
    while (v < o && !__atomic_compare_exchange_n(p, &o, v, false, __ATOMIC_RELAXED, __ATOMIC_RELAXED))
        ;
    return o;
}
inline int atomic_max(int *p, int v)
{
    int o = __atomic_load_n(p, __ATOMIC_RELAXED);
    while (v > o && !__atomic_compare_exchange_n(p, &o, v, false, __ATOMIC_RELAXED, __ATOMIC_RELAXED))
        ;
    return o;
}

} // namespace ocl

/* Address-space and kernel qualifiers. */
#define __kernel
#define __global
#define __constant const
#define __local static thread_local

/* wg_sum/wg_max take "__local float *scratch": paste the qualifier into a
 * name that expands to nothing (and the call-site argument "scratch" into
 * itself), so the definitions become plain float* functions. */
#define OCLSHIM_STRIP___local
#define OCLSHIM_STRIP_scratch scratch
#define wg_sum(a, b, c) oclshim_wg_sum(a, OCLSHIM_STRIP_##b, c)
#define wg_max(a, b, c) oclshim_wg_max(a, OCLSHIM_STRIP_##b, c)

