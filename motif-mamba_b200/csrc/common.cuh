// Device-side helpers shared by the selective-scan, conv1d and state-update kernels.
// sm_100a only.  Element types: float, __half, __nv_bfloat16.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>

#include "motif_ssm.h"

namespace mss {

constexpr int kChunkLen = 256;     // timesteps per x chunk (ss_chunk_len)
constexpr int kMaxDstate = 256;    // largest dstate the forward accepts (the reference's limit)
constexpr int kMaxDstateBwd = 256; // largest dstate the backward accepts (blocks of 16)
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kNumSMs = 148;      // B200 SMs (launch shapes are sized for one wave of them)

// ---- scalar conversions ------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// ---- 8-element vector moves between shared memory and fp32 registers ----------------
// p must be 16-byte aligned (8 x 16-bit = 16 B; 8 x fp32 = 2 x 16 B).
template <typename T> struct Vec8;
template <> struct Vec8<float> {
    static __device__ __forceinline__ void load_rounded(const float (&v)[8], float (&r)[8]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = v[i];
    }
    static __device__ __forceinline__ void load(const float *p, float (&v)[8]) {
        float4 a = reinterpret_cast<const float4 *>(p)[0];
        float4 b = reinterpret_cast<const float4 *>(p)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    static __device__ __forceinline__ void store(float *p, const float (&v)[8]) {
        reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
};
template <> struct Vec8<__nv_bfloat16> {
    // v rounded to bf16 and back (the value a store followed by a load would give)
    static __device__ __forceinline__ void load_rounded(const float (&v)[8], float (&r)[8]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
    }
    static __device__ __forceinline__ void load(const __nv_bfloat16 *p, float (&v)[8]) {
        uint4 r = *reinterpret_cast<const uint4 *>(p);
        uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    static __device__ __forceinline__ void store(__nv_bfloat16 *p, const float (&v)[8]) {
        uint4 r;
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t *>(&h);
        }
        r.x = w[0]; r.y = w[1]; r.z = w[2]; r.w = w[3];
        *reinterpret_cast<uint4 *>(p) = r;
    }
};
template <> struct Vec8<__half> {
    static __device__ __forceinline__ void load_rounded(const float (&v)[8], float (&r)[8]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = __half2float(__float2half_rn(v[i]));
    }
    static __device__ __forceinline__ void load(const __half *p, float (&v)[8]) {
        uint4 r = *reinterpret_cast<const uint4 *>(p);
        uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float2 f = __half22float2(*reinterpret_cast<__half2 *>(&w[i]));
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    static __device__ __forceinline__ void store(__half *p, const float (&v)[8]) {
        uint4 r;
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t *>(&h);
        }
        r.x = w[0]; r.y = w[1]; r.z = w[2]; r.w = w[3];
        *reinterpret_cast<uint4 *>(p) = r;
    }
};

// ---- math ----------------------------------------------------------------------------
// 2^x on the SFU (PTX ex2.approx, flush-to-zero): the scan's decay factors.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// softplus with torch's threshold of 20 (the reference kernel uses the same rule,
// selective_scan_fwd_kernel.cuh:388-390): log(1 + e^x) for x <= 20, x above.
// log(1 + y), y = e^x, is taken from the SFU logarithm where the result is >= ~0.06; for
// smaller y the SFU log of (1 + y) would lose relative accuracy (its error is absolute), so
// the Taylor series y - y^2/2 + y^3/3 - y^4/4 + y^5/5 is used (truncation < y^6/6, i.e.
// < 1e-8 relative for y < 1/16).
__device__ __forceinline__ float softplus20(float x) {
    const float y = __expf(x);
    const float big = __logf(1.f + y);
    const float small = y * fmaf(y, fmaf(y, fmaf(y, fmaf(y, 0.2f, -0.25f), 1.f / 3.f), -0.5f), 1.f);
    const float r = y < 0.0625f ? small : big;
    return x <= 20.f ? r : x;
}
// softplus'(x) = sigmoid(x) = 1 - e^(-s) from the softplus output s = softplus(x) >= 0.  For
// s < 1/16 the difference 1 - e^(-s) would cancel (and be 0 once e^(-s) rounds to 1, i.e. for
// x below about -16), so the series s - s^2/2 + s^3/6 - s^4/24 is used there (truncation
// < s^5/120, i.e. < 2e-7 relative).
__device__ __forceinline__ float softplus_grad_from_out(float s) {
    const float big = 1.f - ex2(-s * kLog2e);
    const float small = s * fmaf(s, fmaf(s, fmaf(s, -1.f / 24.f, 1.f / 6.f), -0.5f), 1.f);
    return s < 0.0625f ? small : big;
}
// 1 / (1 + e^-x) with the SFU exponential and a fast reciprocal (relative error ~1e-7).
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// ---- packed fp32 pairs (Blackwell fma/mul .f32x2: one instruction for two lanes of math) ----
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pack2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 unpack2(f32x2 v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// 2^x of both halves (two SFU ex2).
__device__ __forceinline__ f32x2 ex2x2(f32x2 x) {
    const float2 v = unpack2(x);
    return pack2(ex2(v.x), ex2(v.y));
}

// ---- cp.async (16-byte, zero-filling) ---------------------------------------------------
// Copies src_bytes (0..16) from global to shared and zero-fills the rest of the 16 bytes.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes) {
    unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Vector fp32 reduction into global memory (sm_90+): 4 consecutive floats, 16-B aligned.
__device__ __forceinline__ void red_add_v4(float *gptr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(gptr), "f"(a), "f"(b), "f"(c),
                 "f"(d)
                 : "memory");
}

// ---- tile staging ------------------------------------------------------------------------
// Copies rows [0, nrows) x timesteps [t0, t0 + TT) of a (row, t) array whose rows start
// at g0 + r * rstride (t unit-stride) into shared memory rows of pitch rp bytes.
// Rows >= nrows_valid and timesteps >= tvalid (relative to t0) are zero-filled; nothing
// outside the valid box is read.  `aligned` says that every row start and t0 are 16-byte
// aligned, so 16-byte cp.async can be used; otherwise plain element loads are used.
template <typename T, int TT>
__device__ __forceinline__ void stage_tile(char *sdst, int rp, const T *g0, int64_t rstride, int nrows,
                                           int nrows_valid, int64_t t0, int tvalid, bool aligned,
                                           int tid, int nthr) {
    constexpr int EPC = 16 / sizeof(T);  // elements per 16-byte chunk
    constexpr int CPR = TT / EPC;        // chunks per row
    static_assert(TT % EPC == 0, "tile length must hold whole 16-byte chunks");
    if (aligned) {
        for (int i = tid; i < nrows * CPR; i += nthr) {
            const int r = i / CPR, c = i - r * CPR;
            const int tt = c * EPC;
            int nb = 0;
            if (r < nrows_valid) nb = max(0, min(EPC, tvalid - tt)) * (int)sizeof(T);
            const T *src = nb > 0 ? g0 + (int64_t)r * rstride + t0 + tt : g0;
            cp_async16(sdst + r * rp + tt * (int)sizeof(T), src, nb);
        }
    } else {
        for (int i = tid; i < nrows * TT; i += nthr) {
            const int r = i / TT, tt = i - r * TT;
            T v = from_f<T>(0.f);
            if (r < nrows_valid && tt < tvalid) v = g0[(int64_t)r * rstride + t0 + tt];
            *reinterpret_cast<T *>(sdst + r * rp + tt * (int)sizeof(T)) = v;
        }
    }
}

// Writes rows [0, nrows_valid) x timesteps [t0, t0 + tvalid) from shared rows (pitch rp)
// to global rows g0 + r * rstride.  16-byte stores where the row start is aligned.
template <typename T, int TT>
__device__ __forceinline__ void store_tile(T *g0, int64_t rstride, const char *ssrc, int rp, int nrows_valid,
                                           int64_t t0, int tvalid, bool aligned, int tid, int nthr) {
    constexpr int EPC = 16 / sizeof(T);
    constexpr int CPR = TT / EPC;
    if (aligned) {
        for (int i = tid; i < nrows_valid * CPR; i += nthr) {
            const int r = i / CPR, c = i - r * CPR;
            const int tt = c * EPC;
            const char *s = ssrc + r * rp + tt * (int)sizeof(T);
            T *g = g0 + (int64_t)r * rstride + t0 + tt;
            if (tt + EPC <= tvalid) {
                *reinterpret_cast<uint4 *>(g) = *reinterpret_cast<const uint4 *>(s);
            } else {
                for (int e = 0; e < EPC && tt + e < tvalid; ++e)
                    g[e] = reinterpret_cast<const T *>(s)[e];
            }
        }
    } else {
        for (int i = tid; i < nrows_valid * TT; i += nthr) {
            const int r = i / TT, tt = i - r * TT;
            if (tt < tvalid)
                g0[(int64_t)r * rstride + t0 + tt] = *reinterpret_cast<const T *>(ssrc + r * rp + tt * (int)sizeof(T));
        }
    }
}

// Raises a kernel's dynamic shared-memory limit once per device (the attribute is per device
// context); `mask` is the call site's record of the devices already done.
inline cudaError_t set_smem_once(std::atomic<unsigned long long> &mask, const void *fn, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) mask.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

}  // namespace mss
