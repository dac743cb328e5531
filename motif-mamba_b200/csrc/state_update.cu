// Single-token SSM state update (decode) for sm_100a.
//
// Semantics of mamba_ssm's selective_state_update, which the reference calls at
// mamba_ssm/modules/mamba_simplemotif.py:396-399 (the Triton source is not in the
// reference); restated from the module's torch fallback (:367-376):
//   dt    = softplus(dt + dt_bias)                      (if dt_softplus)
//   state = state * exp(dt * A) + dt * B * x            (in place, state dtype)
//   out   = sum_n state[n] * C[n] + D * x,   out *= silu(z)
// With state_batch_indices (mamba_ssm's continuous-batching argument), batch row b reads and
// updates state row state_batch_indices[b]; a negative index marks a padding row.
// One thread per (batch, channel) keeps its dstate states in registers (fp32 math).
// Decode is latency bound (a few MB per layer), so the kernel is one short launch.
#include "common.cuh"
#include "kernels.h"

namespace mss {

// Fast path for the common layout: 16 states, every per-state row (state, A, B, C) unit
// stride and 16-byte aligned, so each thread moves its rows with 16-byte vector accesses
// (a warp touches whole sectors) instead of 16 scalar strided ones.
// With DTP the dt of each channel is the dt_proj product of the row's dt inputs (folded in;
// rounded to T like the GEMM's output), otherwise it is read from a.dt.
template <typename T, typename ST, bool DTP>
__global__ void __launch_bounds__(128) state_update16_vec_kernel(const ssm_state_update_args a,
                                                                 const ssm_dtproj_args dp) {
    constexpr int NS = 16;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= a.batch * a.dim) return;
    const int64_t b = i / a.dim, d = i - b * a.dim;
    const int64_t g = d / (a.dim / a.n_groups);
    const int64_t sb = a.state_batch_indices ? (int64_t)a.state_batch_indices[b] : b;  // state row
    if (sb < 0 || (a.state_batch_indices && sb >= a.state_batch)) {  // padding / out of range: skipped
        reinterpret_cast<T *>(a.out)[b * a.out_bs + d] = from_f<T>(0.f);
        return;
    }
    const float xv = to_f<T>(reinterpret_cast<const T *>(a.x)[b * a.x_bs + d]);
    float dt;
    if constexpr (DTP) {
        const T *w = reinterpret_cast<const T *>(dp.weight) + d * dp.rank;
        const T *di = reinterpret_cast<const T *>(dp.dt_in) + b * dp.dt_in_bs;
        float acc = 0.f;
        for (int64_t k0 = 0; k0 < dp.rank; k0 += 8) {
            float w8[8], x8[8];
            Vec8<T>::load(w + k0, w8);
            Vec8<T>::load(di + k0, x8);
#pragma unroll
            for (int k = 0; k < 8; ++k) acc = fmaf(w8[k], x8[k], acc);
        }
        dt = to_f<T>(from_f<T>(acc));
    } else {
        dt = to_f<T>(reinterpret_cast<const T *>(a.dt)[b * a.dt_bs + d]);
    }
    if (a.dt_bias) dt += a.dt_bias[d];
    if (a.dt_softplus) dt = softplus20(dt);
    const T *Bp = reinterpret_cast<const T *>(a.B) + b * a.B_bs + g * a.B_gs;
    const T *Cp = reinterpret_cast<const T *>(a.C) + b * a.C_bs + g * a.C_gs;
    ST *st = reinterpret_cast<ST *>(a.state) + sb * a.st_bs + d * a.st_ds;
    const float *Ar = a.A + d * a.A_ds;
    float A[NS], Bv[NS], Cv[NS], sv[NS];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float t8[8];
        Vec8<float>::load(Ar + 8 * h, t8);
#pragma unroll
        for (int j = 0; j < 8; ++j) A[8 * h + j] = t8[j];
        Vec8<T>::load(Bp + 8 * h, t8);
#pragma unroll
        for (int j = 0; j < 8; ++j) Bv[8 * h + j] = t8[j];
        Vec8<T>::load(Cp + 8 * h, t8);
#pragma unroll
        for (int j = 0; j < 8; ++j) Cv[8 * h + j] = t8[j];
        Vec8<ST>::load(st + 8 * h, t8);
#pragma unroll
        for (int j = 0; j < 8; ++j) sv[8 * h + j] = t8[j];
    }
    const float dtx = dt * xv, dl = dt * kLog2e;
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float t8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int n = 8 * h + j;
            t8[j] = fmaf(ex2(dl * A[n]), sv[n], dtx * Bv[n]);
        }
        Vec8<ST>::store(st + 8 * h, t8);
        float r8[8];
        Vec8<ST>::load_rounded(t8, r8);  // the state as stored (state dtype) feeds the output
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
            y0 = fmaf(r8[j], Cv[8 * h + j], y0);
            y1 = fmaf(r8[j + 1], Cv[8 * h + j + 1], y1);
        }
    }
    float y = y0 + y1;
    if (a.D) y = fmaf(a.D[d], xv, y);
    if (a.z) {
        const float zv = to_f<T>(reinterpret_cast<const T *>(a.z)[b * a.z_bs + d]);
        y *= zv * sigmoidf_(zv);
    }
    reinterpret_cast<T *>(a.out)[b * a.out_bs + d] = from_f<T>(y);
}

template <typename T, typename ST, int NS>
__global__ void __launch_bounds__(128) state_update_kernel(const ssm_state_update_args a) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= a.batch * a.dim) return;
    const int64_t b = i / a.dim, d = i - b * a.dim;
    const int64_t g = d / (a.dim / a.n_groups);
    const int64_t sb = a.state_batch_indices ? (int64_t)a.state_batch_indices[b] : b;  // state row
    if (sb < 0 || (a.state_batch_indices && sb >= a.state_batch)) {  // padding / out of range: skipped
        reinterpret_cast<T *>(a.out)[b * a.out_bs + d] = from_f<T>(0.f);
        return;
    }
    const T *X = reinterpret_cast<const T *>(a.x);
    const T *DT = reinterpret_cast<const T *>(a.dt);
    const float xv = to_f<T>(X[b * a.x_bs + d]);
    float dt = to_f<T>(DT[b * a.dt_bs + d]);
    if (a.dt_bias) dt += a.dt_bias[d];
    if (a.dt_softplus) dt = softplus20(dt);
    const T *Bp = reinterpret_cast<const T *>(a.B) + b * a.B_bs + g * a.B_gs;
    const T *Cp = reinterpret_cast<const T *>(a.C) + b * a.C_bs + g * a.C_gs;
    ST *st = reinterpret_cast<ST *>(a.state) + sb * a.st_bs + d * a.st_ds;
    const float dtx = dt * xv;
    float y = 0.f;
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        if (n < a.dstate) {
            const float A = a.A[d * a.A_ds + n * a.A_ns];
            float s = to_f<ST>(st[n * a.st_ns]);
            s = fmaf(ex2(dt * A * kLog2e), s, dtx * to_f<T>(Bp[n]));
            const ST sr = from_f<ST>(s);
            st[n * a.st_ns] = sr;
            y = fmaf(to_f<ST>(sr), to_f<T>(Cp[n]), y);
        }
    }
    if (a.D) y = fmaf(a.D[d], xv, y);
    if (a.z) {
        const float zv = to_f<T>(reinterpret_cast<const T *>(a.z)[b * a.z_bs + d]);
        y *= zv * sigmoidf_(zv);
    }
    reinterpret_cast<T *>(a.out)[b * a.out_bs + d] = from_f<T>(y);
}

template <typename T, typename ST>
static bool su_vec_ok(const ssm_state_update_args &a) {
    auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    return a.dstate == 16 && a.st_ns == 1 && a.A_ns == 1 && al16(a.state) && al16(a.A) && al16(a.B) && al16(a.C) &&
           (a.st_bs * sizeof(ST)) % 16 == 0 && (a.st_ds * sizeof(ST)) % 16 == 0 && (a.A_ds * 4) % 16 == 0 &&
           (a.B_bs * sizeof(T)) % 16 == 0 && (a.B_gs * sizeof(T)) % 16 == 0 && (a.C_bs * sizeof(T)) % 16 == 0 &&
           (a.C_gs * sizeof(T)) % 16 == 0;
}

template <typename T, typename ST>
static cudaError_t su_st(const ssm_state_update_args &a, const ssm_dtproj_args *dp, cudaStream_t st) {
    const int64_t n = a.batch * a.dim;
    const int threads = 128;
    const unsigned blocks = (unsigned)((n + threads - 1) / threads);
    if (n == 0) return cudaSuccess;
    const bool vec = su_vec_ok<T, ST>(a);
    if (dp) {
        auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
        if (!vec || dp->rank % 8 != 0 || dp->rank > 256 || !al16(dp->weight) || !al16(dp->dt_in) ||
            (dp->dt_in_bs * sizeof(T)) % 16 != 0)
            return cudaErrorInvalidValue;
        state_update16_vec_kernel<T, ST, true><<<blocks, threads, 0, st>>>(a, *dp);
        return cudaGetLastError();
    }
    if (vec)
        state_update16_vec_kernel<T, ST, false><<<blocks, threads, 0, st>>>(a, ssm_dtproj_args{});
    else if (a.dstate <= 16)
        state_update_kernel<T, ST, 16><<<blocks, threads, 0, st>>>(a);
    else if (a.dstate <= 32)
        state_update_kernel<T, ST, 32><<<blocks, threads, 0, st>>>(a);
    else if (a.dstate <= 64)
        state_update_kernel<T, ST, 64><<<blocks, threads, 0, st>>>(a);
    else
        state_update_kernel<T, ST, 256><<<blocks, threads, 0, st>>>(a);
    return cudaGetLastError();
}
template <typename T>
static cudaError_t su_t(const ssm_state_update_args &a, const ssm_dtproj_args *dp, cudaStream_t st) {
    switch (a.stype) {
        case MSS_F32: return su_st<T, float>(a, dp, st);
        case MSS_F16: return su_st<T, __half>(a, dp, st);
        default: return su_st<T, __nv_bfloat16>(a, dp, st);
    }
}
cudaError_t launch_state_update(const ssm_state_update_args &a, const ssm_dtproj_args *dp, cudaStream_t st) {
    switch (a.itype) {
        case MSS_F32: return su_t<float>(a, dp, st);
        case MSS_F16: return su_t<__half>(a, dp, st);
        default: return su_t<__nv_bfloat16>(a, dp, st);
    }
}

}  // namespace mss
