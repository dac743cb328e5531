// Fused residual add + RMSNorm for the pre-norm stack (sm_100a).
//
// The reference stack runs Add -> Norm with one fused kernel when fused_add_norm is set
// (mamba_ssm/models/mixer_seq_simple.py:190-211, layer_norm_fn with prenorm=True and
// residual_in_fp32): residual = x + residual (in fp32 when residual_in_fp32), out =
// residual * rsqrt(mean(residual^2) + eps) * weight in x's type.  One warp per row: the row
// is read once (x and the incoming residual, 16-byte vectors), the new residual written
// once, the sum of squares reduced with shuffles, and the normalised row written; the fp32
// row stays in registers between the two halves.  HBM-bound.
#include "common.cuh"
#include "kernels.h"

namespace mss {

namespace nrm {
constexpr int NT = 256;      // 8 rows (warps) per CTA
constexpr int MAXV = 16;     // up to 16 vectors of 8 per lane: rows of up to 4096 elements in registers
}  // namespace nrm

template <typename T, typename RIN, typename ROUT, typename WT, int NV>
__global__ void __launch_bounds__(nrm::NT) add_rms_norm_kernel(const add_rms_norm_args a) {
    const int lane = threadIdx.x & 31;
    const int64_t row = blockIdx.x * (int64_t)(nrm::NT / 32) + (threadIdx.x >> 5);
    if (row >= a.rows) return;
    const int64_t D = a.dim;
    const T *x = reinterpret_cast<const T *>(a.x) + row * a.x_rs;
    const RIN *rin = a.residual_in ? reinterpret_cast<const RIN *>(a.residual_in) + row * a.rin_rs : nullptr;
    ROUT *rout = reinterpret_cast<ROUT *>(a.residual_out) + row * a.rout_rs;
    T *out = reinterpret_cast<T *>(a.out) + row * a.out_rs;
    const WT *w = reinterpret_cast<const WT *>(a.weight);
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < NV; ++q) {
        const int64_t c = (int64_t)(q * 32 + lane) * 8;
        if (c < D) {
            Vec8<T>::load(x + c, v[q]);
            if (rin) {
                float r8[8];
                Vec8<RIN>::load(rin + c, r8);
#pragma unroll
                for (int i = 0; i < 8; ++i) v[q][i] += r8[i];
            }
            Vec8<ROUT>::store(rout + c, v[q]);
            float rr[8];
            Vec8<ROUT>::load_rounded(v[q], rr);  // the residual as stored feeds the norm
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[q][i] = rr[i];
                ss = fmaf(rr[i], rr[i], ss);
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float rstd = rsqrtf(ss / (float)D + a.eps);
    if (a.rstd && lane == 0) a.rstd[row] = rstd;
#pragma unroll
    for (int q = 0; q < NV; ++q) {
        const int64_t c = (int64_t)(q * 32 + lane) * 8;
        if (c < D) {
            float w8[8], o8[8];
            Vec8<WT>::load(w + c, w8);
#pragma unroll
            for (int i = 0; i < 8; ++i) o8[i] = v[q][i] * rstd * w8[i];
            Vec8<T>::store(out + c, o8);
        }
    }
}

template <typename T, typename RIN, typename ROUT, typename WT>
static cudaError_t arn_nv(const add_rms_norm_args &a, cudaStream_t st) {
    const unsigned blocks = (unsigned)((a.rows + nrm::NT / 32 - 1) / (nrm::NT / 32));
    const int64_t nv = (a.dim + 255) / 256;
    if (nv <= 1) add_rms_norm_kernel<T, RIN, ROUT, WT, 1><<<blocks, nrm::NT, 0, st>>>(a);
    else if (nv <= 2) add_rms_norm_kernel<T, RIN, ROUT, WT, 2><<<blocks, nrm::NT, 0, st>>>(a);
    else if (nv <= 4) add_rms_norm_kernel<T, RIN, ROUT, WT, 4><<<blocks, nrm::NT, 0, st>>>(a);
    else if (nv <= 8) add_rms_norm_kernel<T, RIN, ROUT, WT, 8><<<blocks, nrm::NT, 0, st>>>(a);
    else if (nv <= 12) add_rms_norm_kernel<T, RIN, ROUT, WT, 12><<<blocks, nrm::NT, 0, st>>>(a);
    else add_rms_norm_kernel<T, RIN, ROUT, WT, 16><<<blocks, nrm::NT, 0, st>>>(a);
    return cudaGetLastError();
}
template <typename T, typename RIN, typename ROUT>
static cudaError_t arn_w(const add_rms_norm_args &a, cudaStream_t st) {
    return a.wtype == MSS_F32 ? arn_nv<T, RIN, ROUT, float>(a, st) : arn_nv<T, RIN, ROUT, T>(a, st);
}
template <typename T, typename RIN>
static cudaError_t arn_ro(const add_rms_norm_args &a, cudaStream_t st) {
    return a.rout_type == MSS_F32 ? arn_w<T, RIN, float>(a, st) : arn_w<T, RIN, T>(a, st);
}
template <typename T>
static cudaError_t arn_ri(const add_rms_norm_args &a, cudaStream_t st) {
    return a.rin_type == MSS_F32 ? arn_ro<T, float>(a, st) : arn_ro<T, T>(a, st);
}
cudaError_t launch_add_rms_norm(const add_rms_norm_args &a, cudaStream_t st) {
    switch (a.itype) {
        case MSS_F32: return arn_ri<float>(a, st);
        case MSS_F16: return arn_ri<__half>(a, st);
        default: return arn_ri<__nv_bfloat16>(a, st);
    }
}

}  // namespace mss
