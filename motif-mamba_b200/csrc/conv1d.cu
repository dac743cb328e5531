// Depthwise causal conv1d (+SiLU) forward / backward / single-step update for sm_100a.
//
// Semantics of the external causal-conv1d package the reference calls
// (mamba_ssm/ops/selective_scan_interface.py:482-484, 567-569, 635-637;
//  mamba_ssm/modules/mamba_simplemotif.py:298-303, 352-358), restated from the
// module's own torch fallbacks (mamba_simplemotif.py:75-83, 294-295, 344-350):
//   pre[b,c,t] = bias_c + sum_{k<W} w[c,k] * x[b,c,t-W+1+k]      (x = 0 for t < 0)
//   out        = silu(pre) if silu else pre
// Backward:  dpre = dout * silu'(pre);  dx[t] = sum_k w[k] dpre[t+W-1-k];
//            dw[c,k] = sum_{b,t} dpre[t] x[t-W+1+k];  dbias[c] = sum_{b,t} dpre[t].
//
// Both directions are HBM-streaming: one warp walks one (b, c) row in steps of 256
// timesteps, each lane owning 8 consecutive outputs read with 16-byte vector loads.  The
// W-1 halo comes from the neighbouring vector (an L1 hit).  Weight gradients are kept
// per lane, reduced across the warp with shuffles and added once per row.
#include "common.cuh"
#include "kernels.h"

namespace mss {

template <typename T>
__device__ __forceinline__ void load8_row(const T *row, int64_t t, int64_t L, bool vec, float (&v)[8]) {
    if (vec && t >= 0 && t + 8 <= L) {
        Vec8<T>::load(row + t, v);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (t + i >= 0 && t + i < L) ? to_f<T>(row[t + i]) : 0.f;
    }
}
template <typename T>
__device__ __forceinline__ void store8_row(T *row, int64_t t, int64_t L, bool vec, const float (&v)[8]) {
    if (vec && t + 8 <= L) {
        Vec8<T>::store(row + t, v);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (t + i < L) row[t + i] = from_f<T>(v[i]);
    }
}

template <typename W>
__device__ __forceinline__ float ldw(const void *p, int64_t i) {
    return to_f<W>(reinterpret_cast<const W *>(p)[i]);
}

template <typename T, typename WT, int KW>
__global__ void __launch_bounds__(256) conv1d_fwd_kernel(const conv1d_args a, int vec) {
    const int lane = threadIdx.x & 31;
    const int64_t nrows = a.batch * a.dim;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < nrows; r += nwarps) {
        const int64_t b = r / a.dim, c = r - b * a.dim;
        float w[KW];
#pragma unroll
        for (int k = 0; k < KW; ++k) w[k] = ldw<WT>(a.weight, c * a.w_ds + k * a.w_ks);
        const float bias = a.bias ? ldw<WT>(a.bias, c) : 0.f;
        const T *xr = reinterpret_cast<const T *>(a.x) + b * a.x_bs + c * a.x_ds;
        T *orow = reinterpret_cast<T *>(a.out) + b * a.out_bs + c * a.out_ds;
        for (int64_t t0 = (int64_t)lane * 8; t0 < a.seqlen; t0 += 256) {
            float cur[8], prev[8];
            load8_row(xr, t0, a.seqlen, vec, cur);
            load8_row(xr, t0 - 8, a.seqlen, vec, prev);
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float acc = bias;
#pragma unroll
                for (int k = 0; k < KW; ++k) {
                    const int j = i - (KW - 1) + k;  // offset relative to t0
                    const float xv = j >= 0 ? cur[j] : prev[8 + j];
                    acc = fmaf(w[k], xv, acc);
                }
                o[i] = a.silu ? acc * sigmoidf_(acc) : acc;
            }
            store8_row(orow, t0, a.seqlen, vec, o);
        }
    }
}

template <typename T, typename WT, int KW>
__global__ void __launch_bounds__(256) conv1d_bwd_kernel(const conv1d_args a, int vec) {
    const int lane = threadIdx.x & 31;
    const int64_t nrows = a.batch * a.dim;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t r = warp; r < nrows; r += nwarps) {
        const int64_t b = r / a.dim, c = r - b * a.dim;
        float w[KW];
#pragma unroll
        for (int k = 0; k < KW; ++k) w[k] = ldw<WT>(a.weight, c * a.w_ds + k * a.w_ks);
        const float bias = a.bias ? ldw<WT>(a.bias, c) : 0.f;
        const T *xr = reinterpret_cast<const T *>(a.x) + b * a.x_bs + c * a.x_ds;
        const T *dor = reinterpret_cast<const T *>(a.dout) + b * a.dout_bs + c * a.dout_ds;
        T *dxr = reinterpret_cast<T *>(a.dx) + b * a.dx_bs + c * a.dx_ds;
        float dw[KW], db = 0.f;
#pragma unroll
        for (int k = 0; k < KW; ++k) dw[k] = 0.f;
        for (int64_t t0 = (int64_t)lane * 8; t0 < a.seqlen; t0 += 256) {
            // x over [t0-8, t0+16), dout over [t0, t0+16)
            float xp[8], xc[8], xn[8], dc[8], dn[8];
            load8_row(xr, t0 - 8, a.seqlen, vec, xp);
            load8_row(xr, t0, a.seqlen, vec, xc);
            load8_row(xr, t0 + 8, a.seqlen, vec, xn);
            load8_row(dor, t0, a.seqlen, vec, dc);
            load8_row(dor, t0 + 8, a.seqlen, vec, dn);
            auto xat = [&](int j) -> float {  // x at t0 + j, j in [-8, 16)
                return j < 0 ? xp[8 + j] : (j < 8 ? xc[j] : xn[j - 8]);
            };
            // dpre at t0 + i for i in [0, 8 + KW - 1)
            float dpre[8 + KW - 1];
#pragma unroll
            for (int i = 0; i < 8 + KW - 1; ++i) {
                float pre = bias;
#pragma unroll
                for (int k = 0; k < KW; ++k) pre = fmaf(w[k], xat(i - (KW - 1) + k), pre);
                const float dov = i < 8 ? dc[i] : dn[i - 8];  // zero beyond L (load8_row fills 0)
                float g = dov;
                if (a.silu) {
                    const float s = sigmoidf_(pre);
                    g = dov * s * (1.f + pre * (1.f - s));
                }
                dpre[i] = g;
            }
            float dxv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < KW; ++k) acc = fmaf(w[k], dpre[i + (KW - 1) - k], acc);
                dxv[i] = acc;
            }
            store8_row(dxr, t0, a.seqlen, vec, dxv);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (t0 + i < a.seqlen) {
                    db += dpre[i];
#pragma unroll
                    for (int k = 0; k < KW; ++k) dw[k] = fmaf(dpre[i], xat(i - (KW - 1) + k), dw[k]);
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            db += __shfl_xor_sync(0xffffffffu, db, off);
#pragma unroll
            for (int k = 0; k < KW; ++k) dw[k] += __shfl_xor_sync(0xffffffffu, dw[k], off);
        }
        if (lane == 0) {
#pragma unroll
            for (int k = 0; k < KW; ++k) atomicAdd(a.dweight + c * KW + k, dw[k]);
            if (a.dbias) atomicAdd(a.dbias + c, db);
        }
    }
}

template <typename T, typename WT, typename ST>
__global__ void conv1d_update_kernel(const conv1d_update_args a) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= a.batch * a.dim) return;
    const int64_t b = i / a.dim, c = i - b * a.dim;
    ST *st = reinterpret_cast<ST *>(a.conv_state) + b * a.cs_bs + c * a.cs_ds;
    const float xv = to_f<T>(reinterpret_cast<const T *>(a.x)[b * a.x_bs + c]);
    const int S = (int)a.state_len, KW = (int)a.width;
    float acc = a.bias ? ldw<WT>(a.bias, c) : 0.f;
    // shift left by one and append x; the taps read the newest KW entries
    for (int s = 0; s < S; ++s) {
        const float v = s + 1 < S ? to_f<ST>(st[s + 1]) : xv;
        st[s] = from_f<ST>(v);
        const int k = s - (S - KW);
        if (k >= 0) acc = fmaf(ldw<WT>(a.weight, c * a.w_ds + k * a.w_ks), to_f<ST>(st[s]), acc);
    }
    if (a.silu) acc = acc * sigmoidf_(acc);
    reinterpret_cast<T *>(a.out)[b * a.out_bs + c] = from_f<T>(acc);
}

// ---- dispatch -----------------------------------------------------------------------------
template <typename T, typename WT, int KW>
static cudaError_t conv_dir(const conv1d_args &a, bool vec, bool bwd, cudaStream_t st) {
    const int64_t nrows = a.batch * a.dim;
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((nrows * 32 + threads - 1) / threads, 148 * 16);
    if (blocks <= 0) return cudaSuccess;
    if (bwd)
        conv1d_bwd_kernel<T, WT, KW><<<(int)blocks, threads, 0, st>>>(a, vec ? 1 : 0);
    else
        conv1d_fwd_kernel<T, WT, KW><<<(int)blocks, threads, 0, st>>>(a, vec ? 1 : 0);
    return cudaGetLastError();
}
template <typename T, typename WT>
static cudaError_t conv_w(const conv1d_args &a, bool vec, bool bwd, cudaStream_t st) {
    switch (a.width) {
        case 2: return conv_dir<T, WT, 2>(a, vec, bwd, st);
        case 3: return conv_dir<T, WT, 3>(a, vec, bwd, st);
        default: return conv_dir<T, WT, 4>(a, vec, bwd, st);
    }
}
template <typename T>
static cudaError_t conv_t(const conv1d_args &a, bool vec, bool bwd, cudaStream_t st) {
    switch (a.wtype) {
        case MSS_F32: return conv_w<T, float>(a, vec, bwd, st);
        case MSS_F16: return conv_w<T, __half>(a, vec, bwd, st);
        default: return conv_w<T, __nv_bfloat16>(a, vec, bwd, st);
    }
}
static cudaError_t conv_any(const conv1d_args &a, bool vec, bool bwd, cudaStream_t st) {
    switch (a.itype) {
        case MSS_F32: return conv_t<float>(a, vec, bwd, st);
        case MSS_F16: return conv_t<__half>(a, vec, bwd, st);
        default: return conv_t<__nv_bfloat16>(a, vec, bwd, st);
    }
}
cudaError_t launch_conv1d_fwd(const conv1d_args &a, bool vec, cudaStream_t st) { return conv_any(a, vec, false, st); }
cudaError_t launch_conv1d_bwd(const conv1d_args &a, bool vec, cudaStream_t st) { return conv_any(a, vec, true, st); }

template <typename T, typename WT>
static cudaError_t upd_w(const conv1d_update_args &a, cudaStream_t st) {
    const int64_t n = a.batch * a.dim;
    const int threads = 256;
    const int64_t blocks = (n + threads - 1) / threads;
    if (blocks <= 0) return cudaSuccess;
    switch (a.stype) {
        case MSS_F32: conv1d_update_kernel<T, WT, float><<<(unsigned)blocks, threads, 0, st>>>(a); break;
        case MSS_F16: conv1d_update_kernel<T, WT, __half><<<(unsigned)blocks, threads, 0, st>>>(a); break;
        default: conv1d_update_kernel<T, WT, __nv_bfloat16><<<(unsigned)blocks, threads, 0, st>>>(a); break;
    }
    return cudaGetLastError();
}
template <typename T>
static cudaError_t upd_t(const conv1d_update_args &a, cudaStream_t st) {
    switch (a.wtype) {
        case MSS_F32: return upd_w<T, float>(a, st);
        case MSS_F16: return upd_w<T, __half>(a, st);
        default: return upd_w<T, __nv_bfloat16>(a, st);
    }
}
cudaError_t launch_conv1d_update(const conv1d_update_args &a, cudaStream_t st) {
    switch (a.itype) {
        case MSS_F32: return upd_t<float>(a, st);
        case MSS_F16: return upd_t<__half>(a, st);
        default: return upd_t<__nv_bfloat16>(a, st);
    }
}

}  // namespace mss
