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
// forward reads its W-1 halo from the neighbouring vector (an L1 hit); the backward takes
// both halos from neighbouring lanes by shuffle.  Weight gradients are kept per lane,
// reduced across the warp with shuffles and added once per row.
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

// Work item: one row's block of `tblk` steps (a multiple of 256; the whole row unless rows are
// too few to give every SM enough warps, see conv_dir).
template <typename T, typename WT, int KW>
__global__ void __launch_bounds__(256) conv1d_fwd_kernel(const conv1d_args a, int vec, int tblk) {
    const int lane = threadIdx.x & 31;
    const int64_t nrows = a.batch * a.dim;
    const int nblk = (int)((a.seqlen + tblk - 1) / tblk);
    const int64_t items = nrows * nblk;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t it = warp; it < items; it += nwarps) {
        int64_t r = it;
        int blk = 0;
        if (nblk > 1) {  // few rows: items < 2^31 (conv_dir)
            r = (int64_t)((unsigned)it / (unsigned)nblk);
            blk = (int)(it - r * nblk);
        }
        const int64_t b = r / a.dim, c = r - b * a.dim;
        float w[KW];
#pragma unroll
        for (int k = 0; k < KW; ++k) w[k] = ldw<WT>(a.weight, c * a.w_ds + k * a.w_ks);
        const float bias = a.bias ? ldw<WT>(a.bias, c) : 0.f;
        const T *xr = reinterpret_cast<const T *>(a.x) + b * a.x_bs + c * a.x_ds;
        T *orow = reinterpret_cast<T *>(a.out) + b * a.out_bs + c * a.out_ds;
        const int64_t tend = min(a.seqlen, (int64_t)(blk + 1) * tblk);
        for (int64_t t0 = (int64_t)blk * tblk + (int64_t)lane * 8; t0 < tend; t0 += 256) {
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

// Backward: each lane computes dpre only at its own 8 positions.  The W-1 values of x before
// its block come from the lane below by shuffle (lane 0: lane 31 of the previous 256-step
// step, kept in registers), and the W-1 values of dpre after its block from the lane above;
// lane 31's next values belong to lane 0 of the NEXT step, so lane 31 writes its dx one step
// late.  Per 8 outputs: two 16-byte loads (x, dout) and 8 sigmoids.  The kernel is bound by
// load latency, so it is held to 64 registers for 4 resident CTAs per SM (3 at 80: 11 % slower).
template <typename T, typename WT, int KW>
__global__ void __launch_bounds__(256, 4) conv1d_bwd_kernel(const conv1d_args a, int vec) {
    constexpr int H = KW - 1;  // halo
    constexpr unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const int64_t nrows = a.batch * a.dim;
    const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const int64_t L = a.seqlen;
    for (int64_t r = warp; r < nrows; r += nwarps) {  // uniform per warp
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
        float xcarry[H + 1], dprev[8];  // lane 31's last x of the previous step; lane 31's pending dpre
#pragma unroll
        for (int h = 0; h <= H; ++h) xcarry[h] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) dprev[i] = 0.f;
        int64_t tb = 0;
        for (; tb < L; tb += 256) {  // uniform: lanes past L see zeros
            const int64_t t0 = tb + (int64_t)lane * 8;
            float xc[8], dc[8];
            load8_row(xr, t0, L, vec, xc);
            load8_row(dor, t0, L, vec, dc);
            float xh[H + 1];  // x at t0 - H .. t0 - 1 (index H unused)
#pragma unroll
            for (int h = 0; h < H; ++h) {
                const float up = __shfl_up_sync(FULL, xc[8 - H + h], 1);
                xh[h] = lane == 0 ? xcarry[h] : up;
                xcarry[h] = __shfl_sync(FULL, xc[8 - H + h], 31);
            }
            auto xat = [&](int j) -> float { return j < 0 ? xh[H + j] : xc[j]; };  // x at t0 + j
            float dpre[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float pre = bias;
#pragma unroll
                for (int k = 0; k < KW; ++k) pre = fmaf(w[k], xat(i - H + k), pre);
                float g = dc[i];  // zero beyond L
                if (a.silu) {
                    const float s = sigmoidf_(pre);
                    g = g * s * (1.f + pre * (1.f - s));
                }
                dpre[i] = g;
                db += g;
#pragma unroll
                for (int k = 0; k < KW; ++k) dw[k] = fmaf(g, xat(i - H + k), dw[k]);
            }
            // dx[t] = sum_k w[k] dpre[t + H - k]: lanes 0-30 finish this step's block, lane 31
            // the previous step's, with the first H dpre of lane 0 of this step
            float nxt[H + 1];
#pragma unroll
            for (int h = 0; h < H; ++h) {
                const float dn = __shfl_down_sync(FULL, dpre[h], 1);
                const float d0 = __shfl_sync(FULL, dpre[h], 0);
                nxt[h] = lane == 31 ? d0 : dn;
            }
            float src[8], dxv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) src[i] = lane == 31 ? dprev[i] : dpre[i];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < KW; ++k) {
                    const int j = i + H - k;
                    acc = fmaf(w[k], j < 8 ? src[j] : nxt[j - 8], acc);
                }
                dxv[i] = acc;
            }
            const int64_t ts = lane == 31 ? t0 - 256 : t0;
            if (ts >= 0 && ts < L) store8_row(dxr, ts, L, vec, dxv);
            if (lane == 31) {
#pragma unroll
                for (int i = 0; i < 8; ++i) dprev[i] = dpre[i];
            }
        }
        if (lane == 31) {  // the last step's block: nothing follows it (dpre beyond L is zero)
            const int64_t ts = tb - 256 + 248;
            float dxv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < KW; ++k) {
                    const int j = i + H - k;
                    acc = fmaf(w[k], j < 8 ? dprev[j] : 0.f, acc);
                }
                dxv[i] = acc;
            }
            if (ts >= 0 && ts < L) store8_row(dxr, ts, L, vec, dxv);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            db += __shfl_xor_sync(FULL, db, off);
#pragma unroll
            for (int k = 0; k < KW; ++k) dw[k] += __shfl_xor_sync(FULL, dw[k], off);
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
    if (S <= 8) {  // the window in registers: all loads issue before the first store
        float v[8];
#pragma unroll
        for (int s = 0; s < 8; ++s) v[s] = s < S ? to_f<ST>(st[s]) : 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            if (s < S) {
                const ST nv = from_f<ST>(s + 1 < 8 && s + 1 < S ? v[s + 1] : xv);
                st[s] = nv;
                const int k = s - (S - KW);
                if (k >= 0) acc = fmaf(ldw<WT>(a.weight, c * a.w_ds + k * a.w_ks), to_f<ST>(nv), acc);
            }
        }
        if (a.silu) acc = acc * sigmoidf_(acc);
        reinterpret_cast<T *>(a.out)[b * a.out_bs + c] = from_f<T>(acc);
        return;
    }
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
    // Forward with fewer rows than ~48 warps per SM (e.g. a 2 x 1536 batch): a warp walking a
    // whole row keeps one load in flight at a time, so rows are cut into 1024-step items.
    const int64_t row_blk = (a.seqlen + 255) / 256 * 256;
    const int tblk = (!bwd && nrows < 148 * 48 && a.seqlen > 1024) ? 1024 : (int)std::min<int64_t>(row_blk, 1 << 30);
    const int64_t work = nrows * ((a.seqlen + tblk - 1) / tblk);
    const int64_t blocks = std::min<int64_t>(((bwd ? nrows : work) * 32 + threads - 1) / threads, 148 * 16);
    if (blocks <= 0) return cudaSuccess;
    if (bwd)
        conv1d_bwd_kernel<T, WT, KW><<<(int)blocks, threads, 0, st>>>(a, vec ? 1 : 0);
    else
        conv1d_fwd_kernel<T, WT, KW><<<(int)blocks, threads, 0, st>>>(a, vec ? 1 : 0, tblk);
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
