// Motif regulariser of the P/Q coupling, forward and backward, for a batch of matrices.
//
// Semantics of motifRegular.cal (motif/train_kpq_motif_pile_lm.py:405-466), which the
// training script calls once per sampled channel and layer (:590-642):
//   w   = sigmoid(amplitude (a^2 - bias)) with the diagonal zeroed,  m = offdiag - w
//   X0 = m o m^T,  X1 = w o m^T,  X2 = m o w^T,  X3 = w o w^T          (o: elementwise)
//   q_k = c_k * sum(Xa o (Xb Xc))   for the 13 (a, b, c, c_k) of the term tables below
//   obs_k = q_k / (cc (cc-1) (cc-2) / 6);  loss = sum_{target_k > 0} weight_k diff_k^2
// One CTA owns one matrix and keeps w, m and X0..X3 in shared memory; each thread owns
// entries (i, j) and forms the nine distinct products (Xb Xc)(i, j) in one pass over l.
// The backward is the analytic gradient: for S = sum(Xa o (Xb Xc)),
//   dS/dXa = Xb Xc,  dS/dXb = Xa Xc^T,  dS/dXc = Xb^T Xa,
// chained through the transposed products X0..X3 to w and m, then to a.
// The work is a few hundred thousand FMAs per matrix, so one launch covers every matrix
// of every layer (the reference issues ~60 small kernels and a host sync per matrix).
#include "common.cuh"
#include "kernels.h"

namespace mss {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxCC = 32;

// Distinct products Xb Xc used by the 13 terms.
enum Prod { P10, P12, P02, P20, P21, P30, P22, P32, P33, NPROD };

// Term k: S_k = sum(X_a o (X_b X_c)), q_k = coef * S_k; tp(k) indexes the product X_b X_c.
// constexpr tables, so that after unrolling every index into a register array is static.
__device__ constexpr int ta(int k) { constexpr int v[13] = {1, 0, 1, 1, 3, 3, 3, 3, 3, 1, 3, 3, 3}; return v[k]; }
__device__ constexpr int tb(int k) { constexpr int v[13] = {1, 1, 0, 1, 1, 2, 1, 2, 3, 2, 2, 3, 3}; return v[k]; }
__device__ constexpr int tc(int k) { constexpr int v[13] = {0, 2, 2, 2, 0, 0, 2, 1, 0, 2, 2, 2, 3}; return v[k]; }
__device__ constexpr int tp(int k) {
    constexpr int v[13] = {P10, P12, P02, P12, P10, P20, P12, P21, P30, P22, P22, P32, P33};
    return v[k];
}
__device__ constexpr float tcoef(int k) {
    constexpr float v[13] = {0.5f, 0.5f, 1.f, 1.f, 1.f, 1.f, 0.5f, 0.5f, 0.5f, 1.f / 3.f, 1.f, 1.f, 1.f / 6.f};
    return v[k];
}

template <bool BWD>
__global__ void __launch_bounds__(kThreads) motif_regular_kernel(const motif_regular_args a) {
    extern __shared__ float sm[];
    const int cc = (int)a.cc, N = cc * cc;
    float *W = sm, *M = W + N, *X = M + N;  // X[k * N + e] = Xk
    float *G = X + 4 * N;                   // backward: dL/dXk
    __shared__ float red[kThreads / 32][13];
    __shared__ float gam[13];  // dL/dS_k (coefficient folded in)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t mat = blockIdx.x;
    const float *A = a.a + mat * a.a_ms;

    for (int e = tid; e < N; e += kThreads) {
        const int i = e / cc, j = e - i * cc;
        const float av = A[e];
        const float s = 1.f / (1.f + expf(-a.amplitude * (av * av - a.bias)));
        const float w = i != j ? s : 0.f;
        W[e] = w;
        M[e] = (i != j ? 1.f : 0.f) - w;
    }
    __syncthreads();
    for (int e = tid; e < N; e += kThreads) {
        const int i = e / cc, j = e - i * cc, t = j * cc + i;
        X[e] = M[e] * M[t];
        X[N + e] = W[e] * M[t];
        X[2 * N + e] = M[e] * W[t];
        X[3 * N + e] = W[e] * W[t];
    }
    __syncthreads();

    // The entries a thread owns (at most kMaxCC^2 / kThreads = 4).
    constexpr int EPT = kMaxCC * kMaxCC / kThreads;
    float prod[EPT][NPROD];
    float part[13];
#pragma unroll
    for (int k = 0; k < 13; ++k) part[k] = 0.f;
#pragma unroll
    for (int r = 0; r < EPT; ++r) {
        const int e = tid + r * kThreads;
#pragma unroll
        for (int p = 0; p < NPROD; ++p) prod[r][p] = 0.f;
        if (e < N) {
            const int i = e / cc, j = e - i * cc;
            for (int l = 0; l < cc; ++l) {
                float xr[4], xc[4];  // Xk(i, l) and Xk(l, j)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    xr[k] = X[k * N + i * cc + l];
                    xc[k] = X[k * N + l * cc + j];
                }
                prod[r][P10] = fmaf(xr[1], xc[0], prod[r][P10]);
                prod[r][P12] = fmaf(xr[1], xc[2], prod[r][P12]);
                prod[r][P02] = fmaf(xr[0], xc[2], prod[r][P02]);
                prod[r][P20] = fmaf(xr[2], xc[0], prod[r][P20]);
                prod[r][P21] = fmaf(xr[2], xc[1], prod[r][P21]);
                prod[r][P30] = fmaf(xr[3], xc[0], prod[r][P30]);
                prod[r][P22] = fmaf(xr[2], xc[2], prod[r][P22]);
                prod[r][P32] = fmaf(xr[3], xc[2], prod[r][P32]);
                prod[r][P33] = fmaf(xr[3], xc[3], prod[r][P33]);
            }
#pragma unroll
            for (int k = 0; k < 13; ++k) part[k] = fmaf(X[ta(k) * N + e], prod[r][tp(k)], part[k]);
        }
    }
#pragma unroll
    for (int k = 0; k < 13; ++k) {
        float v = part[k];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp][k] = v;
    }
    __syncthreads();
    if (tid < 32) {
        // lane k < 13 finishes motif k; lane 0 sums the loss
        const float ncomb = (float)((int64_t)cc * (cc - 1) * (cc - 2) / 6);
        float obs = 0.f, contrib = 0.f, g = 0.f;
        if (lane < 13) {
            float S = 0.f;
            for (int w = 0; w < kThreads / 32; ++w) S += red[w][lane];
            obs = tcoef(lane) * S / ncomb;
            const float tgt = a.target[lane];
            if (tgt > 0.f) {
                const float wt = a.weight ? a.weight[lane] : 1.f;
                float diff, ddiff;  // diff and d diff / d obs
                if (a.log_mse) {
                    const float oc = fmaxf(obs, a.log_eps);
                    diff = logf(oc) - logf(fmaxf(tgt, a.log_eps));
                    ddiff = obs >= a.log_eps ? 1.f / obs : 0.f;
                } else {
                    diff = obs - tgt;
                    ddiff = 1.f;
                }
                contrib = wt * diff * diff;
                g = wt * 2.f * diff * ddiff * tcoef(lane) / ncomb;
            }
        }
        const float obs_up = __shfl_up_sync(0xffffffffu, obs, 1);  // motif k at slot k + 1
        if (a.obs && lane < 14) a.obs[mat * 14 + lane] = lane == 0 ? 0.f : obs_up;
        float lsum = contrib;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
        if (lane == 0) a.loss[mat] = lsum;
        if (BWD && lane < 13) gam[lane] = g * a.dloss[mat];
    }
    if constexpr (BWD) {
        __syncthreads();
        // dL/dXk(i, j): direct terms from the products, then the two transposed contractions
#pragma unroll
        for (int r = 0; r < EPT; ++r) {
            const int e = tid + r * kThreads;
            if (e >= N) continue;
            const int i = e / cc, j = e - i * cc;
            float g4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < 13; ++k) g4[ta(k)] = fmaf(gam[k], prod[r][tp(k)], g4[ta(k)]);
            float gl[13][2];  // per term: sum_l Xa(i,l) Xc(j,l) and sum_l Xb(l,i) Xa(l,j)
#pragma unroll
            for (int k = 0; k < 13; ++k) gl[k][0] = gl[k][1] = 0.f;
            for (int l = 0; l < cc; ++l) {
                float ri[4], rj[4], ci[4], cj[4];  // Xk(i,l), Xk(j,l), Xk(l,i), Xk(l,j)
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    ri[k] = X[k * N + i * cc + l];
                    rj[k] = X[k * N + j * cc + l];
                    ci[k] = X[k * N + l * cc + i];
                    cj[k] = X[k * N + l * cc + j];
                }
#pragma unroll
                for (int k = 0; k < 13; ++k) {
                    gl[k][0] = fmaf(ri[ta(k)], rj[tc(k)], gl[k][0]);
                    gl[k][1] = fmaf(ci[tb(k)], cj[ta(k)], gl[k][1]);
                }
            }
#pragma unroll
            for (int k = 0; k < 13; ++k) {
                g4[tb(k)] = fmaf(gam[k], gl[k][0], g4[tb(k)]);
                g4[tc(k)] = fmaf(gam[k], gl[k][1], g4[tc(k)]);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) G[k * N + e] = g4[k];
        }
        __syncthreads();
        float *dA = a.da + mat * a.da_ms;
        for (int e = tid; e < N; e += kThreads) {
            const int i = e / cc, j = e - i * cc, t = j * cc + i;
            // X0 = m o m^T, X1 = w o m^T, X2 = m o w^T, X3 = w o w^T
            const float gm = (G[e] + G[t]) * M[t] + G[N + t] * W[t] + G[2 * N + e] * W[t];
            const float gw = G[N + e] * M[t] + G[2 * N + t] * M[t] + (G[3 * N + e] + G[3 * N + t]) * W[t];
            float d = 0.f;
            if (i != j) {
                const float av = A[e];
                const float s = W[e];
                d = (gw - gm) * s * (1.f - s) * a.amplitude * 2.f * av;
            }
            dA[e] = d;
        }
    }
}

}  // namespace

cudaError_t launch_motif_regular(const motif_regular_args &a, cudaStream_t st) {
    const size_t smem = (size_t)(a.dloss ? 10 : 6) * a.cc * a.cc * sizeof(float);
    const dim3 grid((unsigned)a.n_mat);
    if (a.dloss)
        motif_regular_kernel<true><<<grid, kThreads, smem, st>>>(a);
    else
        motif_regular_kernel<false><<<grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace mss
