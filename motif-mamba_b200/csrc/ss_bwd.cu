// Selective-scan backward for sm_100a.
//
// Gradients of the forward in ss_fwd.cu (reference semantics:
// selective_scan_bwd_kernel.cuh:405-880, selective_scan_interface.py:64-91):
//   dh_t   = doutg_t * C_t + exp(dt_{t+1} A) * dh_{t+1}          (reverse recurrence, per state)
//   du_t   = dt_t * sum_n dh_t B_t + D * doutg_t
//   ddelta = (u_t * sum_n dh_t B_t + sum_n A_n dh_t * exp(dt_t A_n) h_{t-1}) * softplus'(.)
//   dA_n  += dt_t * dh_t * exp(dt_t A_n) h_{t-1}
//   dB_nt  = sum_d dh_t dt_t u_t      dC_nt = sum_d doutg_t h_t      (reductions over channels)
//   dD    += doutg_t u_t              ddelta_bias += ddelta_t
//   dz     = dout * out * sigma(z) (1 + z (1 - sigma(z))),   doutg = dout * silu(z)
//
// Design (B200).  One warp owns one channel for one 256-step chunk: lane l owns the 8
// consecutive timesteps 8l..8l+7, so every per-element quantity (softplus, z gate, du,
// ddelta, dz) lives in the owning lane's registers, is loaded and stored with 16-byte
// vector accesses, and the sums over states (sum_n dh B, sum_n A dh p) are in-register
// FMA accumulations across the state loop.  For each state n the forward state is
// rebuilt from the chunk state that ss_fwd stored in x (one every 256 steps): each lane
// folds its 8 steps sequentially, a 5-level warp scan of (decay, state) pairs gives each
// lane its incoming state, and the 8 steps are replayed; the reverse recurrence is the
// mirror image (local fold, reverse warp scan, replay), seeded by the carry from the
// later chunk.  A CTA runs 8 warps on 8 channels of one batch row at a time and K such
// channel groups per chunk: dB / dC (sums over channels) are reduced over the 8 warps
// through shared memory into a per-chunk fp32 accumulator that also sums the K groups,
// and leave once per chunk as vector red.global.add.v4.f32, 1/(8K) of the traffic of a
// per-channel scheme.  B / C of the chunk are staged once per CTA and chunk, converted
// to fp32 in a bank-conflict-free lane-interleaved layout.
#include "common.cuh"
#include "kernels.h"

namespace mss {

namespace bwd {
constexpr int W = 8;              // warps (channels) per CTA pass
constexpr int NT = W * 32;        // threads per CTA
constexpr int IT = 8;             // timesteps per lane
constexpr int CK = kChunkLen;     // timesteps per chunk (= 32 lanes x IT)
constexpr int NS = 16;            // states per thread loop (dstate <= 16)
constexpr int KMAX = 8;           // channel groups per CTA
static_assert(CK == 32 * IT, "a warp covers one chunk");
}  // namespace bwd

// Lane-interleaved chunk layout: timestep t = 8 l + 4 h + j (lane l, half h, j < 4) lives at
// h * 128 + 4 l + j, so each lane reads its 8 steps as two conflict-free 16-byte loads.
struct BwdSmem {
    float BC[2][bwd::NS][bwd::CK];            // B, C of the chunk, fp32
    float RED[2][bwd::W][2][bwd::CK];         // double-buffered per-state dB / dC partials
    float ACC[2][bwd::NS][bwd::CK];           // chunk accumulator of dB / dC
    float DHC[bwd::KMAX][bwd::W][bwd::NS];    // reverse-recurrence carry into the previous chunk
    float DAACC[bwd::KMAX][bwd::W][bwd::NS];  // dA accumulators
    float PBD[bwd::KMAX][bwd::W][2];          // dD, ddelta_bias accumulators
};

template <typename T>
__device__ __forceinline__ void load_items(const T *row, int64_t t0, int64_t L, bool vec, float (&v)[8]) {
    if (vec && t0 + 8 <= L) {
        Vec8<T>::load(row + t0, v);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (t0 + i < L) ? to_f<T>(row[t0 + i]) : 0.f;
    }
}
template <typename T>
__device__ __forceinline__ void store_items(T *row, int64_t t0, int64_t L, bool vec, const float (&v)[8]) {
    if (vec && t0 + 8 <= L) {
        Vec8<T>::store(row + t0, v);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (t0 + i < L) row[t0 + i] = from_f<T>(v[i]);
    }
}
__device__ __forceinline__ void ld8(const float *base, int lane, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(base + lane * 4);
    const float4 c = *reinterpret_cast<const float4 *>(base + 128 + lane * 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
}
__device__ __forceinline__ void st8(float *base, int lane, const float (&v)[8]) {
    *reinterpret_cast<float4 *>(base + lane * 4) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4 *>(base + 128 + lane * 4) = make_float4(v[4], v[5], v[6], v[7]);
}

template <typename T, bool HAS_Z>
__global__ void __launch_bounds__(bwd::NT, 2) ss_bwd_kernel(const BwdParams p) {
    using namespace bwd;
    extern __shared__ __align__(16) char smem_raw[];
    BwdSmem &S = *reinterpret_cast<BwdSmem *>(smem_raw);
    const unsigned FULL = 0xffffffffu;

    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int g = blockIdx.x / p.tiles_per_group;
    const int tile = blockIdx.x - g * p.tiles_per_group;
    const int b = blockIdx.y;
    const int64_t L = p.seqlen;
    const bool vec = p.aligned != 0;
    const int K = p.kgroups;

    for (int i = tid; i < 2 * NS * CK; i += NT) (&S.ACC[0][0][0])[i] = 0.f;
    for (int i = tid; i < KMAX * W * NS; i += NT) {
        (&S.DHC[0][0][0])[i] = 0.f;
        (&S.DAACC[0][0][0])[i] = 0.f;
    }
    for (int i = tid; i < KMAX * W * 2; i += NT) (&S.PBD[0][0][0])[i] = 0.f;

    const T *gB = reinterpret_cast<const T *>(p.B) + (int64_t)b * p.B_bs + (int64_t)g * p.B_gs;
    const T *gC = reinterpret_cast<const T *>(p.C) + (int64_t)b * p.C_bs + (int64_t)g * p.C_gs;

    for (int k = p.n_chunks - 1; k >= 0; --k) {
        const int64_t kt0 = (int64_t)k * CK;
        __syncthreads();  // previous chunk's accumulator flush and B/C reads are done
        // ---- stage B, C of this chunk (fp32; zero beyond dstate / seqlen)
        for (int i = tid; i < 2 * NS * 32; i += NT) {
            const int q = i / (NS * 32), rem = i - q * NS * 32, n = rem >> 5, l = rem & 31;
            float v[8];
            if (n < p.dstate) {
                const T *row = (q == 0 ? gB + (int64_t)n * p.B_ns : gC + (int64_t)n * p.C_ns);
                load_items(row, kt0 + l * 8, L, vec, v);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = 0.f;
            }
            st8(&S.BC[q][n][0], l, v);
        }
        __syncthreads();

        for (int cg = 0; cg < K; ++cg) {
            const int cin = (tile * K + cg) * W + w;  // channel within the group
            const bool valid = cin < p.dpg;
            const int d = g * p.dpg + (valid ? cin : 0);
            const int64_t row = (int64_t)b * p.dim + d;
            const int64_t t0 = kt0 + lane * IT;

            // ---- per-element prologue (this lane's 8 steps)
            float uf[8], dtf[8], dtu[8], dog[8];
            {
                float dv[8], dov[8];
                load_items(reinterpret_cast<const T *>(p.u) + (int64_t)b * p.u_bs + (int64_t)d * p.u_ds, t0, L,
                           vec, uf);
                load_items(reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs + (int64_t)d * p.delta_ds,
                           t0, L, vec, dv);
                load_items(reinterpret_cast<const T *>(p.dout) + (int64_t)b * p.dout_bs + (int64_t)d * p.dout_ds,
                           t0, L, vec, dov);
                const float bias = p.delta_bias ? p.delta_bias[(int64_t)d * p.delta_bias_s] : 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float x = dv[i] + bias;
                    if (p.softplus) x = softplus20(x);
                    dtf[i] = (valid && t0 + i < L) ? x : 0.f;
                    dtu[i] = dtf[i] * uf[i];
                    dog[i] = valid ? dov[i] : 0.f;
                }
                if constexpr (HAS_Z) {
                    float zv[8], ov[8], dzv[8], ozv[8];
                    load_items(reinterpret_cast<const T *>(p.z) + (int64_t)b * p.z_bs + (int64_t)d * p.z_ds, t0, L,
                               vec, zv);
                    load_items(reinterpret_cast<const T *>(p.out) + (int64_t)b * p.out_bs + (int64_t)d * p.out_ds,
                               t0, L, vec, ov);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float sz = sigmoidf_(zv[i]);
                        const float silu = zv[i] * sz;
                        dzv[i] = dog[i] * ov[i] * sz * (1.f + zv[i] * (1.f - sz));
                        ozv[i] = ov[i] * silu;
                        dog[i] *= silu;
                    }
                    if (valid) {
                        store_items(reinterpret_cast<T *>(p.dz) + (int64_t)b * p.dz_bs + (int64_t)d * p.dz_ds, t0, L,
                                    vec, dzv);
                        if (p.recompute_out_z)
                            store_items(reinterpret_cast<T *>(p.out_z) + (int64_t)b * p.out_z_bs +
                                            (int64_t)d * p.out_z_ds, t0, L, vec, ozv);
                    }
                }
            }
            float sdt = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) sdt += dtf[i];

            float S1[8], S2[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) S1[i] = S2[i] = 0.f;

#pragma unroll 1
            for (int n = 0; n < p.dstate; ++n) {  // uniform over the CTA
                const float An = valid ? p.A[(int64_t)d * p.A_ds + (int64_t)n * p.A_ns] : 0.f;
                const float A2 = An * kLog2e;
                float Bv[8], a[8], h[8];
                ld8(&S.BC[0][n][0], lane, Bv);
                // forward: local fold, warp scan of (decay, state), replay
                float H = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    a[i] = ex2(dtf[i] * A2);
                    h[i] = dtu[i] * Bv[i];  // b_i, replaced by the state below
                    H = fmaf(a[i], H, h[i]);
                }
                const float Pl = ex2(A2 * sdt);  // decay over the lane's 8 steps
                float Ad = Pl, Hd = H;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float Ap = __shfl_up_sync(FULL, Ad, off), Hp = __shfl_up_sync(FULL, Hd, off);
                    if (lane >= off) {
                        Hd = fmaf(Ad, Hp, Hd);
                        Ad *= Ap;
                    }
                }
                const float h_chunk =
                    (k > 0 && valid) ? p.x[(row * p.n_chunks + (k - 1)) * 2 * p.dstate + 2 * n + 1] : 0.f;
                float h_in;
                {
                    const float Ae = __shfl_up_sync(FULL, Ad, 1), He = __shfl_up_sync(FULL, Hd, 1);
                    h_in = lane == 0 ? h_chunk : fmaf(Ae, h_chunk, He);
                }
                float hp = h_in;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    h[i] = fmaf(a[i], hp, h[i]);
                    hp = h[i];
                }
                // reverse: local fold of dh (without the carry), reverse warp scan, replay
                float Cv[8];
                ld8(&S.BC[1][n][0], lane, Cv);
                float Dl = 0.f;
#pragma unroll
                for (int i = 7; i >= 0; --i) {
                    Cv[i] *= dog[i];  // e_i = doutg_i C_i
                    Dl = fmaf(i < 7 ? a[i + 1] : 0.f, Dl, Cv[i]);
                }
                float Pd = Pl, Qd = a[0] * Dl;  // lane aggregate: passes Q + P * carry_in to the left
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float Pr = __shfl_down_sync(FULL, Pd, off), Qr = __shfl_down_sync(FULL, Qd, off);
                    if (lane + off < 32) {
                        Qd = fmaf(Pd, Qr, Qd);
                        Pd *= Pr;
                    }
                }
                const float c_chunk = S.DHC[cg][w][n];
                float carry;
                {
                    const float Pe = __shfl_down_sync(FULL, Pd, 1), Qe = __shfl_down_sync(FULL, Qd, 1);
                    carry = lane == 31 ? c_chunk : fmaf(Pe, c_chunk, Qe);
                }
                float dAp = 0.f;
#pragma unroll
                for (int i = 7; i >= 0; --i) {
                    const float dh = Cv[i] + carry;
                    carry = a[i] * dh;
                    const float pv = a[i] * (i > 0 ? h[i - 1] : h_in);  // a_t h_{t-1}
                    const float gv = dh * pv;
                    S1[i] = fmaf(dh, Bv[i], S1[i]);
                    S2[i] = fmaf(An, gv, S2[i]);
                    dAp = fmaf(dtf[i], gv, dAp);
                    Cv[i] = dh;
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) dAp += __shfl_xor_sync(FULL, dAp, off);
                if (lane == 0) {
                    S.DHC[cg][w][n] = carry;  // carry into the previous chunk
                    S.DAACC[cg][w][n] += dAp;
                }
                // dB / dC partials of this warp's channel -> reduce over the CTA's warps
                {
                    float dBv[8], dCv[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        dBv[i] = Cv[i] * dtu[i];
                        dCv[i] = dog[i] * h[i];
                    }
                    st8(&S.RED[n & 1][w][0][0], lane, dBv);
                    st8(&S.RED[n & 1][w][1][0], lane, dCv);
                }
                __syncthreads();
                {
                    const int q = tid >> 7, pp = (tid & 127) * 2;
                    float2 s = make_float2(0.f, 0.f);
#pragma unroll
                    for (int ww = 0; ww < W; ++ww) {
                        const float2 v = *reinterpret_cast<const float2 *>(&S.RED[n & 1][ww][q][pp]);
                        s.x += v.x;
                        s.y += v.y;
                    }
                    float2 *acc = reinterpret_cast<float2 *>(&S.ACC[q][n][pp]);
                    float2 cur = *acc;
                    cur.x += s.x;
                    cur.y += s.y;
                    *acc = cur;
                }
            }
            // ---- per-element epilogue
            {
                const float Dv = p.D ? p.D[(int64_t)d * p.D_s] : 0.f;
                float du[8], dd[8], dv[8], dDp = 0.f, dbp = 0.f;
                load_items(reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs + (int64_t)d * p.delta_ds,
                           t0, L, vec, dv);
                const float bias = p.delta_bias ? p.delta_bias[(int64_t)d * p.delta_bias_s] : 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float x = dv[i] + bias;
                    const float gate = (p.softplus && x <= 20.f) ? sigmoidf_(x) : 1.f;
                    du[i] = fmaf(dtf[i], S1[i], Dv * dog[i]);
                    dd[i] = fmaf(uf[i], S1[i], S2[i]) * gate;
                    if (t0 + i < L) {
                        dDp = fmaf(dog[i], uf[i], dDp);
                        dbp += dd[i];
                    }
                }
                if (valid) {
                    store_items(reinterpret_cast<T *>(p.du) + (int64_t)b * p.du_bs + (int64_t)d * p.du_ds, t0, L,
                                vec, du);
                    store_items(reinterpret_cast<T *>(p.ddelta) + (int64_t)b * p.ddelta_bs + (int64_t)d * p.ddelta_ds,
                                t0, L, vec, dd);
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    dDp += __shfl_xor_sync(FULL, dDp, off);
                    dbp += __shfl_xor_sync(FULL, dbp, off);
                }
                if (lane == 0) {
                    S.PBD[cg][w][0] += dDp;
                    S.PBD[cg][w][1] += dbp;
                }
            }
            __syncthreads();
        }
        // ---- flush the chunk's dB / dC (summed over this CTA's channels)
        __syncthreads();
        const int clen = (int)min((int64_t)CK, L - kt0);
        for (int i = tid; i < 2 * NS * (CK / 4); i += NT) {
            const int q = i / (NS * (CK / 4)), rem = i - q * NS * (CK / 4);
            const int n = rem / (CK / 4), pos = (rem - n * (CK / 4)) * 4;
            const int t = ((pos >> 2) & 31) * 8 + (pos >> 7) * 4;  // first timestep of this 4-group
            float *src = &S.ACC[q][n][pos];
            if (n < p.dstate && t < clen) {
                float *dst = (q == 0 ? p.acc_dB : p.acc_dC) +
                             (((int64_t)b * p.n_groups + g) * p.dstate + n) * p.lpitch + kt0 + t;
                red_add_v4(dst, src[0], src[1], src[2], src[3]);
            }
            src[0] = src[1] = src[2] = src[3] = 0.f;
        }
    }
    __syncthreads();
    for (int i = tid; i < K * W * NS; i += NT) {
        const int cg = i / (W * NS), rem = i - cg * W * NS, ww = rem / NS, n = rem - ww * NS;
        const int cin = (tile * K + cg) * W + ww;
        if (cin < p.dpg && n < p.dstate)
            atomicAdd(p.dA + (int64_t)(g * p.dpg + cin) * p.dstate + n, S.DAACC[cg][ww][n]);
    }
    for (int i = tid; i < K * W; i += NT) {
        const int cg = i / W, ww = i - cg * W;
        const int cin = (tile * K + cg) * W + ww;
        if (cin < p.dpg) {
            if (p.dD) atomicAdd(p.dD + g * p.dpg + cin, S.PBD[cg][ww][0]);
            if (p.ddelta_bias) atomicAdd(p.ddelta_bias + g * p.dpg + cin, S.PBD[cg][ww][1]);
        }
    }
}

// fp32 accumulator rows (pitch lpitch) -> output rows (pitch seqlen) in the input dtype.
template <typename T>
__global__ void acc_to_out_kernel(const float *__restrict__ acc, int64_t lpitch, T *__restrict__ out,
                                  int64_t rows, int64_t seqlen) {
    const int64_t total = rows * seqlen;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / seqlen, t = i - r * seqlen;
        out[i] = from_f<T>(acc[r * lpitch + t]);
    }
}

cudaError_t launch_acc_to_out(const float *acc, int64_t lpitch, void *out, int itype, int64_t rows,
                              int64_t seqlen, cudaStream_t st) {
    const int64_t total = rows * seqlen;
    if (total == 0) return cudaSuccess;
    const int threads = 256;
    const int blocks = (int)std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
    switch (itype) {
        case MSS_F32: acc_to_out_kernel<float><<<blocks, threads, 0, st>>>(acc, lpitch, (float *)out, rows, seqlen); break;
        case MSS_F16: acc_to_out_kernel<__half><<<blocks, threads, 0, st>>>(acc, lpitch, (__half *)out, rows, seqlen); break;
        default: acc_to_out_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(acc, lpitch, (__nv_bfloat16 *)out, rows, seqlen); break;
    }
    return cudaGetLastError();
}

template <typename T, bool HAS_Z>
static cudaError_t launch_bwd_t(const BwdParams &p, cudaStream_t st) {
    auto kern = ss_bwd_kernel<T, HAS_Z>;
    constexpr int SMEM = (int)sizeof(BwdSmem);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    dim3 grid(p.tiles_per_group * p.n_groups, p.batch);
    kern<<<grid, bwd::NT, SMEM, st>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_ss_bwd(const BwdParams &p, int itype, bool has_z, cudaStream_t st) {
    switch (itype) {
        case MSS_F32: return has_z ? launch_bwd_t<float, true>(p, st) : launch_bwd_t<float, false>(p, st);
        case MSS_F16: return has_z ? launch_bwd_t<__half, true>(p, st) : launch_bwd_t<__half, false>(p, st);
        default: return has_z ? launch_bwd_t<__nv_bfloat16, true>(p, st) : launch_bwd_t<__nv_bfloat16, false>(p, st);
    }
}

}  // namespace mss
