// Selective scan with the motif low-rank state coupling, forward and backward, sm_100a.
//
//   h_t = exp(dt_t A) * h_{t-1} + dt_t * P (Q h_{t-1}) + dt_t u_t B_t,   y_t = <C_t, h_t>
//
// (reference: selective_scan_ref with P/Q, mamba_ssm/ops/selective_scan_interface.py:402-433;
// full-matrix path :262-350).  P is (dstate, r) shared or (dim, dstate, r) per channel, Q is
// (r, dstate) or (dim, r, dstate), r <= 8, dstate <= 64.  The coupling mixes states, so the
// diagonal-scan tricks of ss_fwd / ss_bwd do not apply and time stays sequential per channel.
// To give the GPU enough warps, a channel's states (padded to 16, 32 or 64) are split over
// 4, 8 or 16 adjacent lanes, 4 states each: per step q = Q h is a sum over those lanes
// (shuffles), pq = P q, the diagonal update and the output's sum.  Each lane keeps its slice of P and Q in
// registers (rows n of P, columns n of Q for its 4 states), and in the backward also its
// slice of dP and dQ, so nothing is accumulated through shared memory per step.
//
// Forward: B/C tiles of 32 steps are staged in shared memory for the CTA's channels;
// u/delta/z rows are read by the channel's lanes with 16-byte loads; x gets the state every
// 256 steps as in ss_fwd.
// Backward (O(L)): a forward sweep stores the state at every 16-step segment start in a
// workspace; then segments are processed in reverse: the 16 states of each step are
// recomputed into shared memory and the adjoint g_t = C_t doutg_t + M_{t+1}^T g_{t+1}
// (M = diag(a) + dt P Q, M^T g = a g + dt Q^T (P^T g)) runs backwards, accumulating du,
// ddelta, dA, dD, ddelta_bias, dP = sum dt g (Q h_prev)^T and dQ = sum dt (P^T g) h_prev^T.
// dB / dC (sums over channels) are reduce-scattered over the warp's channels with shuffles, summed over the CTA's 4 warps per segment in shared memory, and added to the
// fp32 accumulators with one vector atomic per thread and segment.
#include "common.cuh"
#include "kernels.h"

namespace mss {

namespace pq {
constexpr int SPT = 4;   // states per lane
constexpr int NT = 128;  // threads per CTA
constexpr int TT = 32;   // forward tile (divides the 256-step x chunk)
constexpr int SEG = 16;  // backward segment length
// A channel's NSX states (dstate padded to 16, 32 or 64) sit on LPC = NSX / 4 adjacent lanes.
template <int NSX> struct Geo {
    static constexpr int LPC = NSX / SPT;      // lanes per channel
    static constexpr int CH = NT / LPC;        // channels per CTA
    static constexpr int CPW = 32 / LPC;       // channels per warp
    static constexpr int VPL = 8 / CPW;        // dB / dC values a lane keeps after the warp reduction
};
}  // namespace pq

template <typename T>
__device__ __forceinline__ void pq_load8(const T *row, int64_t t0, int64_t L, bool vec, float (&v)[8]) {
    if (vec && t0 + 8 <= L) {
        Vec8<T>::load(row + t0, v);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (t0 + i < L) ? to_f<T>(row[t0 + i]) : 0.f;
    }
}
template <typename T>
__device__ __forceinline__ void pq_store8(T *row, int64_t t0, int64_t L, bool vec, const float (&v)[8]) {
    if (vec && t0 + 8 <= L) {
        Vec8<T>::store(row + t0, v);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (t0 + i < L) row[t0 + i] = from_f<T>(v[i]);
    }
}
// Sum over the LPC lanes of a channel.
template <int LPC> __device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int off = 1; off < LPC; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// This lane's slice of P (rows n = 4 qt + j) and Q (columns n), zero beyond dstate / r.
template <int RM>
__device__ __forceinline__ void load_pq_slice(const float *P, const float *Q, bool per_dim, int64_t d, int dstate,
                                              int r, int qt, bool valid, float (&Pr)[pq::SPT][RM],
                                              float (&Qr)[RM][pq::SPT]) {
    const float *Pb = per_dim ? P + d * dstate * r : P;
    const float *Qb = per_dim ? Q + d * r * dstate : Q;
#pragma unroll
    for (int j = 0; j < pq::SPT; ++j) {
        const int n = pq::SPT * qt + j;
#pragma unroll
        for (int k = 0; k < RM; ++k) {
            const bool ok = valid && n < dstate && k < r;
            Pr[j][k] = ok ? Pb[n * r + k] : 0.f;
            Qr[k][j] = ok ? Qb[k * dstate + n] : 0.f;
        }
    }
}

// One step of the coupled recurrence for this lane's 4 states (h holds h_{t-1} on entry).
template <int RM, int LPC>
__device__ __forceinline__ void pq_step(float (&h)[pq::SPT], const float (&Pr)[pq::SPT][RM],
                                        const float (&Qr)[RM][pq::SPT], const float (&A2)[pq::SPT], float dt,
                                        float dtu, const float *bt) {
    float q[RM];
#pragma unroll
    for (int k = 0; k < RM; ++k) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < pq::SPT; ++j) s = fmaf(Qr[k][j], h[j], s);
        q[k] = group_sum<LPC>(s);
    }
#pragma unroll
    for (int j = 0; j < pq::SPT; ++j) {
        float pqn = 0.f;
#pragma unroll
        for (int k = 0; k < RM; ++k) pqn = fmaf(Pr[j][k], q[k], pqn);
        h[j] = fmaf(ex2(dt * A2[j]), h[j], fmaf(dt, pqn, dtu * bt[j]));
    }
}

template <typename T, bool HAS_Z, int RM, int NSX>
__global__ void __launch_bounds__(pq::NT) ss_pq_fwd_kernel(const FwdParams p) {
    using namespace pq;
    constexpr int NS = NSX, LPC = Geo<NSX>::LPC, CH = Geo<NSX>::CH;
    __shared__ __align__(16) float Bs[TT][NS], Cs[TT][NS];
    const int tid = threadIdx.x, ch = tid / LPC, qt = tid % LPC;
    const int g = blockIdx.x / p.tiles_per_group, tile = blockIdx.x - g * p.tiles_per_group;
    const int b = blockIdx.y;
    const int cin = tile * CH + ch;
    const bool valid = cin < p.dpg;
    const int d = g * p.dpg + (valid ? cin : 0);
    const int64_t L = p.seqlen, row = (int64_t)b * p.dim + d;
    const bool vec = p.aligned != 0;
    const int r = p.pq_rank;
    float Pr[SPT][RM], Qr[RM][SPT];
    load_pq_slice<RM>(p.P, p.Q, p.pq_per_dim != 0, d, p.dstate, r, qt, valid, Pr, Qr);
    float A2[SPT], h[SPT];
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const int n = SPT * qt + j;
        A2[j] = (valid && n < p.dstate) ? p.A[(int64_t)d * p.A_ds + (int64_t)n * p.A_ns] * kLog2e : 0.f;
        h[j] = 0.f;
    }
    const float Dv = (p.D && valid) ? p.D[(int64_t)d * p.D_s] : 0.f;
    const float bias = (p.delta_bias && valid) ? p.delta_bias[(int64_t)d * p.delta_bias_s] : 0.f;
    const T *ur = reinterpret_cast<const T *>(p.u) + (int64_t)b * p.u_bs + (int64_t)d * p.u_ds;
    const T *dr = reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs + (int64_t)d * p.delta_ds;
    const T *zr = HAS_Z ? reinterpret_cast<const T *>(p.z) + (int64_t)b * p.z_bs + (int64_t)d * p.z_ds : nullptr;
    T *orow = reinterpret_cast<T *>(p.out) + (int64_t)b * p.out_bs + (int64_t)d * p.out_ds;
    T *ozr = HAS_Z ? reinterpret_cast<T *>(p.out_z) + (int64_t)b * p.out_z_bs + (int64_t)d * p.out_z_ds : nullptr;
    const T *gB = reinterpret_cast<const T *>(p.B) + (int64_t)b * p.B_bs + (int64_t)g * p.B_gs;
    const T *gC = reinterpret_cast<const T *>(p.C) + (int64_t)b * p.C_bs + (int64_t)g * p.C_gs;
    float cum = 0.f;

    for (int64_t t0 = 0; t0 < L; t0 += TT) {
        __syncthreads();
        for (int i = tid; i < TT * NS; i += NT) {
            const int t = i / NS, n = i - t * NS;
            const bool ok = t0 + t < L && n < p.dstate;
            Bs[t][n] = ok ? to_f<T>(gB[(int64_t)n * p.B_ns + t0 + t]) : 0.f;
            Cs[t][n] = ok ? to_f<T>(gC[(int64_t)n * p.C_ns + t0 + t]) : 0.f;
        }
        __syncthreads();
#pragma unroll 1
        for (int g8 = 0; g8 < TT && t0 + g8 < L; g8 += 8) {
            const int64_t tg = t0 + g8;
            float uf[8], dv[8], y[8];
            pq_load8(ur, tg, L, vec, uf);
            pq_load8(dr, tg, L, vec, dv);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float dt = dv[j] + bias;
                if (p.softplus) dt = softplus20(dt);
                dt = (valid && tg + j < L) ? dt : 0.f;
                cum += dt;
                const float *bt = &Bs[g8 + j][SPT * qt], *ct = &Cs[g8 + j][SPT * qt];
                pq_step<RM, LPC>(h, Pr, Qr, A2, dt, dt * uf[j], bt);
                float yp = 0.f;
#pragma unroll
                for (int k = 0; k < SPT; ++k) yp = fmaf(ct[k], h[k], yp);
                y[j] = fmaf(Dv, uf[j], group_sum<LPC>(yp));
            }
            if (valid && qt == 0) {
                pq_store8(orow, tg, L, vec, y);
                if constexpr (HAS_Z) {
                    float zf[8];
                    pq_load8(zr, tg, L, vec, zf);
#pragma unroll
                    for (int j = 0; j < 8; ++j) zf[j] = y[j] * zf[j] * sigmoidf_(zf[j]);
                    pq_store8(ozr, tg, L, vec, zf);
                }
            }
        }
        const int64_t te = min(L, t0 + TT);
        if (valid && (te % kChunkLen == 0 || te == L)) {
            float *xr = p.x + (row * p.n_chunks + (te - 1) / kChunkLen) * 2 * p.dstate;
#pragma unroll
            for (int j = 0; j < SPT; ++j) {
                const int n = SPT * qt + j;
                if (n < p.dstate) {
                    xr[2 * n] = ex2(A2[j] * cum);
                    xr[2 * n + 1] = h[j];
                }
            }
        }
    }
}

template <int NSX> struct PqBwdSmem {
    using G = pq::Geo<NSX>;
    float HS[pq::SEG + 1][pq::NT][pq::SPT];      // states of the segment, per lane
    float Bs[pq::SEG][NSX], Cs[pq::SEG][NSX];
    float SV[5][pq::SEG][G::CH];                 // per channel and step: u, dt, dt u, doutg, gate
    float DU[pq::SEG][G::CH], DD[pq::SEG][G::CH];
    float WACC[pq::NT / 32][pq::SEG][32][G::VPL];  // warp sums of dB / dC per step
};

// After the warp's reduce-scatter over channels, lane `ln` keeps the dB / dC values
// [base, base + VPL) of its channel-group slot: halving on lane bits 16, 8, 4 (those above
// the LPC lanes of a channel), the set bit keeping the upper half.
template <int LPC> __device__ __forceinline__ int rs_base(int ln) {
    int base = 0;
#pragma unroll
    for (int m = 16, half = 4; m >= LPC; m >>= 1, half >>= 1)
        if (ln & m) base += half;
    return base;
}

template <typename T, bool HAS_Z, int RM, int NSX>
__global__ void __launch_bounds__(pq::NT) ss_pq_bwd_kernel(const BwdParams p) {
    using namespace pq;
    constexpr int NW = NT / 32, NS = NSX, LPC = Geo<NSX>::LPC, CH = Geo<NSX>::CH, VPL = Geo<NSX>::VPL;
    extern __shared__ __align__(16) char pq_smem[];
    PqBwdSmem<NSX> &S = *reinterpret_cast<PqBwdSmem<NSX> *>(pq_smem);
    auto &HS = S.HS;
    auto &Bs = S.Bs;
    auto &Cs = S.Cs;
    auto &SV = S.SV;
    auto &DU = S.DU;
    auto &DD = S.DD;
    auto &WACC = S.WACC;
    float(&SU)[SEG][CH] = SV[0];
    float(&SDT)[SEG][CH] = SV[1];
    float(&SDTU)[SEG][CH] = SV[2];
    float(&SDG)[SEG][CH] = SV[3];
    float(&SGT)[SEG][CH] = SV[4];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, ch = tid / LPC, qt = tid % LPC;
    const int g = blockIdx.x / p.tiles_per_group, tile = blockIdx.x - g * p.tiles_per_group;
    const int b = blockIdx.y;
    const int cin = tile * CH + ch;
    const bool valid = cin < p.dpg;
    const int d = g * p.dpg + (valid ? cin : 0);
    const int64_t L = p.seqlen, row = (int64_t)b * p.dim + d;
    const bool vec = p.aligned != 0;
    const int r = p.pq_rank;
    const int nseg = (int)((L + SEG - 1) / SEG);
    float Pr[SPT][RM], Qr[RM][SPT];
    load_pq_slice<RM>(p.P, p.Q, p.pq_per_dim != 0, d, p.dstate, r, qt, valid, Pr, Qr);
    float A2[SPT], An[SPT];
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const int n = SPT * qt + j;
        An[j] = (valid && n < p.dstate) ? p.A[(int64_t)d * p.A_ds + (int64_t)n * p.A_ns] : 0.f;
        A2[j] = An[j] * kLog2e;
    }
    const float Dv = (p.D && valid) ? p.D[(int64_t)d * p.D_s] : 0.f;
    const float bias = (p.delta_bias && valid) ? p.delta_bias[(int64_t)d * p.delta_bias_s] : 0.f;
    const T *ur = reinterpret_cast<const T *>(p.u) + (int64_t)b * p.u_bs + (int64_t)d * p.u_ds;
    const T *dr = reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs + (int64_t)d * p.delta_ds;
    const T *dor = reinterpret_cast<const T *>(p.dout) + (int64_t)b * p.dout_bs + (int64_t)d * p.dout_ds;
    const T *gB = reinterpret_cast<const T *>(p.B) + (int64_t)b * p.B_bs + (int64_t)g * p.B_gs;
    const T *gC = reinterpret_cast<const T *>(p.C) + (int64_t)b * p.C_bs + (int64_t)g * p.C_gs;
    float *ck = p.ckpt + row * (int64_t)nseg * NS + SPT * qt;

    auto stage_bc = [&](int64_t t0) {  // caller syncs
        for (int i = tid; i < SEG * NS; i += NT) {
            const int t = i / NS, n = i - t * NS;
            const bool ok = t0 + t < L && n < p.dstate;
            Bs[t][n] = ok ? to_f<T>(gB[(int64_t)n * p.B_ns + t0 + t]) : 0.f;
            Cs[t][n] = ok ? to_f<T>(gC[(int64_t)n * p.C_ns + t0 + t]) : 0.f;
        }
    };
    // Per-step inputs of this channel for a segment (the quad's first lane computes them);
    // with `full` also doutg, the z outputs and the softplus gate.
    auto load_seg = [&](int64_t t0, bool full) {
        if (qt != 0) return;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            float uf[8], dv[8];
            pq_load8(ur, t0 + 8 * hh, L, vec, uf);
            pq_load8(dr, t0 + 8 * hh, L, vec, dv);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int t = 8 * hh + j;
                float x = dv[j] + bias;
                float gate = 1.f;
                if (p.softplus) {
                    gate = x <= 20.f ? sigmoidf_(x) : 1.f;
                    x = softplus20(x);
                }
                x = (valid && t0 + t < L) ? x : 0.f;
                SU[t][ch] = uf[j];
                SDT[t][ch] = x;
                SDTU[t][ch] = x * uf[j];
                SGT[t][ch] = gate;
            }
            if (!full) continue;
            float dov[8];
            pq_load8(dor, t0 + 8 * hh, L, vec, dov);
            if constexpr (HAS_Z) {
                const T *zr = reinterpret_cast<const T *>(p.z) + (int64_t)b * p.z_bs + (int64_t)d * p.z_ds;
                const T *outr = reinterpret_cast<const T *>(p.out) + (int64_t)b * p.out_bs + (int64_t)d * p.out_ds;
                float zv[8], ov[8], dzv[8], ozv[8];
                pq_load8(zr, t0 + 8 * hh, L, vec, zv);
                pq_load8(outr, t0 + 8 * hh, L, vec, ov);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float sz = sigmoidf_(zv[j]);
                    dzv[j] = dov[j] * ov[j] * sz * (1.f + zv[j] * (1.f - sz));
                    ozv[j] = ov[j] * zv[j] * sz;
                    dov[j] *= zv[j] * sz;
                }
                if (valid) {
                    pq_store8(reinterpret_cast<T *>(p.dz) + (int64_t)b * p.dz_bs + (int64_t)d * p.dz_ds, t0 + 8 * hh,
                              L, vec, dzv);
                    if (p.recompute_out_z)
                        pq_store8(reinterpret_cast<T *>(p.out_z) + (int64_t)b * p.out_z_bs + (int64_t)d * p.out_z_ds,
                                  t0 + 8 * hh, L, vec, ozv);
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) SDG[8 * hh + j][ch] = valid ? dov[j] : 0.f;
        }
    };

    // ---- forward sweep: the state at the start of every segment
    {
        float h[SPT] = {0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < nseg; ++s) {
            const int64_t t0 = (int64_t)s * SEG;
            if (valid)  // a lane of a padding channel aliases channel 0's row: it must not write
                *reinterpret_cast<float4 *>(ck + (int64_t)s * NS) = make_float4(h[0], h[1], h[2], h[3]);
            __syncthreads();
            stage_bc(t0);
            load_seg(t0, false);
            __syncthreads();
            const int tv = (int)min((int64_t)SEG, L - t0);
            for (int t = 0; t < tv; ++t)
                pq_step<RM, LPC>(h, Pr, Qr, A2, SDT[t][ch], SDTU[t][ch], &Bs[t][SPT * qt]);
        }
    }

    // ---- reverse sweep over segments
    float carry[SPT] = {0.f, 0.f, 0.f, 0.f}, dA[SPT] = {0.f, 0.f, 0.f, 0.f};
    float dP[SPT][RM], dQ[RM][SPT];
#pragma unroll
    for (int j = 0; j < SPT; ++j)
#pragma unroll
        for (int k = 0; k < RM; ++k) dP[j][k] = dQ[k][j] = 0.f;
    float dDs = 0.f, dbs = 0.f;
    for (int s = nseg - 1; s >= 0; --s) {
        const int64_t t0 = (int64_t)s * SEG;
        const int tv = (int)min((int64_t)SEG, L - t0);
        __syncthreads();
        stage_bc(t0);
        load_seg(t0, true);
        __syncthreads();
        {  // states of the segment: HS[0] = h before it, HS[t+1] = h_t
            const float4 c4 = valid ? *reinterpret_cast<const float4 *>(ck + (int64_t)s * NS)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            float h[SPT] = {c4.x, c4.y, c4.z, c4.w};
            *reinterpret_cast<float4 *>(&HS[0][tid][0]) = c4;
            for (int t = 0; t < tv; ++t) {
                pq_step<RM, LPC>(h, Pr, Qr, A2, SDT[t][ch], SDTU[t][ch], &Bs[t][SPT * qt]);
                *reinterpret_cast<float4 *>(&HS[t + 1][tid][0]) = make_float4(h[0], h[1], h[2], h[3]);
            }
        }
        for (int t = tv - 1; t >= 0; --t) {
            const float dt = SDT[t][ch], dtu = SDTU[t][ch], dg = SDG[t][ch];
            const float4 hp4 = *reinterpret_cast<const float4 *>(&HS[t][tid][0]);
            const float4 hn4 = *reinterpret_cast<const float4 *>(&HS[t + 1][tid][0]);
            const float hp[SPT] = {hp4.x, hp4.y, hp4.z, hp4.w}, hn[SPT] = {hn4.x, hn4.y, hn4.z, hn4.w};
            const float *bt = &Bs[t][SPT * qt], *ct = &Cs[t][SPT * qt];
            float gv[SPT];
#pragma unroll
            for (int j = 0; j < SPT; ++j) gv[j] = fmaf(dg, ct[j], carry[j]);
            float qh[RM], ptg[RM];
#pragma unroll
            for (int k = 0; k < RM; ++k) {
                float s1 = 0.f, s2 = 0.f;
#pragma unroll
                for (int j = 0; j < SPT; ++j) {
                    s1 = fmaf(Qr[k][j], hp[j], s1);
                    s2 = fmaf(Pr[j][k], gv[j], s2);
                }
                qh[k] = group_sum<LPC>(s1);
                ptg[k] = group_sum<LPC>(s2);
            }
            float S1 = 0.f, S2 = 0.f, red[2 * SPT];
#pragma unroll
            for (int j = 0; j < SPT; ++j) {
                const float a = ex2(dt * A2[j]);
                float pqn = 0.f, qtp = 0.f;
#pragma unroll
                for (int k = 0; k < RM; ++k) {
                    pqn = fmaf(Pr[j][k], qh[k], pqn);
                    qtp = fmaf(Qr[k][j], ptg[k], qtp);
                }
                const float ahp = a * hp[j], dtg = dt * gv[j];
                S1 = fmaf(gv[j], bt[j], S1);
                S2 = fmaf(gv[j], fmaf(An[j], ahp, pqn), S2);
                dA[j] = fmaf(dtg, ahp, dA[j]);
                red[j] = dtu * gv[j];        // dB contribution
                red[SPT + j] = dg * hn[j];   // dC contribution
                carry[j] = fmaf(a, gv[j], dt * qtp);
#pragma unroll
                for (int k = 0; k < RM; ++k) {
                    dP[j][k] = fmaf(dtg, qh[k], dP[j][k]);
                    dQ[k][j] = fmaf(dt * ptg[k], hp[j], dQ[k][j]);
                }
            }
            S1 = group_sum<LPC>(S1);
            S2 = group_sum<LPC>(S2);
            if (qt == 0) {
                const float uu = SU[t][ch];
                const float ddt = fmaf(uu, S1, S2) * SGT[t][ch];
                DU[t][ch] = fmaf(dt, S1, Dv * dg);
                DD[t][ch] = ddt;
                dDs = fmaf(dg, uu, dDs);
                dbs += ddt;
            }
            // dB / dC: reduce-scatter the 8 values over the warp's channels (lanes with this
            // qt): after it the lane keeps values [rs_base(lane), + VPL), summed
            {
#pragma unroll
                for (int m = 16, half = 4; m >= LPC; m >>= 1, half >>= 1) {
                    const bool up = (lane & m) != 0;
#pragma unroll
                    for (int i = 0; i < half; ++i) {
                        const float send = up ? red[i] : red[half + i], keep = up ? red[half + i] : red[i];
                        red[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                    }
                }
#pragma unroll
                for (int i = 0; i < VPL; ++i) WACC[wid][t][lane][i] = red[i];
            }
        }
        __syncthreads();
        // du / ddelta of the segment (the quad leader of each channel), dB / dC flush
        if (qt == 0 && valid) {
            T *dur = reinterpret_cast<T *>(p.du) + (int64_t)b * p.du_bs + (int64_t)d * p.du_ds;
            T *ddr = reinterpret_cast<T *>(p.ddelta) + (int64_t)b * p.ddelta_bs + (int64_t)d * p.ddelta_ds;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float a1[8], a2[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    a1[j] = DU[8 * hh + j][ch];
                    a2[j] = DD[8 * hh + j][ch];
                }
                pq_store8(dur, t0 + 8 * hh, L, vec, a1);
                pq_store8(ddr, t0 + 8 * hh, L, vec, a2);
            }
        }
        // WACC entry (lane ln, value i): state SPT * (ln % LPC) + (idx & 3) with idx =
        // rs_base(ln) + i, dB for idx < 4 and dC above; 4 steps per item, one vector atomic each
        for (int it = tid; it < 32 * VPL * 4; it += NT) {
            const int sv = it >> 2, tq = it & 3, ln = sv / VPL, vi = sv - ln * VPL;
            const int idx = rs_base<LPC>(ln) + vi;
            const int n = SPT * (ln % LPC) + (idx & 3);
            const bool isC = idx >= 4;
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float sum = 0.f;
#pragma unroll
                for (int ww = 0; ww < NW; ++ww) sum += WACC[ww][4 * tq + i][ln][vi];
                v[i] = sum;
            }
            if (n < p.dstate && 4 * tq < tv) {
                float *dst = (isC ? p.acc_dC : p.acc_dB) + (((int64_t)b * p.n_groups + g) * p.dstate + n) * p.lpitch +
                             t0 + 4 * tq;
                if (4 * tq + 4 <= tv) {
                    red_add_v4(dst, v[0], v[1], v[2], v[3]);
                } else {
                    for (int i = 0; i < 4; ++i)
                        if (4 * tq + i < tv) atomicAdd(dst + i, v[i]);
                }
            }
        }
    }
    // per-channel sums
    if (valid) {
#pragma unroll
        for (int j = 0; j < SPT; ++j) {
            const int n = SPT * qt + j;
            if (n < p.dstate) atomicAdd(p.dA + (int64_t)d * p.dstate + n, dA[j]);
        }
        if (qt == 0) {
            if (p.dD) atomicAdd(p.dD + d, dDs);
            if (p.ddelta_bias) atomicAdd(p.ddelta_bias + d, dbs);
        }
    }
    // dP / dQ: per channel, or summed over the warp's channels when shared (and over the batch)
#pragma unroll
    for (int j = 0; j < SPT; ++j) {
        const int n = SPT * qt + j;
#pragma unroll
        for (int k = 0; k < RM; ++k) {
            float vp = valid ? dP[j][k] : 0.f, vq = valid ? dQ[k][j] : 0.f;
            if (p.pq_per_dim) {  // summed over the batch rows (one CTA row each)
                if (valid && n < p.dstate && k < r) {
                    atomicAdd(p.dP + ((int64_t)d * p.dstate + n) * r + k, vp);
                    atomicAdd(p.dQ + ((int64_t)d * r + k) * p.dstate + n, vq);
                }
            } else {
#pragma unroll
                for (int off = LPC; off < 32; off <<= 1) {
                    vp += __shfl_xor_sync(0xffffffffu, vp, off);
                    vq += __shfl_xor_sync(0xffffffffu, vq, off);
                }
                if (lane < LPC && n < p.dstate && k < r) {
                    atomicAdd(p.dP + n * r + k, vp);
                    atomicAdd(p.dQ + k * p.dstate + n, vq);
                }
            }
        }
    }
}

template <typename T, bool HAS_Z, int RM, int NSX>
static cudaError_t pq_fwd_t(FwdParams p, cudaStream_t st) {
    constexpr int CH = pq::Geo<NSX>::CH;
    p.tiles_per_group = (p.dpg + CH - 1) / CH;
    dim3 grid(p.tiles_per_group * p.n_groups, p.batch);
    ss_pq_fwd_kernel<T, HAS_Z, RM, NSX><<<grid, pq::NT, 0, st>>>(p);
    return cudaGetLastError();
}

template <typename T, bool HAS_Z, int RM, int NSX>
static cudaError_t pq_bwd_t(BwdParams p, cudaStream_t st) {
    auto kern = ss_pq_bwd_kernel<T, HAS_Z, RM, NSX>;
    constexpr int SMEM = (int)sizeof(PqBwdSmem<NSX>);
    constexpr int CH = pq::Geo<NSX>::CH;
    static std::atomic<unsigned long long> smem_set{0};
    {
        const cudaError_t e = set_smem_once(smem_set, reinterpret_cast<const void *>(kern), SMEM);
        if (e != cudaSuccess) return e;
    }
    p.tiles_per_group = (p.dpg + CH - 1) / CH;
    dim3 grid(p.tiles_per_group * p.n_groups, p.batch);
    kern<<<grid, pq::NT, SMEM, st>>>(p);
    return cudaGetLastError();
}

template <typename T, int NSX>
static cudaError_t pq_fwd_ns(const FwdParams &p, bool has_z, cudaStream_t st) {
    if (p.pq_rank <= 4) return has_z ? pq_fwd_t<T, true, 4, NSX>(p, st) : pq_fwd_t<T, false, 4, NSX>(p, st);
    return has_z ? pq_fwd_t<T, true, 8, NSX>(p, st) : pq_fwd_t<T, false, 8, NSX>(p, st);
}
template <typename T, int NSX>
static cudaError_t pq_bwd_ns(const BwdParams &p, bool has_z, cudaStream_t st) {
    if (p.pq_rank <= 4) return has_z ? pq_bwd_t<T, true, 4, NSX>(p, st) : pq_bwd_t<T, false, 4, NSX>(p, st);
    return has_z ? pq_bwd_t<T, true, 8, NSX>(p, st) : pq_bwd_t<T, false, 8, NSX>(p, st);
}
template <typename T>
static cudaError_t pq_fwd_dispatch(const FwdParams &p, bool has_z, cudaStream_t st) {
    if (p.dstate <= 16) return pq_fwd_ns<T, 16>(p, has_z, st);
    if (p.dstate <= 32) return pq_fwd_ns<T, 32>(p, has_z, st);
    return pq_fwd_ns<T, 64>(p, has_z, st);
}
template <typename T>
static cudaError_t pq_bwd_dispatch(const BwdParams &p, bool has_z, cudaStream_t st) {
    if (p.dstate <= 16) return pq_bwd_ns<T, 16>(p, has_z, st);
    if (p.dstate <= 32) return pq_bwd_ns<T, 32>(p, has_z, st);
    return pq_bwd_ns<T, 64>(p, has_z, st);
}

cudaError_t launch_ss_fwd_pq(const FwdParams &p, int itype, bool has_z, cudaStream_t st) {
    switch (itype) {
        case MSS_F32: return pq_fwd_dispatch<float>(p, has_z, st);
        case MSS_F16: return pq_fwd_dispatch<__half>(p, has_z, st);
        default: return pq_fwd_dispatch<__nv_bfloat16>(p, has_z, st);
    }
}
cudaError_t launch_ss_bwd_pq(const BwdParams &p, int itype, bool has_z, cudaStream_t st) {
    switch (itype) {
        case MSS_F32: return pq_bwd_dispatch<float>(p, has_z, st);
        case MSS_F16: return pq_bwd_dispatch<__half>(p, has_z, st);
        default: return pq_bwd_dispatch<__nv_bfloat16>(p, has_z, st);
    }
}

}  // namespace mss
