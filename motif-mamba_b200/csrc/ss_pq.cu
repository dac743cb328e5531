// Selective scan with the motif low-rank state coupling, forward and backward, sm_100a.
//
//   h_t = exp(dt_t A) * h_{t-1} + dt_t * P (Q h_{t-1}) + dt_t u_t B_t,   y_t = <C_t, h_t>
//
// (reference: selective_scan_ref with P/Q, mamba_ssm/ops/selective_scan_interface.py:402-433;
// full-matrix path :262-350).  P is (dstate, r) shared or (dim, dstate, r) per channel, Q is
// (r, dstate) or (dim, r, dstate), r <= 8, dstate <= 16.  The coupling mixes states, so the
// diagonal-scan tricks of ss_fwd / ss_bwd do not apply: one thread owns one channel and
// walks the sequence with all 16 states in registers.
//
// Forward: per step q = Q h (r x 16 FMAs), pq = P q, the diagonal update, y = <C, h>, the
// D-skip and z gate; B/C tiles are staged in shared memory, u/delta/z rows are read by their
// owning thread with 16-byte loads; x gets the state every 256 steps as in ss_fwd.
// Backward (O(L)): a forward sweep stores the state at every 16-step segment start in a
// workspace; then segments are processed in reverse: the 16 states of each step are
// recomputed into shared memory and the adjoint g_t = C_t doutg_t + M_{t+1}^T g_{t+1}
// (M = diag(a) + dt P Q, M^T g = a g + dt Q^T (P^T g)) runs backwards, accumulating
// du, ddelta, dA, dD, ddelta_bias, dP = sum dt g (Q h_{t-1})^T, dQ = sum dt (P^T g) h_{t-1}^T;
// dB / dC are summed over the warp's 32 channels through a shared-memory transpose and
// added once per lane with an fp32 atomic into the same accumulators ss_bwd uses.
#include "common.cuh"
#include "kernels.h"

namespace mss {

namespace pq {
constexpr int NS = 16;   // states (dstate <= 16, zero padded)
constexpr int RM = 8;    // max rank
constexpr int TT = 32;   // forward tile (divides the 256-step x chunk)
constexpr int CHF = 64;  // forward channels per CTA
constexpr int CHB = 32;  // backward channels per CTA (one warp)
constexpr int SEG = 16;  // backward segment length
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

// Fill P (index n*RM+k) and Q (index k*NS+n) into shared memory, zero-padded to NS x RM.
// Per-channel layout is [index][thread] (conflict-free); shared layout is [index].
template <bool PER_DIM, int CH>
__device__ __forceinline__ void pq_fill(float *Pm, float *Qm, const float *P, const float *Q, int d, bool valid,
                                        int dstate, int r, int tid) {
    using namespace pq;
    if constexpr (PER_DIM) {
        for (int idx = 0; idx < NS * RM; ++idx) {
            const int n = idx / RM, k = idx - n * RM;
            Pm[idx * CH + tid] = (valid && n < dstate && k < r) ? P[((int64_t)d * dstate + n) * r + k] : 0.f;
            const int k2 = idx / NS, n2 = idx - k2 * NS;
            Qm[idx * CH + tid] = (valid && n2 < dstate && k2 < r) ? Q[((int64_t)d * r + k2) * dstate + n2] : 0.f;
        }
    } else {
        for (int idx = tid; idx < NS * RM; idx += CH) {
            const int n = idx / RM, k = idx - n * RM;
            Pm[idx] = (n < dstate && k < r) ? P[n * r + k] : 0.f;
            const int k2 = idx / NS, n2 = idx - k2 * NS;
            Qm[idx] = (n2 < dstate && k2 < r) ? Q[k2 * dstate + n2] : 0.f;
        }
    }
}

template <typename T, bool HAS_Z, bool PER_DIM>
__global__ void __launch_bounds__(pq::CHF) ss_pq_fwd_kernel(const FwdParams p) {
    using namespace pq;
    constexpr int CH = CHF, PW = PER_DIM ? CH : 1;
    extern __shared__ __align__(16) float sm[];
    float *Bs = sm, *Cs = Bs + TT * NS, *Pm = Cs + TT * NS, *Qm = Pm + NS * RM * PW;
    const int tid = threadIdx.x, pi = PER_DIM ? tid : 0;
    const int g = blockIdx.x / p.tiles_per_group, tile = blockIdx.x - g * p.tiles_per_group;
    const int b = blockIdx.y;
    const int cin = tile * CH + tid;
    const bool valid = cin < p.dpg;
    const int d = g * p.dpg + (valid ? cin : 0);
    const int64_t L = p.seqlen, row = (int64_t)b * p.dim + d;
    const bool vec = p.aligned != 0;
    const int r = p.pq_rank;
    pq_fill<PER_DIM, CH>(Pm, Qm, p.P, p.Q, d, valid, p.dstate, r, tid);

    float A2[NS], h[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        A2[n] = (valid && n < p.dstate) ? p.A[(int64_t)d * p.A_ds + (int64_t)n * p.A_ns] * kLog2e : 0.f;
        h[n] = 0.f;
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
        for (int i = tid; i < TT * NS; i += CH) {
            const int t = i / NS, n = i - t * NS;
            const bool ok = t0 + t < L && n < p.dstate;
            Bs[i] = ok ? to_f<T>(gB[(int64_t)n * p.B_ns + t0 + t]) : 0.f;
            Cs[i] = ok ? to_f<T>(gC[(int64_t)n * p.C_ns + t0 + t]) : 0.f;
        }
        __syncthreads();
#pragma unroll 1
        for (int g8 = 0; g8 < TT && t0 + g8 < L; g8 += 8) {
            const int64_t tg = t0 + g8;
            float uf[8], dv[8], y[8];
            pq_load8(ur, tg, L, vec, uf);
            pq_load8(dr, tg, L, vec, dv);
#pragma unroll 1
            for (int j = 0; j < 8; ++j) {
                float dt = dv[j] + bias;
                if (p.softplus) dt = softplus20(dt);
                dt = (valid && tg + j < L) ? dt : 0.f;
                cum += dt;
                const float dtu = dt * uf[j];
                float q[RM];
#pragma unroll
                for (int k = 0; k < RM; ++k) {
                    q[k] = 0.f;
                    if (k < r) {
#pragma unroll
                        for (int n = 0; n < NS; ++n) q[k] = fmaf(Qm[(k * NS + n) * PW + pi], h[n], q[k]);
                    }
                }
                const float *bt = Bs + (g8 + j) * NS, *ct = Cs + (g8 + j) * NS;
                float acc = 0.f;
#pragma unroll
                for (int n = 0; n < NS; ++n) {
                    float pqn = 0.f;
#pragma unroll
                    for (int k = 0; k < RM; ++k)
                        if (k < r) pqn = fmaf(Pm[(n * RM + k) * PW + pi], q[k], pqn);
                    h[n] = fmaf(ex2(dt * A2[n]), h[n], fmaf(dt, pqn, dtu * bt[n]));
                    acc = fmaf(ct[n], h[n], acc);
                }
                y[j] = fmaf(Dv, uf[j], acc);
            }
            if (valid) {
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
            for (int n = 0; n < NS; ++n)
                if (n < p.dstate) {
                    xr[2 * n] = ex2(A2[n] * cum);
                    xr[2 * n + 1] = h[n];
                }
        }
    }
}

template <typename T, bool HAS_Z, bool PER_DIM>
struct PqBwdLayout {
    static constexpr int PW = PER_DIM ? pq::CHB : 1;
    static constexpr int P_OFF = 0, Q_OFF = P_OFF + pq::NS * pq::RM * PW;
    static constexpr int DP_OFF = Q_OFF + pq::NS * pq::RM * PW;                 // [idx][lane]
    static constexpr int DQ_OFF = DP_OFF + pq::NS * pq::RM * pq::CHB;
    static constexpr int HS_OFF = DQ_OFF + pq::NS * pq::RM * pq::CHB;            // [SEG+1][NS][lane]
    static constexpr int SV_OFF = HS_OFF + (pq::SEG + 1) * pq::NS * pq::CHB;     // [5][SEG][lane]
    static constexpr int BS_OFF = SV_OFF + 5 * pq::SEG * pq::CHB;                // B, C [SEG][NS]
    static constexpr int RD_OFF = BS_OFF + 2 * pq::SEG * pq::NS;                 // [32][33]
    static constexpr int FLOATS = RD_OFF + 32 * 33;
};

template <typename T, bool HAS_Z, bool PER_DIM>
__global__ void __launch_bounds__(pq::CHB) ss_pq_bwd_kernel(const BwdParams p) {
    using namespace pq;
    using Ly = PqBwdLayout<T, HAS_Z, PER_DIM>;
    constexpr int PW = Ly::PW;
    extern __shared__ __align__(16) float sm[];
    float *Pm = sm + Ly::P_OFF, *Qm = sm + Ly::Q_OFF, *dPm = sm + Ly::DP_OFF, *dQm = sm + Ly::DQ_OFF;
    float *HS = sm + Ly::HS_OFF, *SV = sm + Ly::SV_OFF, *Bs = sm + Ly::BS_OFF, *Cs = Bs + SEG * NS;
    float *RD = sm + Ly::RD_OFF;
    float *SU = SV, *SDT = SV + SEG * CHB, *SDU = SV + 2 * SEG * CHB, *SDG = SV + 3 * SEG * CHB,
          *SGT = SV + 4 * SEG * CHB;  // u, dt, dt*u, doutg, softplus gate: [SEG][lane]
    const int lane = threadIdx.x, pi = PER_DIM ? lane : 0;
    const int g = blockIdx.x / p.tiles_per_group, tile = blockIdx.x - g * p.tiles_per_group;
    const int b = blockIdx.y;
    const int cin = tile * CHB + lane;
    const bool valid = cin < p.dpg;
    const int d = g * p.dpg + (valid ? cin : 0);
    const int64_t L = p.seqlen, row = (int64_t)b * p.dim + d;
    const bool vec = p.aligned != 0;
    const int r = p.pq_rank;
    const int nseg = (int)((L + SEG - 1) / SEG);
    pq_fill<PER_DIM, CHB>(Pm, Qm, p.P, p.Q, d, valid, p.dstate, r, lane);
    for (int i = lane; i < NS * RM * CHB; i += CHB) dPm[i] = dQm[i] = 0.f;

    float A2[NS], An[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) {
        An[n] = (valid && n < p.dstate) ? p.A[(int64_t)d * p.A_ds + (int64_t)n * p.A_ns] : 0.f;
        A2[n] = An[n] * kLog2e;
    }
    const float Dv = (p.D && valid) ? p.D[(int64_t)d * p.D_s] : 0.f;
    const float bias = (p.delta_bias && valid) ? p.delta_bias[(int64_t)d * p.delta_bias_s] : 0.f;
    const T *ur = reinterpret_cast<const T *>(p.u) + (int64_t)b * p.u_bs + (int64_t)d * p.u_ds;
    const T *dr = reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs + (int64_t)d * p.delta_ds;
    const T *dor = reinterpret_cast<const T *>(p.dout) + (int64_t)b * p.dout_bs + (int64_t)d * p.dout_ds;
    const T *gB = reinterpret_cast<const T *>(p.B) + (int64_t)b * p.B_bs + (int64_t)g * p.B_gs;
    const T *gC = reinterpret_cast<const T *>(p.C) + (int64_t)b * p.C_bs + (int64_t)g * p.C_gs;
    float *ck = p.ckpt + row * (int64_t)nseg * NS;

    auto stage_bc = [&](int64_t t0) {
        __syncwarp();
        for (int i = lane; i < SEG * NS; i += CHB) {
            const int t = i / NS, n = i - t * NS;
            const bool ok = t0 + t < L && n < p.dstate;
            Bs[i] = ok ? to_f<T>(gB[(int64_t)n * p.B_ns + t0 + t]) : 0.f;
            Cs[i] = ok ? to_f<T>(gC[(int64_t)n * p.C_ns + t0 + t]) : 0.f;
        }
        __syncwarp();
    };
    auto step_fwd = [&](float (&h)[NS], float dt, float dtu, const float *bt) {
        float q[RM];
#pragma unroll
        for (int k = 0; k < RM; ++k) {
            q[k] = 0.f;
            if (k < r) {
#pragma unroll
                for (int n = 0; n < NS; ++n) q[k] = fmaf(Qm[(k * NS + n) * PW + pi], h[n], q[k]);
            }
        }
#pragma unroll
        for (int n = 0; n < NS; ++n) {
            float pqn = 0.f;
#pragma unroll
            for (int k = 0; k < RM; ++k)
                if (k < r) pqn = fmaf(Pm[(n * RM + k) * PW + pi], q[k], pqn);
            h[n] = fmaf(ex2(dt * A2[n]), h[n], fmaf(dt, pqn, dtu * bt[n]));
        }
    };
    auto load_seg = [&](int64_t t0) {  // per-step inputs of this lane's row -> SV
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
                SU[t * CHB + lane] = uf[j];
                SDT[t * CHB + lane] = x;
                SDU[t * CHB + lane] = x * uf[j];
                SGT[t * CHB + lane] = gate;
            }
        }
    };

    // ---- forward sweep: the state at the start of every segment
    {
        float h[NS];
#pragma unroll
        for (int n = 0; n < NS; ++n) h[n] = 0.f;
        for (int s = 0; s < nseg; ++s) {
            const int64_t t0 = (int64_t)s * SEG;
#pragma unroll
            for (int n = 0; n < NS; ++n) ck[(int64_t)s * NS + n] = h[n];
            stage_bc(t0);
            load_seg(t0);
            __syncwarp();
            for (int t = 0; t < SEG && t0 + t < L; ++t)
                step_fwd(h, SDT[t * CHB + lane], SDU[t * CHB + lane], Bs + t * NS);
        }
    }

    // ---- reverse sweep over segments
    float carry[NS], dA[NS];
#pragma unroll
    for (int n = 0; n < NS; ++n) carry[n] = dA[n] = 0.f;
    float dDs = 0.f, dbs = 0.f;
    for (int s = nseg - 1; s >= 0; --s) {
        const int64_t t0 = (int64_t)s * SEG;
        const int tv = (int)min((int64_t)SEG, L - t0);
        stage_bc(t0);
        load_seg(t0);
        // doutg and the z gate outputs
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
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
            for (int j = 0; j < 8; ++j) SDG[(8 * hh + j) * CHB + lane] = valid ? dov[j] : 0.f;
        }
        // states of the segment: HS[0] = h before it, HS[t+1] = h_t
        {
            float h[NS];
#pragma unroll
            for (int n = 0; n < NS; ++n) {
                h[n] = ck[(int64_t)s * NS + n];
                HS[n * CHB + lane] = h[n];
            }
            __syncwarp();
            for (int t = 0; t < tv; ++t) {
                step_fwd(h, SDT[t * CHB + lane], SDU[t * CHB + lane], Bs + t * NS);
#pragma unroll
                for (int n = 0; n < NS; ++n) HS[((t + 1) * NS + n) * CHB + lane] = h[n];
            }
        }
        for (int t = tv - 1; t >= 0; --t) {
            const float dt = SDT[t * CHB + lane], uu = SU[t * CHB + lane], dg = SDG[t * CHB + lane];
            const float *bt = Bs + t * NS, *ct = Cs + t * NS;
            float gv[NS], hp[NS];
#pragma unroll
            for (int n = 0; n < NS; ++n) {
                gv[n] = fmaf(dg, ct[n], carry[n]);
                hp[n] = HS[(t * NS + n) * CHB + lane];
            }
            float qh[RM], ptg[RM];
#pragma unroll
            for (int k = 0; k < RM; ++k) {
                qh[k] = ptg[k] = 0.f;
                if (k < r) {
#pragma unroll
                    for (int n = 0; n < NS; ++n) {
                        qh[k] = fmaf(Qm[(k * NS + n) * PW + pi], hp[n], qh[k]);
                        ptg[k] = fmaf(Pm[(n * RM + k) * PW + pi], gv[n], ptg[k]);
                    }
                }
            }
            float S1 = 0.f, S2 = 0.f;
            float red[2 * NS];
#pragma unroll
            for (int n = 0; n < NS; ++n) {
                const float a = ex2(dt * A2[n]);
                float pqn = 0.f, qtp = 0.f;
#pragma unroll
                for (int k = 0; k < RM; ++k)
                    if (k < r) {
                        pqn = fmaf(Pm[(n * RM + k) * PW + pi], qh[k], pqn);
                        qtp = fmaf(Qm[(k * NS + n) * PW + pi], ptg[k], qtp);
                    }
                const float ahp = a * hp[n];
                S1 = fmaf(gv[n], bt[n], S1);
                S2 = fmaf(gv[n], fmaf(An[n], ahp, pqn), S2);
                dA[n] = fmaf(dt * gv[n], ahp, dA[n]);
                red[n] = dt * uu * gv[n];                                  // dB contribution
                red[NS + n] = dg * HS[((t + 1) * NS + n) * CHB + lane];    // dC contribution
                carry[n] = fmaf(a, gv[n], dt * qtp);
            }
            // dP[n][k] += dt g_n qh_k ; dQ[k][n] += dt ptg_k hp_n   (this lane's channel)
            for (int k = 0; k < r; ++k) {
#pragma unroll
                for (int n = 0; n < NS; ++n) {
                    dPm[(n * RM + k) * CHB + lane] = fmaf(dt * gv[n], qh[k], dPm[(n * RM + k) * CHB + lane]);
                    dQm[(k * NS + n) * CHB + lane] = fmaf(dt * ptg[k], hp[n], dQm[(k * NS + n) * CHB + lane]);
                }
            }
            // sum dB / dC contributions over the warp's channels: lane j takes column j
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 2 * NS; ++j) RD[lane * 33 + j] = red[j];
            __syncwarp();
            {
                float sacc = 0.f;
#pragma unroll 8
                for (int i = 0; i < 32; ++i) sacc += RD[i * 33 + lane];
                const int n = lane & (NS - 1);
                if (n < p.dstate) {
                    float *dst = (lane < NS ? p.acc_dB : p.acc_dC) +
                                 (((int64_t)b * p.n_groups + g) * p.dstate + n) * p.lpitch + t0 + t;
                    atomicAdd(dst, sacc);
                }
            }
            const float ddt = fmaf(uu, S1, S2) * SGT[t * CHB + lane];
            const float du = fmaf(dt, S1, Dv * dg);
            dDs = fmaf(dg, uu, dDs);
            dbs += ddt;
            SU[t * CHB + lane] = du;    // reuse: du and ddelta of step t
            SDT[t * CHB + lane] = ddt;
        }
        if (valid) {
            T *dur = reinterpret_cast<T *>(p.du) + (int64_t)b * p.du_bs + (int64_t)d * p.du_ds;
            T *ddr = reinterpret_cast<T *>(p.ddelta) + (int64_t)b * p.ddelta_bs + (int64_t)d * p.ddelta_ds;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float a1[8], a2[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    a1[j] = SU[(8 * hh + j) * CHB + lane];
                    a2[j] = SDT[(8 * hh + j) * CHB + lane];
                }
                pq_store8(dur, t0 + 8 * hh, L, vec, a1);
                pq_store8(ddr, t0 + 8 * hh, L, vec, a2);
            }
        }
        __syncwarp();
    }
    if (valid) {
#pragma unroll
        for (int n = 0; n < NS; ++n)
            if (n < p.dstate) atomicAdd(p.dA + (int64_t)d * p.dstate + n, dA[n]);
        if (p.dD) atomicAdd(p.dD + d, dDs);
        if (p.ddelta_bias) atomicAdd(p.ddelta_bias + d, dbs);
    }
    // dP / dQ: per channel, or summed over the warp's channels when shared
    for (int idx = 0; idx < NS * RM; ++idx) {
        const int n = idx / RM, k = idx - n * RM;
        const int k2 = idx / NS, n2 = idx - k2 * NS;
        float vp = valid ? dPm[idx * CHB + lane] : 0.f;
        float vq = valid ? dQm[idx * CHB + lane] : 0.f;
        if constexpr (PER_DIM) {
            if (valid && n < p.dstate && k < r) atomicAdd(p.dP + ((int64_t)d * p.dstate + n) * r + k, vp);
            if (valid && n2 < p.dstate && k2 < r) atomicAdd(p.dQ + ((int64_t)d * r + k2) * p.dstate + n2, vq);
        } else {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                vp += __shfl_xor_sync(0xffffffffu, vp, off);
                vq += __shfl_xor_sync(0xffffffffu, vq, off);
            }
            if (lane == 0) {
                if (n < p.dstate && k < r) atomicAdd(p.dP + n * r + k, vp);
                if (n2 < p.dstate && k2 < r) atomicAdd(p.dQ + k2 * p.dstate + n2, vq);
            }
        }
    }
}

template <typename T, bool HAS_Z, bool PER_DIM>
static cudaError_t pq_fwd_t(FwdParams p, cudaStream_t st) {
    constexpr int CH = pq::CHF, PW = PER_DIM ? CH : 1;
    const int smem = (2 * pq::TT * pq::NS + 2 * pq::NS * pq::RM * PW) * 4;
    auto kern = ss_pq_fwd_kernel<T, HAS_Z, PER_DIM>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    p.tiles_per_group = (p.dpg + CH - 1) / CH;
    dim3 grid(p.tiles_per_group * p.n_groups, p.batch);
    kern<<<grid, CH, smem, st>>>(p);
    return cudaGetLastError();
}

template <typename T, bool HAS_Z, bool PER_DIM>
static cudaError_t pq_bwd_t(BwdParams p, cudaStream_t st) {
    using Ly = PqBwdLayout<T, HAS_Z, PER_DIM>;
    const int smem = Ly::FLOATS * 4;
    auto kern = ss_pq_bwd_kernel<T, HAS_Z, PER_DIM>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    p.tiles_per_group = (p.dpg + pq::CHB - 1) / pq::CHB;
    dim3 grid(p.tiles_per_group * p.n_groups, p.batch);
    kern<<<grid, pq::CHB, smem, st>>>(p);
    return cudaGetLastError();
}

template <typename T>
static cudaError_t pq_fwd_dispatch(const FwdParams &p, bool has_z, cudaStream_t st) {
    if (p.pq_per_dim) return has_z ? pq_fwd_t<T, true, true>(p, st) : pq_fwd_t<T, false, true>(p, st);
    return has_z ? pq_fwd_t<T, true, false>(p, st) : pq_fwd_t<T, false, false>(p, st);
}
template <typename T>
static cudaError_t pq_bwd_dispatch(const BwdParams &p, bool has_z, cudaStream_t st) {
    if (p.pq_per_dim) return has_z ? pq_bwd_t<T, true, true>(p, st) : pq_bwd_t<T, false, true>(p, st);
    return has_z ? pq_bwd_t<T, true, false>(p, st) : pq_bwd_t<T, false, false>(p, st);
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
