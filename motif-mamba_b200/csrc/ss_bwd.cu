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
// Design (B200): a CTA of 256 threads covers 16 channels x 16 states per pass; thread
// (cl, n) owns state n of channel cl and walks the sequence serially, so every
// recurrence is a register FMA chain.  The forward's chunk states x (one every 256
// steps) seed each chunk; a forward pre-pass over the chunk stores the state at every
// 16-step tile start in shared memory, then the tiles are processed in reverse: the
// 16-step forward is recomputed into registers (decay a_t and state h_t), then the
// reverse recurrence runs over them.  Per-element work (softplus, z gate, du, ddelta,
// dz) is done once per element by "element threads" (one per (t, channel) of the tile);
// the sums over states (sum_n dh B, sum_n A dh p) go through a padded shared-memory
// transpose.  dB / dC are first summed over the CTA's channels on chip (warp shuffle +
// shared memory) into a per-chunk fp32 accumulator that also sums the CTA's K channel
// groups, and leave as one vector red.global.add.v4.f32 per 4 timesteps per chunk, so
// the global atomic traffic is 1/(16 K) of a per-channel scheme.
#include "common.cuh"
#include "kernels.h"

namespace mss {

namespace bwd {
constexpr int NT = 256;   // threads per CTA
constexpr int NSP = 16;   // state lanes per channel (dstate <= 16, zero padded)
constexpr int CL = 16;    // channels per pass
constexpr int SEG = 16;   // timesteps per tile
constexpr int FP = 20;    // padded row pitch (floats) of the fp32 per-tile arrays
constexpr int XP = 36;    // padded row pitch (floats) of the (S1, S2) transpose rows
constexpr int TILES_PER_CHUNK = kChunkLen / SEG;
}  // namespace bwd

template <typename T, bool HAS_Z>
struct BwdLayout {
    static constexpr int RP = bwd::SEG * (int)sizeof(T) + 16;
    static constexpr int NARR = HAS_Z ? 5 : 3;  // u, delta, dout, (z, out)
    static constexpr int U_OFF = 0, DT_OFF = 16 * RP, DO_OFF = 32 * RP, Z_OFF = 48 * RP, OUT_OFF = 64 * RP;
    static constexpr int B_OFF = NARR * 16 * RP, C_OFF = B_OFF + 16 * RP;
    static constexpr int BUF = (NARR * 16 + 32) * RP;
    static constexpr int F_OFF = 2 * BUF;                                // DTF, DTU, DOG [16][FP]
    static constexpr int BCF_OFF = F_OFF + 3 * 16 * bwd::FP * 4;         // B, C fp32 [2][16][FP]
    static constexpr int XCH_OFF = BCF_OFF + 2 * 16 * bwd::FP * 4;       // (S1,S2) transpose | dB/dC partials
    static constexpr int XCH_BYTES = 256 * bwd::XP * 4;                  // >= 8*2*16*16*4
    static constexpr int ACC_OFF = XCH_OFF + XCH_BYTES;                  // [2][16][256] fp32
    static constexpr int CK_OFF = ACC_OFF + 2 * 16 * kChunkLen * 4;      // [16 tiles][256] fp32
    static constexpr int PB_OFF = CK_OFF + bwd::TILES_PER_CHUNK * bwd::NT * 4;  // [2][16 t][16 cl]
    static constexpr int SMEM = PB_OFF + 2 * 16 * 16 * 4;
};

template <typename T, bool HAS_Z>
__global__ void __launch_bounds__(bwd::NT, 2) ss_bwd_kernel(const BwdParams p) {
    using namespace bwd;
    using Ly = BwdLayout<T, HAS_Z>;
    constexpr int RP = Ly::RP;
    extern __shared__ __align__(16) char smem[];
    float *DTF = reinterpret_cast<float *>(smem + Ly::F_OFF);
    float *DTU = DTF + 16 * FP;
    float *DOG = DTU + 16 * FP;
    float *BF = reinterpret_cast<float *>(smem + Ly::BCF_OFF);
    float *CF = BF + 16 * FP;
    float *XCH = reinterpret_cast<float *>(smem + Ly::XCH_OFF);
    float *ACC = reinterpret_cast<float *>(smem + Ly::ACC_OFF);
    float *CKPT = reinterpret_cast<float *>(smem + Ly::CK_OFF);
    float *PB = reinterpret_cast<float *>(smem + Ly::PB_OFF);

    const int tid = threadIdx.x;
    // state-thread coordinates
    const int s_cl = tid >> 4, s_n = tid & 15;
    // element-thread coordinates (prologue / epilogue): t-major so a warp holds 2 timesteps
    const int e_t = tid >> 4, e_cl = tid & 15;

    const int g = blockIdx.x / p.tiles_per_group;
    const int tile = blockIdx.x - g * p.tiles_per_group;
    const int b = blockIdx.y;
    const int64_t L = p.seqlen;
    const bool aligned = p.aligned != 0;

    for (int i = tid; i < 2 * 16 * kChunkLen; i += NT) ACC[i] = 0.f;

    const T *gB = reinterpret_cast<const T *>(p.B) + (int64_t)b * p.B_bs + (int64_t)g * p.B_gs;
    const T *gC = reinterpret_cast<const T *>(p.C) + (int64_t)b * p.C_bs + (int64_t)g * p.C_gs;

    for (int k = p.n_chunks - 1; k >= 0; --k) {
        const int64_t kt0 = (int64_t)k * kChunkLen;
        const int clen = (int)min((int64_t)kChunkLen, L - kt0);
        const int ntile = (clen + SEG - 1) / SEG;
        for (int cgi = 0; cgi < p.kgroups; ++cgi) {
            const int cbase = (tile * p.kgroups + cgi) * CL;  // within the group
            const int nvalid = min(CL, p.dpg - cbase);
            if (nvalid <= 0) break;  // uniform over the CTA
            const int c0 = g * p.dpg + cbase;

            // per-state-thread constants
            const bool s_vch = s_cl < nvalid;
            const int s_d = c0 + (s_vch ? s_cl : 0);
            const bool s_vst = s_vch && s_n < p.dstate;
            const float An = s_vst ? p.A[(int64_t)s_d * p.A_ds + (int64_t)s_n * p.A_ns] : 0.f;
            const float A2 = An * kLog2e;
            const int64_t s_row = (int64_t)b * p.dim + s_d;
            // per-element-thread constants
            const bool e_vch = e_cl < nvalid;
            const int e_d = c0 + (e_vch ? e_cl : 0);
            const float bias = (p.delta_bias && e_vch) ? p.delta_bias[(int64_t)e_d * p.delta_bias_s] : 0.f;
            const float Dv = (p.D && e_vch) ? p.D[(int64_t)e_d * p.D_s] : 0.f;

            const T *gu = reinterpret_cast<const T *>(p.u) + (int64_t)b * p.u_bs + (int64_t)c0 * p.u_ds;
            const T *gdt = reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs + (int64_t)c0 * p.delta_ds;
            const T *gdo = reinterpret_cast<const T *>(p.dout) + (int64_t)b * p.dout_bs + (int64_t)c0 * p.dout_ds;
            const T *gz = HAS_Z ? reinterpret_cast<const T *>(p.z) + (int64_t)b * p.z_bs + (int64_t)c0 * p.z_ds : nullptr;
            const T *gout = HAS_Z ? reinterpret_cast<const T *>(p.out) + (int64_t)b * p.out_bs + (int64_t)c0 * p.out_ds : nullptr;

            auto stage = [&](int buf, int j, bool full) {
                char *rb = smem + buf * Ly::BUF;
                const int64_t t0 = kt0 + (int64_t)j * SEG;
                const int tv = (int)min((int64_t)SEG, L - t0);
                stage_tile<T, SEG>(rb + Ly::U_OFF, RP, gu, p.u_ds, 16, nvalid, t0, tv, aligned, tid, NT);
                stage_tile<T, SEG>(rb + Ly::DT_OFF, RP, gdt, p.delta_ds, 16, nvalid, t0, tv, aligned, tid, NT);
                stage_tile<T, SEG>(rb + Ly::B_OFF, RP, gB, p.B_ns, 16, p.dstate, t0, tv, aligned, tid, NT);
                if (full) {
                    stage_tile<T, SEG>(rb + Ly::DO_OFF, RP, gdo, p.dout_ds, 16, nvalid, t0, tv, aligned, tid, NT);
                    stage_tile<T, SEG>(rb + Ly::C_OFF, RP, gC, p.C_ns, 16, p.dstate, t0, tv, aligned, tid, NT);
                    if constexpr (HAS_Z) {
                        stage_tile<T, SEG>(rb + Ly::Z_OFF, RP, gz, p.z_ds, 16, nvalid, t0, tv, aligned, tid, NT);
                        stage_tile<T, SEG>(rb + Ly::OUT_OFF, RP, gout, p.out_ds, 16, nvalid, t0, tv, aligned, tid, NT);
                    }
                }
            };
            auto elem = [&](const char *rb, int off) -> float {
                return to_f<T>(reinterpret_cast<const T *>(rb + off + e_cl * RP)[e_t]);
            };

            // ---------------- forward pre-pass over the chunk: tile-start checkpoints -------------
            float h = 0.f;
            if (k > 0 && s_vst) h = p.x[(s_row * p.n_chunks + (k - 1)) * 2 * p.dstate + 2 * s_n + 1];
            stage(0, 0, false);
            cp_async_commit();
            for (int j = 0; j < ntile; ++j) {
                if (j + 1 < ntile) {
                    stage((j + 1) & 1, j + 1, false);
                    cp_async_commit();
                    cp_async_wait<1>();
                } else {
                    cp_async_wait<0>();
                }
                __syncthreads();
                {
                    const char *rb = smem + (j & 1) * Ly::BUF;
                    const bool vt = kt0 + j * SEG + e_t < L;
                    float dv = elem(rb, Ly::DT_OFF) + bias;
                    if (p.softplus) dv = softplus20(dv);
                    dv = vt ? dv : 0.f;
                    DTF[e_cl * FP + e_t] = dv;
                    DTU[e_cl * FP + e_t] = dv * elem(rb, Ly::U_OFF);
                    // B tile to fp32 [n][t] (thread -> (n = tid>>4, t = tid&15))
                    BF[(tid >> 4) * FP + (tid & 15)] =
                        to_f<T>(reinterpret_cast<const T *>(rb + Ly::B_OFF + (tid >> 4) * RP)[tid & 15]);
                }
                __syncthreads();
                CKPT[j * NT + tid] = h;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 f = *reinterpret_cast<const float4 *>(DTF + s_cl * FP + 4 * q);
                    const float4 w = *reinterpret_cast<const float4 *>(DTU + s_cl * FP + 4 * q);
                    const float4 bb = *reinterpret_cast<const float4 *>(BF + s_n * FP + 4 * q);
                    h = fmaf(ex2(f.x * A2), h, w.x * bb.x);
                    h = fmaf(ex2(f.y * A2), h, w.y * bb.y);
                    h = fmaf(ex2(f.z * A2), h, w.z * bb.z);
                    h = fmaf(ex2(f.w * A2), h, w.w * bb.w);
                }
            }
            __syncthreads();

            // ---------------- reverse pass over the chunk's tiles ----------------------------------
            float carry = (k < p.n_chunks - 1 && s_vch) ? p.ws_dh[s_row * NSP + s_n] : 0.f;
            float dA_acc = 0.f, dD_part = 0.f, db_part = 0.f;
            stage(0, ntile - 1, true);
            cp_async_commit();
            for (int it = 0; it < ntile; ++it) {
                const int j = ntile - 1 - it;
                const int64_t t0 = kt0 + (int64_t)j * SEG;
                const int tv = (int)min((int64_t)SEG, L - t0);
                if (j > 0) {
                    stage((it + 1) & 1, j - 1, true);
                    cp_async_commit();
                    cp_async_wait<1>();
                } else {
                    cp_async_wait<0>();
                }
                __syncthreads();
                char *rb = smem + (it & 1) * Ly::BUF;
                // -- prologue: one thread per (t, channel) element
                const bool vt = e_t < tv;
                const float uf = elem(rb, Ly::U_OFF);
                const float dtv = elem(rb, Ly::DT_OFF) + bias;
                float dtf = p.softplus ? softplus20(dtv) : dtv;
                const float dgate = (p.softplus && dtv <= 20.f) ? sigmoidf_(dtv) : 1.f;
                dtf = vt ? dtf : 0.f;
                const float dout = vt ? elem(rb, Ly::DO_OFF) : 0.f;
                float doutg = dout, dzv = 0.f, outz = 0.f;
                if constexpr (HAS_Z) {
                    const float zv = elem(rb, Ly::Z_OFF);
                    const float ov = elem(rb, Ly::OUT_OFF);
                    const float sz = sigmoidf_(zv);
                    const float silu = zv * sz;
                    doutg = dout * silu;
                    dzv = dout * ov * sz * (1.f + zv * (1.f - sz));
                    outz = ov * silu;
                }
                DTF[e_cl * FP + e_t] = dtf;
                DTU[e_cl * FP + e_t] = dtf * uf;
                DOG[e_cl * FP + e_t] = doutg;
                BF[(tid >> 4) * FP + (tid & 15)] =
                    to_f<T>(reinterpret_cast<const T *>(rb + Ly::B_OFF + (tid >> 4) * RP)[tid & 15]);
                CF[(tid >> 4) * FP + (tid & 15)] =
                    to_f<T>(reinterpret_cast<const T *>(rb + Ly::C_OFF + (tid >> 4) * RP)[tid & 15]);
                __syncthreads();

                // -- state threads: recompute the tile forward, then the reverse recurrence
                float a[SEG], hs[SEG];
                {
                    float hh = CKPT[j * NT + tid];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 f = *reinterpret_cast<const float4 *>(DTF + s_cl * FP + 4 * q);
                        const float4 w = *reinterpret_cast<const float4 *>(DTU + s_cl * FP + 4 * q);
                        const float4 bb = *reinterpret_cast<const float4 *>(BF + s_n * FP + 4 * q);
                        const float fv[4] = {f.x, f.y, f.z, f.w}, wv[4] = {w.x, w.y, w.z, w.w};
                        const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            a[4 * q + i] = ex2(fv[i] * A2);
                            hh = fmaf(a[4 * q + i], hh, wv[i] * bv[i]);
                            hs[4 * q + i] = hh;
                        }
                    }
                }
                float dBv[SEG], dCv[SEG];
#pragma unroll
                for (int q = 3; q >= 0; --q) {
                    const float4 f = *reinterpret_cast<const float4 *>(DTF + s_cl * FP + 4 * q);
                    const float4 w = *reinterpret_cast<const float4 *>(DTU + s_cl * FP + 4 * q);
                    const float4 o = *reinterpret_cast<const float4 *>(DOG + s_cl * FP + 4 * q);
                    const float4 bb = *reinterpret_cast<const float4 *>(BF + s_n * FP + 4 * q);
                    const float4 cc = *reinterpret_cast<const float4 *>(CF + s_n * FP + 4 * q);
                    const float fv[4] = {f.x, f.y, f.z, f.w}, wv[4] = {w.x, w.y, w.z, w.w};
                    const float ov[4] = {o.x, o.y, o.z, o.w}, bv[4] = {bb.x, bb.y, bb.z, bb.w};
                    const float cv[4] = {cc.x, cc.y, cc.z, cc.w};
#pragma unroll
                    for (int i = 3; i >= 0; --i) {
                        const int t = 4 * q + i;
                        const float dh = fmaf(ov[i], cv[i], carry);
                        carry = a[t] * dh;
                        const float pv = fmaf(-wv[i], bv[i], hs[t]);  // a_t * h_{t-1}
                        const float gv = dh * pv;
                        dA_acc = fmaf(fv[i], gv, dA_acc);
                        *reinterpret_cast<float2 *>(XCH + (t * 16 + s_cl) * XP + 2 * s_n) =
                            make_float2(dh * bv[i], An * gv);
                        dBv[t] = dh * wv[i];
                        dCv[t] = ov[i] * hs[t];
                    }
                }
                __syncthreads();

                // -- epilogue: element threads reduce (S1, S2) over states and form du, ddelta
                {
                    const float4 *xr = reinterpret_cast<const float4 *>(XCH + (e_t * 16 + e_cl) * XP);
                    float S1 = 0.f, S2 = 0.f;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 v = xr[q];
                        S1 += v.x + v.z;
                        S2 += v.y + v.w;
                    }
                    const float du = fmaf(dtf, S1, Dv * doutg);
                    const float ddelta = fmaf(uf, S1, S2) * dgate;
                    if (vt && e_vch) {
                        dD_part = fmaf(doutg, uf, dD_part);
                        db_part += ddelta;
                    }
                    reinterpret_cast<T *>(rb + Ly::U_OFF + e_cl * RP)[e_t] = from_f<T>(du);
                    reinterpret_cast<T *>(rb + Ly::DT_OFF + e_cl * RP)[e_t] = from_f<T>(ddelta);
                    if constexpr (HAS_Z) {
                        reinterpret_cast<T *>(rb + Ly::Z_OFF + e_cl * RP)[e_t] = from_f<T>(dzv);
                        reinterpret_cast<T *>(rb + Ly::OUT_OFF + e_cl * RP)[e_t] = from_f<T>(outz);
                    }
                }
                __syncthreads();

                // -- dB / dC: sum the warp's two channels, then park per-warp partials
#pragma unroll
                for (int t = 0; t < SEG; ++t) {
                    dBv[t] += __shfl_xor_sync(0xffffffffu, dBv[t], 16);
                    dCv[t] += __shfl_xor_sync(0xffffffffu, dCv[t], 16);
                }
                if ((s_cl & 1) == 0) {
                    float *rbB = XCH + ((s_cl >> 1) * 2 + 0) * 256 + s_n * 16;
                    float *rbC = XCH + ((s_cl >> 1) * 2 + 1) * 256 + s_n * 16;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        reinterpret_cast<float4 *>(rbB)[q] = make_float4(dBv[4 * q], dBv[4 * q + 1], dBv[4 * q + 2], dBv[4 * q + 3]);
                        reinterpret_cast<float4 *>(rbC)[q] = make_float4(dCv[4 * q], dCv[4 * q + 1], dCv[4 * q + 2], dCv[4 * q + 3]);
                    }
                }
                {
                    T *gdu = reinterpret_cast<T *>(p.du) + (int64_t)b * p.du_bs + (int64_t)c0 * p.du_ds;
                    T *gdd = reinterpret_cast<T *>(p.ddelta) + (int64_t)b * p.ddelta_bs + (int64_t)c0 * p.ddelta_ds;
                    store_tile<T, SEG>(gdu, p.du_ds, rb + Ly::U_OFF, RP, nvalid, t0, tv, aligned, tid, NT);
                    store_tile<T, SEG>(gdd, p.ddelta_ds, rb + Ly::DT_OFF, RP, nvalid, t0, tv, aligned, tid, NT);
                    if constexpr (HAS_Z) {
                        T *gdz = reinterpret_cast<T *>(p.dz) + (int64_t)b * p.dz_bs + (int64_t)c0 * p.dz_ds;
                        store_tile<T, SEG>(gdz, p.dz_ds, rb + Ly::Z_OFF, RP, nvalid, t0, tv, aligned, tid, NT);
                        if (p.recompute_out_z) {
                            T *goz = reinterpret_cast<T *>(p.out_z) + (int64_t)b * p.out_z_bs + (int64_t)c0 * p.out_z_ds;
                            store_tile<T, SEG>(goz, p.out_z_ds, rb + Ly::OUT_OFF, RP, nvalid, t0, tv, aligned, tid, NT);
                        }
                    }
                }
                __syncthreads();
                {   // thread (n, t): sum the 8 warps' partials into the chunk accumulator
                    const int rn = tid >> 4, rt = tid & 15;
                    float sb = 0.f, sc = 0.f;
#pragma unroll
                    for (int w = 0; w < 8; ++w) {
                        sb += XCH[(w * 2 + 0) * 256 + rn * 16 + rt];
                        sc += XCH[(w * 2 + 1) * 256 + rn * 16 + rt];
                    }
                    ACC[rn * kChunkLen + j * SEG + rt] += sb;
                    ACC[16 * kChunkLen + rn * kChunkLen + j * SEG + rt] += sc;
                }
            }
            // -- end of the (chunk, channel group) pass
            if (s_vch) {
                p.ws_dh[s_row * NSP + s_n] = carry;
                if (s_vst) atomicAdd(p.dA + (int64_t)s_d * p.dstate + s_n, dA_acc);
            }
            PB[e_t * 16 + e_cl] = dD_part;
            PB[256 + e_t * 16 + e_cl] = db_part;
            __syncthreads();
            if (tid < 32) {
                const int q = tid >> 4, cl = tid & 15;
                float sum = 0.f;
#pragma unroll
                for (int t = 0; t < 16; ++t) sum += PB[q * 256 + t * 16 + cl];
                if (cl < nvalid) {
                    float *dst = q == 0 ? p.dD : p.ddelta_bias;
                    if (dst) atomicAdd(dst + c0 + cl, sum);
                }
            }
            __syncthreads();
        }
        // -- flush the chunk's dB / dC (summed over this CTA's channels) to global
        for (int i = tid; i < 2 * 16 * (kChunkLen / 4); i += NT) {
            const int q = i / (16 * (kChunkLen / 4));
            const int rem = i - q * 16 * (kChunkLen / 4);
            const int n = rem / (kChunkLen / 4), t4 = (rem - n * (kChunkLen / 4)) * 4;
            float *src = ACC + q * 16 * kChunkLen + n * kChunkLen + t4;
            if (n < p.dstate && t4 < clen) {
                float *dst = (q == 0 ? p.acc_dB : p.acc_dC) +
                             (((int64_t)b * p.n_groups + g) * p.dstate + n) * p.lpitch + kt0 + t4;
                red_add_v4(dst, src[0], src[1], src[2], src[3]);
            }
            src[0] = 0.f; src[1] = 0.f; src[2] = 0.f; src[3] = 0.f;
        }
        __syncthreads();
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
    using Ly = BwdLayout<T, HAS_Z>;
    auto kern = ss_bwd_kernel<T, HAS_Z>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Ly::SMEM);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    dim3 grid(p.tiles_per_group * p.n_groups, p.batch);
    kern<<<grid, bwd::NT, Ly::SMEM, st>>>(p);
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
