// Selective-scan forward for sm_100a.
//
// Computes, for every (batch b, channel d) row and every timestep t (reference
// semantics: selective_scan_fwd_kernel.cuh:301-544, selective_scan_interface.py:353-451):
//   dt_t  = softplus(delta_t + delta_bias_d)                (or delta_t + bias without softplus)
//   h_t   = exp(dt_t * A_dn) * h_{t-1} + dt_t * u_t * B_nt   for n < dstate
//   out_t = sum_n C_nt h_t[n] + D_d u_t                     (stored in the input dtype)
//   out_z = out_t * silu(z_t)                               (when z is given)
// and, at the end of every kChunkLen-step chunk, x = (prod_t exp(dt_t A_dn), h[n]).
//
// Design (B200): one thread owns one (b, d) row and keeps all of its dstate fp32 states
// in registers, so the recurrence needs no cross-thread scan and y = <C, h> is an
// in-thread FMA chain.  A CTA owns CH consecutive channels of one (batch, group); tiles
// of TT timesteps of u / delta / z (rows of the CTA's channels) and of B / C (rows of the
// group's states, shared by all CH channels) are staged into shared memory with 16-byte
// cp.async into a single buffer (six co-resident CTAs per SM hide each other's load
// latency; the small footprint is what lets config 4 run as one wave).  The states are
// updated in pairs with Blackwell's packed fma/mul.f32x2.  B/C are converted to fp32 once per tile into a [t][n] layout that every
// thread reads with broadcast 16-byte loads.  Outputs are written in place into the
// staged u / z rows and leave through coalesced 16-byte stores.
//
// When batch * dim is too small to fill 148 SMs, the sequence is split into up to 128
// segments (whole 16-step tiles): a carry pass computes each segment's end state from zero
// and its summed dt, a pass over segments (seg_carry_scan_kernel) composes them into
// every segment's initial state (h_in = prod(decay) * h_in + H), and the main pass runs the
// full scan of each segment from its initial state.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace mss {

int fwd_state_pad(int dstate) {
    if (dstate <= 4) return 4;
    if (dstate <= 8) return 8;
    if (dstate <= 16) return 16;
    if (dstate <= 32) return 32;
    if (dstate <= 64) return 64;
    if (dstate <= 128) return 128;
    return 256;
}

template <int NS, int SPT> struct FwdCfg {
    // SPT states per thread: a row with more states than that is split over LPC adjacent
    // lanes, and y = <C, h> is summed over the row's lanes by shuffles.  Splitting multiplies
    // the per-step work that does not depend on the state (dt, softplus, the decay base) by
    // LPC, so it pays only when rows are few: dstate 32 / 64 runs whole rows per thread when
    // there are at least a wave of them and halves otherwise (fwd_spt).
    static_assert(NS % SPT == 0, "whole lanes per row");
    static constexpr int LPC = NS / SPT;  // threads (lanes) per row
    // threads per CTA: for dstate <= 16, 96 x 8 resident CTAs per SM; at config 4 the 1024
    // CTAs spread as 6 or 7 per SM (128-channel CTAs would leave 5 or 6, the SMs with 6
    // setting the pace at 86 % of the mean load)
    static constexpr int NT = NS <= 16 ? 96 : 128;
    static constexpr int CH = NT / LPC;   // channels (rows) per CTA
    static constexpr int TT = 16;         // timesteps per staged tile
    // resident CTAs per SM: registers per thread grow with SPT (~80 at 16, ~170 at 32 split
    // in two, ~250 for 32 or 64 states in one thread)
    static constexpr int MINB = NS <= 16 ? 8 : (SPT == 16 ? 4 : (LPC == 1 ? 2 : 3));
};

// Resident rows per SM of the variant fwd_spt picks (sizes the time split).  dstate 128 / 256
// rows run 8 / 16 lanes of 16 states, 3 CTAs per SM (shared memory: the fp32 B / C tile).
static int rows_per_sm(int ns, int spt) {
    if (ns <= 16) return 768;
    const int lpc = ns / spt, minb = ns > 64 ? 3 : (spt == 16 ? 4 : (lpc == 1 ? 2 : 3));
    return minb * 128 / lpc;
}

int fwd_spt(int ns, int64_t rows) {
    if (ns <= 16) return ns;
    if (ns > 64) return 16;         // 8 or 16 lanes of 16 states per row
    const int whole = ns;           // one thread per row
    const int half = ns / 2;        // two threads per row
    return rows >= (int64_t)kNumSMs * rows_per_sm(ns, whole) ? whole : half;
}

int fwd_rows_per_sm(int dstate, int64_t rows) {
    const int ns = fwd_state_pad(dstate);
    return rows_per_sm(ns, fwd_spt(ns, rows));
}

template <typename T, int NS, int SPT, bool HAS_Z, bool CARRY>
struct FwdLayout {
    static constexpr int CH = FwdCfg<NS, SPT>::CH;
    static constexpr int NT = FwdCfg<NS, SPT>::NT;
    static constexpr int TT = FwdCfg<NS, SPT>::TT;
    static constexpr int RP = TT * (int)sizeof(T) + 16;  // padded row pitch (conflict-free 16-B reads)
    static constexpr int NCH_ARR = CARRY ? 2 : (HAS_Z ? 3 : 2);  // u, delta, (z)
    static constexpr int NST_ARR = CARRY ? 1 : 2;                // B, (C)
    static constexpr int NROWS = CH * NCH_ARR + NS * NST_ARR;
    static constexpr int BUF = NROWS * RP;
    static constexpr int BCW = NS * NST_ARR;  // floats per timestep in the fp32 B/C tile
    static constexpr int U_OFF = 0, DT_OFF = CH * RP, Z_OFF = 2 * CH * RP;
    static constexpr int B_OFF = CH * NCH_ARR * RP, C_OFF = B_OFF + NS * RP;
    static constexpr int SMEM = BUF + TT * BCW * 4;  // single-buffered: co-resident CTAs hide the loads
};

template <typename T, int NS, int SPT, bool HAS_Z, bool CARRY>
__global__ void __launch_bounds__(FwdCfg<NS, SPT>::NT, FwdCfg<NS, SPT>::MINB) ss_fwd_kernel(const FwdParams p) {
    using Ly = FwdLayout<T, NS, SPT, HAS_Z, CARRY>;
    constexpr int CH = Ly::CH, NT = Ly::NT, TT = Ly::TT, RP = Ly::RP, BCW = Ly::BCW;
    constexpr int LPC = FwdCfg<NS, SPT>::LPC;
    extern __shared__ __align__(16) char smem[];
    float *bc = reinterpret_cast<float *>(smem + Ly::BUF);

    const int tid = threadIdx.x;
    const int ch = tid / LPC;                  // this thread's row within the CTA
    const int n0 = (tid - ch * LPC) * SPT;     // and its first state
    const int g = blockIdx.x / p.tiles_per_group;
    const int tile = blockIdx.x - g * p.tiles_per_group;
    const int s = blockIdx.y;
    const int b = blockIdx.z;
    const int cg0 = tile * CH;                 // first channel of this CTA within its group
    const int c0 = g * p.dpg + cg0;            // first channel overall
    const int nvalid_ch = min(CH, p.dpg - cg0);
    const bool valid = ch < nvalid_ch;
    const int d = c0 + (valid ? ch : 0);
    const int64_t L = p.seqlen;
    const int64_t t_begin = (int64_t)s * p.seg_len;
    const int64_t t_end = min(L, t_begin + (int64_t)p.seg_len);
    const bool aligned = p.aligned != 0;

    float A2[SPT];  // rates of states n0 .. n0 + SPT - 1 (times log2 e)
#pragma unroll
    for (int j = 0; j < SPT; ++j)
        A2[j] = (valid && n0 + j < p.dstate) ? p.A[(int64_t)d * p.A_ds + (int64_t)(n0 + j) * p.A_ns] * kLog2e : 0.f;
    const float A2r = LPC == 1 ? A2[0] : (valid ? p.A[(int64_t)d * p.A_ds] * kLog2e : 0.f);  // state 0's rate
    const float Dv = (p.D != nullptr && valid) ? p.D[(int64_t)d * p.D_s] : 0.f;
    const float bias = (p.delta_bias != nullptr && valid) ? p.delta_bias[(int64_t)d * p.delta_bias_s] : 0.f;

    // State and decay rates as packed pairs (states 2m, 2m+1).
    constexpr int NP = SPT / 2;
    f32x2 h2[NP], A2p[NP];
#pragma unroll
    for (int m = 0; m < NP; ++m) {
        h2[m] = pack2(0.f, 0.f);
        A2p[m] = pack2(A2[2 * m], A2[2 * m + 1]);
    }
    // S4D-real structure A[d, n] = (n + 1) A[d, 0] (the module's init, and every BASELINE
    // config): then exp(dt A_n) = r^(n+1) with r = exp(dt A_0), one SFU ex2 per step instead
    // of one per state.  Checked per channel to 1e-6 relative (the -exp(log(n+1)) round trip
    // of the module's A_log deviates by < 2e-7); a CTA takes the chained path only if all its
    // channels qualify, otherwise every state gets its own ex2.
    bool chain_ok = A2r != 0.f || !valid;
#pragma unroll
    for (int j = 0; j < SPT; ++j)
        if (n0 + j > 0 && n0 + j < p.dstate)
            chain_ok = chain_ok && fabsf(A2[j] - (float)(n0 + j + 1) * A2r) <= 1e-6f * fabsf(A2[j]);
    const bool chain = __syncthreads_and(chain_ok) != 0;
    float cum = 0.f;  // sum of dt since t = 0 (main pass) or since the segment start (carry pass)
    const int64_t row = (int64_t)b * p.dim + d;
    if (!CARRY && s > 0 && valid) {
        // initial state of this segment and the summed dt before it, left in the workspace by
        // seg_carry_scan_kernel (the carries of the earlier segments composed in order)
        const float *H = p.ws_h + (row * p.n_seg + s) * NS + n0;
#pragma unroll
        for (int m = 0; m < NP; ++m) h2[m] = pack2(H[2 * m], H[2 * m + 1]);
        cum = p.ws_dts[(int64_t)p.batch * p.dim * p.n_seg + row * p.n_seg + s];
    } else if (!CARRY && p.h0 != nullptr && valid) {  // the caller's state before the first step
        const float *H = p.h0 + row * p.dstate + n0;
#pragma unroll
        for (int m = 0; m < NP; ++m)
            h2[m] = pack2(n0 + 2 * m < p.dstate ? H[2 * m] : 0.f, n0 + 2 * m + 1 < p.dstate ? H[2 * m + 1] : 0.f);
    }

    const T *gu = reinterpret_cast<const T *>(p.u) + (int64_t)b * p.u_bs + (int64_t)c0 * p.u_ds;
    const T *gdt = reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs + (int64_t)c0 * p.delta_ds;
    const T *gz = HAS_Z ? reinterpret_cast<const T *>(p.z) + (int64_t)b * p.z_bs + (int64_t)c0 * p.z_ds : nullptr;
    const T *gB = reinterpret_cast<const T *>(p.B) + (int64_t)b * p.B_bs + (int64_t)g * p.B_gs;
    const T *gC = reinterpret_cast<const T *>(p.C) + (int64_t)b * p.C_bs + (int64_t)g * p.C_gs;

    auto stage = [&](int buf, int64_t t0) {
        char *rb = smem + buf * Ly::BUF;
        const int tv = (int)min((int64_t)TT, t_end - t0);
        stage_tile<T, TT>(rb + Ly::U_OFF, RP, gu, p.u_ds, CH, nvalid_ch, t0, tv, aligned, tid, NT);
        stage_tile<T, TT>(rb + Ly::DT_OFF, RP, gdt, p.delta_ds, CH, nvalid_ch, t0, tv, aligned, tid, NT);
        if constexpr (HAS_Z && !CARRY)
            stage_tile<T, TT>(rb + Ly::Z_OFF, RP, gz, p.z_ds, CH, nvalid_ch, t0, tv, aligned, tid, NT);
        stage_tile<T, TT>(rb + Ly::B_OFF, RP, gB, p.B_ns, NS, p.dstate, t0, tv, aligned, tid, NT);
        if constexpr (!CARRY)
            stage_tile<T, TT>(rb + Ly::C_OFF, RP, gC, p.C_ns, NS, p.dstate, t0, tv, aligned, tid, NT);
    };

    const int ntiles = (int)((t_end - t_begin + TT - 1) / TT);
    for (int it = 0; it < ntiles; ++it) {
        const int64_t t0 = t_begin + (int64_t)it * TT;
        const int tv = (int)min((int64_t)TT, t_end - t0);
        stage(0, t0);
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        char *rb = smem;
        // B / C tile -> fp32 [t][n] (C after B), once per CTA.
        for (int i = tid; i < TT * NS; i += NT) {
            const int n = i % NS, t = i / NS;
            bc[t * BCW + n] = to_f<T>(reinterpret_cast<const T *>(rb + Ly::B_OFF + n * RP)[t]);
            if constexpr (!CARRY)
                bc[t * BCW + NS + n] = to_f<T>(reinterpret_cast<const T *>(rb + Ly::C_OFF + n * RP)[t]);
        }
        __syncthreads();

        T *ur = reinterpret_cast<T *>(rb + Ly::U_OFF + ch * RP);
        const T *dr = reinterpret_cast<const T *>(rb + Ly::DT_OFF + ch * RP);
#pragma unroll 1
        for (int g8 = 0; g8 < TT; g8 += 8) {
            float uf[8], dv[8], dtu[8];
            Vec8<T>::load(ur + g8, uf);
            Vec8<T>::load(dr + g8, dv);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float v = dv[j] + bias;
                if (p.softplus) v = softplus20(v);
                v = (g8 + j < tv) ? v : 0.f;  // padded steps: decay 1, input 0
                dv[j] = v;
                dtu[j] = v * uf[j];
                cum += v;
            }
            float y[8];
            auto steps = [&](auto chained) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const f32x2 *bcr = reinterpret_cast<const f32x2 *>(bc + (g8 + j) * BCW + n0);  // B[n0..]
                    const f32x2 *ccr = reinterpret_cast<const f32x2 *>(bc + (g8 + j) * BCW + NS + n0);  // C[n0..]
                    const f32x2 du2 = pack2(dtu[j], dtu[j]);
                    f32x2 acc2[2] = {pack2(0.f, 0.f), pack2(0.f, 0.f)};  // two chains of pair sums
                    f32x2 ap, q;  // chained path: (r^(2m+1), r^(2m+2)) and the step (r^2, r^2)
                    if constexpr (decltype(chained)::value) {
                        const float r = ex2(dv[j] * A2r);
                        const float r2 = r * r;
                        const float rs = LPC == 1 ? r : ex2(dv[j] * A2[0]);  // r^(n0 + 1)
                        ap = pack2(rs, rs * r);
                        q = pack2(r2, r2);
                    }
                    const f32x2 dt2 = pack2(dv[j], dv[j]);
#pragma unroll
                    for (int m = 0; m < NP; ++m) {
                        f32x2 a2;
                        if constexpr (decltype(chained)::value) {
                            if (m > 0) ap = mul2(ap, q);
                            a2 = ap;
                        } else {
                            a2 = ex2x2(mul2(dt2, A2p[m]));
                        }
                        h2[m] = fma2(a2, h2[m], mul2(du2, bcr[m]));
                        if constexpr (!CARRY) acc2[m & 1] = fma2(ccr[m], h2[m], acc2[m & 1]);
                    }
                    const float2 accv = unpack2(add2(acc2[0], acc2[1]));
                    y[j] = accv.x + accv.y;
                }
            };
            if (chain)
                steps(std::true_type{});
            else
                steps(std::false_type{});
            if constexpr (!CARRY) {
                if constexpr (LPC > 1) {  // sum the row's lanes (adjacent lanes of one warp)
#pragma unroll
                    for (int o = 1; o < LPC; o <<= 1)
#pragma unroll
                        for (int j = 0; j < 8; ++j) y[j] += __shfl_xor_sync(0xffffffffu, y[j], o);
                }
                float o[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) o[j] = fmaf(Dv, uf[j], y[j]);
                if (LPC == 1 || n0 == 0) Vec8<T>::store(ur + g8, o);  // out, in place of u
                if constexpr (HAS_Z) {
                    if (LPC == 1 || n0 == 0) {
                        T *zr = reinterpret_cast<T *>(rb + Ly::Z_OFF + ch * RP);
                        float zf[8];
                        Vec8<T>::load(zr + g8, zf);
#pragma unroll
                        for (int j = 0; j < 8; ++j) zf[j] = o[j] * zf[j] * sigmoidf_(zf[j]);
                        Vec8<T>::store(zr + g8, zf);  // out_z, in place of z
                    }
                }
            }
        }
        if constexpr (!CARRY) {
            const int64_t te = t0 + tv;
            if (valid && (te % kChunkLen == 0 || te == L)) {
                const int64_t k = (te - 1) / kChunkLen;
                float *xr = p.x + (row * p.n_chunks + k) * 2 * p.dstate;
#pragma unroll
                for (int j = 0; j < SPT; ++j)
                    if (n0 + j < p.dstate) {
                        xr[2 * (n0 + j)] = ex2(A2[j] * cum);
                        const float2 hv = unpack2(h2[j >> 1]);
                        xr[2 * (n0 + j) + 1] = (j & 1) ? hv.y : hv.x;
                    }
            }
            __syncthreads();
            T *go = reinterpret_cast<T *>(p.out) + (int64_t)b * p.out_bs + (int64_t)c0 * p.out_ds;
            store_tile<T, TT>(go, p.out_ds, rb + Ly::U_OFF, RP, nvalid_ch, t0, tv, aligned, tid, NT);
            if constexpr (HAS_Z) {
                T *goz = reinterpret_cast<T *>(p.out_z) + (int64_t)b * p.out_z_bs + (int64_t)c0 * p.out_z_ds;
                store_tile<T, TT>(goz, p.out_z_ds, rb + Ly::Z_OFF, RP, nvalid_ch, t0, tv, aligned, tid, NT);
            }
        }
        __syncthreads();
    }
    if (CARRY && valid) {
        float *H = p.ws_h + (row * p.n_seg + s) * NS + n0;
#pragma unroll
        for (int m = 0; m < NP; ++m) {
            const float2 hv = unpack2(h2[m]);
            H[2 * m] = hv.x;
            H[2 * m + 1] = hv.y;
        }
        if (n0 == 0) p.ws_dts[row * p.n_seg + s] = cum;
    }
}

// Turns the per-segment carries into per-segment initial states.  On entry, for every row and
// segment s < n_seg - 1, ws_h[row][s][n] holds H_s[n], the state at the end of segment s started
// from zero, and ws_dts[row][s] the summed dt over it; segment s's decay of state n is
// exp(A_n * dts_s).  On exit, slot s + 1 of ws_h holds the state at the start of segment s + 1
// (the composition h = exp(A_n dts_s) h + H_s over segments 0..s, applied to the caller's
// initial state h0 when there is one), and slot s + 1 of the second half of ws_dts (offset
// rows * n_seg) the summed dt before segment s + 1; the raw sums stay untouched, because every
// thread of a row reads them while its state-0 thread writes the composed sums.
// One thread per (row, state), consecutive threads on consecutive states (coalesced rows of
// ws_h), walking the segments in order: the dependency between segments is one FMA.  The
// carries of kSegBatch segments are loaded together and the next batch's loads are issued
// before the current batch is composed, so the kernel costs about one memory latency per
// batch (kSegBatch = 4 when there are at most 4 carries: fewer registers, more resident
// threads).  A thread reads slot s + 1 of ws_h (segment s + 1's carry) before it overwrites
// that slot with segment s + 1's initial state.
template <int kSegBatch>
__global__ void __launch_bounds__(256) seg_carry_scan_kernel(float *__restrict__ ws_h, float *__restrict__ ws_dts,
                                                             const float *__restrict__ A, int64_t A_ds, int64_t A_ns,
                                                             int64_t rows, int dim, int dstate, int ns, int n_seg,
                                                             const float *__restrict__ h0) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (tid >= rows * ns) return;
    const int64_t row = tid / ns;
    const int n = (int)(tid - row * ns);
    const int d = (int)(row % dim);
    const float a2 = n < dstate ? A[(int64_t)d * A_ds + (int64_t)n * A_ns] * kLog2e : 0.f;
    float h = (h0 != nullptr && n < dstate) ? h0[row * dstate + n] : 0.f;
    float cum = 0.f;
    const int ncarry = n_seg - 1;
    float *H = ws_h + row * n_seg * ns + n;           // slot s at H[s * ns]
    const float *S = ws_dts + row * n_seg;            // raw sums
    float *Sc = ws_dts + rows * n_seg + row * n_seg;  // composed sums
    float hk[kSegBatch], sk[kSegBatch], hn[kSegBatch] = {}, sn[kSegBatch] = {};
    auto load = [&](int s0, float (&hv)[kSegBatch], float (&sv)[kSegBatch]) {
#pragma unroll
        for (int k = 0; k < kSegBatch; ++k) {
            const bool live = s0 + k < ncarry;
            hv[k] = live ? H[(int64_t)(s0 + k) * ns] : 0.f;
            sv[k] = live ? S[s0 + k] : 0.f;
        }
    };
    load(0, hk, sk);
    for (int s0 = 0; s0 < ncarry; s0 += kSegBatch) {
        // the next batch's carries (slot s0 + kSegBatch included) before any store of this batch
        if (s0 + kSegBatch < ncarry) load(s0 + kSegBatch, hn, sn);
#pragma unroll
        for (int k = 0; k < kSegBatch; ++k) {
            if (s0 + k < ncarry) {
                h = fmaf(ex2(a2 * sk[k]), h, hk[k]);
                cum += sk[k];
                H[(int64_t)(s0 + k + 1) * ns] = h;
                if (n == 0) Sc[s0 + k + 1] = cum;
            }
        }
#pragma unroll
        for (int k = 0; k < kSegBatch; ++k) {
            hk[k] = hn[k];
            sk[k] = sn[k];
        }
    }
}

template <typename T, int NS, int SPT, bool HAS_Z, bool CARRY>
static cudaError_t launch_one(const FwdParams &p, dim3 grid, cudaStream_t st) {
    using Ly = FwdLayout<T, NS, SPT, HAS_Z, CARRY>;
    auto kern = ss_fwd_kernel<T, NS, SPT, HAS_Z, CARRY>;
    static std::atomic<unsigned long long> smem_set{0};
    {
        const cudaError_t e = set_smem_once(smem_set, reinterpret_cast<const void *>(kern), Ly::SMEM);
        if (e != cudaSuccess) return e;
    }
    kern<<<grid, Ly::NT, Ly::SMEM, st>>>(p);
    return cudaGetLastError();
}

template <typename T, int NS, int SPT>
static cudaError_t launch_spt(FwdParams p, bool has_z, cudaStream_t st) {
    constexpr int CH = FwdCfg<NS, SPT>::CH;
    p.tiles_per_group = (p.dpg + CH - 1) / CH;
    dim3 grid(p.tiles_per_group * p.n_groups, p.n_seg, p.batch);
    cudaError_t e = cudaSuccess;
    if (p.n_seg > 1) {
        dim3 gc(grid.x, p.n_seg - 1, grid.z);
        e = launch_one<T, NS, SPT, false, true>(p, gc, st);
        if (e != cudaSuccess) return e;
        const int64_t threads = (int64_t)p.batch * p.dim * NS;
        const unsigned nb = (unsigned)((threads + 255) / 256);
        if (p.n_seg - 1 <= 4)
            seg_carry_scan_kernel<4><<<nb, 256, 0, st>>>(p.ws_h, p.ws_dts, p.A, p.A_ds, p.A_ns,
                                                        (int64_t)p.batch * p.dim, p.dim, p.dstate, NS, p.n_seg, p.h0);
        else
            seg_carry_scan_kernel<16><<<nb, 256, 0, st>>>(p.ws_h, p.ws_dts, p.A, p.A_ds, p.A_ns,
                                                         (int64_t)p.batch * p.dim, p.dim, p.dstate, NS, p.n_seg, p.h0);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    if (has_z) return launch_one<T, NS, SPT, true, false>(p, grid, st);
    return launch_one<T, NS, SPT, false, false>(p, grid, st);
}

template <typename T, int NS>
static cudaError_t launch_ns(const FwdParams &p, bool has_z, cudaStream_t st) {
    if constexpr (NS <= 16) {
        return launch_spt<T, NS, NS>(p, has_z, st);
    } else if constexpr (NS > 64) {
        return launch_spt<T, NS, 16>(p, has_z, st);
    } else {
        if (fwd_spt(NS, (int64_t)p.batch * p.dim) == NS) return launch_spt<T, NS, NS>(p, has_z, st);
        return launch_spt<T, NS, NS / 2>(p, has_z, st);
    }
}


template <typename T>
static cudaError_t launch_t(const FwdParams &p, bool has_z, cudaStream_t st) {
    switch (fwd_state_pad(p.dstate)) {
        case 4: return launch_ns<T, 4>(p, has_z, st);
        case 8: return launch_ns<T, 8>(p, has_z, st);
        case 16: return launch_ns<T, 16>(p, has_z, st);
        case 32: return launch_ns<T, 32>(p, has_z, st);
        case 64: return launch_ns<T, 64>(p, has_z, st);
        case 128: return launch_ns<T, 128>(p, has_z, st);
        default: return launch_ns<T, 256>(p, has_z, st);
    }
}

cudaError_t launch_ss_fwd(const FwdParams &p, int itype, bool has_z, cudaStream_t st) {
    switch (itype) {
        case MSS_F32: return launch_t<float>(p, has_z, st);
        case MSS_F16: return launch_t<__half>(p, has_z, st);
        default: return launch_t<__nv_bfloat16>(p, has_z, st);
    }
}

}  // namespace mss
