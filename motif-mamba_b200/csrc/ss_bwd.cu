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
#include <type_traits>

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
// 16-bit inputs keep B / C in their own type here (converted when read: measured 0.7 % faster
// than fp32 staging, whose doubled shared-memory reads raise the short-scoreboard stalls more
// than the saved conversions gain), which also leaves room for the per-warp prefetch buffers
// of the next pass's per-step inputs.
template <typename T> struct BwdSmemT {
    static constexpr bool kPrefetch = sizeof(T) == 2;
    using BCT = typename std::conditional<kPrefetch, T, float>::type;
    BCT BC[2][bwd::NS][bwd::CK];              // B, C of the chunk
    float ACC[2][bwd::NS][bwd::CK];           // chunk accumulator of dB / dC
    float DHC[bwd::KMAX][bwd::W][bwd::NS];    // reverse-recurrence carry into the previous chunk
    float DAACC[bwd::KMAX][bwd::W][bwd::NS];  // dA accumulators
    float PBD[bwd::KMAX][bwd::W][2];          // dD, ddelta_bias accumulators
    float AX[bwd::W][2][bwd::NS];             // this pass's A row and chunk-start states, per warp
    float AXP[2][bwd::W][3 * bwd::NS];        // prefetched A row and raw x pairs, by pass parity
    T PF[kPrefetch ? bwd::W : 1][5][bwd::CK]; // next pass's u, delta, dout, z, out (lane slices)
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
// One Kogge-Stone level of the warp scans of (decay, value) pairs, with the shuffle's own
// in-range predicate guarding the combine (predicated instructions instead of compare + select):
// up:   lanes >= off combine with lane - off:  H = A H' + H, A = A A'   (forward states)
// down: lanes < 32 - off combine with lane + off: Q = P Q' + Q, P = P P' (reverse adjoints)
__device__ __forceinline__ void scan_up_level(float &A, float &H, int off) {
    asm("{\n\t.reg .pred p;\n\t.reg .f32 ap, hp;\n\t"
        "shfl.sync.up.b32 ap|p, %0, %2, 0, 0xffffffff;\n\t"
        "shfl.sync.up.b32 hp, %1, %2, 0, 0xffffffff;\n\t"
        "@p fma.rn.f32 %1, %0, hp, %1;\n\t"
        "@p mul.rn.f32 %0, %0, ap;\n\t}"
        : "+f"(A), "+f"(H) : "r"(off));
}
__device__ __forceinline__ void scan_down_level(float &P, float &Q, int off) {
    asm("{\n\t.reg .pred p;\n\t.reg .f32 pr, qr;\n\t"
        "shfl.sync.down.b32 pr|p, %0, %2, 31, 0xffffffff;\n\t"
        "shfl.sync.down.b32 qr, %1, %2, 31, 0xffffffff;\n\t"
        "@p fma.rn.f32 %1, %0, qr, %1;\n\t"
        "@p mul.rn.f32 %0, %0, pr;\n\t}"
        : "+f"(P), "+f"(Q) : "r"(off));
}

template <typename T> __device__ __forceinline__ void bc_ld8(const T *base, int lane, float (&v)[8]) {
    // 16-bit layout: 4 values at [4 lane, 4 lane + 4) and 4 at [128 + 4 lane, ...)
    const uint2 a = *reinterpret_cast<const uint2 *>(base + lane * 4);
    const uint2 c = *reinterpret_cast<const uint2 *>(base + 128 + lane * 4);
    const T *pa = reinterpret_cast<const T *>(&a), *pc = reinterpret_cast<const T *>(&c);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[j] = to_f<T>(pa[j]);
        v[4 + j] = to_f<T>(pc[j]);
    }
}
template <> __device__ __forceinline__ void bc_ld8<float>(const float *base, int lane, float (&v)[8]) {
    ld8(base, lane, v);
}
template <typename T> __device__ __forceinline__ void bc_st8(T *base, int lane, const float (&v)[8]) {
    T a[4], c[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        a[j] = from_f<T>(v[j]);
        c[j] = from_f<T>(v[4 + j]);
    }
    *reinterpret_cast<uint2 *>(base + lane * 4) = *reinterpret_cast<const uint2 *>(a);
    *reinterpret_cast<uint2 *>(base + 128 + lane * 4) = *reinterpret_cast<const uint2 *>(c);
}
__device__ __forceinline__ void st8(float *base, int lane, const float (&v)[8]) {
    *reinterpret_cast<float4 *>(base + lane * 4) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4 *>(base + 128 + lane * 4) = make_float4(v[4], v[5], v[6], v[7]);
}

template <typename T, bool HAS_Z>
__global__ void __launch_bounds__(bwd::NT, 2) ss_bwd_kernel(const BwdParams p) {
    using namespace bwd;
    extern __shared__ __align__(16) char smem_raw[];
    using Smem = BwdSmemT<T>;
    Smem &S = *reinterpret_cast<Smem *>(smem_raw);
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

    // Per-step inputs of a pass: each lane copies its own 8 steps of u, delta, dout (z, out)
    // for the NEXT pass into its warp's slice of S.PF while the current pass computes.
    const bool pf = Smem::kPrefetch && vec;
    const T *arr_base[5] = {reinterpret_cast<const T *>(p.u) + (int64_t)b * p.u_bs,
                            reinterpret_cast<const T *>(p.delta) + (int64_t)b * p.delta_bs,
                            reinterpret_cast<const T *>(p.dout) + (int64_t)b * p.dout_bs,
                            HAS_Z ? reinterpret_cast<const T *>(p.z) + (int64_t)b * p.z_bs : nullptr,
                            HAS_Z ? reinterpret_cast<const T *>(p.out) + (int64_t)b * p.out_bs : nullptr};
    const int64_t arr_ds[5] = {p.u_ds, p.delta_ds, p.dout_ds, p.z_ds, p.out_ds};
    constexpr int NARR = HAS_Z ? 5 : 3;
    // The A row and the chunk-start states (16 states, dense 16-byte-aligned rows) come the
    // same way: lanes 0-3 copy A, lanes 4-11 the (decay, state) pairs of the previous chunk.
    const bool axpf = pf && p.nblk == NS && p.A_ns == 1 && (p.A_ds & 3) == 0 &&
                      (reinterpret_cast<uintptr_t>(p.A) & 15) == 0 && (p.state_lo & 1) == 0 && (p.dstate & 1) == 0;
    auto prefetch = [&](int kk, int cgg, int par) {
        const int cin = (tile * K + cgg) * W + w;
        const bool cv = cin < p.dpg;
        const int dd = g * p.dpg + (cv ? cin : 0);
        const int64_t tt = (int64_t)kk * CK + lane * IT;
        const int nb = (int)max((int64_t)0, min((int64_t)IT, L - tt)) * (int)sizeof(T);
#pragma unroll
        for (int a = 0; a < NARR; ++a) {
            const T *src = arr_base[a] + (int64_t)dd * arr_ds[a] + (nb > 0 ? tt : 0);
            cp_async16(&S.PF[Smem::kPrefetch ? w : 0][a][lane * IT], src, nb);
        }
        if (axpf && lane < 12) {
            const float *src;
            int nbx;
            if (lane < 4) {
                src = p.A + (int64_t)dd * p.A_ds + p.state_lo + 4 * lane;
                nbx = cv ? 16 : 0;
            } else {
                const int64_t rw = (int64_t)b * p.dim + dd;
                src = p.x + (rw * p.n_chunks + (kk > 0 ? kk - 1 : 0)) * 2 * p.dstate + 2 * p.state_lo + 4 * (lane - 4);
                nbx = (cv && kk > 0) ? 16 : 0;
            }
            cp_async16(&S.AXP[par][w][4 * lane], src, nbx);
        }
        cp_async_commit();
    };
    if (pf && p.n_chunks > 0) prefetch(p.n_chunks - 1, 0, 0);
    int pass = 0;

    for (int k = p.n_chunks - 1; k >= 0; --k) {
        const int64_t kt0 = (int64_t)k * CK;
        __syncthreads();  // previous chunk's accumulator flush and B/C reads are done
        // ---- stage B, C of this chunk (fp32; zero beyond dstate / seqlen)
        for (int i = tid; i < 2 * NS * 32; i += NT) {
            const int q = i / (NS * 32), rem = i - q * NS * 32, n = rem >> 5, l = rem & 31;
            float v[8];
            if (n < p.nblk) {
                const int ng = p.state_lo + n;
                const T *row = (q == 0 ? gB + (int64_t)ng * p.B_ns : gC + (int64_t)ng * p.C_ns);
                load_items(row, kt0 + l * 8, L, vec, v);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = 0.f;
            }
            if constexpr (Smem::kPrefetch) bc_st8(&S.BC[q][n][0], l, v); else st8(&S.BC[q][n][0], l, v);
        }
        __syncthreads();

        for (int cg = 0; cg < K; ++cg) {
            const int cin = (tile * K + cg) * W + w;  // channel within the group
            const bool valid = cin < p.dpg;
            const int d = g * p.dpg + (valid ? cin : 0);
            const int64_t row = (int64_t)b * p.dim + d;
            const int64_t t0 = kt0 + lane * IT;

            // ---- per-element prologue (this lane's 8 steps).  Per-step arrays are held as
            // packed pairs (steps 2m, 2m+1) so independent per-step math issues as f32x2.
            f32x2 uf2[4], dtf2[4], dtu2[4], dog2[4];
            {
                float uf[8], dv[8], dov[8], zv[8], ov[8];
                if (pf) {
                    cp_async_wait<0>();
                    const T *pw = &S.PF[Smem::kPrefetch ? w : 0][0][lane * IT];
                    Vec8<T>::load(pw, uf);
                    Vec8<T>::load(pw + CK, dv);
                    Vec8<T>::load(pw + 2 * CK, dov);
                    if constexpr (HAS_Z) {
                        Vec8<T>::load(pw + 3 * CK, zv);
                        Vec8<T>::load(pw + 4 * CK, ov);
                    }
                    __syncwarp();
                    if (cg + 1 < K) prefetch(k, cg + 1, (pass + 1) & 1);
                    else if (k > 0) prefetch(k - 1, 0, (pass + 1) & 1);
                } else {
                    load_items(arr_base[0] + (int64_t)d * p.u_ds, t0, L, vec, uf);
                    load_items(arr_base[1] + (int64_t)d * p.delta_ds, t0, L, vec, dv);
                    load_items(arr_base[2] + (int64_t)d * p.dout_ds, t0, L, vec, dov);
                    if constexpr (HAS_Z) {
                        load_items(arr_base[3] + (int64_t)d * p.z_ds, t0, L, vec, zv);
                        load_items(arr_base[4] + (int64_t)d * p.out_ds, t0, L, vec, ov);
                    }
                }
                const float bias = p.delta_bias ? p.delta_bias[(int64_t)d * p.delta_bias_s] : 0.f;
                float dtf[8], dog[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float x = dv[i] + bias;
                    if (p.softplus) x = softplus20(x);
                    dtf[i] = (valid && t0 + i < L) ? x : 0.f;
                    dog[i] = valid ? dov[i] : 0.f;
                }
                if constexpr (HAS_Z) {
                    float dzv[8], ozv[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float sz = sigmoidf_(zv[i]);
                        const float silu = zv[i] * sz;
                        dzv[i] = dog[i] * ov[i] * sz * (1.f + zv[i] * (1.f - sz));
                        ozv[i] = ov[i] * silu;
                        dog[i] *= silu;
                    }
                    if (valid && p.blk_first) {
                        store_items(reinterpret_cast<T *>(p.dz) + (int64_t)b * p.dz_bs + (int64_t)d * p.dz_ds, t0, L,
                                    vec, dzv);
                        if (p.recompute_out_z)
                            store_items(reinterpret_cast<T *>(p.out_z) + (int64_t)b * p.out_z_bs +
                                            (int64_t)d * p.out_z_ds, t0, L, vec, ozv);
                    }
                }
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    uf2[m] = pack2(uf[2 * m], uf[2 * m + 1]);
                    dtf2[m] = pack2(dtf[2 * m], dtf[2 * m + 1]);
                    dog2[m] = pack2(dog[2 * m], dog[2 * m + 1]);
                    dtu2[m] = mul2(dtf2[m], uf2[m]);
                }
            }
            float sdt;
            {
                const float2 s = unpack2(add2(add2(dtf2[0], dtf2[1]), add2(dtf2[2], dtf2[3])));
                sdt = s.x + s.y;
            }

            f32x2 S1[4], S2[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) S1[m] = S2[m] = pack2(0.f, 0.f);
            // A row and the chunk-start states of this channel, read once per pass (off the
            // per-state dependency chain)
            if (axpf) {
                if (lane < NS) {
                    S.AX[w][0][lane] = S.AXP[pass & 1][w][lane];
                    S.AX[w][1][lane] = S.AXP[pass & 1][w][NS + 2 * lane + 1];
                }
            } else if (lane < NS) {  // states >= dstate read as zero (A, state), like their zero B / C rows
                const bool st = valid && lane < p.nblk;
                const int ng = p.state_lo + lane;
                S.AX[w][0][lane] = st ? p.A[(int64_t)d * p.A_ds + (int64_t)ng * p.A_ns] : 0.f;
                S.AX[w][1][lane] =
                    (k > 0 && st) ? p.x[(row * p.n_chunks + (k - 1)) * 2 * p.dstate + 2 * ng + 1] : 0.f;
            }
            __syncwarp();

            // Two states per iteration, interleaved through every phase, so each warp always
            // has two independent dependency chains in flight.  An odd dstate pads the last
            // pair with a state whose A, B and C are zero (it contributes nothing), and pairs
            // beyond dstate are such states entirely (A, B, C, x rows are staged as zero).  The W warps
            // walk the state pairs in rotation (warp w takes pair (j + w) mod W at step j), so
            // at every step each warp owns a different pair's rows of the chunk accumulator and
            // adds its dB / dC partials there directly; one barrier per step hands the rows on.
#pragma unroll 1
            for (int j = 0; j < W; ++j) {  // uniform over the CTA; pairs past nblk are all-zero
                const int n0 = 2 * ((j + w) & (W - 1));
                const bool has1 = n0 + 1 < p.nblk;
                float An[2], A2[2], Pl[2];
                f32x2 A2p[2], Anp[2];
                f32x2 Bv[2][4], b2[2][4];
                float a[2][8];
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    const int n = n0 + s;
                    An[s] = S.AX[w][0][n];  // n < NS always (dstate <= 16); padded states are zero
                    A2[s] = An[s] * kLog2e;
                    A2p[s] = pack2(A2[s], A2[s]);
                    Anp[s] = pack2(An[s], An[s]);
                    float bv8[8];
                    bc_ld8(&S.BC[0][n][0], lane, bv8);
#pragma unroll
                    for (int m = 0; m < 4; ++m) Bv[s][m] = pack2(bv8[2 * m], bv8[2 * m + 1]);
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const float2 v = unpack2(ex2x2(mul2(dtf2[m], A2p[s])));
                        a[s][2 * m] = v.x;
                        a[s][2 * m + 1] = v.y;
                        b2[s][m] = mul2(dtu2[m], Bv[s][m]);
                    }
                    Pl[s] = ex2(A2[s] * sdt);  // decay over the lane's 8 steps
                }
                // local folds: forward state from zero, reverse dh without the carry
                float H[2] = {0.f, 0.f}, Dl[2];
                float e[2][8];
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    const int n = n0 + s;
                    float cv8[8];
                    bc_ld8(&S.BC[1][n][0], lane, cv8);
                    const float2 e0 = unpack2(mul2(dog2[0], pack2(cv8[0], cv8[1])));
                    const float2 e1 = unpack2(mul2(dog2[1], pack2(cv8[2], cv8[3])));
                    const float2 e2v = unpack2(mul2(dog2[2], pack2(cv8[4], cv8[5])));
                    const float2 e3 = unpack2(mul2(dog2[3], pack2(cv8[6], cv8[7])));
                    e[s][0] = e0.x; e[s][1] = e0.y; e[s][2] = e1.x; e[s][3] = e1.y;
                    e[s][4] = e2v.x; e[s][5] = e2v.y; e[s][6] = e3.x; e[s][7] = e3.y;
                }
#pragma unroll
                for (int m = 0; m < 4; ++m) {
#pragma unroll
                    for (int s = 0; s < 2; ++s) {
                        const float2 bb = unpack2(b2[s][m]);
                        H[s] = fmaf(a[s][2 * m], H[s], bb.x);
                        H[s] = fmaf(a[s][2 * m + 1], H[s], bb.y);
                    }
                }
                Dl[0] = e[0][7];
                Dl[1] = e[1][7];
#pragma unroll
                for (int i = 6; i >= 0; --i) {
                    Dl[0] = fmaf(a[0][i + 1], Dl[0], e[0][i]);
                    Dl[1] = fmaf(a[1][i + 1], Dl[1], e[1][i]);
                }
                // four independent warp scans, level by level: forward (decay, state) over the
                // lanes below, reverse (decay, carry) over the lanes above, for both states
                float Ad[2], Hd[2], Pd[2], Qd[2];
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    Ad[s] = Pl[s]; Hd[s] = H[s]; Pd[s] = Pl[s]; Qd[s] = a[s][0] * Dl[s];
                }
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
#pragma unroll
                    for (int s = 0; s < 2; ++s) {
                        scan_up_level(Ad[s], Hd[s], off);
                        scan_down_level(Pd[s], Qd[s], off);
                    }
                }
                float h_in[2], carry[2];
#pragma unroll
                for (int s = 0; s < 2; ++s) {
                    const int n = n0 + s;
                    const float h_chunk = S.AX[w][1][n];
                    const float c_chunk = S.DHC[cg][w][n];  // never written for padded states: 0
                    const float Ae = __shfl_up_sync(FULL, Ad[s], 1), He = __shfl_up_sync(FULL, Hd[s], 1);
                    const float Pe = __shfl_down_sync(FULL, Pd[s], 1), Qe = __shfl_down_sync(FULL, Qd[s], 1);
                    h_in[s] = lane == 0 ? h_chunk : fmaf(Ae, h_chunk, He);
                    carry[s] = lane == 31 ? c_chunk : fmaf(Pe, c_chunk, Qe);
                }
                // replays: states forward, dh backward
                f32x2 h2[2][4], dh2[2][4];
                {
                    float hp[2] = {h_in[0], h_in[1]};
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
#pragma unroll
                        for (int s = 0; s < 2; ++s) {
                            const float2 bb = unpack2(b2[s][m]);
                            const float h0 = fmaf(a[s][2 * m], hp[s], bb.x);
                            const float h1 = fmaf(a[s][2 * m + 1], h0, bb.y);
                            h2[s][m] = pack2(h0, h1);
                            hp[s] = h1;
                        }
                    }
#pragma unroll
                    for (int m = 3; m >= 0; --m) {
#pragma unroll
                        for (int s = 0; s < 2; ++s) {
                            const float d1 = e[s][2 * m + 1] + carry[s];
                            carry[s] = a[s][2 * m + 1] * d1;
                            const float d0 = e[s][2 * m] + carry[s];
                            carry[s] = a[s][2 * m] * d0;
                            dh2[s][m] = pack2(d0, d1);
                        }
                    }
                }
                if (lane == 0) {
                    S.DHC[cg][w][n0] = carry[0];  // carries into the previous chunk
                    if (has1) S.DHC[cg][w][n0 + 1] = carry[1];
                }
                // per-step gradients, as pairs; dB / dC partials are added into this pair's rows
                // of the chunk accumulator (no other warp touches them during this step)
                f32x2 dA2[2] = {pack2(0.f, 0.f), pack2(0.f, 0.f)};
#pragma unroll
                for (int s = 0; s < 2; ++s) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {
                        ulonglong2 *ab = reinterpret_cast<ulonglong2 *>(&S.ACC[0][n0 + s][hh * 128 + lane * 4]);
                        ulonglong2 *ac = reinterpret_cast<ulonglong2 *>(&S.ACC[1][n0 + s][hh * 128 + lane * 4]);
                        const bool live = s == 0 || has1;
                        ulonglong2 vb = live ? *ab : make_ulonglong2(0ull, 0ull);
                        ulonglong2 vc = live ? *ac : make_ulonglong2(0ull, 0ull);
#pragma unroll
                        for (int mm = 0; mm < 2; ++mm) {
                            const int m = 2 * hh + mm;
                            const f32x2 pv = fma2(dtu2[m] ^ 0x8000000080000000ull, Bv[s][m], h2[s][m]);  // a_t h_{t-1}
                            const f32x2 gv = mul2(dh2[s][m], pv);
                            S1[m] = fma2(dh2[s][m], Bv[s][m], S1[m]);
                            S2[m] = fma2(Anp[s], gv, S2[m]);
                            dA2[s] = fma2(dtf2[m], gv, dA2[s]);
                            if (mm == 0) {
                                vb.x = fma2(dh2[s][m], dtu2[m], vb.x);
                                vc.x = fma2(dog2[m], h2[s][m], vc.x);
                            } else {
                                vb.y = fma2(dh2[s][m], dtu2[m], vb.y);
                                vc.y = fma2(dog2[m], h2[s][m], vc.y);
                            }
                        }
                        if (live) {
                            *ab = vb;
                            *ac = vc;
                        }
                    }
                }
                {   // this channel's dA for both states: sum over the lanes.  The first level
                    // hands each half-warp one state (lanes < 16 state n0, the others n0 + 1),
                    // so the last four levels reduce one value instead of two.
                    const float2 v0 = unpack2(dA2[0]), v1 = unpack2(dA2[1]);
                    const float p0 = v0.x + v0.y, p1 = v1.x + v1.y;
                    const bool upper = (lane & 16) != 0;
                    float dAp = (upper ? p1 : p0) + __shfl_xor_sync(FULL, upper ? p0 : p1, 16);
#pragma unroll
                    for (int off = 8; off > 0; off >>= 1) dAp += __shfl_xor_sync(FULL, dAp, off);
                    if (lane == 0) S.DAACC[cg][w][n0] += dAp;
                    if (lane == 16 && has1) S.DAACC[cg][w][n0 + 1] += dAp;
                }
                __syncthreads();  // the accumulator rows pass to the next warp
            }
            // ---- per-element epilogue
            {
                const float Dv = p.D ? p.D[(int64_t)d * p.D_s] : 0.f;
                float du[8], dd[8], dDp = 0.f, dbp = 0.f;
                if (p.s12 != nullptr) {
                    // dstate > 16: this launch covers one block of 16 states; the per-step sums
                    // over states are carried between launches in an fp32 scratch (pitch lpitch)
                    float *r1 = p.s12 + ((int64_t)b * p.dim + d) * 2 * p.lpitch;
                    float *r2 = r1 + p.lpitch;
                    if (!p.blk_first) {
                        float a1[8], a2[8];
                        load_items(r1, t0, L, vec, a1);
                        load_items(r2, t0, L, vec, a2);
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            S1[m] = add2(S1[m], pack2(a1[2 * m], a1[2 * m + 1]));
                            S2[m] = add2(S2[m], pack2(a2[2 * m], a2[2 * m + 1]));
                        }
                    }
                    if (!p.blk_last) {
                        float a1[8], a2[8];
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            const float2 v1 = unpack2(S1[m]), v2 = unpack2(S2[m]);
                            a1[2 * m] = v1.x; a1[2 * m + 1] = v1.y;
                            a2[2 * m] = v2.x; a2[2 * m + 1] = v2.y;
                        }
                        if (valid) {
                            store_items(r1, t0, L, vec, a1);
                            store_items(r2, t0, L, vec, a2);
                        }
                    }
                }
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const float2 s1 = unpack2(S1[m]), s2 = unpack2(S2[m]), df = unpack2(dtf2[m]);
                    const float2 dg = unpack2(dog2[m]), u = unpack2(uf2[m]);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int i = 2 * m + h;
                        const float S1v = h ? s1.y : s1.x, S2v = h ? s2.y : s2.x, dtv = h ? df.y : df.x;
                        const float dgv = h ? dg.y : dg.x, uv = h ? u.y : u.x;
                        // softplus'(x) = sigmoid(x) = 1 - exp(-softplus(x)); 1 above the threshold
                        const float gate = p.softplus ? (dtv > 20.f ? 1.f : softplus_grad_from_out(dtv)) : 1.f;
                        du[i] = fmaf(dtv, S1v, Dv * dgv);
                        dd[i] = fmaf(uv, S1v, S2v) * gate;
                        if (t0 + i < L) {
                            dDp = fmaf(dgv, uv, dDp);
                            dbp += dd[i];
                        }
                    }
                }
                if (valid && p.blk_last) {
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
            ++pass;
        }
        // ---- flush the chunk's dB / dC (summed over this CTA's channels)
        __syncthreads();
        const int clen = (int)min((int64_t)CK, L - kt0);
        for (int i = tid; i < 2 * NS * (CK / 4); i += NT) {
            const int q = i / (NS * (CK / 4)), rem = i - q * NS * (CK / 4);
            const int n = rem / (CK / 4), pos = (rem - n * (CK / 4)) * 4;
            const int t = ((pos >> 2) & 31) * 8 + (pos >> 7) * 4;  // first timestep of this 4-group
            float *src = &S.ACC[q][n][pos];
            if (n < p.nblk && t < clen) {
                float *dst = (q == 0 ? p.acc_dB : p.acc_dC) +
                             (((int64_t)b * p.n_groups + g) * p.dstate + p.state_lo + n) * p.lpitch + kt0 + t;
                red_add_v4(dst, src[0], src[1], src[2], src[3]);
            }
            src[0] = src[1] = src[2] = src[3] = 0.f;
        }
    }
    __syncthreads();
    for (int i = tid; i < K * W * NS; i += NT) {
        const int cg = i / (W * NS), rem = i - cg * W * NS, ww = rem / NS, n = rem - ww * NS;
        const int cin = (tile * K + cg) * W + ww;
        if (cin < p.dpg && n < p.nblk)
            atomicAdd(p.dA + (int64_t)(g * p.dpg + cin) * p.dstate + p.state_lo + n, S.DAACC[cg][ww][n]);
    }
    for (int i = tid; i < K * W; i += NT) {
        const int cg = i / W, ww = i - cg * W;
        const int cin = (tile * K + cg) * W + ww;
        if (cin < p.dpg) {
            if (p.dD && p.blk_last) atomicAdd(p.dD + g * p.dpg + cin, S.PBD[cg][ww][0]);
            if (p.ddelta_bias && p.blk_last) atomicAdd(p.ddelta_bias + g * p.dpg + cin, S.PBD[cg][ww][1]);
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
    constexpr int SMEM = (int)sizeof(BwdSmemT<T>);
    static std::atomic<unsigned long long> smem_set{0};
    {
        const cudaError_t e = set_smem_once(smem_set, reinterpret_cast<const void *>(kern), SMEM);
        if (e != cudaSuccess) return e;
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
