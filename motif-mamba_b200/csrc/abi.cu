// C-ABI entry points (include/motif_ssm.h): argument validation, workspace carving,
// launch-shape decisions and dispatch to the kernels.  Mirrors the checks of the
// reference binding (csrc/selective_scan/selective_scan.cpp:270-413, 415-618): the
// same conditions fail, but as a status code plus ss_last_error() text instead of a
// C++ exception, and nothing here allocates.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.h"

using namespace mss;

namespace {

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}
int cuda_fail(cudaError_t e, const char *what) {
    return fail(MSS_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}
int esize(int itype) { return itype == MSS_F32 ? 4 : 2; }
bool valid_type(int t) { return t == MSS_F32 || t == MSS_F16 || t == MSS_BF16; }
bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool st16(int64_t stride, int es) { return ((stride * es) & 15) == 0; }
int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// ---------------- forward launch shape ----------------
struct FwdShape {
    int n_seg, seg_len;
    int64_t ws_h_bytes, ws_dts_bytes;
};
FwdShape fwd_shape(const ss_fwd_args *a) {
    FwdShape s{1, (int)a->seqlen, 0, 0};
    const int64_t rows = a->batch * a->dim;
    // Few rows (small batch x channels): split the sequence into segments so that rows x
    // segments fills up to one wave of resident rows; segments are whole 16-step tiles.  A
    // carry pass gives every segment its initial state.
    const int64_t capacity = (int64_t)kNumSMs * fwd_rows_per_sm((int)a->dstate, rows);
    const int64_t n_want = rows > 0 ? capacity / rows : 1;
    if (!a->P && rows > 0 && n_want >= 2 && a->seqlen >= 4 * 64) {
        // at most 128 segments of >= 64 steps
        const int64_t n_max = std::min<int64_t>(std::min<int64_t>(n_want, 128), a->seqlen / 64);
        int64_t seg = round_up((a->seqlen + n_max - 1) / n_max, 16);
        int64_t n = (a->seqlen + seg - 1) / seg;
        if (n > 1) {
            s.n_seg = (int)n;
            s.seg_len = (int)seg;
            const int ns = fwd_state_pad((int)a->dstate);
            s.ws_h_bytes = round_up(rows * n * ns * 4, 256);
            s.ws_dts_bytes = round_up(2 * rows * n * 4, 256);  // raw and composed dt sums
        }
    }
    return s;
}

// Motif coupling limits: P and Q both given, rank 1..8, dstate <= 64 (4 states per lane).
int check_pq(const char *who, const float *P, const float *Q, int64_t rank, int64_t dstate) {
    if (!P && !Q) return MSS_OK;
    if (!P || !Q) return fail(MSS_ERR_INVALID, "%s: P and Q must be given together", who);
    if (rank < 1 || rank > 8) return fail(MSS_ERR_UNSUPPORTED, "%s: pq_rank must be in [1, 8]", who);
    if (dstate > 64) return fail(MSS_ERR_UNSUPPORTED, "%s: the P/Q coupling supports dstate <= 64", who);
    return MSS_OK;
}

int check_fwd(const ss_fwd_args *a, bool need_ptrs = true) {
    if (!a) return fail(MSS_ERR_INVALID, "ss_fwd: null argument struct");
    if (!valid_type(a->itype)) return fail(MSS_ERR_INVALID, "ss_fwd: itype must be f32, f16 or bf16");
    if (a->batch < 0 || a->dim < 0 || a->seqlen < 0)
        return fail(MSS_ERR_INVALID, "ss_fwd: negative size");
    if (a->dstate < 1) return fail(MSS_ERR_INVALID, "ss_fwd: dstate must be >= 1");
    if (a->dstate > kMaxDstate)
        return fail(MSS_ERR_UNSUPPORTED, "ss_fwd: dstate %lld > %d is not supported by this build",
                    (long long)a->dstate, kMaxDstate);
    if (a->n_groups < 1 || (a->dim > 0 && a->dim % a->n_groups != 0))
        return fail(MSS_ERR_INVALID, "ss_fwd: n_groups must divide dim");
    if (a->batch * a->dim * a->seqlen == 0 || !need_ptrs) return check_pq("ss_fwd", a->P, a->Q, a->pq_rank, a->dstate);
    if (!a->u || !a->delta || !a->A || !a->B || !a->C || !a->out || !a->x)
        return fail(MSS_ERR_INVALID, "ss_fwd: u, delta, A, B, C, out and x must be non-null");
    if (a->z && !a->out_z) return fail(MSS_ERR_INVALID, "ss_fwd: out_z must be given with z");
    if (a->seqlen > (int64_t)1 << 31 || a->dim > (int64_t)1 << 30)
        return fail(MSS_ERR_UNSUPPORTED, "ss_fwd: size out of range");
    return check_pq("ss_fwd", a->P, a->Q, a->pq_rank, a->dstate);
}

int check_bwd(const ss_bwd_args *a, bool need_ptrs = true) {
    if (!a) return fail(MSS_ERR_INVALID, "ss_bwd: null argument struct");
    if (!valid_type(a->itype)) return fail(MSS_ERR_INVALID, "ss_bwd: itype must be f32, f16 or bf16");
    if (a->batch < 0 || a->dim < 0 || a->seqlen < 0) return fail(MSS_ERR_INVALID, "ss_bwd: negative size");
    if (a->dstate < 1) return fail(MSS_ERR_INVALID, "ss_bwd: dstate must be >= 1");
    if (a->dstate > kMaxDstateBwd)
        return fail(MSS_ERR_UNSUPPORTED, "ss_bwd: dstate %lld > %d is not supported by this build",
                    (long long)a->dstate, kMaxDstateBwd);
    if (a->n_groups < 1 || (a->dim > 0 && a->dim % a->n_groups != 0))
        return fail(MSS_ERR_INVALID, "ss_bwd: n_groups must divide dim");
    if (!need_ptrs) return check_pq("ss_bwd", a->P, a->Q, a->pq_rank, a->dstate);
    if (a->z && (!a->out || !a->dz)) return fail(MSS_ERR_INVALID, "ss_bwd: out and dz must be given with z");
    if (a->recompute_out_z && (!a->z || !a->out_z))
        return fail(MSS_ERR_INVALID, "ss_bwd: recompute_out_z needs z and out_z");
    if (!a->dA || !a->dB || !a->dC) return fail(MSS_ERR_INVALID, "ss_bwd: dA, dB and dC must be non-null");
    if ((a->D != nullptr) != (a->dD != nullptr)) return fail(MSS_ERR_INVALID, "ss_bwd: dD must be given iff D is");
    if ((a->delta_bias != nullptr) != (a->ddelta_bias != nullptr))
        return fail(MSS_ERR_INVALID, "ss_bwd: ddelta_bias must be given iff delta_bias is");
    if (a->batch * a->dim * a->seqlen == 0) return MSS_OK;
    if (!a->u || !a->delta || !a->A || !a->B || !a->C || !a->dout || !a->du || !a->ddelta || !a->x)
        return fail(MSS_ERR_INVALID, "ss_bwd: u, delta, A, B, C, dout, du, ddelta and x must be non-null");
    if (a->seqlen > (int64_t)1 << 31 || a->dim > (int64_t)1 << 30)
        return fail(MSS_ERR_UNSUPPORTED, "ss_bwd: size out of range");
    if (a->P && (!a->dP || !a->dQ)) return fail(MSS_ERR_INVALID, "ss_bwd: dP and dQ must be given with P");
    return check_pq("ss_bwd", a->P, a->Q, a->pq_rank, a->dstate);
}

struct BwdShape {
    int kgroups, tiles_per_group;
    int64_t lpitch, acc_bytes, dh_bytes, ckpt_bytes;
};
BwdShape bwd_shape(const ss_bwd_args *a) {
    BwdShape s;
    const int64_t rows = a->batch * a->dim;
    // K channel groups of kBwdChannelsPerGroup per CTA (more K: fewer accumulator flushes per
    // channel).  Among the K that still give at least ~3 waves of 2 CTAs / SM, take the one whose
    // CTA count fills its last wave best (ties to the larger K): at config 4 the last wave of
    // K = 8 is 19 % full and costs ~5 % of the kernel.
    const int cpg = kBwdChannelsPerGroup;
    const int64_t dpg = a->n_groups > 0 ? a->dim / a->n_groups : a->dim;
    const int64_t slots = 2 * kNumSMs;
    int64_t kmax = rows / (cpg * slots * 3);
    kmax = kmax < 1 ? 1 : (kmax > kBwdMaxGroups ? kBwdMaxGroups : kmax);
    s.kgroups = (int)kmax;
    double best = -1.0;
    for (int64_t k = kmax; k >= 1 && k * 2 >= kmax; --k) {
        const int64_t ctas = ((dpg + cpg * k - 1) / (cpg * k)) * a->n_groups * a->batch;
        const int64_t waves = (ctas + slots - 1) / slots;
        const double fill = waves > 0 ? (double)ctas / (double)(waves * slots) : 0.0;
        if (fill > best + 0.005) {
            best = fill;
            s.kgroups = (int)k;
        }
    }
    s.tiles_per_group = (int)((dpg + cpg * s.kgroups - 1) / (cpg * s.kgroups));
    s.lpitch = round_up(a->seqlen, 4);
    s.acc_bytes = round_up(a->batch * a->n_groups * a->dstate * s.lpitch * 4, 256);
    // dstate > 16: fp32 per-step partial sums over states, carried between state blocks
    s.dh_bytes = a->dstate > 16 ? round_up(rows * 2 * s.lpitch * 4, 256) : 0;
    // P/Q coupling: the 16 states at every 16-step segment start
    const int64_t nsx = a->dstate <= 16 ? 16 : (a->dstate <= 32 ? 32 : 64);  // padded states per checkpoint
    s.ckpt_bytes = a->P ? round_up(rows * ((a->seqlen + 15) / 16) * nsx * 4, 256) : 0;
    return s;
}

}  // namespace

namespace mss {
int set_last_error(int code, const char *msg) { return fail(code, "%s", msg); }
}  // namespace mss

extern "C" {

int32_t ss_chunk_len(void) { return kChunkLen; }
int32_t ss_max_dstate(void) { return kMaxDstate; }
const char *ss_last_error(void) { return g_err.c_str(); }
const char *ss_version(void) { return "motif-mamba-b200 0.1.0 (sm_100a)"; }
void ss_abi_struct_sizes(int64_t out[5]) {
    out[0] = sizeof(ss_fwd_args);
    out[1] = sizeof(ss_bwd_args);
    out[2] = sizeof(conv1d_args);
    out[3] = sizeof(conv1d_update_args);
    out[4] = sizeof(ssm_state_update_args);
}

int ss_fwd_workspace_size(const ss_fwd_args *a, int64_t *bytes) {
    int rc = check_fwd(a, false);
    if (rc) return rc;
    if (!bytes) return fail(MSS_ERR_INVALID, "ss_fwd_workspace_size: null output");
    FwdShape s = fwd_shape(a);
    *bytes = s.ws_h_bytes + s.ws_dts_bytes;
    return MSS_OK;
}

int ss_fwd(const ss_fwd_args *a, void *stream) {
    int rc = check_fwd(a);
    if (rc) return rc;
    if (a->batch * a->dim * a->seqlen == 0) return MSS_OK;
    FwdShape s = fwd_shape(a);
    if (s.ws_h_bytes + s.ws_dts_bytes > 0) {
        if (!a->workspace || a->workspace_bytes < s.ws_h_bytes + s.ws_dts_bytes)
            return fail(MSS_ERR_WORKSPACE, "ss_fwd: workspace of %lld bytes required",
                        (long long)(s.ws_h_bytes + s.ws_dts_bytes));
        if (!al16(a->workspace)) return fail(MSS_ERR_ALIGNMENT, "ss_fwd: workspace must be 16-byte aligned");
    }
    const int es = esize(a->itype);
    FwdParams p{};
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.seqlen = (int)a->seqlen; p.dstate = (int)a->dstate;
    p.n_groups = (int)a->n_groups; p.dpg = (int)(a->dim / a->n_groups);
    p.softplus = a->delta_softplus ? 1 : 0;
    p.n_seg = s.n_seg; p.seg_len = s.seg_len;
    p.n_chunks = (int)((a->seqlen + kChunkLen - 1) / kChunkLen);
    p.u = a->u; p.delta = a->delta; p.B = a->B; p.C = a->C; p.z = a->z; p.out = a->out; p.out_z = a->out_z;
    p.u_bs = a->u_bs; p.u_ds = a->u_ds; p.delta_bs = a->delta_bs; p.delta_ds = a->delta_ds;
    p.B_bs = a->B_bs; p.B_gs = a->B_gs; p.B_ns = a->B_ns; p.C_bs = a->C_bs; p.C_gs = a->C_gs; p.C_ns = a->C_ns;
    p.z_bs = a->z_bs; p.z_ds = a->z_ds; p.out_bs = a->out_bs; p.out_ds = a->out_ds;
    p.out_z_bs = a->out_z_bs; p.out_z_ds = a->out_z_ds;
    p.A = a->A; p.A_ds = a->A_ds; p.A_ns = a->A_ns;
    p.D = a->D; p.D_s = a->D_s; p.delta_bias = a->delta_bias; p.delta_bias_s = a->delta_bias_s;
    p.x = a->x;
    p.h0 = a->h0;
    p.ws_h = s.n_seg > 1 ? reinterpret_cast<float *>(a->workspace) : nullptr;
    p.ws_dts = s.n_seg > 1 ? reinterpret_cast<float *>(reinterpret_cast<char *>(a->workspace) + s.ws_h_bytes) : nullptr;
    bool aligned = al16(a->u) && al16(a->delta) && al16(a->B) && al16(a->C) && al16(a->out) &&
                   st16(a->u_bs, es) && st16(a->u_ds, es) && st16(a->delta_bs, es) && st16(a->delta_ds, es) &&
                   st16(a->B_bs, es) && st16(a->B_gs, es) && st16(a->B_ns, es) && st16(a->C_bs, es) &&
                   st16(a->C_gs, es) && st16(a->C_ns, es) && st16(a->out_bs, es) && st16(a->out_ds, es);
    if (a->z)
        aligned = aligned && al16(a->z) && al16(a->out_z) && st16(a->z_bs, es) && st16(a->z_ds, es) &&
                  st16(a->out_z_bs, es) && st16(a->out_z_ds, es);
    p.aligned = aligned ? 1 : 0;
    if (a->h0 && (reinterpret_cast<uintptr_t>(a->h0) & 3))
        return fail(MSS_ERR_ALIGNMENT, "ss_fwd: h0 must be 4-byte aligned fp32");
    cudaError_t e;
    if (a->P) {
        if (a->h0) return fail(MSS_ERR_UNSUPPORTED, "ss_fwd: an initial state is not supported with P/Q");
        p.P = a->P; p.Q = a->Q; p.pq_rank = (int)a->pq_rank; p.pq_per_dim = a->pq_per_dim ? 1 : 0;
        e = launch_ss_fwd_pq(p, a->itype, a->z != nullptr, static_cast<cudaStream_t>(stream));
    } else {
        e = launch_ss_fwd(p, a->itype, a->z != nullptr, static_cast<cudaStream_t>(stream));
    }
    if (e != cudaSuccess) return cuda_fail(e, "ss_fwd launch");
    return MSS_OK;
}

int ss_bwd_workspace_size(const ss_bwd_args *a, int64_t *bytes) {
    int rc = check_bwd(a, false);
    if (rc) return rc;
    if (!bytes) return fail(MSS_ERR_INVALID, "ss_bwd_workspace_size: null output");
    BwdShape s = bwd_shape(a);
    *bytes = 2 * s.acc_bytes + s.dh_bytes + s.ckpt_bytes;
    return MSS_OK;
}

int ss_bwd(const ss_bwd_args *a, void *stream) {
    int rc = check_bwd(a);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int es = esize(a->itype);
    cudaError_t e;
    // Gradients that are sums are fully overwritten (zeroed here, then accumulated).
    e = cudaMemsetAsync(a->dA, 0, a->dim * a->dstate * 4, st);
    if (e != cudaSuccess) return cuda_fail(e, "ss_bwd memset dA");
    if (a->dD && (e = cudaMemsetAsync(a->dD, 0, a->dim * 4, st)) != cudaSuccess) return cuda_fail(e, "ss_bwd memset dD");
    if (a->ddelta_bias && (e = cudaMemsetAsync(a->ddelta_bias, 0, a->dim * 4, st)) != cudaSuccess)
        return cuda_fail(e, "ss_bwd memset ddelta_bias");
    if (a->P) {
        const int64_t np = (a->pq_per_dim ? a->dim : 1) * a->dstate * a->pq_rank * 4;
        if ((e = cudaMemsetAsync(a->dP, 0, np, st)) != cudaSuccess) return cuda_fail(e, "ss_bwd memset dP");
        if ((e = cudaMemsetAsync(a->dQ, 0, np, st)) != cudaSuccess) return cuda_fail(e, "ss_bwd memset dQ");
    }
    if (a->batch * a->dim * a->seqlen == 0) {
        const int64_t nbc = a->batch * a->n_groups * a->dstate * a->seqlen * es;
        if (nbc > 0) {
            if ((e = cudaMemsetAsync(a->dB, 0, nbc, st)) != cudaSuccess) return cuda_fail(e, "ss_bwd memset dB");
            if ((e = cudaMemsetAsync(a->dC, 0, nbc, st)) != cudaSuccess) return cuda_fail(e, "ss_bwd memset dC");
        }
        return MSS_OK;
    }
    BwdShape s = bwd_shape(a);
    const int64_t need = 2 * s.acc_bytes + s.dh_bytes + s.ckpt_bytes;
    if (!a->workspace || a->workspace_bytes < need)
        return fail(MSS_ERR_WORKSPACE, "ss_bwd: workspace of %lld bytes required", (long long)need);
    if (!al16(a->workspace)) return fail(MSS_ERR_ALIGNMENT, "ss_bwd: workspace must be 16-byte aligned");
    char *ws = reinterpret_cast<char *>(a->workspace);
    float *acc_dB = reinterpret_cast<float *>(ws);
    float *acc_dC = reinterpret_cast<float *>(ws + s.acc_bytes);
    if ((e = cudaMemsetAsync(ws, 0, 2 * s.acc_bytes, st)) != cudaSuccess) return cuda_fail(e, "ss_bwd memset acc");

    BwdParams p{};
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.seqlen = (int)a->seqlen; p.dstate = (int)a->dstate;
    p.n_groups = (int)a->n_groups; p.dpg = (int)(a->dim / a->n_groups);
    p.tiles_per_group = s.tiles_per_group; p.kgroups = s.kgroups;
    p.softplus = a->delta_softplus ? 1 : 0; p.recompute_out_z = a->recompute_out_z ? 1 : 0;
    p.n_chunks = (int)((a->seqlen + kChunkLen - 1) / kChunkLen);
    p.lpitch = s.lpitch;
    p.u = a->u; p.delta = a->delta; p.B = a->B; p.C = a->C; p.z = a->z; p.out = a->out; p.dout = a->dout;
    p.u_bs = a->u_bs; p.u_ds = a->u_ds; p.delta_bs = a->delta_bs; p.delta_ds = a->delta_ds;
    p.B_bs = a->B_bs; p.B_gs = a->B_gs; p.B_ns = a->B_ns; p.C_bs = a->C_bs; p.C_gs = a->C_gs; p.C_ns = a->C_ns;
    p.z_bs = a->z_bs; p.z_ds = a->z_ds; p.out_bs = a->out_bs; p.out_ds = a->out_ds;
    p.dout_bs = a->dout_bs; p.dout_ds = a->dout_ds;
    p.A = a->A; p.A_ds = a->A_ds; p.A_ns = a->A_ns;
    p.D = a->D; p.D_s = a->D_s; p.delta_bias = a->delta_bias; p.delta_bias_s = a->delta_bias_s;
    p.x = a->x;
    p.du = a->du; p.ddelta = a->ddelta; p.dz = a->dz; p.out_z = a->out_z;
    p.du_bs = a->du_bs; p.du_ds = a->du_ds; p.ddelta_bs = a->ddelta_bs; p.ddelta_ds = a->ddelta_ds;
    p.dz_bs = a->dz_bs; p.dz_ds = a->dz_ds; p.out_z_bs = a->out_z_bs; p.out_z_ds = a->out_z_ds;
    p.dA = a->dA; p.dD = a->dD; p.ddelta_bias = a->ddelta_bias;
    p.acc_dB = acc_dB; p.acc_dC = acc_dC;
    p.s12 = s.dh_bytes > 0 ? reinterpret_cast<float *>(ws + 2 * s.acc_bytes) : nullptr;
    bool aligned = al16(a->u) && al16(a->delta) && al16(a->B) && al16(a->C) && al16(a->dout) &&
                   al16(a->du) && al16(a->ddelta) && st16(a->u_bs, es) && st16(a->u_ds, es) &&
                   st16(a->delta_bs, es) && st16(a->delta_ds, es) && st16(a->B_bs, es) && st16(a->B_gs, es) &&
                   st16(a->B_ns, es) && st16(a->C_bs, es) && st16(a->C_gs, es) && st16(a->C_ns, es) &&
                   st16(a->dout_bs, es) && st16(a->dout_ds, es) && st16(a->du_bs, es) && st16(a->du_ds, es) &&
                   st16(a->ddelta_bs, es) && st16(a->ddelta_ds, es);
    if (a->z)
        aligned = aligned && al16(a->z) && al16(a->out) && al16(a->dz) && st16(a->z_bs, es) &&
                  st16(a->z_ds, es) && st16(a->out_bs, es) && st16(a->out_ds, es) && st16(a->dz_bs, es) &&
                  st16(a->dz_ds, es);
    if (a->recompute_out_z)
        aligned = aligned && al16(a->out_z) && st16(a->out_z_bs, es) && st16(a->out_z_ds, es);
    p.aligned = aligned ? 1 : 0;
    if (a->P) {
        p.P = a->P; p.Q = a->Q; p.pq_rank = (int)a->pq_rank; p.pq_per_dim = a->pq_per_dim ? 1 : 0;
        p.dP = a->dP; p.dQ = a->dQ;
        p.ckpt = reinterpret_cast<float *>(ws + 2 * s.acc_bytes + s.dh_bytes);
        e = launch_ss_bwd_pq(p, a->itype, a->z != nullptr, st);
        if (e != cudaSuccess) return cuda_fail(e, "ss_bwd launch");
    }
    // one launch per block of 16 states (a single launch for dstate <= 16)
    for (int lo = 0; !a->P && lo < (int)a->dstate; lo += 16) {
        p.state_lo = lo;
        p.nblk = (int)std::min<int64_t>(16, a->dstate - lo);
        p.blk_first = lo == 0;
        p.blk_last = lo + 16 >= a->dstate;
        e = launch_ss_bwd(p, a->itype, a->z != nullptr, st);
        if (e != cudaSuccess) return cuda_fail(e, "ss_bwd launch");
    }
    const int64_t rows = a->batch * a->n_groups * a->dstate;
    if ((e = launch_acc_to_out(acc_dB, s.lpitch, a->dB, a->itype, rows, a->seqlen, st)) != cudaSuccess)
        return cuda_fail(e, "ss_bwd dB convert");
    if ((e = launch_acc_to_out(acc_dC, s.lpitch, a->dC, a->itype, rows, a->seqlen, st)) != cudaSuccess)
        return cuda_fail(e, "ss_bwd dC convert");
    return MSS_OK;
}

static int check_conv(const conv1d_args *a, const char *who) {
    if (!a) return fail(MSS_ERR_INVALID, "%s: null argument struct", who);
    if (!valid_type(a->itype) || !valid_type(a->wtype)) return fail(MSS_ERR_INVALID, "%s: bad element type", who);
    if (a->width < 2 || a->width > 4) return fail(MSS_ERR_UNSUPPORTED, "%s: width must be 2, 3 or 4", who);
    if (a->batch < 0 || a->dim < 0 || a->seqlen < 0) return fail(MSS_ERR_INVALID, "%s: negative size", who);
    return MSS_OK;
}
static bool conv_vec(const conv1d_args *a, bool bwd) {
    const int es = esize(a->itype);
    bool v = al16(a->x) && st16(a->x_bs, es) && st16(a->x_ds, es);
    if (!bwd) v = v && al16(a->out) && st16(a->out_bs, es) && st16(a->out_ds, es);
    else v = v && al16(a->dout) && al16(a->dx) && st16(a->dout_bs, es) && st16(a->dout_ds, es) &&
             st16(a->dx_bs, es) && st16(a->dx_ds, es);
    return v;
}

int conv1d_fwd(const conv1d_args *a, void *stream) {
    int rc = check_conv(a, "conv1d_fwd");
    if (rc) return rc;
    if (a->batch * a->dim * a->seqlen == 0) return MSS_OK;
    if (!a->x || !a->weight || !a->out) return fail(MSS_ERR_INVALID, "conv1d_fwd: x, weight and out must be non-null");
    cudaError_t e = launch_conv1d_fwd(*a, conv_vec(a, false), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MSS_OK : cuda_fail(e, "conv1d_fwd launch");
}

int conv1d_bwd(const conv1d_args *a, void *stream) {
    int rc = check_conv(a, "conv1d_bwd");
    if (rc) return rc;
    if (!a->dweight) return fail(MSS_ERR_INVALID, "conv1d_bwd: dweight must be non-null");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(a->dweight, 0, a->dim * a->width * 4, st);
    if (e != cudaSuccess) return cuda_fail(e, "conv1d_bwd memset");
    if (a->dbias && (e = cudaMemsetAsync(a->dbias, 0, a->dim * 4, st)) != cudaSuccess)
        return cuda_fail(e, "conv1d_bwd memset");
    if (a->batch * a->dim * a->seqlen == 0) return MSS_OK;
    if (!a->x || !a->weight || !a->dout || !a->dx)
        return fail(MSS_ERR_INVALID, "conv1d_bwd: x, weight, dout and dx must be non-null");
    e = launch_conv1d_bwd(*a, conv_vec(a, true), st);
    return e == cudaSuccess ? MSS_OK : cuda_fail(e, "conv1d_bwd launch");
}

int conv1d_update(const conv1d_update_args *a, void *stream) {
    if (!a) return fail(MSS_ERR_INVALID, "conv1d_update: null argument struct");
    if (!valid_type(a->itype) || !valid_type(a->wtype) || !valid_type(a->stype))
        return fail(MSS_ERR_INVALID, "conv1d_update: bad element type");
    if (a->width < 2 || a->width > 4) return fail(MSS_ERR_UNSUPPORTED, "conv1d_update: width must be 2, 3 or 4");
    if (a->state_len < a->width) return fail(MSS_ERR_INVALID, "conv1d_update: state_len must be >= width");
    if (a->batch * a->dim == 0) return MSS_OK;
    if (!a->x || !a->conv_state || !a->weight || !a->out)
        return fail(MSS_ERR_INVALID, "conv1d_update: x, conv_state, weight and out must be non-null");
    cudaError_t e = launch_conv1d_update(*a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MSS_OK : cuda_fail(e, "conv1d_update launch");
}

int ssm_state_update(const ssm_state_update_args *a, void *stream) {
    if (!a) return fail(MSS_ERR_INVALID, "ssm_state_update: null argument struct");
    if (!valid_type(a->itype) || !valid_type(a->stype)) return fail(MSS_ERR_INVALID, "ssm_state_update: bad element type");
    if (a->dstate < 1 || a->dstate > 256) return fail(MSS_ERR_UNSUPPORTED, "ssm_state_update: dstate must be in [1, 256]");
    if (a->n_groups < 1 || a->dim % a->n_groups != 0)
        return fail(MSS_ERR_INVALID, "ssm_state_update: n_groups must divide dim");
    if (a->batch * a->dim == 0) return MSS_OK;
    if (!a->state || !a->x || !a->dt || !a->A || !a->B || !a->C || !a->out)
        return fail(MSS_ERR_INVALID, "ssm_state_update: state, x, dt, A, B, C and out must be non-null");
    if (a->state_batch_indices && a->state_batch < 1)
        return fail(MSS_ERR_INVALID, "ssm_state_update: state_batch must be given with state_batch_indices");
    cudaError_t e = launch_state_update(*a, nullptr, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MSS_OK : cuda_fail(e, "ssm_state_update launch");
}

int ssm_state_update_dtproj(const ssm_state_update_args *a, const ssm_dtproj_args *p, void *stream) {
    if (!a || !p) return fail(MSS_ERR_INVALID, "ssm_state_update_dtproj: null argument struct");
    if (!valid_type(a->itype) || !valid_type(a->stype))
        return fail(MSS_ERR_INVALID, "ssm_state_update_dtproj: bad element type");
    if (a->dstate != 16) return fail(MSS_ERR_UNSUPPORTED, "ssm_state_update_dtproj: dstate must be 16");
    if (a->n_groups < 1 || a->dim % a->n_groups != 0)
        return fail(MSS_ERR_INVALID, "ssm_state_update_dtproj: n_groups must divide dim");
    if (p->rank < 8 || p->rank % 8 != 0 || p->rank > 256)
        return fail(MSS_ERR_UNSUPPORTED, "ssm_state_update_dtproj: rank must be a multiple of 8 in [8, 256]");
    if (a->batch * a->dim == 0) return MSS_OK;
    if (!a->state || !a->x || !p->dt_in || !p->weight || !a->A || !a->B || !a->C || !a->out)
        return fail(MSS_ERR_INVALID, "ssm_state_update_dtproj: a required pointer is null");
    if (a->state_batch_indices && a->state_batch < 1)
        return fail(MSS_ERR_INVALID, "ssm_state_update_dtproj: state_batch must be given with state_batch_indices");
    cudaError_t e = launch_state_update(*a, p, static_cast<cudaStream_t>(stream));
    if (e == cudaErrorInvalidValue)
        return fail(MSS_ERR_ALIGNMENT, "ssm_state_update_dtproj: rows must be unit-stride and 16-byte aligned");
    return e == cudaSuccess ? MSS_OK : cuda_fail(e, "ssm_state_update_dtproj launch");
}

int64_t add_rms_norm_args_size(void) { return (int64_t)sizeof(add_rms_norm_args); }

int add_rms_norm(const add_rms_norm_args *a, void *stream) {
    if (!a) return fail(MSS_ERR_INVALID, "add_rms_norm: null argument struct");
    if (!valid_type(a->itype)) return fail(MSS_ERR_INVALID, "add_rms_norm: bad element type");
    for (int t : {a->rin_type, a->rout_type, a->wtype})
        if (t != MSS_F32 && t != a->itype) return fail(MSS_ERR_INVALID, "add_rms_norm: residual / weight type must be f32 or itype");
    if (a->rows < 0 || a->dim < 0) return fail(MSS_ERR_INVALID, "add_rms_norm: negative size");
    if (a->dim % 8 != 0 || a->dim > 4096)
        return fail(MSS_ERR_UNSUPPORTED, "add_rms_norm: dim must be a multiple of 8 and at most 4096");
    if (a->rows == 0 || a->dim == 0) return MSS_OK;
    if (!a->x || !a->residual_out || !a->weight || !a->out)
        return fail(MSS_ERR_INVALID, "add_rms_norm: x, residual_out, weight and out must be non-null");
    const int es = esize(a->itype);
    if (!al16(a->x) || !al16(a->residual_out) || !al16(a->weight) || !al16(a->out) ||
        (a->residual_in && !al16(a->residual_in)) || !st16(a->x_rs, es) || !st16(a->out_rs, es) ||
        !st16(a->rout_rs, esize(a->rout_type)) || (a->residual_in && !st16(a->rin_rs, esize(a->rin_type))))
        return fail(MSS_ERR_ALIGNMENT, "add_rms_norm: rows must start on 16-byte boundaries");
    cudaError_t e = launch_add_rms_norm(*a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MSS_OK : cuda_fail(e, "add_rms_norm launch");
}

int64_t motif_regular_args_size(void) { return (int64_t)sizeof(motif_regular_args); }

int motif_regular(const motif_regular_args *a, void *stream) {
    if (!a) return fail(MSS_ERR_INVALID, "motif_regular: null argument struct");
    if (a->n_mat < 0) return fail(MSS_ERR_INVALID, "motif_regular: negative n_mat");
    if (a->cc < 3 || a->cc > 32) return fail(MSS_ERR_UNSUPPORTED, "motif_regular: cc must be in [3, 32]");
    if (a->n_mat > 0x7fffffff) return fail(MSS_ERR_UNSUPPORTED, "motif_regular: n_mat too large");
    if (a->n_mat == 0) return MSS_OK;
    if (!a->a || !a->target || !a->loss) return fail(MSS_ERR_INVALID, "motif_regular: a, target and loss must be non-null");
    if (a->a_ms < a->cc * a->cc) return fail(MSS_ERR_INVALID, "motif_regular: matrix stride below cc * cc");
    if (a->dloss && (!a->da || a->da_ms < a->cc * a->cc))
        return fail(MSS_ERR_INVALID, "motif_regular: da (stride >= cc * cc) is required with dloss");
    if (a->log_mse && !(a->log_eps > 0.f)) return fail(MSS_ERR_INVALID, "motif_regular: log_eps must be > 0");
    cudaError_t e = launch_motif_regular(*a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? MSS_OK : cuda_fail(e, "motif_regular launch");
}

}  // extern "C"
