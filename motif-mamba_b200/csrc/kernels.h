// Internal launch interface between the C-ABI layer (abi.cu) and the kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "motif_ssm.h"

namespace mss {

struct FwdParams {
    int batch, dim, seqlen, dstate, n_groups, dpg, tiles_per_group;
    int softplus, n_seg, seg_len, n_chunks, aligned;
    const void *u, *delta, *B, *C, *z;
    void *out, *out_z;
    int64_t u_bs, u_ds, delta_bs, delta_ds, B_bs, B_gs, B_ns, C_bs, C_gs, C_ns, z_bs, z_ds;
    int64_t out_bs, out_ds, out_z_bs, out_z_ds;
    const float *A;
    int64_t A_ds, A_ns;
    const float *D;
    int64_t D_s;
    const float *delta_bias;
    int64_t delta_bias_s;
    float *x;
    float *ws_h, *ws_dts;  // segment carries (n_seg > 1)
    const float *P, *Q;    // motif coupling (nullptr: none)
    int pq_rank, pq_per_dim;
    const float *h0;       // state before the first step (batch, dim, dstate), or nullptr (zero)
};

struct BwdParams {
    int batch, dim, seqlen, dstate, n_groups, dpg, tiles_per_group, kgroups;
    int softplus, recompute_out_z, n_chunks, aligned;
    int64_t lpitch;  // row pitch (floats) of the fp32 dB/dC accumulators
    const void *u, *delta, *B, *C, *z, *out, *dout;
    int64_t u_bs, u_ds, delta_bs, delta_ds, B_bs, B_gs, B_ns, C_bs, C_gs, C_ns, z_bs, z_ds;
    int64_t out_bs, out_ds, dout_bs, dout_ds;
    const float *A;
    int64_t A_ds, A_ns;
    const float *D;
    int64_t D_s;
    const float *delta_bias;
    int64_t delta_bias_s;
    const float *x;
    void *du, *ddelta, *dz, *out_z;
    int64_t du_bs, du_ds, ddelta_bs, ddelta_ds, dz_bs, dz_ds, out_z_bs, out_z_ds;
    float *dA, *dD, *ddelta_bias;
    float *acc_dB, *acc_dC;  // fp32 accumulators (batch, n_groups, dstate, lpitch)
    int state_lo, nblk;      // this launch's block of states [state_lo, state_lo + nblk), nblk <= 16
    int blk_first, blk_last; // first / last block of the launch sequence
    float *s12;              // dstate > 16: per-step partial sums over states (batch, dim, 2, lpitch)
    const float *P, *Q;      // motif coupling (nullptr: none)
    int pq_rank, pq_per_dim;
    float *dP, *dQ;
    float *ckpt;             // motif backward: states every 16 steps (batch, dim, ceil(L/16), 16)
};

// Sets the text ss_last_error() reports on this thread and returns `code`.
int set_last_error(int code, const char *msg);

int fwd_state_pad(int dstate);
// resident rows per SM of the forward variant chosen for batch x dim = rows
int fwd_rows_per_sm(int dstate, int64_t rows);
int fwd_channels_per_cta(int dstate);
cudaError_t launch_ss_fwd(const FwdParams &p, int itype, bool has_z, cudaStream_t st);

constexpr int kBwdChannelsPerGroup = 8;  // channels (warps) per CTA pass of the backward
constexpr int kBwdMaxGroups = 8;         // channel groups per backward CTA
cudaError_t launch_ss_bwd(const BwdParams &p, int itype, bool has_z, cudaStream_t st);
cudaError_t launch_conv1d_fwd(const conv1d_args &a, bool vec, cudaStream_t st);
cudaError_t launch_conv1d_bwd(const conv1d_args &a, bool vec, cudaStream_t st);
cudaError_t launch_conv1d_update(const conv1d_update_args &a, cudaStream_t st);
cudaError_t launch_state_update(const ssm_state_update_args &a, const ssm_dtproj_args *dp, cudaStream_t st);
cudaError_t launch_add_rms_norm(const add_rms_norm_args &a, cudaStream_t st);
cudaError_t launch_motif_regular(const motif_regular_args &a, cudaStream_t st);
cudaError_t launch_ss_fwd_pq(const FwdParams &p, int itype, bool has_z, cudaStream_t st);
cudaError_t launch_ss_bwd_pq(const BwdParams &p, int itype, bool has_z, cudaStream_t st);
cudaError_t launch_acc_to_out(const float *acc, int64_t lpitch, void *out, int itype, int64_t rows,
                              int64_t seqlen, cudaStream_t st);

}  // namespace mss
