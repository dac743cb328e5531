/*
 * motif_ssm.h -- C ABI of the B200 (sm_100a) selective-scan hot path.
 *
 * Plain pointers, element strides and sizes; no framework types.  Every entry
 * point is asynchronous on the caller's stream, allocates nothing (callers pass
 * every output and, where one is needed, a workspace whose size a *_workspace_size
 * query returns), never aborts, and returns an int status (MSS_OK on success).
 * The message of the last failure on the calling thread is ss_last_error().
 *
 * The reference interfaces each entry point replaces (paths relative to the
 * reference project, 4354ce38/Motif-Mamba, a fork of mamba_ssm 2.2.6.post3):
 *
 *   ss_fwd            selective_scan_cuda.fwd   csrc/selective_scan/selective_scan.cpp:270-413, 621-627
 *   ss_bwd            selective_scan_cuda.bwd   csrc/selective_scan/selective_scan.cpp:415-618, 628-636
 *   conv1d_fwd        causal_conv1d_fwd_function   (external causal-conv1d; call sites
 *                     mamba_ssm/ops/selective_scan_interface.py:482-484, 567-569)
 *   conv1d_bwd        causal_conv1d_bwd_function   (selective_scan_interface.py:635-637)
 *   conv1d_update     causal_conv1d_update_function / causal_conv1d_update
 *                     (mamba_ssm/modules/mamba_simplemotif.py:352-358)
 *   ssm_state_update  mamba_ssm.ops.triton.selective_state_update.selective_state_update
 *                     (mamba_ssm/modules/mamba_simplemotif.py:396-399)
 *
 * Layout conventions.  Sequence tensors are (batch, channels, seqlen) with the
 * sequence dimension unit-stride; strides below are in ELEMENTS.  B and C of the
 * scan are "variable" (batch, groups, dstate, seqlen).  A, D, delta_bias are fp32.
 */
#ifndef MOTIF_SSM_H
#define MOTIF_SSM_H

#include <stdint.h>

#if defined(__GNUC__)
#define MSS_API __attribute__((visibility("default")))
#else
#define MSS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define MSS_OK 0
#define MSS_ERR_INVALID 1       /* bad argument: shape, stride, null pointer, flag combination */
#define MSS_ERR_UNSUPPORTED 2   /* valid for the reference but not implemented here (e.g. complex A) */
#define MSS_ERR_ALIGNMENT 3     /* pointer alignment the kernel needs is not met */
#define MSS_ERR_WORKSPACE 4     /* workspace missing or smaller than *_workspace_size */
#define MSS_ERR_CUDA 5          /* a CUDA runtime call or kernel launch failed */

/* element types of the sequence tensors (u, delta, z, B, C, out, ...) */
#define MSS_F32 0
#define MSS_F16 1
#define MSS_BF16 2

/* Length, in timesteps, of the chunks whose end states ss_fwd writes into x.
 * x has shape (batch, dim, ceil(seqlen / ss_chunk_len()), 2 * dstate) fp32 and
 * holds (cumulative decay, state) pairs; x[:, :, -1, 1::2] is the final state. */
MSS_API int32_t ss_chunk_len(void);

/* Largest dstate the kernels accept. */
MSS_API int32_t ss_max_dstate(void);

typedef struct {
    int64_t batch, dim, seqlen, dstate, n_groups;
    int32_t itype;           /* MSS_F32 / MSS_F16 / MSS_BF16 for u, delta, B, C, z, out, out_z */
    int32_t delta_softplus;  /* 1: delta <- softplus(delta + delta_bias) (threshold 20) */
    const void *u;      int64_t u_bs, u_ds;
    const void *delta;  int64_t delta_bs, delta_ds;
    const float *A;     int64_t A_ds, A_ns;            /* (dim, dstate) */
    const void *B;      int64_t B_bs, B_gs, B_ns;      /* (batch, n_groups, dstate, seqlen) */
    const void *C;      int64_t C_bs, C_gs, C_ns;
    const float *D;     int64_t D_s;                   /* nullable, (dim,) */
    const float *delta_bias; int64_t delta_bias_s;     /* nullable, (dim,) */
    const void *z;      int64_t z_bs, z_ds;            /* nullable */
    void *out;          int64_t out_bs, out_ds;        /* y + D*u, before the z gate */
    void *out_z;        int64_t out_z_bs, out_z_ds;    /* required iff z: out * silu(z) */
    float *x;           /* contiguous (batch, dim, n_chunks, 2*dstate) */
    void *workspace;    int64_t workspace_bytes;
    /* motif low-rank coupling h += dt * P (Q h_prev) (selective_scan_interface.py:402-433);
     * P == NULL disables it.  fp32 contiguous: P (dstate, r) and Q (r, dstate), or per channel
     * P (dim, dstate, r) and Q (dim, r, dstate) when pq_per_dim; r = pq_rank <= 8, dstate <= 64. */
    const float *P;     const float *Q;
    int64_t pq_rank;    int32_t pq_per_dim; int32_t _pad_pq;
    /* nullable: the state before the first step, fp32 contiguous (batch, dim, dstate), so a
     * sequence can be scanned in pieces (the state at the end of one piece, x[:, :, -1, 1::2],
     * starts the next; the decay halves of x then cover this call's steps only).  No
     * counterpart in the reference's binding, which always starts from zero; forward only
     * (ss_bwd assumes a zero initial state) and not with P/Q. */
    const float *h0;
} ss_fwd_args;

typedef struct {
    int64_t batch, dim, seqlen, dstate, n_groups;
    int32_t itype;
    int32_t delta_softplus;
    int32_t recompute_out_z; /* 1: also write out_z = out * silu(z) (needs z) */
    int32_t _pad0;
    const void *u;      int64_t u_bs, u_ds;
    const void *delta;  int64_t delta_bs, delta_ds;
    const float *A;     int64_t A_ds, A_ns;
    const void *B;      int64_t B_bs, B_gs, B_ns;
    const void *C;      int64_t C_bs, C_gs, C_ns;
    const float *D;     int64_t D_s;                   /* nullable */
    const float *delta_bias; int64_t delta_bias_s;     /* nullable */
    const void *z;      int64_t z_bs, z_ds;            /* nullable */
    const void *out;    int64_t out_bs, out_ds;        /* forward's pre-gate out; required iff z */
    const float *x;     /* ss_fwd's chunk states, contiguous (batch, dim, n_chunks, 2*dstate) */
    const void *dout;   int64_t dout_bs, dout_ds;
    void *du;           int64_t du_bs, du_ds;
    void *ddelta;       int64_t ddelta_bs, ddelta_ds;
    float *dA;          /* contiguous (dim, dstate), overwritten */
    void *dB;           /* contiguous (batch, n_groups, dstate, seqlen), itype, overwritten */
    void *dC;
    float *dD;          /* nullable iff D is null, (dim,), overwritten */
    float *ddelta_bias; /* nullable iff delta_bias is null, (dim,), overwritten */
    void *dz;           int64_t dz_bs, dz_ds;          /* required iff z */
    void *out_z;        int64_t out_z_bs, out_z_ds;    /* required iff recompute_out_z */
    void *workspace;    int64_t workspace_bytes;
    const float *P;     const float *Q;                /* as in ss_fwd_args; NULL: no coupling */
    int64_t pq_rank;    int32_t pq_per_dim; int32_t _pad_pq;
    float *dP;          float *dQ;                     /* fp32, shapes of P and Q, overwritten */
} ss_bwd_args;

typedef struct {
    int64_t batch, dim, seqlen, width;
    int32_t itype;              /* x, out (and dout, dx in the backward) */
    int32_t wtype;              /* weight and bias element type */
    int32_t silu;
    int32_t _pad0;
    const void *x;      int64_t x_bs, x_ds;
    const void *weight; int64_t w_ds, w_ks;            /* (dim, width) */
    const void *bias;                                  /* nullable, contiguous (dim,) */
    void *out;          int64_t out_bs, out_ds;        /* forward output */
    const void *dout;   int64_t dout_bs, dout_ds;      /* backward only */
    void *dx;           int64_t dx_bs, dx_ds;          /* backward only */
    float *dweight;     /* backward only: contiguous (dim, width) fp32, overwritten */
    float *dbias;       /* backward only: nullable (dim,) fp32, overwritten */
} conv1d_args;

typedef struct {
    int64_t batch, dim, width, state_len;   /* state_len >= width (reference: == width) */
    int32_t itype;              /* x, out */
    int32_t wtype;              /* weight, bias */
    int32_t stype;              /* conv_state element type */
    int32_t silu;
    const void *x;      int64_t x_bs;                  /* (batch, dim) */
    void *conv_state;   int64_t cs_bs, cs_ds;          /* (batch, dim, state_len), updated in place */
    const void *weight; int64_t w_ds, w_ks;
    const void *bias;                                  /* nullable */
    void *out;          int64_t out_bs;                /* (batch, dim) */
} conv1d_update_args;

typedef struct {
    int64_t batch, dim, dstate, n_groups;
    int32_t itype;              /* x, dt, z, out, B, C */
    int32_t stype;              /* state element type */
    int32_t dt_softplus;
    int32_t _pad0;
    void *state;        int64_t st_bs, st_ds, st_ns;   /* (batch, dim, dstate), updated in place */
    const void *x;      int64_t x_bs;                  /* (batch, dim) */
    const void *dt;     int64_t dt_bs;
    const float *A;     int64_t A_ds, A_ns;
    const void *B;      int64_t B_bs, B_gs;            /* (batch, n_groups, dstate), dstate unit-stride */
    const void *C;      int64_t C_bs, C_gs;
    const float *D;                                    /* nullable (dim,) */
    const void *z;      int64_t z_bs;                  /* nullable */
    const float *dt_bias;                              /* nullable (dim,) */
    void *out;          int64_t out_bs;
    /* nullable (batch,) on the device: row b updates state row state_batch_indices[b]; an index
     * < 0 (a padding slot) or >= state_batch skips the row (state untouched, out row zero) */
    const int32_t *state_batch_indices;
    int64_t state_batch;                               /* rows of state (used with the indices) */
} ssm_state_update_args;

/* Residual add + RMSNorm of the pre-norm stack (the fused Add -> Norm the reference runs with
 * fused_add_norm and residual_in_fp32, mamba_ssm/models/mixer_seq_simple.py:190-211):
 * residual_out = x + residual_in (residual_in NULL: x), out = residual_out * rsqrt(mean(
 * residual_out^2) + eps) * weight, computed in fp32 from residual_out as stored.  Rows of
 * `dim` elements (dim % 8 == 0, <= 4096) with unit stride and 16-byte-aligned row starts. */
typedef struct {
    int64_t rows, dim;
    int32_t itype;      /* x and out */
    int32_t rin_type;   /* residual_in: MSS_F32 or itype */
    int32_t rout_type;  /* residual_out: MSS_F32 or itype */
    int32_t wtype;      /* weight: MSS_F32 or itype */
    const void *x;              int64_t x_rs;
    const void *residual_in;    int64_t rin_rs;        /* nullable */
    void *residual_out;         int64_t rout_rs;
    const void *weight;
    void *out;                  int64_t out_rs;
    float *rstd;                                       /* nullable (rows,): 1 / rms per row */
    float eps;                  int32_t _pad;
} add_rms_norm_args;

/* dt_proj folded into the decode state update: dt[b, c] = sum_k weight[c, k] * dt_in[b, k],
 * rounded to itype (as the separate dt_proj GEMM stores it), then ssm_state_update with that
 * dt.  weight (dim, rank) contiguous in itype, rank % 8 == 0 and <= 256; dt_in rows of `rank`
 * elements of itype with 16-byte-aligned starts.  Needs dstate == 16 and the unit-stride,
 * 16-byte-aligned state / A / B / C rows of ssm_state_update's vector path. */
typedef struct {
    const void *dt_in;  int64_t dt_in_bs;   /* (batch, rank) */
    const void *weight; int64_t rank;       /* (dim, rank) */
} ssm_dtproj_args;

/* Workspace bytes ss_fwd / ss_bwd need for these arguments (0 means none). */
MSS_API int ss_fwd_workspace_size(const ss_fwd_args *a, int64_t *bytes);
MSS_API int ss_bwd_workspace_size(const ss_bwd_args *a, int64_t *bytes);

/* selective scan forward: writes out, out_z (iff z) and x.  (selective_scan.cpp:270-413) */
MSS_API int ss_fwd(const ss_fwd_args *a, void *stream);
/* selective scan backward: writes du, ddelta, dA, dB, dC, dD, ddelta_bias, dz, out_z.  (selective_scan.cpp:415-618) */
MSS_API int ss_bwd(const ss_bwd_args *a, void *stream);
/* Scratch bytes ss_bwd_noalloc owns per GPU (64 MiB).  A call is accepted when
 * ss_bwd_workspace_size() for its arguments is at most this.  For dstate <= 16 without P/Q
 * that is the fp32 dB / dC accumulators, 2 x batch x n_groups x dstate x round_up(seqlen, 4)
 * x 4 bytes (e.g. 32 x 1 x 16 x 16384 fits); dstate > 16 adds a per-step scratch of
 * batch x dim x 2 x round_up(seqlen, 4) x 4 bytes and P/Q a checkpoint array that also
 * grows with batch x dim x seqlen, so those calls reach the limit at much smaller sizes. */
#define MSS_BWD_NOALLOC_SCRATCH_BYTES (64ll << 20)

/* ss_bwd for callers that cannot allocate device memory: code whose device memory is owned
 * by another allocator (a framework's caching pool it may not bypass), or a host runtime
 * that forbids cudaMalloc in its steady state because cudaMalloc can synchronize the device
 * and has no latency bound.  No counterpart in the reference.  Same arguments and results as ss_bwd,
 * but `workspace` / `workspace_bytes` are ignored: the scratch is a static device array of
 * MSS_BWD_NOALLOC_SCRATCH_BYTES in this library's device image: it is placed on a GPU when
 * the library's module is loaded there (at the latest on the first call on that device) and
 * held until the process exits.  Sizes whose ss_bwd_workspace_size() exceeds it fail with
 * MSS_ERR_WORKSPACE.  The first call on a device looks the array's address up and caches it
 * per device (make that call before any stream capture; resetting the device afterwards,
 * e.g. cudaDeviceReset, is not supported).  Every call shares the array, so calls that
 * overlap on the GPU race.  It calls no allocator. */
MSS_API int ss_bwd_noalloc(const ss_bwd_args *a, void *stream);

/* depthwise causal conv1d (+SiLU) forward / backward (causal-conv1d API) */
MSS_API int conv1d_fwd(const conv1d_args *a, void *stream);
MSS_API int conv1d_bwd(const conv1d_args *a, void *stream);
/* one decode step of the conv: shifts conv_state left by one, appends x, writes out */
MSS_API int conv1d_update(const conv1d_update_args *a, void *stream);
/* one decode step of the SSM: updates state in place, writes out */
MSS_API int ssm_state_update(const ssm_state_update_args *a, void *stream);

/* Residual add + RMSNorm above (replaces the reference's fused layer_norm_fn(prenorm=True) call,
 * mamba_ssm/models/mixer_seq_simple.py:190-211, whose Triton source the export lacks). */
MSS_API int add_rms_norm(const add_rms_norm_args *a, void *stream);
/* sizeof(add_rms_norm_args), for binding-side layout checks. */
MSS_API int64_t add_rms_norm_args_size(void);

/* ssm_state_update with dt_proj folded in (the reference step's F.linear(dt, dt_proj.weight)
 * followed by selective_state_update, mamba_simplemotif.py:363-399); a->dt is not read. */
MSS_API int ssm_state_update_dtproj(const ssm_state_update_args *a, const ssm_dtproj_args *p, void *stream);

/* Motif regulariser over a batch of cc x cc fp32 matrices (the P_eff @ Q squares of the
 * coupled layers; replaces motifRegular.cal, motif/train_kpq_motif_pile_lm.py:405-466, one
 * matrix per call there).  Per matrix: soft edges w = sigmoid(amplitude (a^2 - bias)) off the
 * diagonal, the 13 three-node motif densities obs[1..13] (obs[0] = 0) divided by
 * cc (cc-1) (cc-2) / 6, and loss = sum over i with target[i] > 0 of weight[i] diff_i^2,
 * diff_i = obs[i+1] - target[i] (log_mse: log(max(obs, eps)) - log(max(target, eps))).
 * With dloss given, also da = dloss * d loss / d a.  3 <= cc <= 32; rows unit stride. */
typedef struct {
    int64_t n_mat, cc;
    const float *a;       int64_t a_ms;        /* (n_mat, cc, cc): matrix stride, row stride cc */
    const float *target;                       /* (13,) on the device; <= 0 entries are skipped */
    const float *weight;                       /* nullable (13,) on the device: all ones */
    float amplitude, bias;
    int32_t log_mse;      float log_eps;
    float *loss;                               /* (n_mat,) */
    float *obs;                                /* nullable (n_mat, 14) */
    const float *dloss;                        /* nullable (n_mat,): when given, da is written */
    float *da;            int64_t da_ms;       /* (n_mat, cc, cc) */
} motif_regular_args;

MSS_API int motif_regular(const motif_regular_args *a, void *stream);
/* sizeof(motif_regular_args), for binding-side layout checks. */
MSS_API int64_t motif_regular_args_size(void);

/* Message of the last failure on the calling thread ("" if none). */
MSS_API const char *ss_last_error(void);
/* Library version string. */
MSS_API const char *ss_version(void);
/* sizeof() of each argument struct, for binding-side layout checks:
 * out[0..4] = ss_fwd_args, ss_bwd_args, conv1d_args, conv1d_update_args, ssm_state_update_args */
MSS_API void ss_abi_struct_sizes(int64_t out[5]);

#ifdef __cplusplus
}
#endif
#endif /* MOTIF_SSM_H */
