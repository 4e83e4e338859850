/*
 * scope_b200 -- C ABI of the B200 (sm_100a) SCOPE sparse-attention hot path.
 *
 * Three parts, each replacing one piece of the reference (onetensor/scope):
 *   1. the pointer block-mask builder       <- SpectralBias.build_pointer_blockmask
 *                                              (model/attn_bias.py:623-874)
 *   2. the spectral bias inside the tile    <- the score_mod closure / qk_aug
 *                                              augmentation (scoped_medium.py:380-457)
 *   3. block-sparse causal attention fwd/bwd <- flex_attention(q, k, v, block_mask=,
 *                                              score_mod=, scale=) (scoped_medium.py:459-476)
 *
 * Conventions
 *   - Every pointer is a device pointer; every call takes the caller's stream
 *     and launches only on it.  No call synchronises the host.
 *   - The library allocates no device memory.  Buffers (including the
 *     workspace whose size scope_workspace_bytes() returns) belong to the caller.
 *   - Strides are in elements.  The last dimension of q/k/v/out/dO/dq/dk/dv
 *     is contiguous; head and token strides are free, so the [B,H,T,D] views
 *     of [B,T,H,D] tensors that the reference passes work unchanged.
 *   - Return value: SCOPE_OK (0) or a negative scope_status; scope_error_string()
 *     names it.  Kernels that find a bad index or give up a bounded wait set
 *     bits in the optional `err_flag` word (read it after the stream drains).
 */
#ifndef SCOPE_B200_H
#define SCOPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *scope_stream_t; /* == cudaStream_t */

typedef enum scope_status {
    SCOPE_OK = 0,
    SCOPE_ERR_INVALID = -1,     /* bad shape, size or knob (ValueError on the Python side) */
    SCOPE_ERR_DTYPE = -2,       /* unsupported dtype combination */
    SCOPE_ERR_ALIGN = -3,       /* pointer or stride not aligned as required */
    SCOPE_ERR_CUDA = -4,        /* a CUDA launch or runtime call failed */
    SCOPE_ERR_UNSUPPORTED = -5, /* device is not sm_100 or configuration unsupported */
    SCOPE_ERR_WORKSPACE = -6    /* workspace missing or too small */
} scope_status;

typedef enum scope_dtype { SCOPE_F32 = 0, SCOPE_BF16 = 1 } scope_dtype;

typedef enum scope_bias_mode {
    SCOPE_BIAS_NONE = 0,     /* plain block-sparse attention */
    SCOPE_BIAS_SCORE_MOD = 1,/* exact score_mod semantics (scoped_medium.py:425-457) */
    SCOPE_BIAS_QK_AUG = 2    /* qk_aug augmentation (scoped_medium.py:380-423), the reference default */
} scope_bias_mode;

typedef enum scope_gate { SCOPE_GATE_NONE = 0, SCOPE_GATE_SOFTPLUS = 1, SCOPE_GATE_RELU = 2 } scope_gate;

/* device error-word bits */
#define SCOPE_DEVERR_INDEX   0x1  /* a kv / q block index outside [0, QB) was skipped */
#define SCOPE_DEVERR_TIMEOUT 0x2  /* a bounded pipeline wait gave up */
#define SCOPE_DEVERR_SHAPE   0x4  /* a list longer than its buffer was truncated */

/* ------------------------------------------------------------------------ */
/* 1. pointer block-mask builder                                              */
/* ------------------------------------------------------------------------ */

/* Document / reset starts and document ranges per block.
 * Replaces model/attn_bias.py:681-709 (doc_start_blk_ptr / doc_start_blk_local)
 * and adds the per-block document min/max used to classify attention tiles.
 * out: int32 [4, QB] = {doc_start_blk_ptr, doc_start_blk_local, doc_min, doc_max}.
 * docs may be NULL (one document). */
int scope_block_info(const int32_t *docs, int32_t T, int32_t block_size,
                     int32_t doc_clamp, int32_t reset_active, int32_t reset_len,
                     int32_t *out, scope_stream_t stream);

typedef struct ScopeMaskArgs {
    int32_t H, QB, M, block_size;
    /* Pointer source, exactly one of:
     *  (a) selection: Gumbel top-M over causal candidate blocks kb <= qb of
     *      scores = sel_logits / sel_tau + sel_gumbel   (both [H,QB,>=QB] f32)
     *  (b) delta_rep [H,QB,M] f32: the representative Δ* (model/attn_bias.py:714-719) */
    const float *sel_logits, *sel_gumbel;
    int64_t sel_head_stride, sel_row_stride;
    float sel_tau;
    const float *delta_rep;
    int64_t delta_head_stride, delta_row_stride, delta_m_stride;
    /* budget logits of each peak [H,QB,M] (model/attn_bias.py:716) */
    const float *budget_rep;
    int64_t budget_head_stride, budget_row_stride, budget_m_stride;
    /* Gumbel peak masking (model/attn_bias.py:763-777): g [H,QB,M] contiguous, k, tau; NULL = off */
    const float *peak_gumbel;
    int32_t gumbel_k;
    float gumbel_tau;
    /* [4,QB] from scope_block_info */
    const int32_t *block_info;
    /* knobs, already resolved as the reference resolves them */
    int32_t local_blocks;  /* min(max(1, L), QB) */
    int32_t half_blocks;   /* max(0, ptr_half_blocks) */
    int32_t half_active;   /* schedule cap (_pointer_half_blocks_active) */
    int32_t ptr_enabled;   /* _pointer_mask_active */
    int32_t global_max;    /* min(pointer_global_blocks, QB) */
    int32_t global_active; /* clamp(active global blocks, 0, global_max) */
    int32_t radius_mode;   /* 0 = "fixed", 1 = "pi" */
    int32_t budget_rem;    /* integer radius budget (model/attn_bias.py:724-734) */
    float budget_temp;     /* max(pointer_budget_temp, 1e-6) */
    /* outputs */
    int32_t *kv_num;       /* [H,QB] */
    int32_t *kv_indices;   /* [H,QB,kv_stride] */
    int32_t kv_stride;     /* >= max_kv (compact) or == QB with flex_padded */
    int32_t flex_padded;   /* 1: the reference's QB-column layout (model/attn_bias.py:854-862) */
    uint32_t *q_bitmap;    /* optional [H,QB,ceil(QB/32)]: bit qb of row (h,kb) = kb visible from qb */
    int32_t *r_m_out;      /* optional [H,QB,M] radii */
    int32_t *centres_out;  /* optional [H,QB,M] pointer centres */
    int32_t *stats;        /* optional: kv_unique_hist[max_kv+1] | radius_hist[half+1] |
                              extra_sum_hist[max(1,half*M)+1] | zero-radius count (int32, accumulated) */
    int32_t *err_flag;     /* optional device error word */
} ScopeMaskArgs;

/* Number of list entries before de-duplication: L + M*(2p+1) + G (p > 0) or L + M + G. */
int32_t scope_mask_max_kv(int32_t local_blocks, int32_t M, int32_t half_blocks, int32_t global_max);

/* Builds the pointer block mask.  Replaces SpectralBias.build_pointer_blockmask
 * (model/attn_bias.py:623-874) minus BlockMask.from_kv_blocks' dense transpose,
 * which the q_bitmap replaces.  The caller zeroes q_bitmap and stats. */
int scope_mask_build(const ScopeMaskArgs *args, scope_stream_t stream);

/* torch BlockMask q-side layout from the bitmap: q_num [H,KB], q_indices [H,KB,QB]
 * (valid q-blocks ascending, then the rest ascending) -- what
 * BlockMask.from_kv_blocks -> _transpose_ordered produces
 * (torch/nn/attention/flex_attention.py:412-415).  q_indices may be NULL. */
int scope_mask_transpose(const uint32_t *q_bitmap, int32_t H, int32_t QB,
                         int32_t *q_num, int32_t *q_indices, scope_stream_t stream);

/* Kernel tiles of a coarse mask (block_size 2*bs -> bs; the attention kernels
 * tile at 128, config C5 builds its mask at 256).  No counterpart function in
 * the reference: torch's flex kernel likewise runs a BLOCK_SIZE-256 mask on
 * smaller tiles internally (SPARSE_Q/KV_BLOCK_SIZE multiples of its BLOCK_M /
 * BLOCK_N, torch/_inductor/kernel/flex/templates/flex_attention.py.jinja:32-33).  Fine q block 2qb+s gets fine
 * kv blocks 2kb, 2kb+1 of each listed kb, minus those wholly in its causal
 * future; out lists [H, 2QB, kv_stride_out >= 2*kv_stride]; the caller zeroes
 * q_bitmap_out [H, 2QB, ceil(2QB/32)].  Bad indices are skipped and set
 * SCOPE_DEVERR_INDEX in err_flag (may be NULL). */
int scope_mask_refine(const int32_t *kv_num, const int32_t *kv_indices, int32_t H, int32_t QB,
                      int32_t kv_stride, int32_t *kv_num_out, int32_t *kv_indices_out,
                      int32_t kv_stride_out, uint32_t *q_bitmap_out, int32_t *err_flag,
                      scope_stream_t stream);

/* q-side bitmap [H, QB, ceil(QB/32)] of a mask given only its kv lists: the
 * q side of a torch BlockMask handed to the attention drop-in, which the
 * reference builds by BlockMask.from_kv_blocks' dense transpose
 * (model/attn_bias.py:867-874; torch/nn/attention/flex_attention.py:412-415).
 * Bit qb of row (h, kb) is set for each kb among the first kv_num[h, qb]
 * entries of row (h, qb) of kv_indices [H, QB, kv_stride].  The caller zeroes
 * q_bitmap.  Indices outside [0, QB) are skipped (SCOPE_DEVERR_INDEX); counts
 * outside [0, kv_stride] are clamped (SCOPE_DEVERR_SHAPE). */
int scope_mask_bitmap_from_lists(const int32_t *kv_num, const int32_t *kv_indices, int32_t H, int32_t QB,
                                 int32_t kv_stride, uint32_t *q_bitmap, int32_t *err_flag,
                                 scope_stream_t stream);

/* ------------------------------------------------------------------------ */
/* 2. spectral bias helpers                                                   */
/* ------------------------------------------------------------------------ */

/* bf16 trig tables cos/sin(fp32(w_k*d)), d in [0,L)  (model/attn_bias.py:326-340).
 * omegas [K] f32; cos_out/sin_out [K,L] bf16 (raw 16-bit). */
int scope_trig_tables(const float *omegas, int32_t K, int32_t L,
                      uint16_t *cos_out, uint16_t *sin_out, scope_stream_t stream);

/* Augmented dims of the qk_aug mode (scoped_medium.py:380-421):
 *   q_aug[h,t] = s*[A*cos_t + B*sin_t, A*sin_t - B*cos_t, (-slope)], zero padded to d_aug,
 *   k_aug[t]   = s*[cos_t, sin_t, (t)], zero padded,  s = sqrt(beta/scale),
 * rounded to `dtype`.  coeff [H,T,K] f32 contiguous; slope [H,T] or NULL;
 * q_aug [H,T,d_aug]; k_aug [T,d_aug] (head independent). */
int scope_qk_aug_prepare(const float *coeff_cos, const float *coeff_sin, const float *slope,
                         const uint16_t *cos_tab, const uint16_t *sin_tab, int32_t tab_len,
                         int32_t H, int32_t T, int32_t K, int32_t d_aug, float beta, float scale,
                         int32_t dtype, void *q_aug, void *k_aug, scope_stream_t stream);

/* The coefficient block of SpectralBias.forward (model/attn_bias.py:306-324,
 * 419-478): the per-query MLP (two bf16 linears with SiLU, weights shared by
 * all heads or one set per head) and the mixture that produces the bias
 * inputs.  Outputs as the reference returns them, batch 1.  T % 128 == 0,
 * D == 64, hidden == 128, K in {6, 8, 16}, M in {2, 4, 8}. */
typedef struct ScopeCoeffArgs {
    int32_t H, T, D, hidden, K, M;
    int32_t use_slope, subtract_b0;
    const void *q;                    /* bf16 [H,T,D] view: element strides q_sh, q_st, last dim contiguous */
    int64_t q_sh, q_st;
    int32_t w_heads;                  /* 1 (share_across_heads) or H */
    const void *w1, *b1;              /* bf16 [w_heads,hidden,D], [w_heads,hidden] */
    const void *w2, *b2;              /* bf16 [w_heads,n_out,hidden], [w_heads,n_out]; n_out = 5M + use_slope */
    const float *omegas, *log_omegas; /* [K], and their fp32 natural logs */
    float delta_cap;                  /* clamp(delta_star_max_active, 0, T-1) */
    float logw_min, logw_max, c_scale, width_min, width_max, eps;
    float *coeff_cos, *coeff_sin;     /* [H,T,K] */
    float *slope, *b0;                /* [H,T] (zeros when the term is off) */
    float *delta_star, *pi, *budget_logits;   /* [H,T,M] */
    float *delta_main, *width;        /* [H,T] */
    uint16_t *mlp_out;                /* optional bf16 [H,T,n_out]: the MLP output y */
    float *omega_reg;                 /* optional [H,T]: sum_m sum_k omega_k^2 a_mk^2 (a normalised over k),
                                         the per-token term of the training penalty reg_omega */
    int32_t *err_flag;                /* optional device error word */
} ScopeCoeffArgs;
int scope_spectral_coeffs(const ScopeCoeffArgs *args, scope_stream_t stream);

/* Backward of the coefficient block up to the MLP output: dL/dy [H,T,n_out]
 * f32 from the MLP output y (mlp_out of the forward) and the upstream
 * gradients of the block's outputs, each optional (NULL = zero).  The MLP's
 * own backward follows (scope_spectral_mlp_bwd). */
typedef struct ScopeCoeffBwdArgs {
    int32_t H, T, K, M, use_slope, subtract_b0;
    const uint16_t *mlp_out;                       /* bf16 [H,T,n_out] */
    const float *dcoeff_cos, *dcoeff_sin;          /* [H,T,K] */
    const float *db0, *dslope, *ddelta_main, *dwidth;   /* [H,T] */
    const float *ddelta_star, *dpi, *dbudget_logits;    /* [H,T,M] */
    const float *domega_reg;                       /* [H,T]: gradient of the omega_reg output */
    const float *omegas, *log_omegas;              /* [K] */
    float delta_cap, logw_min, logw_max, c_scale, width_min, width_max, eps;
    float *dy;                                     /* [H,T,n_out], or NULL with dy_bf16 */
    void *dy_bf16;                                 /* or bf16 [H,T,dy_ld], zero padded past n_out: the
                                                      rounding the reference's bf16 MLP backward applies,
                                                      in the layout scope_spectral_mlp_bwd reads */
    int32_t dy_ld;                                 /* row stride of dy_bf16: multiple of 8, >= n_out */
    int32_t *err_flag;                             /* optional device error word */
} ScopeCoeffBwdArgs;
int scope_spectral_coeffs_bwd(const ScopeCoeffBwdArgs *args, scope_stream_t stream);

/* Backward of the coefficient block's MLP with weights shared by the heads:
 * from dL/dy to dL/dq, dL/dW1, dL/db1 and dL/dW2 (dL/db2 is the column sum
 * of dy).  Replaces the autograd backward of SpectralBias._mlp_forward
 * (model/attn_bias.py:306-318): linear(q, W1, b1) -> silu -> linear(., W2, b2)
 * in bf16, with the same roundings (each linear's output, the SiLU and its
 * backward rounded to bf16).  The weight gradients are fp32 sums the caller
 * zeroes; the reference's are those sums rounded to bf16. */
typedef struct ScopeCoeffMlpBwdArgs {
    int32_t H, T, n_out;              /* T % 128 == 0, n_out <= 96, hidden 128, head dim 64 */
    const void *q;                    /* bf16 [H,T,64] view (last dim contiguous) */
    int64_t q_sh, q_st;
    const void *w1, *b1, *w2;         /* bf16 [128,64], [128], [n_out,128] */
    const void *dy;                   /* bf16 [H*T, NP]: dL/dy, zero columns from n_out to NP = n_out
                                         rounded up to 16 */
    void *dq;                         /* bf16 [H,T,64] contiguous */
    float *dw1, *db1, *dw2;           /* fp32 [128,64], [128], [n_out,128]: sums added */
    int32_t *err_flag;                /* optional device error word */
} ScopeCoeffMlpBwdArgs;
int scope_spectral_mlp_bwd(const ScopeCoeffMlpBwdArgs *args, scope_stream_t stream);

/* Self-test of the bounded-wait failure path (no counterpart in the
 * reference): one CTA allocates TMEM, waits at most limit_us microseconds
 * (<= 1 s) on an mbarrier nothing arrives on, sets SCOPE_DEVERR_TIMEOUT in
 * *err_flag (device memory), frees TMEM and exits. */
int scope_selftest_wait_timeout(int32_t *err_flag, uint32_t limit_us, scope_stream_t stream);

/* Self-test of the FMA-pipe exponential the attention forward uses for a
 * share of its exponentials (no counterpart in the reference): y[i] = 2^x[i]
 * for n float32 values in device memory, x <= 127 (inputs below -125 give
 * about 2^-125). */
int scope_selftest_exp2_fma(const float *x, float *y, int32_t n, scope_stream_t stream);

/* ------------------------------------------------------------------------ */
/* 3. block-sparse attention                                                  */
/* ------------------------------------------------------------------------ */

typedef struct ScopeAttnArgs {
    int32_t H, T, D, block_size;     /* D == 64; block_size == 128 (or 64/256 on the CUDA-core path) */
    int32_t dtype;                    /* scope_dtype of q,k,v,out,dout,dq,dk,dv */
    const void *q, *k, *v;
    int64_t q_sh, q_st, k_sh, k_st, v_sh, v_st;   /* head / token strides */
    void *out;
    int64_t o_sh, o_st;
    float *lse;                       /* [H,T] natural-log logsumexp (written by fwd, read by bwd) */
    /* block mask (kv side for fwd/dQ, q side for dK/dV) */
    const int32_t *kv_num;            /* [H,QB] */
    const int32_t *kv_indices;        /* [H,QB,kv_stride] */
    int32_t kv_stride;
    const uint32_t *q_bitmap;         /* [H,QB,ceil(QB/32)] (backward) */
    const int32_t *block_info;        /* [4,QB] (rows 2,3: doc min/max) or NULL */
    const int32_t *docs;              /* [T] document ids or NULL (causal only) */
    float scale;
    /* spectral bias */
    int32_t bias_mode;                /* scope_bias_mode */
    int32_t K;
    const float *coeff_cos, *coeff_sin;           /* [H,T,K] */
    const uint16_t *cos_tab, *sin_tab;            /* [K,tab_len] bf16 */
    int32_t tab_len;
    const float *b0, *slope, *delta_main, *width; /* [H,T] each or NULL */
    int32_t gate;                     /* scope_gate */
    float beta, gate_lambda, gate_tau;
    const void *q_aug, *k_aug;        /* qk_aug: from scope_qk_aug_prepare (with the slope column when
                                         there is a slope).  score_mod: optional; from scope_qk_aug_prepare
                                         WITHOUT the slope column (slope = NULL), they put the closure's
                                         Fourier sum on the tensor cores (bf16, 128-token blocks), the
                                         backward reusing what the forward was given */
    int32_t d_aug;                    /* multiple of 16: qk_aug 16..64; score_mod 16 * ceil(2K / 16) with
                                         q_aug, else 0 (CUDA cores); 0 for no bias */
    /* backward only */
    const void *dout;
    int64_t do_sh, do_st;
    void *dq, *dk, *dv;
    int64_t dq_sh, dq_st, dk_sh, dk_st, dv_sh, dv_st;
    float *dcoeff_cos, *dcoeff_sin;   /* [H,T,K] or NULL */
    float *db0, *dslope, *ddelta_main, *dwidth; /* [H,T] or NULL */
    void *workspace;
    size_t workspace_bytes;
    int32_t flags;                    /* SCOPE_FLAG_* */
    int32_t *err_flag;                /* optional device error word */
} ScopeAttnArgs;

/* ScopeAttnArgs.flags: run the CUDA-core kernels even where the tensor-core
 * kernels apply (cross-checking one implementation against the other). */
#define SCOPE_FLAG_CUDA_CORES 0x1

/* Forward: out and lse.  Replaces the flex_attention forward at
 * scoped_medium.py:459-466 (score_mod) and :422 (qk_aug). */
int scope_attn_fwd(const ScopeAttnArgs *args, scope_stream_t stream);

/* Backward: dq, dk, dv and the gradients of the captured bias tensors
 * (dcoeff_cos/dcoeff_sin, db0, dslope, ddelta_main, dwidth when given).
 * Replaces flex_attention's autograd backward (scoped_medium.py:2520). */
int scope_attn_bwd(const ScopeAttnArgs *args, scope_stream_t stream);

/* Workspace bytes scope_attn_bwd needs for these arguments. */
size_t scope_workspace_bytes(const ScopeAttnArgs *args);

/* Teacher block mass.  Replaces the teacher's dense loop at
 * scoped_medium.py:1793-1819: for each head h and 128-row query block qb,
 * the dense document-causal softmax of (q k^T + q_aug k_aug^T) * scale over
 * all keys, summed over the block's rows and over the keys of each kv block
 * kb, into mass[h, qb, kb] ([H, QB, QB] float32; zero above the diagonal;
 * each (h, qb) row sums to 128).  Reads q, k, the strides, docs, block_info
 * (scope_block_info with doc_clamp 1 and no reset), scale, H, T, D (64),
 * block_size (128), dtype (bf16), err_flag and, with bias_mode
 * SCOPE_BIAS_QK_AUG, q_aug [H, T, d_aug] and k_aug [T, d_aug] (the teacher's
 * q_pos / k_pos, zero-padded to d_aug = 16, 32, 48 or 64 columns); the other
 * fields are ignored.  Documents are runs of equal ids (the reference's
 * cumulative count of separator tokens).  Tensor cores only:
 * SCOPE_ERR_UNSUPPORTED off sm_100. */
int scope_block_mass(const ScopeAttnArgs *args, float *mass, scope_stream_t stream);

/* Backward for callers that cannot allocate or pass a workspace (a plugin host
 * that owns all device memory and gives the library no allocator, a binding
 * without a device allocator).  No counterpart in the reference.
 * Same arguments and results as scope_attn_bwd; args->workspace is ignored and
 * the scratch lives in one file-scope device array of
 * scope_static_scratch_bytes() bytes (32 MiB) that every GPU loading the
 * library holds until exit.  Problems whose scratch exceeds it
 * (scope_workspace_bytes(args) > 32 MiB) are rejected with
 * SCOPE_ERR_WORKSPACE.  It calls no allocator.  Its first call on a device
 * looks up the array's device address (make that first call before any stream
 * capture).  All calls share the array: calls whose kernels overlap on the GPU
 * (different streams, or several devices' work on one context) race on it.  The device address is kept per device: cudaDeviceReset() between
 * calls is not supported. */
int scope_attn_bwd_static_scratch(const ScopeAttnArgs *args, scope_stream_t stream);

/* Size in bytes of the array scope_attn_bwd_static_scratch uses. */
size_t scope_static_scratch_bytes(void);

/* Name of a scope_status value. */
const char *scope_error_string(int status);

/* Struct layout self-check for bindings: which = 0 (ScopeMaskArgs), 1
 * (ScopeAttnArgs), 2 (ScopeCoeffArgs), 3 (ScopeCoeffBwdArgs) or 4
 * (ScopeCoeffMlpBwdArgs); what = 0 (sizeof) or 1 (offset of the last field,
 * err_flag). */
size_t scope_abi_layout(int which, int what);

/* Number of kernels this library has launched in this process (all devices).
 * Host-side counter used by benchmarks to report their kernel launches. */
uint64_t scope_launch_count(void);

/* 1 if the current device can run the tensor-core (sm_100a) kernels. */
int scope_device_supported(void);

#ifdef __cplusplus
}
#endif
#endif /* SCOPE_B200_H */
