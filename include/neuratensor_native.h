/*
 * neuratensor_native.h -- C ABI of libneuratensor_native.so
 *
 * B200 (sm_100a) kernels for the FusedSpikeBlock inference path of
 * NeuraTensor 4.0.4.  Every entry point takes plain device pointers, sizes
 * and element strides, runs asynchronously on the given CUDA stream and
 * returns an nt_status code; it never aborts the process.  The caller owns
 * every buffer: inputs, outputs, state buffers and workspaces (sized with
 * the *_workspace_bytes queries).
 *
 * Concurrency: calls on different streams may run concurrently when they use
 * different workspaces and outputs, with two exceptions that are shared
 * per device: nt_rmsnorm_in_proj_noalloc's static scratch (overlapping calls
 * of that entry point race), and the device error word that every kernel
 * with a bounded wait may set (nt_get_error_flag reports the union of all
 * streams' flags since it was last cleared).  The launch counter is a process
 * total.
 *
 * Reference interfaces replaced (paths inside the NeuraTensor source tree):
 *   nt_lif_scan            LIFLayer.forward            neuratensor/core/snn.py:264-312
 *                          (_lif_sequential_scan :167-182, _lif_single_step :64-75)
 *   nt_selective_scan      SelectiveSSMLayer._discretize + _scan_sequential / _scan_single_step
 *                                                      neuratensor/core/ssm.py:106-139,145-221
 *   nt_ssm_forward         SelectiveSSMLayer.forward   neuratensor/core/ssm.py:313-349
 *   nt_sparse_out_proj     FusedSpikeBlock._sparse_out_proj  neuratensor/core/fused.py:149-165
 *   nt_rmsnorm_in_proj     FusedSpikeBlock.norm + in_proj    neuratensor/core/fused.py:118-119
 *   nt_block_forward       FusedSpikeBlock.forward     neuratensor/core/fused.py:101-147
 *   nt_window_attention    SlidingWindowAttention RoPE + SDPA neuratensor/core/model.py:148-178
 *   nt_attention_forward   SlidingWindowAttention.forward neuratensor/core/model.py:148-181
 *   nt_embedding           NeuraTensorModel.embedding  neuratensor/core/model.py:258
 *   nt_lm_head             NeuraTensorModel.norm + lm_head neuratensor/core/model.py:283-284
 *   nt_greedy_tokens       top-k = 1 sampling in NeuraTensorModel.generate model.py:344-359
 *   nt_lif_ssm_fused       LIF spikes driving the selective scan with given dt/B/C
 *                          (snn.py:167-182 feeding ssm.py:106-139,184-221)
 *
 * Layouts: activations are row-major [rows, channels] with unit channel
 * stride; "rows" are (batch, time) pairs in batch-major order.  Weights are
 * the nn.Linear weights, row-major [out_features, in_features].
 */
#ifndef NEURATENSOR_NATIVE_H
#define NEURATENSOR_NATIVE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NT_ABI_VERSION 1

#if defined(__GNUC__)
#define NT_API __attribute__((visibility("default")))
#else
#define NT_API
#endif

typedef enum {
    NT_F32 = 0,   /* float32                                   */
    NT_BF16 = 1,  /* bfloat16                                  */
    NT_U8 = 2     /* uint8 (spike output of nt_lif_ssm_fused)  */
} nt_dtype;

typedef enum {
    NT_OK = 0,
    NT_ERR_ARG = 1,        /* bad shape, stride, null pointer or alignment          */
    NT_ERR_DTYPE = 2,      /* unsupported dtype combination                          */
    NT_ERR_ARCH = 3,       /* device is not sm_100                                   */
    NT_ERR_CUDA = 4,       /* CUDA runtime / launch error                            */
    NT_ERR_TIMEOUT = 5,    /* a bounded device-side wait expired (see error flag)    */
    NT_ERR_WORKSPACE = 6   /* workspace pointer null or smaller than required        */
} nt_status;

/* Library / device queries ------------------------------------------------ */
NT_API int nt_abi_version(void);
/* Message of the last failing call on this host thread ("" if none). */
NT_API const char* nt_last_error(void);
/* NT_OK when `device` is an sm_100 GPU this build can run on. */
NT_API int nt_device_supported(int device);
/* Reads (and optionally clears) the device error word that kernels set when
 * a bounded wait expires.  Synchronises the device.  *flags == 0 means no
 * kernel reported an error. */
NT_API int nt_get_error_flag(int device, unsigned* flags, int clear);
/* Checks the bounded-wait path (no counterpart in the reference, whose code
 * never waits on the device): one CTA waits on a barrier that nothing
 * completes, gives up after limit_ns of wall time (0..1e9), sets bit 16 of the
 * device error word and returns normally.  Every pipeline wait in this
 * library's kernels is bounded the same way (2 s), so a stalled producer shows
 * up as a flag and an error status instead of a hung GPU. */
NT_API int nt_bounded_wait_check(int64_t limit_ns, void* stream);
/* Kernels this library has launched in this process (all devices, all host
 * threads).  Reading it before and after a call counts that call's launches.
 * No counterpart in the reference, which launches no kernels of its own. */
NT_API unsigned long long nt_launch_count(void);

/* (a) LIF membrane recurrence -- LIFLayer.forward (snn.py:264-312).
 * Per channel c and step t:  V = beta[c]*V + x[t,c]  (a product then a sum,
 * each rounded to `dtype`), S = (V >= threshold[c]), V = V - threshold[c]*S.
 * x: [B,T,C] with element strides (x_sb, x_st, 1); spikes written as 0/1 in
 * `dtype` with strides (s_sb, s_st, 1).  beta, threshold: [C] in `dtype`.
 * mem_in: [B,C] in `dtype` or NULL for zeros (snn.py:286-287); mem_out: [B,C].
 * spike_count: optional device uint64 that is incremented by the number of
 * spikes (caller zeroes it). */
NT_API int nt_lif_scan(int dtype, int64_t B, int64_t T, int64_t C,
                const void* x, int64_t x_sb, int64_t x_st,
                const void* beta, const void* threshold,
                const void* mem_in, void* mem_out,
                void* spikes, int64_t s_sb, int64_t s_st,
                unsigned long long* spike_count, void* stream);

/* (b) selective scan -- SelectiveSSMLayer._discretize + _scan_sequential
 * (ssm.py:106-139,184-221).  A = -exp(log_A); A_bar = exp(A*dt);
 * B_bar = (A_bar-1)/A*B (dt*B where |A| < 1e-6); h = A_bar*h + B_bar*u;
 * y = sum_n C[n]*h[n] + D*u.  If gate != NULL the output is y*silu(gate)
 * (fused.py:130).  u, dt, gate, y: [B,T,d] contiguous in `dtype`;
 * Bm, Cm: [B,T,N] contiguous in `dtype`; log_A: [d,N], D: [d] in `dtype`.
 * state_in/state_out: [B,d,N] in `state_dtype` (state_in NULL = zeros); the
 * recurrence itself runs in float32.  d_state N <= 256. */
NT_API int nt_selective_scan(int dtype, int state_dtype, int64_t B, int64_t T, int64_t d, int64_t N,
                      const void* u, const void* dt, const void* Bm, const void* Cm,
                      const void* log_A, const void* D, const void* gate,
                      const void* state_in, void* state_out, void* y, void* stream);

/* SelectiveSSMLayer.forward (ssm.py:313-349): B = u W_B^T, C = u W_C^T,
 * dt = softplus(u W_dt^T + b_dt), then the scan above.  W_proj is the packed
 * projection weight [d + 2N, d] = rows of W_dt, then W_B, then W_C.
 * Workspace: nt_ssm_workspace_bytes(). */
NT_API int64_t nt_ssm_workspace_bytes(int dtype, int64_t B, int64_t T, int64_t d, int64_t N);
NT_API int nt_ssm_forward(int dtype, int state_dtype, int64_t B, int64_t T, int64_t d, int64_t N,
                   const void* u, const void* W_proj, const void* b_dt,
                   const void* log_A, const void* D,
                   const void* state_in, void* state_out, void* y,
                   void* workspace, int64_t workspace_bytes, void* stream);

/* (c) spike-sparse out_proj -- FusedSpikeBlock._sparse_out_proj
 * (fused.py:149-165).  o: [M,K], spikes: [M,K] (0/1), W: [Nout,K], out:
 * [M,Nout], all `dtype`, contiguous.  A row is active when any spike in it
 * is non-zero.  If 2*n_active > M every row is projected (dense branch);
 * otherwise only active rows are projected and inactive rows are zero.
 * n_active_out: optional device int64 receiving n_active.
 * Workspace: nt_sparse_out_proj_workspace_bytes(). */
NT_API int64_t nt_sparse_out_proj_workspace_bytes(int dtype, int64_t M, int64_t K, int64_t Nout);
NT_API int nt_sparse_out_proj(int dtype, int64_t M, int64_t K, int64_t Nout,
                       const void* o, const void* spikes, const void* W, void* out,
                       long long* n_active_out,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* (d) RMSNorm + in_proj -- fused.py:118-119.  xn = RMSNorm(x) (eps = float32
 * machine epsilon, as nn.RMSNorm with eps=None), [h | gate] = xn W_in^T.
 * x: [M,dm]; gamma: [dm]; W_in: [2*di, dm]; h, gate: [M,di], all `dtype`.
 * Workspace: nt_rmsnorm_in_proj_workspace_bytes(). */
NT_API int64_t nt_rmsnorm_in_proj_workspace_bytes(int dtype, int64_t M, int64_t dm, int64_t di);
NT_API int nt_rmsnorm_in_proj(int dtype, int64_t M, int64_t dm, int64_t di,
                       const void* x, const void* gamma, const void* W_in,
                       void* h, void* gate,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* RMSNorm + in_proj without a workspace (no counterpart in the reference).
 * Same computation and arguments as nt_rmsnorm_in_proj, minus the workspace:
 * the normalised activations go to a scratch array the library itself holds
 * in device memory (nt_noalloc_scratch_bytes() bytes per device, 32 MiB), for
 * callers that cannot allocate device memory, e.g. serving runtimes that
 * reserve HBM at start-up and forbid cudaMalloc afterwards.  Requires
 * M*d_model*sizeof(dtype) <= nt_noalloc_scratch_bytes() (else NT_ERR_ARG).
 * The first call on a device, made with that device current, looks up the
 * array's address; make it before any stream capture.  The address is cached
 * for the life of the process and does not survive a device reset
 * (cudaDeviceReset or a re-created primary context): do not call this entry
 * point after one.  Calls share the array: calls that overlap on the GPU race. */
NT_API size_t nt_noalloc_scratch_bytes(void);
NT_API int nt_rmsnorm_in_proj_noalloc(int dtype, int64_t M, int64_t dm, int64_t di,
                       const void* x, const void* gamma, const void* W_in,
                       void* h, void* gate, void* stream);

/* SlidingWindowAttention.forward (model.py:148-181), bf16, head_dim 64 or 128:
 * out = o_proj(attention(qkv(RMSNorm(x)))) + x, with the attention as in
 * nt_window_attention.  x, out: [B,T,dm]; norm_w: [dm]; W_qkv: [3*dm, dm];
 * W_o: [dm, dm]; cos_t, sin_t: [T, dm/n_heads] rotary tables.
 * Workspace: nt_attention_workspace_bytes(). */
NT_API int64_t nt_attention_workspace_bytes(int dtype, int64_t B, int64_t T, int64_t dm);
NT_API int nt_attention_forward(int dtype, int64_t B, int64_t T, int64_t dm, int64_t n_heads, int64_t window,
                                const void* x, const void* norm_w, const void* W_qkv, const void* W_o,
                                const void* cos_t, const void* sin_t, void* out,
                                void* workspace, int64_t workspace_bytes, void* stream);

/* Embedding gather -- NeuraTensorModel.embedding (model.py:258, nn.Embedding):
 * out[r, :] = W[ids[r], :] for r < M.  ids: [M] int64; W: [vocab, dm]; out:
 * [M, dm], both `dtype`.  An id outside [0, vocab) yields a zero row and sets
 * a flag in the device error word (nt_get_error_flag), where the reference
 * raises IndexError. */
NT_API int nt_embedding(int dtype, int64_t M, int64_t dm, int64_t vocab, const int64_t* ids, const void* W,
                        void* out, void* stream);

/* Greedy next tokens -- NeuraTensorModel.generate with top_k = 1, temperature 1,
 * top_p 1 and no repetition penalty (model.py:344-359): per row of logits
 * [B, vocab] (row stride ld elements, `dtype`), the reference keeps the entries
 * equal to the maximum and samples among them; this picks the
 * floor(u[r] * ties)-th tied index in index order, u: [B] float32 in [0, 1).
 * tokens: [B] int64 device output. */
NT_API int nt_greedy_tokens(int dtype, int64_t B, int64_t vocab, const void* logits, int64_t ld, const float* u,
                            int64_t* tokens, void* stream);

/* Final RMSNorm + tied lm_head -- NeuraTensorModel.norm + lm_head
 * (model.py:283-284): logits = RMSNorm(x) W^T, logits in `dtype` (bf16 logits
 * in bf16 mode).  x: [M, dm]; gamma: [dm]; W: [vocab, dm] (the embedding
 * matrix when tied); logits: [M, vocab].  Workspace: nt_lm_head_workspace_bytes(). */
NT_API int64_t nt_lm_head_workspace_bytes(int dtype, int64_t M, int64_t dm, int64_t vocab);
NT_API int nt_lm_head(int dtype, int64_t M, int64_t dm, int64_t vocab, const void* x, const void* gamma,
                      const void* W, void* logits, void* workspace, int64_t workspace_bytes, void* stream);

/* FusedSpikeBlock.forward in eval mode (fused.py:101-147):
 *   out = sparse_out_proj(SSM(LIF(in_proj(RMSNorm(x))_h)) * silu(gate)) * out_scale + x
 * x, out: [B,T,dm]; weights as in the module (W_proj packed as above);
 * beta = sigmoid(beta_logit) and threshold in `dtype`, [di];
 * mem_in/mem_out: [B,di] in `dtype` (mem_in NULL = zeros);
 * state_in/state_out: [B,di,N] in `state_dtype` (state_in NULL = zeros);
 * spike_count: device uint64, incremented by this block's spike count;
 * sparse: 1 = inference sparse out_proj (fused.py:133-134), 0 = dense.
 * Workspace: nt_block_workspace_bytes(). */
NT_API int64_t nt_block_workspace_bytes(int dtype, int64_t B, int64_t T, int64_t dm, int64_t di, int64_t N);
NT_API int nt_block_forward(int dtype, int state_dtype, int64_t B, int64_t T, int64_t dm, int64_t di,
                     int64_t N,
                     const void* x, const void* norm_w, const void* W_in,
                     const void* beta, const void* threshold,
                     const void* log_A, const void* D, const void* W_proj, const void* b_dt,
                     const void* W_out, const void* out_scale,
                     const void* mem_in, void* mem_out,
                     const void* state_in, void* state_out,
                     void* out, unsigned long long* spike_count, int sparse,
                     void* workspace, int64_t workspace_bytes, void* stream);

/* Standalone fused LIF + selective scan: the LIF spikes of x drive the scan
 * with caller-given dt/B/C.  x, delta, y: [B,L,d] bf16; Bm, Cm: [B,L,N] bf16;
 * log_A: [d,N], Dskip, beta, threshold: [d] float32; mem_in/mem_out: [B,d]
 * float32; state_in/state_out: [B,d,N] float32 (NULL inputs = zeros);
 * spikes: optional [B,L,d] output in `spike_dtype` (NT_U8 or NT_BF16);
 * spike_count: optional device uint64 (incremented).  All math in float32. */
NT_API int nt_lif_ssm_fused(int64_t B, int64_t L, int64_t d, int64_t N,
                     const void* x, const void* delta, const void* Bm, const void* Cm,
                     const float* log_A, const float* Dskip,
                     const float* beta, const float* threshold,
                     const float* mem_in, float* mem_out,
                     const float* state_in, float* state_out,
                     void* y, void* spikes, int spike_dtype,
                     unsigned long long* spike_count, void* stream);

/* Sliding-window causal attention with rotary embedding -- the middle of
 * SlidingWindowAttention.forward (model.py:159-178: q/k/v from the qkv
 * projection, apply_rotary on q and k (model.py:119-126), then
 * scaled_dot_product_attention with the causal window mask j in [i-window, i]).
 * bf16 only, head_dim (HD) 64 or 128.  qkv: [B*T, ld_qkv] rows, columns
 * [q | k | v] of n_heads*HD each; cos_t, sin_t: [T, HD] bf16 rotary tables
 * (the module's cached ones); out: [B*T, ld_out], head h in columns
 * h*HD .. h*HD+HD-1 (the transpose(1,2).reshape layout o_proj takes).
 * Softmax scale 1/sqrt(HD).  RoPE
 * rounds like the reference's bf16 ops; scores and softmax in float32, the
 * probabilities rounded to bf16 before the product with v. */
NT_API int nt_window_attention(int dtype, int64_t B, int64_t T, int64_t n_heads, int64_t head_dim,
                        int64_t window, const void* qkv, int64_t ld_qkv, const void* cos_t,
                        const void* sin_t, void* out, int64_t ld_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NEURATENSOR_NATIVE_H */
