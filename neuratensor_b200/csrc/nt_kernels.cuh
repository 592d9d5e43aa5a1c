// Internal kernel argument blocks and launchers (not part of the C ABI).
#pragma once
#include "nt_common.cuh"

namespace nt {

// Channels per LIF CTA; the block path's per-row partial counts have
// ceil(C / kLifChannels) entries per row.
constexpr int kLifChannels = 64;

struct LifArgs {
    int64_t B, T, C;
    const void* x; int64_t x_sb, x_st;
    const void* beta; const void* threshold;
    const void* mem_in; void* mem_out;
    void* spikes; int64_t s_sb, s_st;
    unsigned long long* spike_count;       // optional, += spikes
    // optional row activity: bit (t % 32) of row_bits[(cblk * B + b) * n_words + t / 32]
    // is set when row (b, t) has a spike among the channels of block cblk
    unsigned* row_bits;
    int64_t n_words;                       // = ceil(T / 32)
};
// math: NT_F32 (exact fp32 recurrence) or NT_BF16 (bf16 rounding after each op)
int launch_lif_scan(int dtype, int math, const LifArgs& a, cudaStream_t stream);

struct ScanArgs {
    int64_t B, T, d, N;
    const void* u; const void* dt; const void* Bm; const void* Cm;
    int64_t ld_bc;                          // row stride of Bm / Cm (elements)
    const void* log_A; const void* D; const void* gate;
    const void* state_in; void* state_out;
    void* y;
    // Row compaction (block path): when row_pos != nullptr and *n_active_dense
    // says the sparse branch is taken, output row r goes to row row_pos[r]
    // (inactive rows are skipped).
    const int* row_pos; const int* sparse_flag;
    int gate_is_silu;                       // gate already holds rnd(silu(gate))
    float* seg_decay;                       // state-only segment pass: exp(A*sum(dt)) per state
};
int launch_selective_scan(int dtype, int state_dtype, const ScanArgs& a, cudaStream_t stream);
// Time-segmented variant for small batches (needs the float32 workspace below;
// falls back to launch_selective_scan when one segment suffices).
int scan_segments(int64_t B, int64_t T);
size_t selective_scan_segmented_workspace(int64_t B, int64_t T, int64_t d, int64_t N);
int launch_selective_scan_segmented(int dtype, int state_dtype, const ScanArgs& a, void* ws, size_t ws_bytes,
                                    cudaStream_t stream);

struct FusedArgs {
    int64_t B, L, d, N;
    const void* x; const void* delta; const void* Bm; const void* Cm;
    const float* log_A; const float* Dskip; const float* beta; const float* threshold;
    const float* mem_in; float* mem_out; const float* state_in; float* state_out;
    void* y; void* spikes; int spike_dtype;
    unsigned long long* spike_count;
};
int launch_lif_ssm_fused(const FusedArgs& a, cudaStream_t stream);

// RMSNorm rows (eps = FLT_EPSILON), rounding like torch's rms_norm.
int launch_rmsnorm(int dtype, int64_t M, int64_t D, const void* x, const void* w, void* y,
                   cudaStream_t stream);

// Embedding rows out[r] = W[ids[r]] (ids outside [0, vocab): zero row and ERRF_BAD_ARG).
int launch_embedding(int dtype, int64_t M, int64_t D, int64_t vocab, const int64_t* ids, const void* W, void* out,
                     cudaStream_t stream);

// Greedy choice per row of logits [B, V] (row stride ld): uniform among the tied maxima, u[r] in [0,1).
int launch_greedy(int dtype, int64_t B, int64_t V, const void* logits, int64_t ld, const float* u, int64_t* out,
                  cudaStream_t stream);

// Row compaction (the density decision of _sparse_out_proj): counters[0] =
// n_active, counters[1] = 1 when the sparse branch is taken (2*n_active <= M),
// counters[2] = rows the out_proj GEMM processes.  Only on the sparse branch
// are row_pos (position among active rows, or -1) and row_idx (inverse map,
// first n_active entries) written; consumers treat both as the identity when
// counters[1] == 0.  n_active_out (optional) receives n_active as int64.
// Input: row-activity bits (M = B*T rows, n_cblk channel blocks, the layout of
// LifArgs::row_bits).
int launch_compact_row_bits(int64_t B, int64_t T, int64_t n_cblk, const unsigned* row_bits, int* row_pos,
                            int* row_idx, int* counters, int sparse_enabled, cudaStream_t stream,
                            long long* n_active_out = nullptr);
// Row activity of a dense [M,K] matrix as 32-row words (bit j of words[g]: row 32g + j
// has a non-zero value); the layout of launch_compact_row_bits with B = 1, n_cblk = 1.
int launch_row_any_words(int dtype, int64_t M, int64_t K, const void* spikes, unsigned* words,
                         cudaStream_t stream);
// Gather active rows of src [M,K] into dst [n_active,K] (dst row i = src row row_idx[i];
// every row, in order, when counters[1] == 0).
int launch_gather_rows(int dtype, int64_t M, int64_t K, const void* src, const int* row_idx,
                       const int* counters, void* dst, cudaStream_t stream);
// Rows skipped by the sparse branch: dst[r,:] = fill (0) or src[r,:] (residual copy).
int launch_fill_inactive(int dtype, int64_t M, int64_t N, const int* row_pos, const int* counters,
                         const void* src, void* dst, cudaStream_t stream);

// Sliding-window causal attention with RoPE, bf16, head_dim 64 or 128: qkv row-major
// [B*T, ld_qkv] with columns [q | k | v] (H heads of 64 each), cos/sin [T][64]
// bf16, out [B*T, ld_out] (head h in columns h*64 .. h*64+63).
int launch_window_attention(int64_t B, int64_t T, int64_t H, int64_t head_dim, int64_t window, const void* qkv,
                            int64_t ld_qkv, const void* cos_t, const void* sin_t, void* out, int64_t ld_out,
                            cudaStream_t stream);

// ---------------------------------------------------------------------------
// GEMM: D[M,N] = A[M,K] * B[N,K]^T with a fused epilogue.
// ---------------------------------------------------------------------------
enum EpiKind : int {
    EPI_STORE = 0,        // D -> out (dtype), ldo
    EPI_SPLIT2 = 1,       // cols [0,split) -> out, [split,N) -> out2 (in_proj h | gate)
    EPI_SSM_PROJ = 2,     // cols [0,split): softplus(acc + bias) -> out (dt); rest -> out2 (B|C)
    EPI_OUT_PROJ = 3,     // out[row_map(r)] = rnd(rnd(rnd(acc)*scale) + resid[row_map(r)])
    EPI_SCATTER = 4,      // out[row_map(r)] = acc  (sparse out_proj without scale)
    EPI_SPLIT2_SILU = 5,  // cols [0,split) -> out (h), [split,N) -> out2 as rnd(silu(acc))
    EPI_RESID = 6         // out = rnd(rnd(acc) + resid)  (attention o_proj + residual)
};
struct EpiArgs {
    int kind;
    void* out; int64_t ldo;
    void* out2; int64_t ldo2;
    int64_t split;
    const void* bias;          // EPI_SSM_PROJ
    const void* scale;         // EPI_OUT_PROJ: pointer to one dtype value
    const void* resid; int64_t ldr;
    const int* row_idx;        // row map for compacted A rows (nullptr: identity)
    const int* row_sparse;     // when set and *row_sparse == 0, row_idx is the identity
    int vec;                   // 1: outputs, residual and bias allow 16-byte accesses per 8 columns
};
struct GemmArgs {
    int64_t M, N, K;
    const void* A; int64_t lda;   // [M,K] row-major
    const void* Bw; int64_t ldb;  // [N,K] row-major
    const int* m_count;           // optional device row count (rows >= *m_count are skipped)
    EpiArgs epi;
    // optional float32 scratch for split-K partial sums ([splits][M][N]); a GEMM
    // with fewer output tiles than SMs splits K when it fits (gemm_split_k)
    float* part;
    int64_t part_elems;
};
int launch_gemm(int dtype, const GemmArgs& g, cudaStream_t stream);
// K splits a bf16 GEMM of this shape takes on the current device when given
// partial-sum scratch (1 = none); the scratch it needs is splits * M * N floats.
int gemm_split_k(int64_t M, int64_t N, int64_t K);

}  // namespace nt
