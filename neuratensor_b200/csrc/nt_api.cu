// C ABI of libneuratensor_native.so: argument checks, workspace carving and
// kernel sequencing.  Declarations and the reference interfaces each entry
// point replaces are in include/neuratensor_native.h.
#include "nt_kernels.cuh"

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <mutex>

namespace nt {

// ---------------------------------------------------------------------------
// Errors
// ---------------------------------------------------------------------------
static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

// Every launcher calls check_launch right after its launch, so this counts
// the library's kernel launches.
std::atomic<unsigned long long> g_launches{0};

int check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(NT_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return NT_OK;
}

// One error word per device, in this library's own device memory.
__device__ unsigned g_error_word;

unsigned* device_error_word(int device) {
    static unsigned* ptrs[64] = {};
    static std::mutex mu;
    if (device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_error_word) == cudaSuccess) ptrs[device] = static_cast<unsigned*>(p);
    }
    return ptrs[device];
}

}  // namespace nt

using namespace nt;

namespace {

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t esize(int dtype) { return dtype == NT_F32 ? 4 : (dtype == NT_BF16 ? 2 : 1); }

inline bool act_dtype_ok(int dtype) { return dtype == NT_F32 || dtype == NT_BF16; }

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Sequential carving of a caller-provided workspace.
struct Carve {
    char* base;
    int64_t off = 0;
    explicit Carve(void* b) : base(static_cast<char*>(b)) {}
    template <typename T> T* take(int64_t bytes) {
        T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
        off += align256(bytes);
        return p;
    }
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_gemm_operand(const void* p, int64_t ld, int dtype, const char* name) {
    if (dtype == NT_BF16 && (!aligned16(p) || (ld * 2) % 16))
        return fail(NT_ERR_ARG, "%s: bf16 GEMM operands need 16-byte alignment and a row length multiple of 8", name);
    return NT_OK;
}

// Workspace layouts ---------------------------------------------------------
struct SsmWs { void* dt; void* bc; int64_t bytes; };
SsmWs ssm_ws(void* ws, int dtype, int64_t M, int64_t d, int64_t N) {
    Carve c(ws);
    SsmWs w;
    w.dt = c.take<char>(M * d * esize(dtype));
    w.bc = c.take<char>(M * 2 * N * esize(dtype));
    w.bytes = c.off;
    return w;
}

struct SparseWs { unsigned* words; int* pos; int* idx; int* counters; void* oc; int64_t bytes; };
SparseWs sparse_ws(void* ws, int dtype, int64_t M, int64_t K) {
    Carve c(ws);
    SparseWs w;
    w.words = c.take<unsigned>(4 * ((M + 31) / 32));
    w.pos = c.take<int>(M * 4);
    w.idx = c.take<int>(M * 4);
    w.counters = c.take<int>(64);
    w.oc = c.take<char>(M * K * esize(dtype));
    w.bytes = c.off;
    return w;
}

struct BlockWs {
    void *xn, *h, *gate, *spikes, *dt, *bc, *o;
    unsigned* row_bits;
    int *pos, *idx, *counters;
    void* scanseg;              // float32 end states / decays / carry-ins of the segmented scan
    size_t scanseg_bytes;
    float* part;                // split-K partial sums of the block's GEMMs (small row counts)
    int64_t part_elems;
    int64_t bytes;
};
BlockWs block_ws(void* ws, int dtype, int64_t B, int64_t T, int64_t dm, int64_t di, int64_t N) {
    const int64_t M = B * T;
    Carve c(ws);
    BlockWs w;
    const int64_t es = esize(dtype);
    w.xn = c.take<char>(M * dm * es);
    w.h = c.take<char>(M * di * es);
    w.gate = c.take<char>(M * di * es);
    w.spikes = c.take<char>(M * di * es);
    w.dt = c.take<char>(M * di * es);
    w.bc = c.take<char>(M * 2 * N * es);
    w.o = c.take<char>(M * di * es);
    w.row_bits = c.take<unsigned>(4 * ((di + kLifChannels - 1) / kLifChannels) * B * ((T + 31) / 32));
    w.pos = c.take<int>(M * 4);
    w.idx = c.take<int>(M * 4);
    w.counters = c.take<int>(64);
    w.scanseg_bytes = selective_scan_segmented_workspace(B, T, di, N);
    w.scanseg = w.scanseg_bytes ? c.take<char>((int64_t)w.scanseg_bytes) : nullptr;
    w.part_elems = 0;
    if (dtype == NT_BF16) {
        const int64_t shapes[3][3] = {{2 * di, dm}, {di + 2 * N, di}, {dm, di}};   // N, K of each GEMM
        for (const auto& sh : shapes) {
            const int s = gemm_split_k(M, sh[0], sh[1]);
            if (s > 1) w.part_elems = std::max<int64_t>(w.part_elems, (int64_t)s * M * sh[0]);
        }
    }
    w.part = w.part_elems ? c.take<float>(w.part_elems * (int64_t)sizeof(float)) : nullptr;
    w.bytes = c.off;
    return w;
}

#define NT_TRY(expr)                  \
    do {                              \
        int _rc = (expr);             \
        if (_rc != NT_OK) return _rc; \
    } while (0)

}  // namespace

extern "C" {

int nt_abi_version(void) { return NT_ABI_VERSION; }

const char* nt_last_error(void) { return g_last_error; }

int nt_device_supported(int device) {
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, device);
    if (e != cudaSuccess) return fail(NT_ERR_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
    if (p.major != 10 || p.minor != 0)
        return fail(NT_ERR_ARCH, "device %d is sm_%d%d; this library is built for sm_100a", device, p.major, p.minor);
    return NT_OK;
}

unsigned long long nt_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int nt_get_error_flag(int device, unsigned* flags, int clear) {
    if (!flags) return fail(NT_ERR_ARG, "nt_get_error_flag: flags is NULL");
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) return fail(NT_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    int rc = NT_OK;
    unsigned* w = device_error_word(device);
    if (!w) rc = fail(NT_ERR_CUDA, "error word unavailable");
    else if (cudaDeviceSynchronize() != cudaSuccess ||
             cudaMemcpy(flags, w, sizeof(unsigned), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = fail(NT_ERR_CUDA, "reading the device error word failed: %s", cudaGetErrorString(cudaGetLastError()));
    else if (clear && cudaMemset(w, 0, sizeof(unsigned)) != cudaSuccess)
        rc = fail(NT_ERR_CUDA, "clearing the device error word failed");
    cudaSetDevice(prev);
    return rc;
}

// ---------------------------------------------------------------------------
// Bounded-wait check: one CTA waits on a shared-memory mbarrier that nothing
// ever completes, with a caller-chosen wall-time limit (at most 1 s), the way
// the GEMM's pipeline waits are bounded.  When the limit passes, the kernel
// sets the wait-expired bit of the device error word and returns normally, so
// the context stays usable; nt_get_error_flag then reports the bit.
// ---------------------------------------------------------------------------
namespace {
constexpr unsigned ERRF_WAIT_CHECK = 16u;

__global__ void bounded_wait_check_kernel(uint64_t limit_ns, unsigned* err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);                     // one arrival expected, none ever made
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    const uint64_t t0 = globaltimer_ns();
    bool done = false;
    while (!done && globaltimer_ns() - t0 < limit_ns) done = mbar_try_wait(smem_u32(&bar), 0);
    if (!done) atomicOr(err, ERRF_WAIT_CHECK);
}
}  // namespace

int nt_bounded_wait_check(int64_t limit_ns, void* stream) {
    if (limit_ns < 0 || limit_ns > 1000000000LL)
        return fail(NT_ERR_ARG, "nt_bounded_wait_check: limit %lld ns outside [0, 1 s]", (long long)limit_ns);
    int dev = 0;
    cudaGetDevice(&dev);
    unsigned* w = device_error_word(dev);
    if (!w) return fail(NT_ERR_CUDA, "nt_bounded_wait_check: error word unavailable");
    bounded_wait_check_kernel<<<1, 32, 0, as_stream(stream)>>>((uint64_t)limit_ns, w);
    return check_launch("bounded_wait_check_kernel");
}

// ---------------------------------------------------------------------------
// (a) LIF
// ---------------------------------------------------------------------------
int nt_lif_scan(int dtype, int64_t B, int64_t T, int64_t C, const void* x, int64_t x_sb, int64_t x_st,
                const void* beta, const void* threshold, const void* mem_in, void* mem_out, void* spikes,
                int64_t s_sb, int64_t s_st, unsigned long long* spike_count, void* stream) {
    if (!act_dtype_ok(dtype)) return fail(NT_ERR_DTYPE, "nt_lif_scan: dtype %d", dtype);
    if (B < 1 || T < 1 || C < 1) return fail(NT_ERR_ARG, "nt_lif_scan: B, T, C must be >= 1 (got %lld, %lld, %lld)",
                                             (long long)B, (long long)T, (long long)C);
    if (!x || !beta || !threshold || !mem_out || !spikes) return fail(NT_ERR_ARG, "nt_lif_scan: null pointer");
    if (B > 65535) return fail(NT_ERR_ARG, "nt_lif_scan: B > 65535");
    LifArgs a{B, T, C, x, x_sb, x_st, beta, threshold, mem_in, mem_out, spikes, s_sb, s_st, spike_count, nullptr, 0};
    return launch_lif_scan(dtype, dtype, a, as_stream(stream));
}

// ---------------------------------------------------------------------------
// (b) selective scan
// ---------------------------------------------------------------------------
int nt_selective_scan(int dtype, int state_dtype, int64_t B, int64_t T, int64_t d, int64_t N, const void* u,
                      const void* dt, const void* Bm, const void* Cm, const void* log_A, const void* D,
                      const void* gate, const void* state_in, void* state_out, void* y, void* stream) {
    if (!act_dtype_ok(dtype) || !act_dtype_ok(state_dtype)) return fail(NT_ERR_DTYPE, "nt_selective_scan: dtype");
    if (B < 1 || T < 1 || d < 1 || N < 1) return fail(NT_ERR_ARG, "nt_selective_scan: sizes must be >= 1");
    if (N > 256) return fail(NT_ERR_ARG, "nt_selective_scan: d_state %lld > 256", (long long)N);
    if (B > 65535) return fail(NT_ERR_ARG, "nt_selective_scan: B > 65535");
    if (!u || !dt || !Bm || !Cm || !log_A || !D || !state_out || !y)
        return fail(NT_ERR_ARG, "nt_selective_scan: null pointer");
    ScanArgs a{B, T, d, N, u, dt, Bm, Cm, N, log_A, D, gate, state_in, state_out, y, nullptr, nullptr, 0};
    return launch_selective_scan(dtype, state_dtype, a, as_stream(stream));
}

int64_t nt_ssm_workspace_bytes(int dtype, int64_t B, int64_t T, int64_t d, int64_t N) {
    return ssm_ws(nullptr, dtype, B * T, d, N).bytes;
}

int nt_ssm_forward(int dtype, int state_dtype, int64_t B, int64_t T, int64_t d, int64_t N, const void* u,
                   const void* W_proj, const void* b_dt, const void* log_A, const void* D, const void* state_in,
                   void* state_out, void* y, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!act_dtype_ok(dtype) || !act_dtype_ok(state_dtype)) return fail(NT_ERR_DTYPE, "nt_ssm_forward: dtype");
    if (B < 1 || T < 1 || d < 1 || N < 1 || N > 256) return fail(NT_ERR_ARG, "nt_ssm_forward: bad sizes");
    if (!u || !W_proj || !b_dt || !log_A || !D || !state_out || !y) return fail(NT_ERR_ARG, "nt_ssm_forward: null pointer");
    const int64_t M = B * T;
    SsmWs w = ssm_ws(workspace, dtype, M, d, N);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(NT_ERR_WORKSPACE, "nt_ssm_forward: workspace %lld < %lld bytes", (long long)workspace_bytes,
                    (long long)w.bytes);
    NT_TRY(check_gemm_operand(u, d, dtype, "nt_ssm_forward(u)"));
    NT_TRY(check_gemm_operand(W_proj, d, dtype, "nt_ssm_forward(W_proj)"));
    cudaStream_t st = as_stream(stream);
    GemmArgs g{};
    g.M = M; g.N = d + 2 * N; g.K = d;
    g.A = u; g.lda = d; g.Bw = W_proj; g.ldb = d;
    g.epi.kind = EPI_SSM_PROJ;
    g.epi.out = w.dt; g.epi.ldo = d; g.epi.out2 = w.bc; g.epi.ldo2 = 2 * N; g.epi.split = d; g.epi.bias = b_dt;
    NT_TRY(launch_gemm(dtype, g, st));
    const char* bc = static_cast<const char*>(w.bc);
    ScanArgs a{B, T, d, N, u, w.dt, bc, bc + N * esize(dtype), 2 * N, log_A, D, nullptr, state_in, state_out, y,
               nullptr, nullptr, 0};
    return launch_selective_scan(dtype, state_dtype, a, st);
}

// ---------------------------------------------------------------------------
// (c) sparse out_proj
// ---------------------------------------------------------------------------
int64_t nt_sparse_out_proj_workspace_bytes(int dtype, int64_t M, int64_t K, int64_t Nout) {
    (void)Nout;
    return sparse_ws(nullptr, dtype, M, K).bytes;
}

int nt_sparse_out_proj(int dtype, int64_t M, int64_t K, int64_t Nout, const void* o, const void* spikes,
                       const void* W, void* out, long long* n_active_out, void* workspace, int64_t workspace_bytes,
                       void* stream) {
    if (!act_dtype_ok(dtype)) return fail(NT_ERR_DTYPE, "nt_sparse_out_proj: dtype %d", dtype);
    if (M < 1 || K < 1 || Nout < 1) return fail(NT_ERR_ARG, "nt_sparse_out_proj: sizes must be >= 1");
    if (!o || !spikes || !W || !out) return fail(NT_ERR_ARG, "nt_sparse_out_proj: null pointer");
    SparseWs w = sparse_ws(workspace, dtype, M, K);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(NT_ERR_WORKSPACE, "nt_sparse_out_proj: workspace %lld < %lld bytes", (long long)workspace_bytes,
                    (long long)w.bytes);
    NT_TRY(check_gemm_operand(o, K, dtype, "nt_sparse_out_proj(o)"));
    NT_TRY(check_gemm_operand(W, K, dtype, "nt_sparse_out_proj(W)"));
    if ((K * esize(dtype)) % 16) return fail(NT_ERR_ARG, "nt_sparse_out_proj: row bytes must be a multiple of 16");
    cudaStream_t st = as_stream(stream);
    NT_TRY(launch_row_any_words(dtype, M, K, spikes, w.words, st));
    NT_TRY(launch_compact_row_bits(1, M, 1, w.words, w.pos, w.idx, w.counters, 1, st, n_active_out));
    NT_TRY(launch_gather_rows(dtype, M, K, o, w.idx, w.counters, w.oc, st));
    GemmArgs g{};
    g.M = M; g.N = Nout; g.K = K;
    g.A = w.oc; g.lda = K; g.Bw = W; g.ldb = K; g.m_count = w.counters + 2;
    g.epi.kind = EPI_SCATTER; g.epi.out = out; g.epi.ldo = Nout; g.epi.row_idx = w.idx; g.epi.row_sparse = w.counters + 1;
    NT_TRY(launch_gemm(dtype, g, st));
    return launch_fill_inactive(dtype, M, Nout, w.pos, w.counters, nullptr, out, st);
}

// ---------------------------------------------------------------------------
// (d) RMSNorm + in_proj
// ---------------------------------------------------------------------------
int64_t nt_rmsnorm_in_proj_workspace_bytes(int dtype, int64_t M, int64_t dm, int64_t di) {
    (void)di;
    return align256(M * dm * esize(dtype));
}

int nt_rmsnorm_in_proj(int dtype, int64_t M, int64_t dm, int64_t di, const void* x, const void* gamma,
                       const void* W_in, void* h, void* gate, void* workspace, int64_t workspace_bytes,
                       void* stream) {
    if (!act_dtype_ok(dtype)) return fail(NT_ERR_DTYPE, "nt_rmsnorm_in_proj: dtype %d", dtype);
    if (M < 1 || dm < 1 || di < 1) return fail(NT_ERR_ARG, "nt_rmsnorm_in_proj: sizes must be >= 1");
    if (!x || !gamma || !W_in || !h || !gate) return fail(NT_ERR_ARG, "nt_rmsnorm_in_proj: null pointer");
    const int64_t need = nt_rmsnorm_in_proj_workspace_bytes(dtype, M, dm, di);
    if (!workspace || workspace_bytes < need)
        return fail(NT_ERR_WORKSPACE, "nt_rmsnorm_in_proj: workspace %lld < %lld bytes", (long long)workspace_bytes,
                    (long long)need);
    NT_TRY(check_gemm_operand(workspace, dm, dtype, "nt_rmsnorm_in_proj(x)"));
    NT_TRY(check_gemm_operand(W_in, dm, dtype, "nt_rmsnorm_in_proj(W_in)"));
    cudaStream_t st = as_stream(stream);
    NT_TRY(launch_rmsnorm(dtype, M, dm, x, gamma, workspace, st));
    GemmArgs g{};
    g.M = M; g.N = 2 * di; g.K = dm;
    g.A = workspace; g.lda = dm; g.Bw = W_in; g.ldb = dm;
    g.epi.kind = EPI_SPLIT2; g.epi.out = h; g.epi.ldo = di; g.epi.out2 = gate; g.epi.ldo2 = di; g.epi.split = di;
    return launch_gemm(dtype, g, st);
}

// ---------------------------------------------------------------------------
// Model glue: embedding gather, final RMSNorm + tied lm_head
// ---------------------------------------------------------------------------
int nt_embedding(int dtype, int64_t M, int64_t dm, int64_t vocab, const int64_t* ids, const void* W, void* out,
                 void* stream) {
    if (!act_dtype_ok(dtype)) return fail(NT_ERR_DTYPE, "nt_embedding: dtype %d", dtype);
    if (M < 0 || dm < 1 || vocab < 1) return fail(NT_ERR_ARG, "nt_embedding: bad sizes");
    if (M == 0) return NT_OK;
    if (!ids || !W || !out) return fail(NT_ERR_ARG, "nt_embedding: null pointer");
    return launch_embedding(dtype, M, dm, vocab, ids, W, out, as_stream(stream));
}

int nt_greedy_tokens(int dtype, int64_t B, int64_t vocab, const void* logits, int64_t ld, const float* u,
                     int64_t* tokens, void* stream) {
    if (!act_dtype_ok(dtype)) return fail(NT_ERR_DTYPE, "nt_greedy_tokens: dtype %d", dtype);
    if (B < 0 || vocab < 1 || ld < vocab || B > 2147483647LL) return fail(NT_ERR_ARG, "nt_greedy_tokens: bad sizes");
    if (B == 0) return NT_OK;
    if (!logits || !u || !tokens) return fail(NT_ERR_ARG, "nt_greedy_tokens: null pointer");
    return launch_greedy(dtype, B, vocab, logits, ld, u, tokens, as_stream(stream));
}

int64_t nt_lm_head_workspace_bytes(int dtype, int64_t M, int64_t dm, int64_t vocab) {
    (void)vocab;
    return align256(M * dm * esize(dtype));
}

int nt_lm_head(int dtype, int64_t M, int64_t dm, int64_t vocab, const void* x, const void* gamma, const void* W,
               void* logits, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!act_dtype_ok(dtype)) return fail(NT_ERR_DTYPE, "nt_lm_head: dtype %d", dtype);
    if (M < 0 || dm < 1 || vocab < 1) return fail(NT_ERR_ARG, "nt_lm_head: bad sizes");
    if (M == 0) return NT_OK;
    if (!x || !gamma || !W || !logits) return fail(NT_ERR_ARG, "nt_lm_head: null pointer");
    const int64_t need = nt_lm_head_workspace_bytes(dtype, M, dm, vocab);
    if (!workspace || workspace_bytes < need)
        return fail(NT_ERR_WORKSPACE, "nt_lm_head: workspace %lld < %lld bytes", (long long)workspace_bytes,
                    (long long)need);
    NT_TRY(check_gemm_operand(workspace, dm, dtype, "nt_lm_head(x)"));
    NT_TRY(check_gemm_operand(W, dm, dtype, "nt_lm_head(W)"));
    cudaStream_t st = as_stream(stream);
    NT_TRY(launch_rmsnorm(dtype, M, dm, x, gamma, workspace, st));
    GemmArgs g{};
    g.M = M; g.N = vocab; g.K = dm;
    g.A = workspace; g.lda = dm; g.Bw = W; g.ldb = dm;
    g.epi.kind = EPI_STORE; g.epi.out = logits; g.epi.ldo = vocab;
    return launch_gemm(dtype, g, st);
}

// ---------------------------------------------------------------------------
// FusedSpikeBlock.forward
// ---------------------------------------------------------------------------
int64_t nt_block_workspace_bytes(int dtype, int64_t B, int64_t T, int64_t dm, int64_t di, int64_t N) {
    return block_ws(nullptr, dtype, B, T, dm, di, N).bytes;
}

int nt_block_forward(int dtype, int state_dtype, int64_t B, int64_t T, int64_t dm, int64_t di, int64_t N,
                     const void* x, const void* norm_w, const void* W_in, const void* beta, const void* threshold,
                     const void* log_A, const void* D, const void* W_proj, const void* b_dt, const void* W_out,
                     const void* out_scale, const void* mem_in, void* mem_out, const void* state_in,
                     void* state_out, void* out, unsigned long long* spike_count, int sparse, void* workspace,
                     int64_t workspace_bytes, void* stream) {
    if (!act_dtype_ok(dtype) || !act_dtype_ok(state_dtype)) return fail(NT_ERR_DTYPE, "nt_block_forward: dtype");
    if (B < 1 || T < 1 || dm < 1 || di < 1 || N < 1) return fail(NT_ERR_ARG, "nt_block_forward: sizes must be >= 1");
    if (N > 256) return fail(NT_ERR_ARG, "nt_block_forward: d_state %lld > 256", (long long)N);
    if (B > 65535) return fail(NT_ERR_ARG, "nt_block_forward: B > 65535");
    if (!x || !norm_w || !W_in || !beta || !threshold || !log_A || !D || !W_proj || !b_dt || !W_out || !out_scale ||
        !mem_out || !state_out || !out)
        return fail(NT_ERR_ARG, "nt_block_forward: null pointer");
    const int64_t M = B * T;
    BlockWs w = block_ws(workspace, dtype, B, T, dm, di, N);
    if (!workspace || workspace_bytes < w.bytes)
        return fail(NT_ERR_WORKSPACE, "nt_block_forward: workspace %lld < %lld bytes", (long long)workspace_bytes,
                    (long long)w.bytes);
    NT_TRY(check_gemm_operand(W_in, dm, dtype, "nt_block_forward(W_in)"));
    NT_TRY(check_gemm_operand(W_proj, di, dtype, "nt_block_forward(W_proj)"));
    NT_TRY(check_gemm_operand(W_out, di, dtype, "nt_block_forward(W_out)"));
    if (dtype == NT_BF16 && (dm % 8 || di % 8)) return fail(NT_ERR_ARG, "nt_block_forward: bf16 needs d_model, d_inner multiples of 8");
    cudaStream_t st = as_stream(stream);
    const int64_t es = esize(dtype);

    // (d) RMSNorm + in_proj -> h | gate
    NT_TRY(launch_rmsnorm(dtype, M, dm, x, norm_w, w.xn, st));
    {
        GemmArgs g{};
        g.M = M; g.N = 2 * di; g.K = dm;
        g.A = w.xn; g.lda = dm; g.Bw = W_in; g.ldb = dm;
        g.epi.kind = EPI_SPLIT2_SILU; g.epi.out = w.h; g.epi.ldo = di; g.epi.out2 = w.gate; g.epi.ldo2 = di;
        g.epi.split = di; g.part = w.part; g.part_elems = w.part_elems;
        NT_TRY(launch_gemm(dtype, g, st));
    }
    // (a) LIF -> spikes, membrane, row-activity bits
    const int64_t n_cblk = (di + kLifChannels - 1) / kLifChannels, n_words = (T + 31) / 32;
    {
        LifArgs a{B, T, di, w.h, T * di, di, beta, threshold, mem_in, mem_out, w.spikes, T * di, di,
                  spike_count, w.row_bits, n_words};
        NT_TRY(launch_lif_scan(dtype, dtype, a, st));
    }
    // density decision of _sparse_out_proj and, when sparse, the row compaction
    NT_TRY(launch_compact_row_bits(B, T, n_cblk, w.row_bits, w.pos, w.idx, w.counters, sparse ? 1 : 0, st));
    // (b) dt | B | C projections of the spikes
    {
        GemmArgs g{};
        g.M = M; g.N = di + 2 * N; g.K = di;
        g.A = w.spikes; g.lda = di; g.Bw = W_proj; g.ldb = di;
        g.epi.kind = EPI_SSM_PROJ; g.epi.out = w.dt; g.epi.ldo = di; g.epi.out2 = w.bc; g.epi.ldo2 = 2 * N;
        g.epi.split = di; g.epi.bias = b_dt; g.part = w.part; g.part_elems = w.part_elems;
        NT_TRY(launch_gemm(dtype, g, st));
    }
    // (b) selective scan with the gate fused, rows compacted when sparse
    {
        const char* bc = static_cast<const char*>(w.bc);
        ScanArgs a{B, T, di, N, w.spikes, w.dt, bc, bc + N * es, 2 * N, log_A, D, w.gate, state_in, state_out, w.o,
                   w.pos, w.counters + 1, /*gate_is_silu=*/1};
        NT_TRY(launch_selective_scan_segmented(dtype, state_dtype, a, w.scanseg, w.scanseg_bytes, st));
    }
    // (c) out_proj on the processed rows, * out_scale + residual, scattered back
    {
        GemmArgs g{};
        g.M = M; g.N = dm; g.K = di;
        g.A = w.o; g.lda = di; g.Bw = W_out; g.ldb = di; g.m_count = w.counters + 2;
        g.epi.kind = EPI_OUT_PROJ; g.epi.out = out; g.epi.ldo = dm; g.epi.scale = out_scale; g.epi.resid = x;
        g.epi.ldr = dm; g.epi.row_idx = w.idx; g.epi.row_sparse = w.counters + 1;
        g.part = w.part; g.part_elems = w.part_elems;
        NT_TRY(launch_gemm(dtype, g, st));
    }
    // rows skipped by the sparse branch: out = 0 * out_scale + x = x
    return launch_fill_inactive(dtype, M, dm, w.pos, w.counters, x, out, st);
}

// ---------------------------------------------------------------------------
// Standalone fused LIF + selective scan
// ---------------------------------------------------------------------------
int nt_window_attention(int dtype, int64_t B, int64_t T, int64_t n_heads, int64_t head_dim, int64_t window,
                        const void* qkv, int64_t ld_qkv, const void* cos_t, const void* sin_t, void* out,
                        int64_t ld_out, void* stream) {
    if (dtype != NT_BF16) return fail(NT_ERR_DTYPE, "nt_window_attention: bf16 only (dtype %d)", dtype);
    if (head_dim != 64 && head_dim != 128)
        return fail(NT_ERR_ARG, "nt_window_attention: head_dim %lld (64 or 128 supported)", (long long)head_dim);
    if (B < 1 || T < 1 || n_heads < 1 || window < 0 || B > 65535 || n_heads > 65535 || T > (int64_t)INT32_MAX / 2)
        return fail(NT_ERR_ARG, "nt_window_attention: bad sizes");
    if (!qkv || !cos_t || !sin_t || !out) return fail(NT_ERR_ARG, "nt_window_attention: null pointer");
    if (ld_qkv < 3 * n_heads * head_dim || ld_out < n_heads * head_dim)
        return fail(NT_ERR_ARG, "nt_window_attention: leading dimensions too small");
    if (ld_qkv % 8 || ld_out % 2 || !aligned16(qkv) || !aligned16(cos_t) || !aligned16(sin_t) ||
        (reinterpret_cast<uintptr_t>(out) & 3))
        return fail(NT_ERR_ARG, "nt_window_attention: qkv/cos/sin need 16-byte aligned rows, out 4-byte");
    return launch_window_attention(B, T, n_heads, head_dim, window, qkv, ld_qkv, cos_t, sin_t, out, ld_out,
                                   as_stream(stream));
}

int64_t nt_attention_workspace_bytes(int dtype, int64_t B, int64_t T, int64_t dm) {
    const int64_t M = B * T, es = esize(dtype);
    return align256(M * dm * es) + align256(M * 3 * dm * es) + align256(M * dm * es);
}

int nt_attention_forward(int dtype, int64_t B, int64_t T, int64_t dm, int64_t n_heads, int64_t window,
                         const void* x, const void* norm_w, const void* W_qkv, const void* W_o, const void* cos_t,
                         const void* sin_t, void* out, void* workspace, int64_t workspace_bytes, void* stream) {
    if (dtype != NT_BF16) return fail(NT_ERR_DTYPE, "nt_attention_forward: bf16 only (dtype %d)", dtype);
    if (B < 1 || T < 1 || dm < 1 || n_heads < 1 || dm % n_heads)
        return fail(NT_ERR_ARG, "nt_attention_forward: bad sizes");
    const int64_t hd = dm / n_heads;
    if (hd != 64 && hd != 128) return fail(NT_ERR_ARG, "nt_attention_forward: head_dim %lld (64 or 128)", (long long)hd);
    if (!x || !norm_w || !W_qkv || !W_o || !cos_t || !sin_t || !out)
        return fail(NT_ERR_ARG, "nt_attention_forward: null pointer");
    const int64_t need = nt_attention_workspace_bytes(dtype, B, T, dm);
    if (!workspace || workspace_bytes < need)
        return fail(NT_ERR_WORKSPACE, "nt_attention_forward: workspace %lld < %lld bytes", (long long)workspace_bytes,
                    (long long)need);
    NT_TRY(check_gemm_operand(W_qkv, dm, dtype, "nt_attention_forward(W_qkv)"));
    NT_TRY(check_gemm_operand(W_o, dm, dtype, "nt_attention_forward(W_o)"));
    const int64_t M = B * T, es = esize(dtype);
    Carve c(workspace);
    void* xn = c.take<char>(M * dm * es);
    void* qkv = c.take<char>(M * 3 * dm * es);
    void* o = c.take<char>(M * dm * es);
    cudaStream_t st = as_stream(stream);
    // norm -> qkv projection (model.py:156-158)
    NT_TRY(launch_rmsnorm(dtype, M, dm, x, norm_w, xn, st));
    {
        GemmArgs g{};
        g.M = M; g.N = 3 * dm; g.K = dm;
        g.A = xn; g.lda = dm; g.Bw = W_qkv; g.ldb = dm;
        g.epi.kind = EPI_STORE; g.epi.out = qkv; g.epi.ldo = 3 * dm;
        NT_TRY(launch_gemm(dtype, g, st));
    }
    // RoPE + windowed causal softmax attention (model.py:159-179)
    NT_TRY(nt_window_attention(dtype, B, T, n_heads, hd, window, qkv, 3 * dm, cos_t, sin_t, o, dm, stream));
    // o_proj + residual (model.py:180-181)
    GemmArgs g{};
    g.M = M; g.N = dm; g.K = dm;
    g.A = o; g.lda = dm; g.Bw = W_o; g.ldb = dm;
    g.epi.kind = EPI_RESID; g.epi.out = out; g.epi.ldo = dm; g.epi.resid = x; g.epi.ldr = dm;
    return launch_gemm(dtype, g, st);
}

int nt_lif_ssm_fused(int64_t B, int64_t L, int64_t d, int64_t N, const void* x, const void* delta, const void* Bm,
                     const void* Cm, const float* log_A, const float* Dskip, const float* beta,
                     const float* threshold, const float* mem_in, float* mem_out, const float* state_in,
                     float* state_out, void* y, void* spikes, int spike_dtype, unsigned long long* spike_count,
                     void* stream) {
    if (B < 1 || L < 1 || d < 1 || N < 1 || N > 256) return fail(NT_ERR_ARG, "nt_lif_ssm_fused: bad sizes");
    if (B > 65535) return fail(NT_ERR_ARG, "nt_lif_ssm_fused: B > 65535");
    if (!x || !delta || !Bm || !Cm || !log_A || !Dskip || !beta || !threshold || !mem_out || !state_out || !y)
        return fail(NT_ERR_ARG, "nt_lif_ssm_fused: null pointer");
    if (spikes && spike_dtype != NT_U8 && spike_dtype != NT_BF16)
        return fail(NT_ERR_DTYPE, "nt_lif_ssm_fused: spike dtype %d", spike_dtype);
    FusedArgs f{B, L, d, N, x, delta, Bm, Cm, log_A, Dskip, beta, threshold, mem_in, mem_out, state_in, state_out,
                y, spikes, spike_dtype, spike_count};
    return launch_lif_ssm_fused(f, as_stream(stream));
}

}  // extern "C"
