// nt_rmsnorm_in_proj_noalloc: RMSNorm + in_proj with library-owned scratch.
//
// Some callers cannot allocate device memory at the point where they run the
// block: serving runtimes that reserve all of HBM once at start-up and forbid
// cudaMalloc afterwards (it can synchronize the device and fragments their
// pool), or hosts that call through the C ABI without an allocator of their
// own to hand a workspace from.  This entry point needs no workspace: the
// normalised activations live in kNoAllocScratchBytes of device memory that
// the library declares at file scope, so every GPU that loads the library
// holds this array until the process exits.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's device address with cudaGetSymbolAddress and caches it; later
// calls on that device reuse it.  That first call should therefore happen
// before any stream capture.
//
// All calls share the one array and it keeps the last call's contents.
// Nothing in it has to start at zero: the RMSNorm kernel writes every element
// the GEMM reads.  Calls that overlap on the GPU (different streams, or
// different host threads on one device) race on the array.
#include "nt_kernels.cuh"

#include <mutex>

namespace nt {
namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;   // 32 MiB per device

// Host code must not use this name as a pointer: on the host it is only a
// stand-in for the device symbol.  The device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up once).
int scratch_for_current_device(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(NT_ERR_CUDA, "nt_rmsnorm_in_proj_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(NT_ERR_ARG, "nt_rmsnorm_in_proj_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(NT_ERR_CUDA, "nt_rmsnorm_in_proj_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                        cudaGetErrorString(e));
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return NT_OK;
}

}  // namespace
}  // namespace nt

using namespace nt;

extern "C" {

size_t nt_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int nt_rmsnorm_in_proj_noalloc(int dtype, int64_t M, int64_t dm, int64_t di, const void* x, const void* gamma,
                               const void* W_in, void* h, void* gate, void* stream) {
    if (dtype != NT_F32 && dtype != NT_BF16) return fail(NT_ERR_DTYPE, "nt_rmsnorm_in_proj_noalloc: dtype %d", dtype);
    if (M < 1 || dm < 1 || di < 1) return fail(NT_ERR_ARG, "nt_rmsnorm_in_proj_noalloc: sizes must be >= 1");
    if (!x || !gamma || !W_in || !h || !gate) return fail(NT_ERR_ARG, "nt_rmsnorm_in_proj_noalloc: null pointer");
    const int64_t es = dtype == NT_F32 ? 4 : 2;
    const int64_t need = M * dm * es;
    if (need > (int64_t)kNoAllocScratchBytes)
        return fail(NT_ERR_ARG,
                    "nt_rmsnorm_in_proj_noalloc: M*d_model*%lld = %lld bytes exceeds the %zu-byte scratch; "
                    "split the rows or use nt_rmsnorm_in_proj with a workspace",
                    (long long)es, (long long)need, kNoAllocScratchBytes);
    if (dtype == NT_BF16 && ((reinterpret_cast<uintptr_t>(W_in) & 15) || (dm * 2) % 16))
        return fail(NT_ERR_ARG, "nt_rmsnorm_in_proj_noalloc: bf16 GEMM operands need 16-byte alignment and d_model "
                                "a multiple of 8");
    void* xn = nullptr;
    const int rc = scratch_for_current_device(&xn);
    if (rc != NT_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    int r = launch_rmsnorm(dtype, M, dm, x, gamma, xn, st);
    if (r != NT_OK) return r;
    GemmArgs g{};
    g.M = M; g.N = 2 * di; g.K = dm;
    g.A = xn; g.lda = dm; g.Bw = W_in; g.ldb = dm;
    g.epi.kind = EPI_SPLIT2; g.epi.out = h; g.epi.ldo = di; g.epi.out2 = gate; g.epi.ldo2 = di; g.epi.split = di;
    return launch_gemm(dtype, g, st);
}

}  // extern "C"
