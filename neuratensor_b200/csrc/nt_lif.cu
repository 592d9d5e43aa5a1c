// LIF membrane recurrence (neuratensor/core/snn.py:64-75,167-182).
//
// The recurrence is non-linear (threshold + reset), so time stays serial per
// channel: one thread owns one (batch, channel) membrane for the whole
// sequence.  A CTA covers kLifChannels channels of one batch row with two
// membrane warps and one helper warp: the helper streams input tiles into a
// kLifStages-deep shared-memory ring with cp.async and writes the spike tiles
// out, so the membrane warps only run the serial chain.
//
// Arithmetic follows the reference exactly:
//   V = beta*V + x      -- a product then a sum, each rounded to the dtype
//   S = V >= theta
//   V = V - theta*S
// fp32: __fmul_rn/__fadd_rn keep the two roundings (no FMA contraction), so
// spikes and membranes are bit-identical to the reference on equal inputs.
// bf16: native bfloat16 multiply/add/subtract (.rn, round-to-nearest-even), which
// equal torch's compute-in-fp32-then-round for bf16 operands: the product of
// two bf16 values is exact in fp32, and a bf16 sum is either exact in fp32 or
// too far from a rounding midpoint for the second rounding to matter.
#include "nt_kernels.cuh"

namespace nt {

namespace {

constexpr int kLifStages = 3;
// steps per tile: 256 bytes of input per channel (128 bf16 or 64 fp32 steps)
template <typename T> struct LifSteps { static constexpr int value = 256 / (int)sizeof(T); };

__device__ __forceinline__ void cp16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem) : "memory");
}
__device__ __forceinline__ void commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Membrane update for one step.  The membrane lives in the working dtype
// (float for fp32, bfloat16 for bf16) so the serial chain carries no
// conversions.  Returns true when the neuron fires.
__device__ __forceinline__ bool lif_step(float& v, float beta, float th, float x) {
    v = __fadd_rn(__fmul_rn(beta, v), x);
    const bool s = v >= th;
    v = __fsub_rn(v, __fmul_rn(th, s ? 1.f : 0.f));
    return s;
}
__device__ __forceinline__ bool lif_step(__nv_bfloat16& v, __nv_bfloat16 beta, __nv_bfloat16 th, __nv_bfloat16 x) {
    // the _rn forms keep the product and the sum as two separately rounded
    // operations (plain mul/add may be contracted into one fma)
    v = __hadd_rn(__hmul_rn(beta, v), x);
    const bool s = __hge(v, th);
    if (s) v = __hsub_rn(v, th);
    return s;
}

template <typename S> struct MathOf;
template <> struct MathOf<float> {
    static __device__ __forceinline__ float from(float f) { return f; }
    template <typename T> static __device__ __forceinline__ float in(T x) { return Elem<sizeof(T) == 4 ? NT_F32 : NT_BF16>::to_f(x); }
};
template <> struct MathOf<__nv_bfloat16> {
    static __device__ __forceinline__ __nv_bfloat16 from(float f) { return __float2bfloat16_rn(f); }
    template <typename T> static __device__ __forceinline__ __nv_bfloat16 in(T x) { return x; }
};

// Spike tile element: 0/1 in the output dtype.
template <typename T> __device__ __forceinline__ T spike_val(bool s);
template <> __device__ __forceinline__ float spike_val<float>(bool s) { return s ? 1.f : 0.f; }
template <> __device__ __forceinline__ __nv_bfloat16 spike_val<__nv_bfloat16>(bool s) {
    return __ushort_as_bfloat16(s ? (unsigned short)0x3F80 : (unsigned short)0);
}

// Shared-memory layout of one CTA: a kLifStages-deep ring of input tiles,
// two spike tiles, and the mbarriers that hand them between the roles.
template <typename T> struct LifSmem {
    static constexpr int kSteps = LifSteps<T>::value;
    static constexpr size_t tile_bytes = (size_t)kSteps * kLifChannels * sizeof(T);
    static constexpr size_t bar_off = (kLifStages + 2) * tile_bytes;
    static constexpr size_t bytes = bar_off + (2 * kLifStages + 4) * sizeof(uint64_t);
};

// Spikes in one 32-bit word of the spike tile: bit 7 of a bf16 1.0 (0x3F80)
// or bit 23 of a float 1.0 (0x3F800000); a 0 spike is all zero bits.
template <typename T> __device__ __forceinline__ int spikes_in_word(uint32_t w);
template <> __device__ __forceinline__ int spikes_in_word<__nv_bfloat16>(uint32_t w) { return __popc(w & 0x00800080u); }
template <> __device__ __forceinline__ int spikes_in_word<float>(uint32_t w) { return (w >> 23) & 1u; }

__device__ __forceinline__ bool lif_wait(uint64_t* bar, uint32_t parity) {
    const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(bar), parity));
    __syncwarp();
    return ok;
}

// Roles: threads 0..63 (two warps) each own one channel's membrane and run
// the serial chain; thread 64..95 (the helper warp) streams input tiles in
// with cp.async, and writes the spike tiles out together with per-row counts
// and row-activity words.  Input stage s and spike tile b are handed over
// through mbarriers (in_full/in_empty, spk_full/spk_empty); every wait is
// bounded and raises a device error flag on expiry.
constexpr int kLifThreads = kLifChannels + 32;

template <int DT, int MATH>
__global__ void __launch_bounds__(kLifThreads)
lif_scan_kernel(LifArgs a, unsigned* err) {
    using E = Elem<DT>;
    using T = typename E::T;
    using S = typename Elem<MATH>::T;       // state / arithmetic type
    using M = MathOf<S>;
    using L = LifSmem<T>;
    constexpr int EPV = 16 / (int)sizeof(T);
    constexpr int kSteps = L::kSteps;
    extern __shared__ __align__(16) unsigned char lif_smem[];
    T (*tile)[kSteps][kLifChannels] = reinterpret_cast<T (*)[kSteps][kLifChannels]>(lif_smem);
    T (*spk)[kSteps][kLifChannels] =
        reinterpret_cast<T (*)[kSteps][kLifChannels]>(lif_smem + kLifStages * L::tile_bytes);
    uint64_t* in_full = reinterpret_cast<uint64_t*>(lif_smem + L::bar_off);
    uint64_t* in_empty = in_full + kLifStages;
    uint64_t* spk_full = in_empty + kLifStages;
    uint64_t* spk_empty = spk_full + 2;

    const int tid = threadIdx.x, lane = tid & 31;
    const int64_t c0 = (int64_t)blockIdx.x * kLifChannels, b = blockIdx.y;
    const int ntiles = (int)((a.T + kSteps - 1) / kSteps);
    if (tid == 0) {
        for (int i = 0; i < kLifStages; ++i) {
            mbar_init(smem_u32(&in_full[i]), 1);
            mbar_init(smem_u32(&in_empty[i]), kLifChannels / 32);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&spk_full[i]), kLifChannels / 32);
            mbar_init(smem_u32(&spk_empty[i]), 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (tid < kLifChannels) {
        // ======================= membrane warps ==============================
        const int64_t c = c0 + tid;
        const bool live = c < a.C;
        S beta = M::from(0.f), th = M::from(0.f), v = M::from(0.f);
        if (live) {
            beta = M::from(E::load(static_cast<const T*>(a.beta) + c));
            th = M::from(E::load(static_cast<const T*>(a.threshold) + c));
            if (a.mem_in) v = M::from(E::load(static_cast<const T*>(a.mem_in) + b * a.C + c));
        }
        bool ok = true;
        for (int k = 0; k < ntiles; ++k) {
            const int st = k % kLifStages, sb2 = k & 1;
            if (!lif_wait(&in_full[st], (k / kLifStages) & 1)) { ok = false; break; }
            if (k >= 2 && !lif_wait(&spk_empty[sb2], ((k >> 1) - 1) & 1)) { ok = false; break; }
            const T* xt = &tile[st][0][0];
            T (*sp)[kLifChannels] = spk[sb2];
            const int64_t t0 = (int64_t)k * kSteps;
            const int nt = (a.T - t0 < kSteps) ? (int)(a.T - t0) : kSteps;
            // One membrane update and one spike store per step; inputs read eight
            // steps ahead into registers, so no shared-memory latency sits on the
            // chain (the loads of group g+1 precede the stores of group g).
            if (nt == kSteps) {
                constexpr int G = 8;
                T xn[G];
#pragma unroll
                for (int j = 0; j < G; ++j) xn[j] = xt[j * kLifChannels + tid];
#pragma unroll 1
                for (int g = 0; g < kSteps / G; ++g) {
                    T xc[G];
#pragma unroll
                    for (int j = 0; j < G; ++j) xc[j] = xn[j];
                    if (g + 1 < kSteps / G) {
#pragma unroll
                        for (int j = 0; j < G; ++j) xn[j] = xt[((g + 1) * G + j) * kLifChannels + tid];
                    }
#pragma unroll
                    for (int j = 0; j < G; ++j) {
                        const bool fired = lif_step(v, beta, th, M::in(xc[j]));
                        sp[g * G + j][tid] = spike_val<T>(fired && live);
                    }
                }
            } else {
#pragma unroll 4
                for (int tt = 0; tt < nt; ++tt) {
                    const bool fired = lif_step(v, beta, th, M::in(xt[tt * kLifChannels + tid]));
                    sp[tt][tid] = spike_val<T>(fired && live);
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(smem_u32(&in_empty[st]));
                mbar_arrive(smem_u32(&spk_full[sb2]));
            }
        }
        if (!ok) {
            if (lane == 0) atomicOr(err, ERRF_TIMEOUT_EPILOGUE);
            return;
        }
        if (live && a.mem_out) static_cast<T*>(a.mem_out)[b * a.C + c] = E::from_f(Elem<MATH>::to_f(v));
        return;
    }

    // ========================= helper warp ==================================
    const T* xb = static_cast<const T*>(a.x) + b * a.x_sb;
    T* sbase = static_cast<T*>(a.spikes) + b * a.s_sb;
    const bool full_cols = c0 + kLifChannels <= a.C;
    const bool vec_in = full_cols && (a.x_st % EPV == 0) && (a.x_sb % EPV == 0) &&
                        ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
    const bool vec_out = full_cols && (a.s_st % EPV == 0) && (a.s_sb % EPV == 0) &&
                         ((reinterpret_cast<uintptr_t>(a.spikes) & 15) == 0);
    constexpr int VPR = kLifChannels / EPV;      // 16-byte vectors per tile row
    // input tile k into stage k % kLifStages; one commit group per tile slot
    auto issue = [&](int k) {
        if (k < ntiles) {
            T* dst = &tile[k % kLifStages][0][0];
            const int64_t t0 = (int64_t)k * kSteps;
            if (vec_in) {
                for (int i = lane; i < kSteps * VPR; i += 32) {
                    const int tt = i / VPR, vv = i % VPR;
                    const int64_t t = t0 + tt;
                    if (t < a.T) cp16(dst + tt * kLifChannels + vv * EPV, xb + t * a.x_st + c0 + vv * EPV);
                }
            } else {
                for (int i = lane; i < kSteps * kLifChannels; i += 32) {
                    const int tt = i / kLifChannels, cc = i % kLifChannels;
                    const int64_t t = t0 + tt;
                    dst[i] = (t < a.T && c0 + cc < a.C) ? xb[t * a.x_st + c0 + cc] : T(0.f);
                }
            }
        }
        commit();
    };
    unsigned local_count = 0;
    // spike tile j out, its per-row counts, row-activity words; then hand it back
    auto out = [&](int j) -> bool {
        const int sb2 = j & 1;
        if (!lif_wait(&spk_full[sb2], (j >> 1) & 1)) return false;
        T (*sp)[kLifChannels] = spk[sb2];
        const int64_t t0 = (int64_t)j * kSteps;
        const int nt = (a.T - t0 < kSteps) ? (int)(a.T - t0) : kSteps;
        if (vec_out) {
            for (int i = lane; i < nt * VPR; i += 32) {
                const int tt = i / VPR, vv = i % VPR;
                *reinterpret_cast<uint4*>(sbase + (t0 + tt) * a.s_st + c0 + vv * EPV) =
                    *reinterpret_cast<const uint4*>(&sp[tt][vv * EPV]);
            }
        } else {
            for (int i = lane; i < nt * kLifChannels; i += 32) {
                const int tt = i / kLifChannels, cc = i % kLifChannels;
                if (c0 + cc < a.C) sbase[(t0 + tt) * a.s_st + c0 + cc] = sp[tt][cc];
            }
        }
#pragma unroll
        for (int m = 0; m < kSteps / 32; ++m) {
            const int tt = lane + 32 * m;
            int cnt = 0;
            if (tt < nt) {
                // each lane starts at another 16-byte column (rows are 128 or 256 B
                // apart, so equal columns would share banks)
                constexpr int NQ = kLifChannels * (int)sizeof(T) / 16;
                const uint4* row = reinterpret_cast<const uint4*>(&sp[tt][0]);
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    const uint4 w = row[(q + tt) & (NQ - 1)];
                    cnt += spikes_in_word<T>(w.x) + spikes_in_word<T>(w.y) + spikes_in_word<T>(w.z) +
                           spikes_in_word<T>(w.w);
                }
            }
            local_count += cnt;
            if (a.row_bits) {
                const unsigned word = __ballot_sync(0xffffffffu, cnt != 0);
                const int64_t wi = t0 / 32 + m;
                if (lane == 0 && wi < a.n_words) a.row_bits[((int64_t)blockIdx.x * a.B + b) * a.n_words + wi] = word;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&spk_empty[sb2]));
        return true;
    };

    // Tile j is announced (in_full) as soon as it has landed, one tile ahead of
    // the membrane warps; commit groups: one per tile slot, tiles in order.
    static_assert(kLifStages == 3, "wait_group counts below assume three stages");
    for (int k = 0; k < kLifStages; ++k) issue(k);
    asm volatile("cp.async.wait_group 2;" ::: "memory");                  // tile 0 has landed
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&in_full[0]));
    bool ok = true;
    for (int k = 0; k < ntiles && ok; ++k) {
        if (k + 1 < ntiles) {
            asm volatile("cp.async.wait_group 1;" ::: "memory");          // tiles up to k+1 have landed
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&in_full[(k + 1) % kLifStages]));
        }
        if (k >= 1 && !out(k - 1)) { ok = false; break; }
        // stage k % kLifStages takes tile k + kLifStages once the membrane warps are done with tile k
        if (k + kLifStages < ntiles) {
            if (!lif_wait(&in_empty[k % kLifStages], (k / kLifStages) & 1)) { ok = false; break; }
        }
        issue(k + kLifStages);
    }
    if (ok && ntiles > 0 && !out(ntiles - 1)) ok = false;
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (!ok) {
        if (lane == 0) atomicOr(err, ERRF_TIMEOUT_PRODUCER);
        return;
    }
    if (a.spike_count) {
        const unsigned wsum = __reduce_add_sync(0xffffffffu, local_count);
        if (lane == 0 && wsum) atomicAdd(a.spike_count, (unsigned long long)wsum);
    }
}

// Short sequences (T <= 32, e.g. decode steps): the tile ring above costs far
// more than a few steps, so one thread owns one (batch, channel) membrane and
// reads its inputs directly (consecutive channels: coalesced).  A 256-thread
// CTA covers four 64-channel blocks of one batch row; each warp's ballot per
// step gives the row-activity bit of its 32 channels, and the two warps of a
// block combine their words through shared memory (T <= 32: one word).
constexpr int kLifShortMaxT = 32;

template <int DT, int MATH>
__global__ void __launch_bounds__(256)
lif_short_kernel(LifArgs a) {
    using E = Elem<DT>;
    using T = typename E::T;
    using S = typename Elem<MATH>::T;
    using M = MathOf<S>;
    __shared__ unsigned s_bits[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t c = (int64_t)blockIdx.x * 256 + tid, b = blockIdx.y;
    const bool live = c < a.C;
    S beta = M::from(0.f), th = M::from(0.f), v = M::from(0.f);
    if (live) {
        beta = M::from(E::load(static_cast<const T*>(a.beta) + c));
        th = M::from(E::load(static_cast<const T*>(a.threshold) + c));
        if (a.mem_in) v = M::from(E::load(static_cast<const T*>(a.mem_in) + b * a.C + c));
    }
    const T* xb = static_cast<const T*>(a.x) + b * a.x_sb;
    T* sb = static_cast<T*>(a.spikes) + b * a.s_sb;
    unsigned bits = 0, count = 0;
    for (int64_t t = 0; t < a.T; ++t) {
        bool fired = false;
        if (live) {
            fired = lif_step(v, beta, th, M::in(xb[t * a.x_st + c]));
            sb[t * a.s_st + c] = spike_val<T>(fired);
        }
        count += fired;
        if (__ballot_sync(0xffffffffu, fired)) bits |= 1u << t;
    }
    if (live && a.mem_out) static_cast<T*>(a.mem_out)[b * a.C + c] = E::from_f(Elem<MATH>::to_f(v));
    if (a.spike_count) {
        const unsigned wsum = __reduce_add_sync(0xffffffffu, count);
        if (lane == 0 && wsum) atomicAdd(a.spike_count, (unsigned long long)wsum);
    }
    if (a.row_bits) {
        if (lane == 0) s_bits[warp] = bits;
        __syncthreads();
        // warps 2k and 2k+1 hold the 64 channels of block blockIdx.x*4 + k; thread k writes it
        const int64_t cblk = (int64_t)blockIdx.x * 4 + tid;
        if (tid < 4 && cblk * kLifChannels < a.C)
            a.row_bits[(cblk * a.B + b) * a.n_words] = s_bits[2 * tid] | s_bits[2 * tid + 1];
    }
}

}  // namespace

template <int DT, int MATH>
int launch_lif_typed(const LifArgs& a, cudaStream_t stream) {
    using T = typename Elem<DT>::T;
    constexpr size_t smem = LifSmem<T>::bytes;
    auto kern = lif_scan_kernel<DT, MATH>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NT_ERR_CUDA, "lif_scan: smem attribute: %s", cudaGetErrorString(e));
    int dev = 0;
    cudaGetDevice(&dev);
    if (a.T <= kLifShortMaxT) {
        dim3 grid((unsigned)((a.C + 255) / 256), (unsigned)a.B);
        lif_short_kernel<DT, MATH><<<grid, 256, 0, stream>>>(a);
        return check_launch("lif_short_kernel");
    }
    dim3 grid((unsigned)((a.C + kLifChannels - 1) / kLifChannels), (unsigned)a.B);
    kern<<<grid, kLifThreads, smem, stream>>>(a, device_error_word(dev));
    return check_launch("lif_scan_kernel");
}

int launch_lif_scan(int dtype, int math, const LifArgs& a, cudaStream_t stream) {
    if (dtype == NT_F32 && math == NT_F32) return launch_lif_typed<NT_F32, NT_F32>(a, stream);
    if (dtype == NT_BF16 && math == NT_BF16) return launch_lif_typed<NT_BF16, NT_BF16>(a, stream);
    if (dtype == NT_BF16 && math == NT_F32) return launch_lif_typed<NT_BF16, NT_F32>(a, stream);
    return fail(NT_ERR_DTYPE, "lif_scan: unsupported dtype %d / math %d", dtype, math);
}

}  // namespace nt
