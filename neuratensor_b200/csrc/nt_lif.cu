// LIF membrane recurrence (neuratensor/core/snn.py:64-75,167-182).
//
// The recurrence is non-linear (threshold + reset), so time stays serial per
// channel: one thread owns one (batch, channel) membrane for the whole
// sequence.  A CTA covers kLifChannels channels of one batch row.  Input
// tiles of kLifSteps steps x kLifChannels channels stream into a
// kLifStages-deep shared-memory ring with cp.async, so the only latency on
// the serial path is the membrane update itself.
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

constexpr int kLifStages = 4;
// steps per tile: 32 KB of staging for the whole ring in either dtype
template <typename T> struct LifSteps { static constexpr int value = 128 / (int)sizeof(T); };

__device__ __forceinline__ void cp16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem) : "memory");
}
__device__ __forceinline__ void commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void wait_stages() {
    asm volatile("cp.async.wait_group %0;" ::"n"(kLifStages - 2) : "memory");
}

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

template <int DT, int MATH>
__global__ void __launch_bounds__(kLifChannels)
lif_scan_kernel(LifArgs a) {
    using E = Elem<DT>;
    using T = typename E::T;
    using S = typename Elem<MATH>::T;       // state / arithmetic type
    using M = MathOf<S>;
    constexpr int EPV = 16 / (int)sizeof(T);
    constexpr int kLifSteps = LifSteps<T>::value;
    __shared__ __align__(16) T tile[kLifStages][kLifSteps][kLifChannels];
    __shared__ __align__(16) T spk_tile[kLifSteps][kLifChannels];
    __shared__ unsigned row_mask[kLifSteps][kLifChannels / 32];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t c0 = (int64_t)blockIdx.x * kLifChannels, c = c0 + tid, b = blockIdx.y;
    const bool live = c < a.C;
    const T* xb = static_cast<const T*>(a.x) + b * a.x_sb;
    T* sb = static_cast<T*>(a.spikes) + b * a.s_sb;

    S beta = M::from(0.f), th = M::from(0.f), v = M::from(0.f);
    if (live) {
        beta = M::from(E::load(static_cast<const T*>(a.beta) + c));
        th = M::from(E::load(static_cast<const T*>(a.threshold) + c));
        if (a.mem_in) v = M::from(E::load(static_cast<const T*>(a.mem_in) + b * a.C + c));
    }
    // 16-byte copies when every row segment of the tile is aligned
    const bool full_cols = c0 + kLifChannels <= a.C;
    const bool vec_in = full_cols && (a.x_st % EPV == 0) && (a.x_sb % EPV == 0) &&
                        ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
    const bool vec_out = full_cols && (a.s_st % EPV == 0) && (a.s_sb % EPV == 0) &&
                         ((reinterpret_cast<uintptr_t>(a.spikes) & 15) == 0);
    const int ntiles = (int)((a.T + kLifSteps - 1) / kLifSteps);
    constexpr int VPR = kLifChannels / EPV;      // 16-byte vectors per tile row

    auto issue = [&](int k) {
        if (k < ntiles) {
            T* dst = &tile[k % kLifStages][0][0];
            const int64_t t0 = (int64_t)k * kLifSteps;
            if (vec_in) {
                for (int i = tid; i < kLifSteps * VPR; i += kLifChannels) {
                    const int tt = i / VPR, vv = i % VPR;
                    const int64_t t = t0 + tt;
                    if (t < a.T) cp16(dst + tt * kLifChannels + vv * EPV, xb + t * a.x_st + c0 + vv * EPV);
                }
            } else {
                for (int i = tid; i < kLifSteps * kLifChannels; i += kLifChannels) {
                    const int tt = i / kLifChannels, cc = i % kLifChannels;
                    const int64_t t = t0 + tt;
                    dst[i] = (t < a.T && c0 + cc < a.C) ? xb[t * a.x_st + c0 + cc] : T(0.f);
                }
            }
        }
        commit();   // one group per tile slot (possibly empty) keeps the wait count uniform
    };

    for (int k = 0; k < kLifStages - 1; ++k) issue(k);
    unsigned local_count = 0;
    for (int k = 0; k < ntiles; ++k) {
        issue(k + kLifStages - 1);
        wait_stages();
        __syncthreads();
        const T* xt = &tile[k % kLifStages][0][0];
        const int64_t t0 = (int64_t)k * kLifSteps;
        const int nt = (a.T - t0 < kLifSteps) ? (int)(a.T - t0) : kLifSteps;
#pragma unroll 8
        for (int tt = 0; tt < nt; ++tt) {
            const bool fired = lif_step(v, beta, th, M::in(xt[tt * kLifChannels + tid])) && live;
            spk_tile[tt][tid] = spike_val<T>(fired);
            const unsigned m = __ballot_sync(0xffffffffu, fired);
            if (lane == 0) row_mask[tt][warp] = m;
        }
        __syncthreads();   // spike tile complete; input slot k is refilled next iteration
        // spikes out (16-byte stores when aligned) and per-row counts from the tile
        if (vec_out) {
            for (int i = tid; i < nt * VPR; i += kLifChannels) {
                const int tt = i / VPR, vv = i % VPR;
                *reinterpret_cast<uint4*>(sb + (t0 + tt) * a.s_st + c0 + vv * EPV) =
                    *reinterpret_cast<const uint4*>(&spk_tile[tt][vv * EPV]);
            }
        } else {
            for (int i = tid; i < nt * kLifChannels; i += kLifChannels) {
                const int tt = i / kLifChannels, cc = i % kLifChannels;
                if (c0 + cc < a.C) sb[(t0 + tt) * a.s_st + c0 + cc] = spk_tile[tt][cc];
            }
        }
        // per-row spike counts; row-activity words (32 rows each) of this channel block
        static_assert(kLifSteps <= kLifChannels && kLifSteps % 32 == 0, "one thread per tile row");
        {
            const int tt = tid;
            unsigned cnt = 0;
            if (tt < nt) {
#pragma unroll
                for (int w = 0; w < kLifChannels / 32; ++w) cnt += __popc(row_mask[tt][w]);
            }
            local_count += cnt;
            if (a.row_bits && tt < kLifSteps) {
                const unsigned word = __ballot_sync(0xffffffffu, cnt != 0);
                const int64_t wi = t0 / 32 + tt / 32;
                if (lane == 0 && wi < a.n_words) a.row_bits[((int64_t)blockIdx.x * a.B + b) * a.n_words + wi] = word;
            }
        }
        __syncthreads();   // spike tile is rewritten by the next tile
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (live && a.mem_out) static_cast<T*>(a.mem_out)[b * a.C + c] = E::from_f(Elem<MATH>::to_f(v));
    if (a.spike_count) {
        const unsigned wsum = __reduce_add_sync(0xffffffffu, local_count);
        if (lane == 0 && wsum) atomicAdd(a.spike_count, (unsigned long long)wsum);
    }
}

}  // namespace

int launch_lif_scan(int dtype, int math, const LifArgs& a, cudaStream_t stream) {
    dim3 grid((unsigned)((a.C + kLifChannels - 1) / kLifChannels), (unsigned)a.B);
    if (dtype == NT_F32 && math == NT_F32) lif_scan_kernel<NT_F32, NT_F32><<<grid, kLifChannels, 0, stream>>>(a);
    else if (dtype == NT_BF16 && math == NT_BF16) lif_scan_kernel<NT_BF16, NT_BF16><<<grid, kLifChannels, 0, stream>>>(a);
    else if (dtype == NT_BF16 && math == NT_F32) lif_scan_kernel<NT_BF16, NT_F32><<<grid, kLifChannels, 0, stream>>>(a);
    else return fail(NT_ERR_DTYPE, "lif_scan: unsupported dtype %d / math %d", dtype, math);
    return check_launch("lif_scan_kernel");
}

}  // namespace nt
