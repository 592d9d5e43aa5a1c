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
// bf16: native bfloat16 multiply/add/subtract (round-to-nearest-even), which
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

// Membrane update for one step; returns the spike (0/1).
template <int MATH>
__device__ __forceinline__ float lif_step(float& v, float beta, float th, float x) {
    if (MATH == NT_F32) {
        v = __fadd_rn(__fmul_rn(beta, v), x);
        const float s = (v >= th) ? 1.f : 0.f;
        v = __fsub_rn(v, __fmul_rn(th, s));
        return s;
    } else {
        const __nv_bfloat16 vb = __hadd(__hmul(__float2bfloat16_rn(beta), __float2bfloat16_rn(v)),
                                        __float2bfloat16_rn(x));
        const float vf = __bfloat162float(vb);
        const bool s = vf >= th;
        v = s ? __bfloat162float(__hsub(vb, __float2bfloat16_rn(th))) : vf;
        return s ? 1.f : 0.f;
    }
}

template <int DT, int MATH>
__global__ void __launch_bounds__(kLifChannels)
lif_scan_kernel(LifArgs a) {
    using E = Elem<DT>;
    using T = typename E::T;
    constexpr int EPV = 16 / (int)sizeof(T);
    constexpr int kLifSteps = LifSteps<T>::value;
    __shared__ __align__(16) T tile[kLifStages][kLifSteps][kLifChannels];
    __shared__ unsigned short row_cnt[kLifSteps][kLifChannels / 32];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t c0 = (int64_t)blockIdx.x * kLifChannels, c = c0 + tid, b = blockIdx.y;
    const bool live = c < a.C;
    const T* xb = static_cast<const T*>(a.x) + b * a.x_sb;
    T* sp = static_cast<T*>(a.spikes) + b * a.s_sb + c;

    float beta = 0.f, th = 0.f, v = 0.f;
    if (live) {
        beta = E::load(static_cast<const T*>(a.beta) + c);
        th = E::load(static_cast<const T*>(a.threshold) + c);
        if (a.mem_in) v = E::load(static_cast<const T*>(a.mem_in) + b * a.C + c);
    }
    // 16-byte copies when every row segment of the tile is aligned
    const bool vec = (c0 + kLifChannels <= a.C) && (a.x_st % EPV == 0) && (a.x_sb % EPV == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
    const int ntiles = (int)((a.T + kLifSteps - 1) / kLifSteps);

    auto issue = [&](int k) {
        if (k < ntiles) {
            T* dst = &tile[k % kLifStages][0][0];
            const int64_t t0 = (int64_t)k * kLifSteps;
            if (vec) {
                constexpr int VPR = kLifChannels / EPV;
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
            const float spk = lif_step<MATH>(v, beta, th, E::to_f(xt[tt * kLifChannels + tid]));
            const bool fired = live && spk != 0.f;
            if (live) sp[(t0 + tt) * a.s_st] = E::from_f(spk);
            local_count += fired ? 1u : 0u;
            if (a.row_partials) {
                const unsigned ballot = __ballot_sync(0xffffffffu, fired);
                if (lane == 0) row_cnt[tt][warp] = (unsigned short)__popc(ballot);
            }
        }
        __syncthreads();   // tile slot k is refilled next iteration; row counts complete
        if (a.row_partials) {
            for (int i = tid; i < nt; i += kLifChannels) {
                unsigned short sum = 0;
#pragma unroll
                for (int w = 0; w < kLifChannels / 32; ++w) sum += row_cnt[i][w];
                a.row_partials[(b * a.T + t0 + i) * a.n_cblk + blockIdx.x] = sum;
            }
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (live && a.mem_out) static_cast<T*>(a.mem_out)[b * a.C + c] = E::from_f(v);
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
