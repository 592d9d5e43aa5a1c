// LIF membrane recurrence (neuratensor/core/snn.py:64-75,167-182).
//
// One thread owns one (batch, channel) membrane for the whole sequence: the
// recurrence is non-linear (threshold + reset), so time stays serial per
// channel while channels run in parallel.  Loads of the next UNROLL steps are
// issued before the serial chain consumes them so the chain, not memory
// latency, sets the pace.
//
// Arithmetic follows the reference exactly:
//   V = beta*V + x      -- a product then a sum, each rounded to the dtype
//   S = V >= theta
//   V = V - theta*S
// fp32: __fmul_rn/__fadd_rn keep the two roundings (no FMA contraction), so
// spikes and membranes are bit-identical to the reference on equal inputs.
// bf16: each result is rounded to bfloat16, as torch does for bf16 tensors.
#include "nt_kernels.cuh"

namespace nt {

template <int DT, int MATH>
__global__ void __launch_bounds__(128)
lif_scan_kernel(LifArgs a) {
    using E = Elem<DT>;
    using T = typename E::T;
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t b = blockIdx.y;
    const bool live = c < a.C;
    const T* __restrict__ x = static_cast<const T*>(a.x);
    T* __restrict__ s = static_cast<T*>(a.spikes);

    float beta = 0.f, th = 0.f, v = 0.f;
    if (live) {
        beta = E::load(static_cast<const T*>(a.beta) + c);
        th = E::load(static_cast<const T*>(a.threshold) + c);
        if (a.mem_in) v = E::load(static_cast<const T*>(a.mem_in) + b * a.C + c);
    }
    const T* xp = x + b * a.x_sb + c;
    T* sp = s + b * a.s_sb + c;

    // per-row partial spike counts: each warp ballots, lane 0 accumulates into
    // shared memory; flushed every ROWS steps (only used by the block path).
    constexpr int ROWS = 64;
    __shared__ unsigned short row_cnt[ROWS][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    unsigned local_count = 0;

    constexpr int UNROLL = 8;
    for (int64_t t0 = 0; t0 < a.T; t0 += UNROLL) {
        float xv[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int64_t t = t0 + u;
            xv[u] = (live && t < a.T) ? E::load(xp + t * a.x_st) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const int64_t t = t0 + u;
            if (t >= a.T) break;
            float spk = 0.f;
            if (MATH == NT_F32) {
                v = __fadd_rn(__fmul_rn(beta, v), xv[u]);
                spk = (v >= th) ? 1.f : 0.f;
                v = __fsub_rn(v, __fmul_rn(th, spk));
            } else {
                v = bf16_round(bf16_round(beta * v) + xv[u]);
                spk = (v >= th) ? 1.f : 0.f;
                v = bf16_round(v - bf16_round(th * spk));
            }
            if (live) sp[t * a.s_st] = E::from_f(spk);
            const unsigned ballot = __ballot_sync(0xffffffffu, live && spk != 0.f);
            local_count += (live && spk != 0.f) ? 1u : 0u;
            if (a.row_partials) {
                const int r = (int)(t % ROWS);
                if (lane == 0) row_cnt[r][warp] = (unsigned short)__popc(ballot);
                if (r == ROWS - 1 || t == a.T - 1) {
                    __syncthreads();
                    const int64_t tb = t - r;  // first row of this flush window
                    for (int i = threadIdx.x; i <= r; i += blockDim.x) {
                        const unsigned short sum = row_cnt[i][0] + row_cnt[i][1] + row_cnt[i][2] + row_cnt[i][3];
                        a.row_partials[(b * a.T + tb + i) * a.n_cblk + blockIdx.x] = sum;
                    }
                    __syncthreads();
                }
            }
        }
    }
    if (live && a.mem_out) static_cast<T*>(a.mem_out)[b * a.C + c] = E::from_f(v);
    if (a.spike_count) {
        unsigned wsum = __reduce_add_sync(0xffffffffu, local_count);
        if (lane == 0 && wsum) atomicAdd(a.spike_count, (unsigned long long)wsum);
    }
}

int launch_lif_scan(int dtype, int math, const LifArgs& a, cudaStream_t stream) {
    dim3 grid((unsigned)((a.C + 127) / 128), (unsigned)a.B);
    if (dtype == NT_F32 && math == NT_F32) lif_scan_kernel<NT_F32, NT_F32><<<grid, 128, 0, stream>>>(a);
    else if (dtype == NT_BF16 && math == NT_BF16) lif_scan_kernel<NT_BF16, NT_BF16><<<grid, 128, 0, stream>>>(a);
    else if (dtype == NT_BF16 && math == NT_F32) lif_scan_kernel<NT_BF16, NT_F32><<<grid, 128, 0, stream>>>(a);
    else return fail(NT_ERR_DTYPE, "lif_scan: unsupported dtype %d / math %d", dtype, math);
    return check_launch("lif_scan_kernel");
}

}  // namespace nt
