// Selective scan (neuratensor/core/ssm.py:106-139 discretisation,
// ssm.py:184-221 sequential scan, ssm.py:145-182 single step) and the
// standalone LIF -> selective-scan fusion.
//
// Work split: a channel's d_state recurrences are spread over TPC threads
// (8 states each, TPC = next power of two >= N/8), so a 128-thread CTA owns
// CPB = 128/TPC channels of one batch row.  Time is walked serially in
// chunks of TCH steps: each chunk's inputs (u, dt, gate, B, C) are staged in
// shared memory with coalesced loads, the recurrence runs from registers, and
// the chunk's outputs are written back coalesced.  The state never leaves
// registers between chunks; it is float32 whatever the activation dtype.
//
// Discretisation per step (A = -exp(log_A), computed once per state):
//   A_bar = exp(dt*A)             -> ex2(dt * A*log2(e)) on the MUFU pipe
//   B_bar = (A_bar - 1)/A * B     (dt*B where |A| < 1e-6, ssm.py:129-137)
//   h     = A_bar*h + B_bar*u     (the B_bar term is skipped when u == 0)
//   y     = sum_n C[n]*h[n] + D*u
// When A has the HiPPO structure A[c,n] = (n+1)*A[c,0] (the reference's
// initialisation, ssm.py:34-43) the kernel detects it per CTA and replaces
// the per-state exponentials by one exponential per thread and a chain of
// multiplies: exp(dt*A[c,n+1]) = exp(dt*A[c,n]) * exp(dt*A[c,0]).
#include "nt_kernels.cuh"

namespace nt {

namespace {

constexpr int kTch = 32;    // time steps per staged chunk
constexpr int kNpt = 8;     // d_state entries per thread

template <int DT>
__device__ __forceinline__ float ld_act(const void* p, int64_t i) {
    return Elem<DT>::load(static_cast<const typename Elem<DT>::T*>(p) + i);
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

// MODE 0: plain selective scan (u given).  MODE 1: u = LIF spikes of x.
template <int DT, int SDT, int TPC, int MODE>
__global__ void __launch_bounds__(128)
scan_kernel(ScanArgs a, FusedArgs f) {
    constexpr int CPB = 128 / TPC;
    constexpr int NP = kNpt * TPC;
    extern __shared__ float smem[];
    float* s_u = smem;                 // [kTch][CPB]  u (MODE 0) or x (MODE 1)
    float* s_dt = s_u + kTch * CPB;    // [kTch][CPB]
    float* s_g = s_dt + kTch * CPB;    // [kTch][CPB]  gate
    float* s_y = s_g + kTch * CPB;     // [kTch][CPB]  y (and spikes in MODE 1 via s_g)
    float* s_B = s_y + kTch * CPB;     // [kTch][NP]
    float* s_C = s_B + kTch * NP;      // [kTch][NP]

    const int64_t T = MODE ? f.L : a.T, d = MODE ? f.d : a.d, N = MODE ? f.N : a.N;
    const void* p_u = MODE ? f.x : a.u;
    const void* p_dt = MODE ? f.delta : a.dt;
    const void* p_B = MODE ? f.Bm : a.Bm;
    const void* p_C = MODE ? f.Cm : a.Cm;
    const bool has_gate = (MODE == 0) && a.gate != nullptr;
    const int64_t ld_bc = (MODE == 0 && a.ld_bc > 0) ? a.ld_bc : N;

    const int tid = threadIdx.x, cl = tid / TPC, sub = tid % TPC;
    const int64_t c0 = (int64_t)blockIdx.x * CPB, c = c0 + cl, b = blockIdx.y;
    const bool live = c < d;

    // ---- per-state constants ------------------------------------------------
    // A = -exp(log_A), rounded like the reference's own tensor op (ssm.py:121)
    auto load_A = [&](int64_t n) -> float {
        if (MODE == 0) return -Elem<DT>::rnd(expf(ld_act<DT>(a.log_A, c * N + n)));
        return -expf(f.log_A[c * N + n]);
    };
    float A2[kNpt], cinv[kNpt], h[kNpt];
    unsigned lim_mask = 0;
    bool hippo_ok = true;
    const float Abase = live ? load_A(0) : 0.f;
    const void* sin = MODE ? (const void*)f.state_in : a.state_in;
#pragma unroll
    for (int j = 0; j < kNpt; ++j) {
        const int64_t n = (int64_t)sub * kNpt + j;
        float A = 0.f;
        h[j] = 0.f;
        if (live && n < N) {
            A = load_A(n);
            if (sin) {
                const int64_t si = (b * d + c) * N + n;
                if (MODE == 0 && SDT == NT_BF16) h[j] = ld_act<NT_BF16>(sin, si);
                else h[j] = static_cast<const float*>(sin)[si];
            }
            // HiPPO structure check: A[c,n] == (n+1) * A[c,0] to 1e-6 relative
            if (fabsf(A - (float)(n + 1) * Abase) > 1e-6f * fabsf(A)) hippo_ok = false;
        }
        A2[j] = A * kLog2e;
        const bool lim = (live && n < N) && fabsf(A) < 1e-6f;
        if (lim) { lim_mask |= 1u << j; hippo_ok = false; }
        cinv[j] = (A == 0.f) ? 0.f : 1.0f / A;
    }
    const float q2 = Abase * kLog2e;
    const bool hippo = __syncthreads_and(hippo_ok ? 1 : 0) != 0;
    float Dv = 0.f, beta = 0.f, th = 0.f, mem = 0.f;
    if (live) {
        Dv = MODE == 0 ? ld_act<DT>(a.D, c) : f.Dskip[c];
        if (MODE == 1) {
            beta = f.beta[c];
            th = f.threshold[c];
            if (f.mem_in) mem = f.mem_in[b * d + c];
        }
    }
    unsigned spike_local = 0;
    const bool sparse_rows = (MODE == 0) && a.row_pos != nullptr && a.sparse_flag != nullptr && *a.sparse_flag != 0;

    for (int64_t t0 = 0; t0 < T; t0 += kTch) {
        __syncthreads();
        // ---- stage the chunk ----------------------------------------------
        for (int i = tid; i < kTch * CPB; i += 128) {
            const int tt = i / CPB, cc = i % CPB;
            const int64_t t = t0 + tt, cg = c0 + cc;
            const bool ok = t < T && cg < d;
            const int64_t idx = (b * T + t) * d + cg;
            if (MODE == 0) {
                s_u[i] = ok ? ld_act<DT>(p_u, idx) : 0.f;
                s_dt[i] = ok ? ld_act<DT>(p_dt, idx) : 0.f;
                if (has_gate) s_g[i] = ok ? ld_act<DT>(a.gate, idx) : 0.f;
            } else {
                s_u[i] = ok ? ld_act<NT_BF16>(p_u, idx) : 0.f;
                s_dt[i] = ok ? ld_act<NT_BF16>(p_dt, idx) : 0.f;
            }
        }
        for (int i = tid; i < kTch * NP; i += 128) {
            const int tt = i / NP, n = i % NP;
            const int64_t t = t0 + tt;
            const bool ok = t < T && n < N;
            const int64_t idx = (b * T + t) * ld_bc + n;
            s_B[i] = ok ? (MODE == 0 ? ld_act<DT>(p_B, idx) : ld_act<NT_BF16>(p_B, idx)) : 0.f;
            s_C[i] = ok ? (MODE == 0 ? ld_act<DT>(p_C, idx) : ld_act<NT_BF16>(p_C, idx)) : 0.f;
        }
        __syncthreads();
        const int nt = (T - t0 < kTch) ? (int)(T - t0) : kTch;
        for (int tt = 0; tt < nt; ++tt) {
            float u;
            if (MODE == 0) {
                u = s_u[tt * CPB + cl];
            } else {
                // LIF step (snn.py:177-181) in fp32, same in every thread of the channel
                mem = __fadd_rn(__fmul_rn(beta, mem), s_u[tt * CPB + cl]);
                u = (mem >= th) ? 1.f : 0.f;
                mem = __fsub_rn(mem, __fmul_rn(th, u));
            }
            const float dtv = s_dt[tt * CPB + cl];
            float av[kNpt];
            if (hippo) {
                av[0] = ex2(dtv * A2[0]);
                const float qv = ex2(dtv * q2);
#pragma unroll
                for (int j = 1; j < kNpt; ++j) av[j] = av[j - 1] * qv;
            } else {
#pragma unroll
                for (int j = 0; j < kNpt; ++j) av[j] = ex2(dtv * A2[j]);
            }
            const float4* Bp = reinterpret_cast<const float4*>(s_B + tt * NP + sub * kNpt);
            const float4* Cp = reinterpret_cast<const float4*>(s_C + tt * NP + sub * kNpt);
            const float4 b0 = Bp[0], b1 = Bp[1], k0 = Cp[0], k1 = Cp[1];
            const float Bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            const float Cv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
            if (u != 0.f) {
#pragma unroll
                for (int j = 0; j < kNpt; ++j) {
                    const float coef = (lim_mask >> j & 1u) ? dtv : (av[j] - 1.0f) * cinv[j];
                    h[j] = fmaf(av[j], h[j], coef * Bv[j] * u);
                }
            } else {
#pragma unroll
                for (int j = 0; j < kNpt; ++j) h[j] = av[j] * h[j];
            }
            float yp = 0.f;
#pragma unroll
            for (int j = 0; j < kNpt; ++j) yp = fmaf(Cv[j], h[j], yp);
#pragma unroll
            for (int off = TPC / 2; off > 0; off >>= 1) yp += __shfl_xor_sync(0xffffffffu, yp, off);
            if (sub == 0) {
                s_y[tt * CPB + cl] = __fadd_rn(yp, __fmul_rn(Dv, u));
                if (MODE == 1) s_g[tt * CPB + cl] = u;
            }
            if (MODE == 1 && sub == 0 && live) spike_local += (u != 0.f);
        }
        __syncthreads();
        // ---- write the chunk's outputs -------------------------------------
        for (int i = tid; i < kTch * CPB; i += 128) {
            const int tt = i / CPB, cc = i % CPB;
            const int64_t t = t0 + tt, cg = c0 + cc;
            if (t >= T || cg >= d) continue;
            int64_t row = b * T + t;
            if (MODE == 0) {
                using E = Elem<DT>;
                float o = E::rnd(s_y[i]);
                if (has_gate) o = E::rnd(o * E::rnd(silu_f(s_g[i])));
                if (sparse_rows) {
                    const int pos = a.row_pos[row];
                    if (pos < 0) continue;
                    row = pos;
                }
                static_cast<typename E::T*>(a.y)[row * d + cg] = E::from_f(o);
            } else {
                static_cast<__nv_bfloat16*>(f.y)[row * d + cg] = __float2bfloat16_rn(s_y[i]);
                if (f.spikes) {
                    if (f.spike_dtype == NT_U8) static_cast<unsigned char*>(f.spikes)[row * d + cg] = (unsigned char)(s_g[i] != 0.f);
                    else static_cast<__nv_bfloat16*>(f.spikes)[row * d + cg] = __float2bfloat16_rn(s_g[i]);
                }
            }
        }
    }
    // ---- carry-out ------------------------------------------------------------
    void* sout = MODE ? (void*)f.state_out : a.state_out;
    if (live && sout) {
#pragma unroll
        for (int j = 0; j < kNpt; ++j) {
            const int64_t n = (int64_t)sub * kNpt + j;
            if (n >= N) continue;
            const int64_t si = (b * d + c) * N + n;
            if (MODE == 0 && SDT == NT_BF16) static_cast<__nv_bfloat16*>(sout)[si] = __float2bfloat16_rn(h[j]);
            else static_cast<float*>(sout)[si] = h[j];
        }
    }
    if (MODE == 1) {
        if (live && sub == 0 && f.mem_out) f.mem_out[b * d + c] = mem;
        if (f.spike_count) {
            const unsigned w = __reduce_add_sync(0xffffffffu, spike_local);
            if ((tid & 31) == 0 && w) atomicAdd(f.spike_count, (unsigned long long)w);
        }
    }
}

int pow2_tpc(int64_t N) {
    int tpc = 1;
    while (tpc * kNpt < N) tpc <<= 1;
    return tpc;
}

template <int DT, int SDT, int MODE, int TPC>
int launch_tpc(const ScanArgs& a, const FusedArgs& f, cudaStream_t stream) {
    constexpr int CPB = 128 / TPC;
    const size_t smem = sizeof(float) * (size_t)(4 * kTch * CPB + 2 * kTch * kNpt * TPC);
    auto kern = scan_kernel<DT, SDT, TPC, MODE>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return fail(NT_ERR_CUDA, "scan: smem attribute: %s", cudaGetErrorString(e));
    }
    const int64_t d = MODE ? f.d : a.d, B = MODE ? f.B : a.B;
    dim3 grid((unsigned)((d + CPB - 1) / CPB), (unsigned)B);
    kern<<<grid, 128, smem, stream>>>(a, f);
    return check_launch("scan_kernel");
}

template <int DT, int SDT, int MODE>
int launch_mode(const ScanArgs& a, const FusedArgs& f, cudaStream_t stream) {
    const int tpc = pow2_tpc(MODE ? f.N : a.N);
    switch (tpc) {
        case 1: return launch_tpc<DT, SDT, MODE, 1>(a, f, stream);
        case 2: return launch_tpc<DT, SDT, MODE, 2>(a, f, stream);
        case 4: return launch_tpc<DT, SDT, MODE, 4>(a, f, stream);
        case 8: return launch_tpc<DT, SDT, MODE, 8>(a, f, stream);
        case 16: return launch_tpc<DT, SDT, MODE, 16>(a, f, stream);
        case 32: return launch_tpc<DT, SDT, MODE, 32>(a, f, stream);
        default: return fail(NT_ERR_ARG, "scan: d_state %lld > 256 unsupported", (long long)(MODE ? f.N : a.N));
    }
}

}  // namespace

int launch_selective_scan(int dtype, int state_dtype, const ScanArgs& a, cudaStream_t stream) {
    FusedArgs f{};
    if (dtype == NT_F32 && state_dtype == NT_F32) return launch_mode<NT_F32, NT_F32, 0>(a, f, stream);
    if (dtype == NT_BF16 && state_dtype == NT_F32) return launch_mode<NT_BF16, NT_F32, 0>(a, f, stream);
    if (dtype == NT_BF16 && state_dtype == NT_BF16) return launch_mode<NT_BF16, NT_BF16, 0>(a, f, stream);
    return fail(NT_ERR_DTYPE, "selective_scan: unsupported dtype %d / state dtype %d", dtype, state_dtype);
}

int launch_lif_ssm_fused(const FusedArgs& f, cudaStream_t stream) {
    ScanArgs a{};
    return launch_mode<NT_BF16, NT_F32, 1>(a, f, stream);
}

}  // namespace nt
