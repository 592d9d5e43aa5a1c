// Selective scan (neuratensor/core/ssm.py:106-139 discretisation,
// ssm.py:184-221 sequential scan, ssm.py:145-182 single step) and the
// standalone LIF -> selective-scan fusion.
//
// Work split: a channel's d_state recurrences are spread over TPC threads
// (NPT = 8 states each, or 4 when the batch is too small to give every SM
// sub-partition a few warps; TPC = next power of two >= N/NPT).  A
// 128-thread CTA owns CPB = 128/TPC channels of one batch row and walks time
// serially; the state is float32 in registers for the whole sequence.
//
// The recurrence is bound by the FP32 pipe (about four fused multiply-adds
// per state update: the decay chain, the input term, the state update and
// the C.h readout), so everything else is kept off the per-step path:
// B/(n+1) and C are widened once per CTA and chunk into a bank-conflict-free
// layout and read as broadcasts, (u, dt) once per (step, channel), and the
// partial C.h sums of a channel's TPC threads are combined in registers by a
// butterfly over TPC steps at a time (no shared-memory reduction).
//
// Discretisation per step (A = -exp(log_A)):
//   A_bar = exp(dt*A)            -> ex2(dt * A*log2(e)) on the MUFU pipe
//   B_bar = (A_bar - 1)/A * B    (dt*B where |A| < 1e-6, ssm.py:129-137)
//   h     = A_bar*h + B_bar*u    (the B_bar term is skipped when u == 0)
//   y     = sum_n C[n]*h[n] + D*u
// HiPPO fast path: when A[c,n] = (n+1)*A[c,0] for every state of every
// channel of the CTA (the reference's initialisation, ssm.py:34-43), a
// thread needs two exponentials per step and a chain of fmas:
// exp(dt*A[c,n+1]) = exp(dt*A[c,n]) * exp(dt*A[c,0]), carried as e = A_bar - 1.  The structure test is
// 1e-6 relative on A for float32 parameters; for bfloat16 parameters it is
// made on log_A (one bf16 ulp of log(n+1) + log_A[c,0]), because a bf16 model
// stores log(n+1) rounded and exp() of that lands up to ~2% away from n+1.
// On the fast path A is exactly (n+1)*A[c,0].
#include "nt_kernels.cuh"

#include <algorithm>
#include <type_traits>

namespace nt {

namespace {


__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

// Stage rows [t0, t0+TCH) x [col0, col0+NCOLS) of a row-major matrix (leading
// dimension ld elements) into smem rows of NCOLS elements.  16-byte cp.async
// copies when the whole tile is aligned, element copies (zero fill outside
// the matrix) otherwise.
template <typename T, int NCOLS, int TCH>
__device__ __forceinline__ void stage_tile(T* dst, const T* src, int64_t ld, int64_t t0, int64_t T_len,
                                           int64_t col0, int64_t col_lim, bool vec_ok, int tid) {
    constexpr int EPV = 16 / (int)sizeof(T);      // elements per 16-byte vector
    if constexpr (NCOLS % EPV == 0) {
        if (vec_ok) {
            constexpr int VPR = NCOLS / EPV;        // vectors per row
            for (int i = tid; i < TCH * VPR; i += 128) {
                const int tt = i / VPR, v = i % VPR;
                const int64_t t = t0 + tt;
                T* dp = dst + tt * NCOLS + v * EPV;
                if (t < T_len) cp_async16(dp, src + t * ld + col0 + v * EPV);
                else *reinterpret_cast<uint4*>(dp) = make_uint4(0, 0, 0, 0);
            }
            return;
        }
    }
    {
        for (int i = tid; i < TCH * NCOLS; i += 128) {
            const int tt = i / NCOLS, cc = i % NCOLS;
            const int64_t t = t0 + tt, cidx = col0 + cc;
            dst[i] = (t < T_len && cidx < col_lim) ? src[t * ld + cidx] : T(0.f);
        }
    }
}

// f(std::integral_constant<int, 0>) ... f(std::integral_constant<int, N-1>): a
// compile-time unrolled loop (every index is a constant in the body).
template <int I, int N, typename F>
__device__ __forceinline__ void static_for(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        static_for<I + 1, N>(f);
    }
}

// Packed f32x2 arithmetic (sm_100 FFMA2 / FMUL2); NT_SCAN_SCALAR builds the same
// arithmetic from scalar instructions (identical rounding) for comparison.
__device__ __forceinline__ float2 pfma(float2 a, float2 b, float2 c) {
#ifdef NT_SCAN_SCALAR
    return make_float2(__fmaf_rn(a.x, b.x, c.x), __fmaf_rn(a.y, b.y, c.y));
#else
    return __ffma2_rn(a, b, c);
#endif
}
__device__ __forceinline__ float2 pmul(float2 a, float2 b) {
#ifdef NT_SCAN_SCALAR
    return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
#else
    return __fmul2_rn(a, b);
#endif
}

// One unit in the last place of a bf16 value held in a float: 2^(exponent - 7)
// (0 for zero and subnormals, which are then compared exactly).
__device__ __forceinline__ float bf16_ulp(float v) {
    const uint32_t e = __float_as_uint(v) & 0x7f800000u;
    return e <= (7u << 23) ? 0.f : __uint_as_float(e - (7u << 23));
}
// Eight consecutive states at p (16-byte vectors when p is aligned).
__device__ __forceinline__ void load_state8(const __nv_bfloat16* p, float (&h)[8]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const uint4 w = *reinterpret_cast<const uint4*>(p);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            h[2 * i] = __uint_as_float(ww[i] << 16);
            h[2 * i + 1] = __uint_as_float(ww[i] & 0xffff0000u);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = __bfloat162float(p[i]);
    }
}
__device__ __forceinline__ void load_state8(const float* p, float (&h)[8]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        h[0] = a.x; h[1] = a.y; h[2] = a.z; h[3] = a.w; h[4] = b.x; h[5] = b.y; h[6] = b.z; h[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = p[i];
    }
}
__device__ __forceinline__ void store_state8(__nv_bfloat16* p, const float (&h)[8]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            __nv_bfloat162 v = __floats2bfloat162_rn(h[2 * i], h[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = __float2bfloat16_rn(h[i]);
    }
}
__device__ __forceinline__ void store_state8(float* p, const float (&h)[8]) {
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
        *reinterpret_cast<float4*>(p) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(p + 4) = make_float4(h[4], h[5], h[6], h[7]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) p[i] = h[i];
    }
}
// HiPPO test of one state of a bf16 model: log_A[c,n] == log(n+1) + log_A[c,0]
// to one bf16 ulp of the stored value (the HiPPO init up to storage rounding).
__device__ __forceinline__ bool hippo_state_bf16(float la, float la0, float lnp1) {
    return fabsf(la - (lnp1 + la0)) <= bf16_ulp(la);
}
// exp(la) < 2e-6 is impossible above this log_A, so |A| < 1e-6 (the
// reference's dt*B branch, ssm.py:129-137) needs A itself only below it.
constexpr float kLimLogA = -13.0f;

// Shared-memory plan of one CTA: CPB = K*128/TPC channels of one batch row,
// 128 threads, TPC threads per channel slice holding NPT states each (NP =
// TPC*NPT >= d_state), K channels per thread.
template <int TPC, int NPT, int K, typename T>
struct ScanLayout {
    static constexpr int TCH = 32;                 // time steps per staged chunk
    static constexpr int SLOTS = 128 / TPC;        // channel slots per CTA
    static constexpr int CPB = K * SLOTS;          // channels per CTA
    static constexpr int NP = TPC * NPT;           // padded d_state
    // raw staging (double-buffered): u|x, dt, gate tiles [TCH][CPB]; B, C tiles [TCH][NP]
    static constexpr int RAW = 3 * TCH * CPB + 2 * TCH * NP;
    static constexpr int RAW_BYTES = ((RAW * (int)sizeof(T)) + 15) & ~15;
    // output tile [TCH][CPB] of T; row positions [TCH]; spike masks [CPB];
    // general-path per-state constants [3][K][NPT/2][128] float2
    static constexpr int YO_BYTES = ((TCH * CPB * (int)sizeof(T)) + 15) & ~15;
    static constexpr size_t BYTES =
        2 * (size_t)RAW_BYTES + YO_BYTES + 4 * TCH + 4 * CPB + 8 * 3 * K * (NPT / 2) * 128 + 4 * NP;
};

// Load NPT consecutive elements of a staged row as floats (16-byte vector loads).
template <int NPT>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[NPT]) {
#pragma unroll
    for (int q = 0; q < NPT / 8; ++q) {
        const uint4 w = *reinterpret_cast<const uint4*>(p + 8 * q);
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[8 * q + 2 * i] = __uint_as_float(ww[i] << 16);
            v[8 * q + 2 * i + 1] = __uint_as_float(ww[i] & 0xffff0000u);
        }
    }
    if constexpr (NPT % 8 == 4) {
        const uint2 w = *reinterpret_cast<const uint2*>(p + NPT - 4);
        v[NPT - 4] = __uint_as_float(w.x << 16);
        v[NPT - 3] = __uint_as_float(w.x & 0xffff0000u);
        v[NPT - 2] = __uint_as_float(w.y << 16);
        v[NPT - 1] = __uint_as_float(w.y & 0xffff0000u);
    }
}
template <int NPT>
__device__ __forceinline__ void load_row(const float* p, float (&v)[NPT]) {
#pragma unroll
    for (int q = 0; q < NPT / 4; ++q) {
        const float4 w = *reinterpret_cast<const float4*>(p + 4 * q);
        v[4 * q] = w.x; v[4 * q + 1] = w.y; v[4 * q + 2] = w.z; v[4 * q + 3] = w.w;
    }
}

// Sum of TPC per-step partials across the TPC consecutive lanes of a channel:
// on entry v[j] is this lane's partial C.h of step j of the group; on exit
// v[0] is the complete sum for step `sub` (a butterfly reduce-scatter: at
// each level a lane keeps the half of the steps its bit of `sub` selects and
// adds the partner's partials for them).
template <int TPC>
__device__ __forceinline__ void reduce_scatter(float (&v)[TPC], int sub, unsigned gmask) {
    static_for<0, 5>([&](auto lv) {
        constexpr int half = TPC >> (decltype(lv)::value + 1);
        if constexpr (half >= 1) {
            const bool upper = (sub & half) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const float send = upper ? v[i] : v[i + half];
                const float keep = upper ? v[i + half] : v[i];
                v[i] = keep + __shfl_xor_sync(gmask, send, half);
            }
        }
    });
}

// MODE 0: selective scan with given u.  MODE 1: u = LIF spikes of x (fused op).
// OUT = 0 (MODE 0 only): the state-only pass of the time-segmented scan -- no
// C, no outputs; writes the segment's end state (float32, from a zero start)
// to state_out and its total decay exp(A*sum(dt)) per state to a.seg_decay.
//
// Thread (slot, sub) owns states [NPT*sub, NPT*sub + NPT) of the K channels
// c0 + k*SLOTS + slot.  What bounds this kernel is shared memory: a warp's
// 16-byte load costs four wavefronts even when its lanes share addresses, so
// the cost of a step is the bytes each lane reads.  Each thread therefore
// reads the staged raw tiles directly -- its slice of the step's B and C rows
// (bf16: 16 bytes per 8 states, shared by its K channels) and u, dt of its
// channels -- and derives everything else in registers: B/(n+1), and per
// channel u/A0, dt*A0*log2(e), q = exp(dt*A0) and the decay chain.  In MODE 1
// every thread of a channel runs that channel's LIF membrane itself (the same
// arithmetic in each, so they agree), which keeps the chunk free of a serial
// per-channel pass.  Per chunk of TCH steps:
//   1. cp.async stages the next chunk's raw inputs while this one computes;
//   2. each thread advances its states through the chunk, in groups of TPC
//      steps whose partial C.h sums are combined by a register butterfly
//      (reduce_scatter); the sums stay in registers until the chunk is done;
//   3. D*u, the gate and the rounding, into the output tile, which goes to
//      global memory with 16-byte stores.
#ifndef NT_SCAN_MINB8
#define NT_SCAN_MINB8 3
#endif
template <int DT, int SDT, int TPC, int NPT, int K, int MODE, int OUT = 1>
__global__ void __launch_bounds__(128, NPT == 8 ? NT_SCAN_MINB8 : 4)
ssm_scan_kernel(ScanArgs a, FusedArgs f) {
    static_assert(OUT == 1 || MODE == 0, "state-only pass is a MODE 0 variant");
    static_assert(NPT == 4 || NPT == 8, "4 or 8 states per thread");
    using T = typename Elem<MODE == 0 ? DT : NT_BF16>::T;
    using L = ScanLayout<TPC, NPT, K, T>;
    constexpr int CPB = L::CPB, SLOTS = L::SLOTS, NP = L::NP, kTch = L::TCH, NPR = NPT / 2;
    constexpr int EPV = 16 / (int)sizeof(T);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* w_yo = reinterpret_cast<T*>(smem_raw + 2 * L::RAW_BYTES);                     // [kTch][CPB]
    int* w_pos = reinterpret_cast<int*>(smem_raw + 2 * L::RAW_BYTES + L::YO_BYTES);  // [kTch]
    unsigned* w_spk = reinterpret_cast<unsigned*>(w_pos + kTch);                     // [CPB] MODE 1 spike masks
    // general path, per thread, channel and state pair: (A*log2e), ((n+1)/A), ((n+1) for |A| < 1e-6 else 0)
    float2* w_gen = reinterpret_cast<float2*>(w_spk + CPB);                          // [3][K][NPR][128]
    float* w_lnp1 = reinterpret_cast<float*>(w_gen + 3 * K * NPR * 128);             // [NP] log(n+1)

    const int64_t T_len = MODE ? f.L : a.T, d = MODE ? f.d : a.d, N = MODE ? f.N : a.N;
    const T* p_u = static_cast<const T*>(MODE ? f.x : a.u);
    const T* p_dt = static_cast<const T*>(MODE ? f.delta : a.dt);
    const T* p_B = static_cast<const T*>(MODE ? f.Bm : a.Bm);
    const T* p_C = static_cast<const T*>(MODE ? f.Cm : a.Cm);
    const T* p_g = MODE == 0 ? static_cast<const T*>(a.gate) : nullptr;
    const bool has_gate = p_g != nullptr;
    const int64_t ld_bc = (MODE == 0 && a.ld_bc > 0) ? a.ld_bc : N;

    const int tid = threadIdx.x, slot = tid / TPC, sub = tid % TPC, lane = tid & 31;
    const unsigned gmask = TPC >= 32 ? 0xffffffffu : (((1u << TPC) - 1u) << (lane & ~(TPC - 1)));
    const int64_t c0 = (int64_t)blockIdx.x * CPB, b = blockIdx.y;
    auto chan = [&](int k) -> int64_t { return c0 + k * SLOTS + slot; };

    // ---- per-channel, per-state constants -------------------------------------
    // A = -exp(log_A), rounded like the reference's own tensor op (ssm.py:121).
    // HiPPO structure test, per channel.  fp32 parameters: A[c,n] == (n+1)*A[c,0]
    // to 1e-6 relative.  bf16 parameters: log_A[c,n] == log(n+1) + log_A[c,0] to
    // one bf16 ulp of the stored value (the HiPPO init up to storage rounding),
    // tested in the log domain against a per-CTA table of log(n+1), so a HiPPO
    // channel costs no exponential per state; the general path's per-state
    // constants are formed only for channels that need them.
    constexpr bool kBf16Params = (MODE == 0 && DT == NT_BF16);
    auto load_logA = [&](int64_t c, int64_t n) -> float {
        if (MODE == 0) return Elem<DT>::load(static_cast<const typename Elem<DT>::T*>(a.log_A) + c * N + n);
        return f.log_A[c * N + n];
    };
    auto A_of = [&](float la) -> float { return MODE == 0 ? -Elem<DT>::rnd(expf(la)) : -expf(la); };
    for (int i = tid; i < NP; i += 128) w_lnp1[i] = logf((float)(i + 1));
    __syncthreads();
    const void* sin = MODE ? (const void*)f.state_in : a.state_in;
    float2 hv[K][NPR];                               // the thread's states, as packed pairs
    float a0l[K], ra0[K], Dv[K];
    bool live[K], hippo[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int64_t c = chan(k);
        live[k] = c < d;
        bool ok = true;
        const float la0 = live[k] ? load_logA(c, 0) : 0.f;
        const float Abase = live[k] ? A_of(la0) : -1.f;
        a0l[k] = Abase * kLog2e;
        ra0[k] = 1.0f / Abase;
        Dv[k] = 0.f;
        if (live[k]) Dv[k] = MODE == 0 ? Elem<DT>::load(static_cast<const typename Elem<DT>::T*>(a.D) + c) : f.Dskip[c];
        const bool full_slice = NPT == 8 && live[k] && (int64_t)(sub + 1) * NPT <= N;
        float hs[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) hs[j] = 0.f;
        if (sin && full_slice) {
            const int64_t s0 = (b * d + c) * N + (int64_t)sub * NPT;
            if (MODE == 0 && SDT == NT_BF16) load_state8(static_cast<const __nv_bfloat16*>(sin) + s0, hs);
            else load_state8(static_cast<const float*>(sin) + s0, hs);
        }
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int64_t n = (int64_t)sub * NPT + j;
            float h0 = hs[j];
            const bool on = live[k] && n < N;
            if (on) {
                const float la = load_logA(c, n);
                if (sin && !full_slice) {
                    const int64_t si = (b * d + c) * N + n;
                    if (MODE == 0 && SDT == NT_BF16) h0 = __bfloat162float(static_cast<const __nv_bfloat16*>(sin)[si]);
                    else h0 = static_cast<const float*>(sin)[si];
                }
                if (kBf16Params) {
                    if (!hippo_state_bf16(la, la0, w_lnp1[n])) ok = false;
                    if (la <= kLimLogA && fabsf(A_of(la)) < 1e-6f) ok = false;
                } else {
                    const float A = A_of(la);
                    if (fabsf(A - (float)(n + 1) * Abase) > 1e-6f * fabsf(A) || fabsf(A) < 1e-6f) ok = false;
                }
            }
            if (j & 1) hv[k][j / 2].y = h0;
            else hv[k][j / 2].x = h0;
        }
        // one decision per channel: every state of the channel must qualify
        const unsigned okm = __ballot_sync(0xffffffffu, ok);
        hippo[k] = (okm & gmask) == gmask;
    }
    bool all_hippo = true;
#pragma unroll
    for (int k = 0; k < K; ++k) all_hippo = all_hippo && hippo[k];
    // the HiPPO path needs every channel of the thread to qualify (else the
    // general path, which is exact for any A, runs for all of them)
    const bool use_hippo = all_hippo;
    if (!use_hippo) {
        // general path on B' = B/(n+1): B_bar*u = (A_bar - 1) * ((n+1)/A) * B' * u,
        // or dt * (n+1) * B' * u for the |A| < 1e-6 states (ssm.py:129-137)
#pragma unroll
        for (int k = 0; k < K; ++k) {
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int64_t n = (int64_t)sub * NPT + j;
                const bool on = live[k] && n < N;
                const float A = on ? A_of(load_logA(chan(k), n)) : 0.f;
                const bool lim = on && fabsf(A) < 1e-6f;
                const float np1 = (float)(n + 1);
                const float ci = (lim || A == 0.f) ? 0.f : np1 / A;
                const int gi = (k * NPR + j / 2) * 128 + tid, gs = K * NPR * 128;
                reinterpret_cast<float*>(w_gen + gi)[j & 1] = A * kLog2e;
                reinterpret_cast<float*>(w_gen + gi + gs)[j & 1] = ci;
                reinterpret_cast<float*>(w_gen + gi + 2 * gs)[j & 1] = lim ? np1 : 0.f;
            }
        }
    }
    float rn[NPT];                                   // 1/(n+1) of the thread's states
#pragma unroll
    for (int j = 0; j < NPT; ++j) rn[j] = 1.0f / (float)(sub * NPT + j + 1);
    // HiPPO: exponents of the thread's first two states, (n0+1) and (n0+2) times dt*A0*log2(e)
    const float np1a = (float)(sub * NPT + 1), np1b = (float)(sub * NPT + 2);

    float beta[K], th[K], mem[K];                    // MODE 1: every thread of a channel runs its LIF
#pragma unroll
    for (int k = 0; k < K; ++k) {
        beta[k] = th[k] = mem[k] = 0.f;
        if (MODE == 1 && live[k]) {
            beta[k] = f.beta[chan(k)];
            th[k] = f.threshold[chan(k)];
            if (f.mem_in) mem[k] = f.mem_in[b * d + chan(k)];
        }
    }
    unsigned spike_local = 0;
    float dt_sum[K];                                 // state-only pass: sum of dt over the segment
#pragma unroll
    for (int k = 0; k < K; ++k) dt_sum[k] = 0.f;
    const bool sparse_rows = (MODE == 0) && a.row_pos != nullptr && a.sparse_flag != nullptr && *a.sparse_flag != 0;

    // 16-byte staging is possible when every tile row starts 16-byte aligned
    const bool act_vec = (d % EPV == 0) && (c0 + CPB <= d) && (CPB % EPV == 0) &&
                         ((reinterpret_cast<uintptr_t>(p_u) | reinterpret_cast<uintptr_t>(p_dt) |
                           reinterpret_cast<uintptr_t>(p_g)) & 15) == 0;
    const bool bc_vec = (NP == N) && (ld_bc % EPV == 0) &&
                        ((reinterpret_cast<uintptr_t>(p_B) | reinterpret_cast<uintptr_t>(p_C)) & 15) == 0;
    const int64_t row0 = b * T_len;   // first (batch, time) row of this batch element

    auto raw_buf = [&](int kk) { return reinterpret_cast<T*>(smem_raw + (kk & 1) * L::RAW_BYTES); };
    auto issue = [&](int64_t t0, T* rb) {
        T* r_u = rb;
        T* r_dt = r_u + kTch * CPB;
        T* r_g = r_dt + kTch * CPB;
        T* r_B = r_g + kTch * CPB;
        T* r_C = r_B + kTch * NP;
        stage_tile<T, CPB, kTch>(r_u, p_u + row0 * d, d, t0, T_len, c0, d, act_vec, tid);
        stage_tile<T, CPB, kTch>(r_dt, p_dt + row0 * d, d, t0, T_len, c0, d, act_vec, tid);
        if (has_gate) stage_tile<T, CPB, kTch>(r_g, p_g + row0 * d, d, t0, T_len, c0, d, act_vec, tid);
        stage_tile<T, NP, kTch>(r_B, p_B + row0 * ld_bc, ld_bc, t0, T_len, 0, N, bc_vec, tid);
        if (OUT) stage_tile<T, NP, kTch>(r_C, p_C + row0 * ld_bc, ld_bc, t0, T_len, 0, N, bc_vec, tid);
        cp_async_commit();
    };

    const int nchunks = (int)((T_len + kTch - 1) / kTch);
    issue(0, raw_buf(0));
    for (int kc = 0; kc < nchunks; ++kc) {
        const int64_t t0 = (int64_t)kc * kTch;
        if (kc + 1 < nchunks) {
            issue(t0 + kTch, raw_buf(kc + 1));
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        if (sparse_rows && tid < kTch) w_pos[tid] = (t0 + tid < T_len) ? a.row_pos[row0 + t0 + tid] : -1;
        __syncthreads();
        const int nt = (T_len - t0 < kTch) ? (int)(T_len - t0) : kTch;
        const T* rb = raw_buf(kc);
        const T* r_u = rb;
        const T* r_dt = r_u + kTch * CPB;
        const T* r_g = r_dt + kTch * CPB;
        const T* r_B = r_g + kTch * CPB;
        const T* r_C = r_B + kTch * NP;
        unsigned smask[K];                           // MODE 1: this chunk's spikes, bit tt
#pragma unroll
        for (int k = 0; k < K; ++k) smask[k] = 0;

        // One step of this thread's K x NPT states; returns the K partial C.h
        // sums.  Steps past the end of the sequence see u = dt = B = 0, which
        // leaves the state unchanged.
        auto step = [&](int tt, auto hip, float (&yk)[K]) {
            constexpr bool HIP = decltype(hip)::value;
            float Bv[NPT], Cv[NPT];
            load_row<NPT>(r_B + tt * NP + sub * NPT, Bv);
            if (OUT) load_row<NPT>(r_C + tt * NP + sub * NPT, Cv);
            float2 Bp[NPR];
#pragma unroll
            for (int j = 0; j < NPR; ++j)
                Bp[j] = pmul(make_float2(Bv[2 * j], Bv[2 * j + 1]), make_float2(rn[2 * j], rn[2 * j + 1]));
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int cc = k * SLOTS + slot;
                float u;
                const float dtv = to_f(r_dt[tt * CPB + cc]);
                if (MODE == 0) {
                    u = to_f(r_u[tt * CPB + cc]);
                } else {
                    // LIF step (snn.py:177-181) in fp32
                    const float m1 = __fadd_rn(__fmul_rn(beta[k], mem[k]), to_f(r_u[tt * CPB + cc]));
                    const float s1 = (m1 >= th[k]) ? 1.f : 0.f;
                    const bool in_seq = live[k] && tt < nt;
                    u = in_seq ? s1 : 0.f;
                    mem[k] = in_seq ? __fsub_rn(m1, __fmul_rn(th[k], s1)) : mem[k];
                    smask[k] |= (u != 0.f ? 1u : 0u) << tt;
                }
                float2 av[NPR];
                if (HIP) {
                    // A[n] = (n+1) A0.  With e = A_bar - 1 = exp(dt A[n]) - 1 and
                    // w = u B/((n+1) A0) = u B_bar / e, the update A_bar h + B_bar u is
                    //     h' = h + e (h + w)      (two fmas: t = B' * u/A0 + h, h + e t)
                    // and e follows the chain e[n+2] = e[n] q^2 + (q^2 - 1), q = exp(dt A0),
                    // seeded by the exponentials of the thread's first two states.
                    const float x0 = dtv * a0l[k], s = u * ra0[k];
                    const float q = ex2(x0);
                    const float qs = q * q, qm = __fmaf_rn(q, q, -1.0f);
                    av[0] = make_float2(ex2(x0 * np1a) - 1.0f, ex2(x0 * np1b) - 1.0f);
                    const float2 qq = make_float2(qs, qs), qqm = make_float2(qm, qm), ss = make_float2(s, s);
#pragma unroll
                    for (int j = 1; j < NPR; ++j) av[j] = pfma(av[j - 1], qq, qqm);
#pragma unroll
                    for (int j = 0; j < NPR; ++j) hv[k][j] = pfma(av[j], pfma(Bp[j], ss, hv[k][j]), hv[k][j]);
                } else {
                    const float2 uu = make_float2(u, u), dd = make_float2(dtv, dtv);
                    constexpr int gs = K * NPR * 128;
#pragma unroll
                    for (int j = 0; j < NPR; ++j) {
                        const int gi = (k * NPR + j) * 128 + tid;
                        const float2 A2 = w_gen[gi], ci = w_gen[gi + gs], lm = w_gen[gi + 2 * gs];
                        av[j] = make_float2(ex2(dtv * A2.x), ex2(dtv * A2.y));
                        const float2 coef = pfma(dd, lm, pfma(av[j], ci, make_float2(-ci.x, -ci.y)));
                        hv[k][j] = pfma(av[j], hv[k][j], pmul(coef, pmul(Bp[j], uu)));
                    }
                }
                if constexpr (OUT) {
                    // C.h as two packed fma chains (halving the dependent depth), then the lanes
                    float2 ya = pmul(make_float2(Cv[0], Cv[1]), hv[k][0]);
                    float2 yb = pmul(make_float2(Cv[2], Cv[3]), hv[k][1]);
#pragma unroll
                    for (int j = 2; j < NPR; j += 2) {
                        ya = pfma(make_float2(Cv[2 * j], Cv[2 * j + 1]), hv[k][j], ya);
                        yb = pfma(make_float2(Cv[2 * j + 2], Cv[2 * j + 3]), hv[k][j + 1], yb);
                    }
                    yk[k] = (ya.x + yb.x) + (ya.y + yb.y);
                } else {
                    dt_sum[k] += dtv;                  // the segment's total decay exponent
                    yk[k] = 0.f;
                }
            }
        };
        // ---- recurrence: groups of TPC steps, partial sums combined in registers
        constexpr int NG = kTch / TPC;
        float yfin[K][NG];
        auto run = [&](auto hip) {
            static_for<0, NG>([&](auto grp) {
                constexpr int g = decltype(grp)::value;
                float yp[K][TPC];
                static_for<0, TPC>([&](auto j) {
                    float yk[K];
                    step(g * TPC + decltype(j)::value, hip, yk);
#pragma unroll
                    for (int k = 0; k < K; ++k) yp[k][decltype(j)::value] = yk[k];
                });
                if constexpr (OUT) {
#pragma unroll
                    for (int k = 0; k < K; ++k) {
                        if constexpr (TPC > 1) reduce_scatter<TPC>(yp[k], sub, gmask);
                        yfin[k][g] = yp[k][0];
                    }
                }
            });
        };
        if (use_hippo) run(std::true_type{});
        else run(std::false_type{});
        if constexpr (OUT) {
            // D*u, the gate and the rounding (thread (slot, sub) holds step g*TPC + sub
            // of each of its channels for every group g)
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int cc = k * SLOTS + slot;
#pragma unroll
                for (int g = 0; g < NG; ++g) {
                    const int tt = g * TPC + (TPC > 1 ? sub : 0);
                    const float uu = MODE == 0 ? to_f(r_u[tt * CPB + cc]) : (float)((smask[k] >> tt) & 1u);
                    const float yv = __fadd_rn(yfin[k][g], __fmul_rn(Dv[k], uu));
                    if constexpr (MODE == 0) {
                        using E = Elem<DT>;
                        float o = E::rnd(yv);
                        if (has_gate) {
                            const float gv = to_f(r_g[tt * CPB + cc]);
                            o = E::rnd(o * (a.gate_is_silu ? gv : E::rnd(silu_f(gv))));
                        }
                        w_yo[tt * CPB + cc] = E::from_f(o);
                    } else {
                        w_yo[tt * CPB + cc] = __float2bfloat16_rn(yv);
                    }
                }
                if (MODE == 1 && sub == 0) {
                    w_spk[cc] = smask[k];
                    spike_local += __popc(smask[k]);
                }
            }
            __syncthreads();
            // ---- output tile -> global (16-byte stores where rows allow) -------
            constexpr int VPR = (CPB * (int)sizeof(T)) % 16 == 0 ? CPB * (int)sizeof(T) / 16 : 1;
            constexpr bool kRowVec = (CPB * (int)sizeof(T)) % 16 == 0;
            using OT = typename Elem<MODE == 0 ? DT : NT_BF16>::T;
            OT* p_y = static_cast<OT*>(MODE ? f.y : a.y);
            const bool vec_out = kRowVec && act_vec && (reinterpret_cast<uintptr_t>(p_y) & 15) == 0;
            if (vec_out) {
                for (int i = tid; i < kTch * VPR; i += 128) {
                    const int tt = i / VPR, v = i % VPR;
                    if (tt >= nt) continue;
                    int64_t row = row0 + t0 + tt;
                    if (sparse_rows) {
                        row = w_pos[tt];
                        if (row < 0) continue;
                    }
                    *reinterpret_cast<uint4*>(p_y + row * d + c0 + v * EPV) =
                        *reinterpret_cast<const uint4*>(w_yo + tt * CPB + v * EPV);
                }
            } else {
                for (int i = tid; i < kTch * CPB; i += 128) {
                    const int tt = i / CPB, cc = i % CPB;
                    if (tt >= nt || c0 + cc >= d) continue;
                    int64_t row = row0 + t0 + tt;
                    if (sparse_rows) {
                        row = w_pos[tt];
                        if (row < 0) continue;
                    }
                    p_y[row * d + c0 + cc] = w_yo[tt * CPB + cc];
                }
            }
            if (MODE == 1 && f.spikes) {
                // the chunk's spikes, one byte (or bf16) per (step, channel), consecutive channels per thread
                for (int i = tid; i < kTch * CPB; i += 128) {
                    const int tt = i / CPB, cc = i % CPB;
                    if (tt >= nt || c0 + cc >= d) continue;
                    const unsigned sbit = (w_spk[cc] >> tt) & 1u;
                    const int64_t idx = (row0 + t0 + tt) * d + c0 + cc;
                    if (f.spike_dtype == NT_U8) static_cast<unsigned char*>(f.spikes)[idx] = (unsigned char)sbit;
                    else static_cast<__nv_bfloat16*>(f.spikes)[idx] = __float2bfloat16_rn((float)sbit);
                }
            }
        }
        __syncthreads();   // raw_buf(kc) and the tiles are refilled by the next chunk
    }
    // ---- carry-out -----------------------------------------------------------
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int64_t c = chan(k);
        if (!live[k]) continue;
        if constexpr (!OUT) {
            // end state of the segment (float32) and its decay exp(A*sum(dt)) per state
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int64_t n = (int64_t)sub * NPT + j;
                if (n >= N) continue;
                const int64_t si = (b * d + c) * N + n;
                const float2 A2 = w_gen[(k * NPR + j / 2) * 128 + tid];
                const float a2 = use_hippo ? (float)(n + 1) * a0l[k] : ((j & 1) ? A2.y : A2.x);
                static_cast<float*>(a.state_out)[si] = (j & 1) ? hv[k][j / 2].y : hv[k][j / 2].x;
                a.seg_decay[si] = ex2(a2 * dt_sum[k]);
            }
        } else {
            void* sout = MODE ? (void*)f.state_out : a.state_out;
            if (sout) {
#pragma unroll
                for (int j = 0; j < NPT; ++j) {
                    const int64_t n = (int64_t)sub * NPT + j;
                    if (n >= N) continue;
                    const int64_t si = (b * d + c) * N + n;
                    const float hj = (j & 1) ? hv[k][j / 2].y : hv[k][j / 2].x;
                    if (MODE == 0 && SDT == NT_BF16) static_cast<__nv_bfloat16*>(sout)[si] = __float2bfloat16_rn(hj);
                    else static_cast<float*>(sout)[si] = hj;
                }
            }
            if (MODE == 1 && sub == 0 && f.mem_out) f.mem_out[b * d + c] = mem[k];
        }
    }
    if (MODE == 1 && f.spike_count) {
        const unsigned w = __reduce_add_sync(0xffffffffu, spike_local);
        if ((tid & 31) == 0 && w) atomicAdd(f.spike_count, (unsigned long long)w);
    }
}

int pow2_at_least(int64_t x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

template <int DT, int SDT, int MODE, int TPC, int NPT, int K, int OUT>
int launch_tpc(const ScanArgs& a, const FusedArgs& f, cudaStream_t stream) {
    using T = typename Elem<MODE == 0 ? DT : NT_BF16>::T;
    using L = ScanLayout<TPC, NPT, K, T>;
    auto kern = ssm_scan_kernel<DT, SDT, TPC, NPT, K, MODE, OUT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::BYTES);
    if (e != cudaSuccess) return fail(NT_ERR_CUDA, "scan: smem attribute: %s", cudaGetErrorString(e));
    const int64_t d = MODE ? f.d : a.d, B = MODE ? f.B : a.B;
    dim3 grid((unsigned)((d + L::CPB - 1) / L::CPB), (unsigned)B);
    kern<<<grid, 128, L::BYTES, stream>>>(a, f);
    return check_launch("ssm_scan_kernel");
}

#ifndef NT_SCAN_WIDE_WARPS
#define NT_SCAN_WIDE_WARPS 6
#endif
#ifndef NT_SCAN_NARROW_WARPS
#define NT_SCAN_NARROW_WARPS 2
#endif
// Slicing: 8 states per thread (TPC = N/8 threads per channel).  Two channels
// per thread (their B and C slices loaded once) when that still leaves every
// SM sub-partition NT_SCAN_WIDE_WARPS warps or more: the recurrence of one
// warp is a serial chain over T, so warps per sub-partition, and how evenly
// they divide, set the time when the batch is small.
template <int DT, int SDT, int MODE, int OUT = 1>
int launch_mode(const ScanArgs& a, const FusedArgs& f, cudaStream_t stream) {
    const int64_t N = MODE ? f.N : a.N, d = MODE ? f.d : a.d, B = MODE ? f.B : a.B;
    if (N > 256) return fail(NT_ERR_ARG, "scan: d_state %lld > 256 unsupported", (long long)N);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tpc = pow2_at_least((N + 7) / 8);
    const int64_t warps2 = B * ((d + 2 * 128 / tpc - 1) / (2 * 128 / tpc)) * 4;
    // (bf16 inputs only: the float32 path is the parity configuration)
    const bool wide = (MODE == 1 || DT == NT_BF16) && OUT == 1 && tpc <= 16 &&
                      warps2 >= (int64_t)NT_SCAN_WIDE_WARPS * 4 * sms;
    if constexpr (MODE == 0 && DT == NT_BF16 && OUT == 1) {
        // fewer than two warps per SM sub-partition with 8 states per thread:
        // 4 states per thread doubles the warps (d_state <= 32 only)
        const int64_t warps1 = B * ((d + 128 / tpc - 1) / (128 / tpc)) * 4;
        if (N > 4 && N <= 32 && warps1 < (int64_t)NT_SCAN_NARROW_WARPS * 4 * sms) {
            switch (pow2_at_least((N + 3) / 4)) {
                case 2: return launch_tpc<DT, SDT, MODE, 2, 4, 1, OUT>(a, f, stream);
                case 4: return launch_tpc<DT, SDT, MODE, 4, 4, 1, OUT>(a, f, stream);
                case 8: return launch_tpc<DT, SDT, MODE, 8, 4, 1, OUT>(a, f, stream);
                default: break;
            }
        }
    }
    if constexpr (MODE == 1 || (DT == NT_BF16 && OUT == 1)) {
      if (wide) {
        switch (tpc) {
            case 1: return launch_tpc<DT, SDT, MODE, 1, 8, 2, OUT>(a, f, stream);
            case 2: return launch_tpc<DT, SDT, MODE, 2, 8, 2, OUT>(a, f, stream);
            case 4: return launch_tpc<DT, SDT, MODE, 4, 8, 2, OUT>(a, f, stream);
            case 8: return launch_tpc<DT, SDT, MODE, 8, 8, 2, OUT>(a, f, stream);
            case 16: return launch_tpc<DT, SDT, MODE, 16, 8, 2, OUT>(a, f, stream);
            default: break;
        }
      }
    }
    switch (tpc) {
        case 1: return launch_tpc<DT, SDT, MODE, 1, 8, 1, OUT>(a, f, stream);
        case 2: return launch_tpc<DT, SDT, MODE, 2, 8, 1, OUT>(a, f, stream);
        case 4: return launch_tpc<DT, SDT, MODE, 4, 8, 1, OUT>(a, f, stream);
        case 8: return launch_tpc<DT, SDT, MODE, 8, 8, 1, OUT>(a, f, stream);
        case 16: return launch_tpc<DT, SDT, MODE, 16, 8, 1, OUT>(a, f, stream);
        case 32: return launch_tpc<DT, SDT, MODE, 32, 8, 1, OUT>(a, f, stream);
        default: return fail(NT_ERR_ARG, "scan: d_state %lld > 256 unsupported", (long long)N);
    }
}

// ---------------------------------------------------------------------------
// Short sequences (decode steps, T <= kStepMaxT).  The chunked kernel stages
// and steps through a whole 32-step chunk and pays its per-CTA set-up for a
// few channels, which for one step costs many times the step itself; this
// kernel is bounded by reading and writing the state.  A 256-thread CTA owns
// CPS = 256/TPC channels of one batch row; thread (channel, sub) keeps states
// [8 sub, 8 sub + 8) in registers, exactly the slice a thread of the chunked
// kernel holds with 8 states per thread, and B/(n+1) and C of the step are
// read once per CTA into shared memory.  The arithmetic is the chunked
// kernel's, operation for operation (per-channel HiPPO decision, the same
// records and decay chain, the same C.h summation tree), so a sequence
// stepped through this kernel reproduces the chunked kernel's 8-state-per-
// thread results bit for bit.
constexpr int kStepMaxT = 4;
constexpr int kStepThreads = 256;

template <int DT, int SDT, int TPC>
__global__ void __launch_bounds__(kStepThreads, 4)
ssm_step_kernel(ScanArgs a) {
    using E = Elem<DT>;
    using T = typename E::T;
    constexpr int NPT = 8, NPR = 4, NP = TPC * NPT, CPS = kStepThreads / TPC;
    __shared__ __align__(16) float s_B[NP];
    __shared__ __align__(16) float s_C[NP];
    const int tid = threadIdx.x, cl = tid / TPC, sub = tid % TPC, lane = tid & 31;
    const unsigned gmask = TPC >= 32 ? 0xffffffffu : (((1u << TPC) - 1u) << (lane & ~(TPC - 1)));
    const int64_t c = (int64_t)blockIdx.x * CPS + cl, b = blockIdx.y;
    const int64_t d = a.d, N = a.N, Tl = a.T;
    const bool live = c < d;
    const int64_t ld_bc = a.ld_bc > 0 ? a.ld_bc : N;
    const T* logA = static_cast<const T*>(a.log_A) + (live ? c : 0) * N;
    __shared__ float s_lnp1[NP];
    for (int i = tid; i < NP; i += kStepThreads) s_lnp1[i] = logf((float)(i + 1));
    __syncthreads();
    const float la0 = live ? E::load(logA) : 0.f;
    const float Abase = live ? -E::rnd(expf(la0)) : -1.f;
    float2 hv[NPR], A2v[NPR], civ[NPR], lmv[NPR];
    using ST = typename Elem<SDT>::T;
    const bool full_slice = live && (int64_t)(sub + 1) * NPT <= N;
    float hs[NPT];
#pragma unroll
    for (int j = 0; j < NPT; ++j) hs[j] = 0.f;
    if (a.state_in && full_slice) load_state8(static_cast<const ST*>(a.state_in) + (b * d + c) * N + sub * NPT, hs);
    bool ok = true;
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int64_t n = (int64_t)sub * NPT + j;
        const bool on = live && n < N;
        float h0 = hs[j];
        if (on) {
            const float la = E::load(logA + n);
            if (a.state_in && !full_slice) {
                const int64_t si = (b * d + c) * N + n;
                h0 = SDT == NT_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.state_in)[si])
                                    : static_cast<const float*>(a.state_in)[si];
            }
            if (DT == NT_BF16) {
                if (!hippo_state_bf16(la, la0, s_lnp1[n])) ok = false;
                if (la <= kLimLogA && fabsf(E::rnd(expf(la))) < 1e-6f) ok = false;
            } else {
                const float A = -E::rnd(expf(la));
                if (fabsf(A - (float)(n + 1) * Abase) > 1e-6f * fabsf(A) || fabsf(A) < 1e-6f) ok = false;
            }
        }
        if (j & 1) hv[j / 2].y = h0;
        else hv[j / 2].x = h0;
    }
    const unsigned okm = __ballot_sync(0xffffffffu, ok);
    const bool hippo = (okm & gmask) == gmask;
    if (!hippo) {
        // the general path's per-state constants (only channels that need them pay for the exponentials)
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int64_t n = (int64_t)sub * NPT + j;
            const bool on = live && n < N;
            const float A = on ? -E::rnd(expf(E::load(logA + n))) : 0.f;
            const bool lim = on && fabsf(A) < 1e-6f;
            const float np1 = (float)(n + 1);
            const float ci = (lim || A == 0.f) ? 0.f : np1 / A;
            if (j & 1) { A2v[j / 2].y = A * kLog2e; civ[j / 2].y = ci; lmv[j / 2].y = lim ? np1 : 0.f; }
            else { A2v[j / 2].x = A * kLog2e; civ[j / 2].x = ci; lmv[j / 2].x = lim ? np1 : 0.f; }
        }
    }
    const float a0l = Abase * kLog2e, ra0 = 1.0f / Abase;
    const float np1a = (float)(sub * NPT + 1), np1b = (float)(sub * NPT + 2);
    const float Dv = live ? E::load(static_cast<const T*>(a.D) + c) : 0.f;
    const bool sparse_rows = a.row_pos != nullptr && a.sparse_flag != nullptr && *a.sparse_flag != 0;
    const T* p_u = static_cast<const T*>(a.u);
    const T* p_dt = static_cast<const T*>(a.dt);
    const T* p_B = static_cast<const T*>(a.Bm);
    const T* p_C = static_cast<const T*>(a.Cm);
    const T* p_g = static_cast<const T*>(a.gate);
    for (int64_t t = 0; t < Tl; ++t) {
        const int64_t row = b * Tl + t;
        __syncthreads();                                    // the previous step's B/C reads are done
        for (int i = tid; i < NP; i += kStepThreads) {
            const bool in = i < N;
            s_B[i] = in ? E::to_f(p_B[row * ld_bc + i]) * (1.0f / (float)(i + 1)) : 0.f;
            s_C[i] = in ? E::to_f(p_C[row * ld_bc + i]) : 0.f;
        }
        __syncthreads();
        const float u = live ? E::to_f(p_u[row * d + c]) : 0.f;
        const float dtv = live ? E::to_f(p_dt[row * d + c]) : 0.f;
        float2 Bp[NPR], Cp[NPR], av[NPR];
#pragma unroll
        for (int j = 0; j < NPR; ++j) {
            Bp[j] = *reinterpret_cast<const float2*>(s_B + sub * NPT + 2 * j);
            Cp[j] = *reinterpret_cast<const float2*>(s_C + sub * NPT + 2 * j);
        }
        if (hippo) {
            // the chunked kernel's record and chain (put_rec, step)
            const float x0 = dtv * a0l, s = u * ra0;
            const float q = ex2(x0);
            const float qs = q * q, qm = __fmaf_rn(q, q, -1.0f);
            av[0] = make_float2(ex2(x0 * np1a) - 1.0f, ex2(x0 * np1b) - 1.0f);
            const float2 qq = make_float2(qs, qs), qqm = make_float2(qm, qm), ss = make_float2(s, s);
#pragma unroll
            for (int j = 1; j < NPR; ++j) av[j] = pfma(av[j - 1], qq, qqm);
#pragma unroll
            for (int j = 0; j < NPR; ++j) hv[j] = pfma(av[j], pfma(Bp[j], ss, hv[j]), hv[j]);
        } else {
            const float2 uu = make_float2(u, u), dd = make_float2(dtv, dtv);
#pragma unroll
            for (int j = 0; j < NPR; ++j) {
                av[j] = make_float2(ex2(dtv * A2v[j].x), ex2(dtv * A2v[j].y));
                const float2 coef = pfma(dd, lmv[j], pfma(av[j], civ[j], make_float2(-civ[j].x, -civ[j].y)));
                const float2 bu = pmul(coef, pmul(Bp[j], uu));
                hv[j] = pfma(av[j], hv[j], bu);
            }
        }
        float2 ya = pmul(Cp[0], hv[0]), yb = pmul(Cp[1], hv[1]);
        ya = pfma(Cp[2], hv[2], ya);
        yb = pfma(Cp[3], hv[3], yb);
        float y = (ya.x + yb.x) + (ya.y + yb.y);
#pragma unroll
        for (int half = TPC / 2; half >= 1; half >>= 1) y += __shfl_xor_sync(gmask, y, half);
        if (sub == 0 && live) {
            const float yv = __fadd_rn(y, __fmul_rn(Dv, u));
            float o = E::rnd(yv);
            if (p_g) {
                const float gv = E::to_f(p_g[row * d + c]);
                o = E::rnd(o * (a.gate_is_silu ? gv : E::rnd(silu_f(gv))));
            }
            int64_t orow = row;
            if (sparse_rows) orow = a.row_pos[row];
            if (orow >= 0) static_cast<T*>(a.y)[orow * d + c] = E::from_f(o);
        }
    }
    if (a.state_out && live) {
        float ho[NPT];
#pragma unroll
        for (int j = 0; j < NPT; ++j) ho[j] = (j & 1) ? hv[j / 2].y : hv[j / 2].x;
        if (full_slice) {
            store_state8(static_cast<ST*>(a.state_out) + (b * d + c) * N + sub * NPT, ho);
        } else {
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int64_t n = (int64_t)sub * NPT + j;
                if (n >= N) continue;
                const int64_t si = (b * d + c) * N + n;
                if (SDT == NT_BF16) static_cast<__nv_bfloat16*>(a.state_out)[si] = __float2bfloat16_rn(ho[j]);
                else static_cast<float*>(a.state_out)[si] = ho[j];
            }
        }
    }
}

// The same step for many rows: one CTA per group of CPS channels walks a
// range of rows (decode with many streams).  A channel's set-up -- log_A, the
// HiPPO test, the general path's constants, D -- is done once for all its
// rows instead of once per (row, channel), and a thread reads its own B/C
// slice of each row (the CTA's channels share them through L1), so the row
// loop has no barrier.  Per (row, channel, state) the arithmetic is the one of
// ssm_step_kernel above, so both give the same results.
template <int DT, int SDT, int TPC>
__global__ void __launch_bounds__(kStepThreads, 4)
ssm_step_rows_kernel(ScanArgs a, int rows_per_cta) {
    using E = Elem<DT>;
    using T = typename E::T;
    using ST = typename Elem<SDT>::T;
    constexpr int NPT = 8, NPR = 4, NP = TPC * NPT, CPS = kStepThreads / TPC;
    const int tid = threadIdx.x, cl = tid / TPC, sub = tid % TPC, lane = tid & 31;
    const unsigned gmask = TPC >= 32 ? 0xffffffffu : (((1u << TPC) - 1u) << (lane & ~(TPC - 1)));
    const int64_t c = (int64_t)blockIdx.x * CPS + cl;
    const int64_t d = a.d, N = a.N, Tl = a.T;
    const int64_t b0 = (int64_t)blockIdx.y * rows_per_cta;
    const int64_t b1 = b0 + rows_per_cta < a.B ? b0 + rows_per_cta : a.B;
    const bool live = c < d;
    const int64_t ld_bc = a.ld_bc > 0 ? a.ld_bc : N;
    const T* logA = static_cast<const T*>(a.log_A) + (live ? c : 0) * N;
    __shared__ float s_lnp1[NP];
    for (int i = tid; i < NP; i += kStepThreads) s_lnp1[i] = logf((float)(i + 1));
    __syncthreads();
    const float la0 = live ? E::load(logA) : 0.f;
    const float Abase = live ? -E::rnd(expf(la0)) : -1.f;
    float2 A2v[NPR], civ[NPR], lmv[NPR];
    float rn[NPT];                                   // 1/(n+1): B enters the HiPPO update as B/(n+1)
    bool ok = true;
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int64_t n = (int64_t)sub * NPT + j;
        const bool on = live && n < N;
        rn[j] = 1.0f / (float)(n + 1);
        if (on) {
            const float la = E::load(logA + n);
            if (DT == NT_BF16) {
                if (!hippo_state_bf16(la, la0, s_lnp1[n])) ok = false;
                if (la <= kLimLogA && fabsf(E::rnd(expf(la))) < 1e-6f) ok = false;
            } else {
                const float A = -E::rnd(expf(la));
                if (fabsf(A - (float)(n + 1) * Abase) > 1e-6f * fabsf(A) || fabsf(A) < 1e-6f) ok = false;
            }
        }
    }
    const unsigned okm = __ballot_sync(0xffffffffu, ok);
    const bool hippo = (okm & gmask) == gmask;
    if (!hippo) {
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int64_t n = (int64_t)sub * NPT + j;
            const bool on = live && n < N;
            const float A = on ? -E::rnd(expf(E::load(logA + n))) : 0.f;
            const bool lim = on && fabsf(A) < 1e-6f;
            const float np1 = (float)(n + 1);
            const float ci = (lim || A == 0.f) ? 0.f : np1 / A;
            if (j & 1) { A2v[j / 2].y = A * kLog2e; civ[j / 2].y = ci; lmv[j / 2].y = lim ? np1 : 0.f; }
            else { A2v[j / 2].x = A * kLog2e; civ[j / 2].x = ci; lmv[j / 2].x = lim ? np1 : 0.f; }
        }
    }
    const float a0l = Abase * kLog2e, ra0 = 1.0f / Abase;
    const float np1a = (float)(sub * NPT + 1), np1b = (float)(sub * NPT + 2);
    const float Dv = live ? E::load(static_cast<const T*>(a.D) + c) : 0.f;
    const bool sparse_rows = a.row_pos != nullptr && a.sparse_flag != nullptr && *a.sparse_flag != 0;
    const bool full_slice = live && (int64_t)(sub + 1) * NPT <= N;
    // 16-byte B/C slice loads when every row's slice starts 16-byte aligned
    const bool vec_bc = full_slice && sizeof(T) == 2 && ld_bc % 8 == 0 &&
                        ((reinterpret_cast<uintptr_t>(a.Bm) | reinterpret_cast<uintptr_t>(a.Cm)) & 15) == 0;
    const T* p_u = static_cast<const T*>(a.u);
    const T* p_dt = static_cast<const T*>(a.dt);
    const T* p_B = static_cast<const T*>(a.Bm);
    const T* p_C = static_cast<const T*>(a.Cm);
    const T* p_g = static_cast<const T*>(a.gate);
    auto slice = [&](const T* p, int64_t row, float (&v)[NPT]) {
        const T* q = p + row * ld_bc + sub * NPT;
        if (vec_bc) {
            const uint4 w = *reinterpret_cast<const uint4*>(q);
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = __uint_as_float(ww[i] << 16);
                v[2 * i + 1] = __uint_as_float(ww[i] & 0xffff0000u);
            }
        } else {
#pragma unroll
            for (int j = 0; j < NPT; ++j) v[j] = (live && (int64_t)sub * NPT + j < N) ? E::to_f(q[j]) : 0.f;
        }
    };
    for (int64_t bi = b0; bi < b1; ++bi) {
        float hs[NPT];
#pragma unroll
        for (int j = 0; j < NPT; ++j) hs[j] = 0.f;
        if (a.state_in && full_slice) {
            load_state8(static_cast<const ST*>(a.state_in) + (bi * d + c) * N + sub * NPT, hs);
        } else if (a.state_in && live) {
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int64_t n = (int64_t)sub * NPT + j;
                if (n >= N) continue;
                const int64_t si = (bi * d + c) * N + n;
                hs[j] = SDT == NT_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.state_in)[si])
                                       : static_cast<const float*>(a.state_in)[si];
            }
        }
        float2 hv[NPR];
#pragma unroll
        for (int j = 0; j < NPR; ++j) hv[j] = make_float2(hs[2 * j], hs[2 * j + 1]);
        for (int64_t t = 0; t < Tl; ++t) {
            const int64_t row = bi * Tl + t;
            float Bv[NPT], Cv[NPT];
            slice(p_B, row, Bv);
            slice(p_C, row, Cv);
            const float u = live ? E::to_f(p_u[row * d + c]) : 0.f;
            const float dtv = live ? E::to_f(p_dt[row * d + c]) : 0.f;
            float2 Bp[NPR], Cp[NPR], av[NPR];
#pragma unroll
            for (int j = 0; j < NPR; ++j) {
                Bp[j] = make_float2(Bv[2 * j] * rn[2 * j], Bv[2 * j + 1] * rn[2 * j + 1]);
                Cp[j] = make_float2(Cv[2 * j], Cv[2 * j + 1]);
            }
            if (hippo) {
                const float x0 = dtv * a0l, s = u * ra0;
                const float q = ex2(x0);
                const float qs = q * q, qm = __fmaf_rn(q, q, -1.0f);
                av[0] = make_float2(ex2(x0 * np1a) - 1.0f, ex2(x0 * np1b) - 1.0f);
                const float2 qq = make_float2(qs, qs), qqm = make_float2(qm, qm), ss = make_float2(s, s);
#pragma unroll
                for (int j = 1; j < NPR; ++j) av[j] = pfma(av[j - 1], qq, qqm);
#pragma unroll
                for (int j = 0; j < NPR; ++j) hv[j] = pfma(av[j], pfma(Bp[j], ss, hv[j]), hv[j]);
            } else {
                const float2 uu = make_float2(u, u), dd = make_float2(dtv, dtv);
#pragma unroll
                for (int j = 0; j < NPR; ++j) {
                    av[j] = make_float2(ex2(dtv * A2v[j].x), ex2(dtv * A2v[j].y));
                    const float2 coef = pfma(dd, lmv[j], pfma(av[j], civ[j], make_float2(-civ[j].x, -civ[j].y)));
                    const float2 bu = pmul(coef, pmul(Bp[j], uu));
                    hv[j] = pfma(av[j], hv[j], bu);
                }
            }
            float2 ya = pmul(Cp[0], hv[0]), yb = pmul(Cp[1], hv[1]);
            ya = pfma(Cp[2], hv[2], ya);
            yb = pfma(Cp[3], hv[3], yb);
            float y = (ya.x + yb.x) + (ya.y + yb.y);
#pragma unroll
            for (int half = TPC / 2; half >= 1; half >>= 1) y += __shfl_xor_sync(gmask, y, half);
            if (sub == 0 && live) {
                const float yv = __fadd_rn(y, __fmul_rn(Dv, u));
                float o = E::rnd(yv);
                if (p_g) {
                    const float gv = E::to_f(p_g[row * d + c]);
                    o = E::rnd(o * (a.gate_is_silu ? gv : E::rnd(silu_f(gv))));
                }
                int64_t orow = row;
                if (sparse_rows) orow = a.row_pos[row];
                if (orow >= 0) static_cast<T*>(a.y)[orow * d + c] = E::from_f(o);
            }
        }
        if (a.state_out && live) {
            float ho[NPT];
#pragma unroll
            for (int j = 0; j < NPT; ++j) ho[j] = (j & 1) ? hv[j / 2].y : hv[j / 2].x;
            if (full_slice) {
                store_state8(static_cast<ST*>(a.state_out) + (bi * d + c) * N + sub * NPT, ho);
            } else {
#pragma unroll
                for (int j = 0; j < NPT; ++j) {
                    const int64_t n = (int64_t)sub * NPT + j;
                    if (n >= N) continue;
                    const int64_t si = (bi * d + c) * N + n;
                    if (SDT == NT_BF16) static_cast<__nv_bfloat16*>(a.state_out)[si] = __float2bfloat16_rn(ho[j]);
                    else static_cast<float*>(a.state_out)[si] = ho[j];
                }
            }
        }
    }
}

#ifndef NT_STEP_ROWS_MIN_B
#define NT_STEP_ROWS_MIN_B 16
#endif
template <int DT, int SDT>
int launch_step(const ScanArgs& a, cudaStream_t stream) {
    const int tpc = pow2_at_least((a.N + 7) / 8);
    if (a.B >= NT_STEP_ROWS_MIN_B) {
        // many rows: channel groups walk row ranges, about four CTAs per SM in all
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int64_t groups = (a.d + kStepThreads / tpc - 1) / (kStepThreads / tpc);
        int64_t rg = (4LL * sms + groups - 1) / groups;
        rg = rg < 1 ? 1 : (rg > a.B ? a.B : rg);
        const int rows = (int)((a.B + rg - 1) / rg);
        rg = (a.B + rows - 1) / rows;
        auto go = [&](auto kern) {
            kern<<<dim3((unsigned)groups, (unsigned)rg), kStepThreads, 0, stream>>>(a, rows);
        };
        switch (tpc) {
            case 1: go(ssm_step_rows_kernel<DT, SDT, 1>); break;
            case 2: go(ssm_step_rows_kernel<DT, SDT, 2>); break;
            case 4: go(ssm_step_rows_kernel<DT, SDT, 4>); break;
            case 8: go(ssm_step_rows_kernel<DT, SDT, 8>); break;
            case 16: go(ssm_step_rows_kernel<DT, SDT, 16>); break;
            case 32: go(ssm_step_rows_kernel<DT, SDT, 32>); break;
            default: return fail(NT_ERR_ARG, "scan: d_state %lld > 256 unsupported", (long long)a.N);
        }
        return check_launch("ssm_step_rows_kernel");
    }
    auto go = [&](auto kern, int tpc_) {
        dim3 grid((unsigned)((a.d + kStepThreads / tpc_ - 1) / (kStepThreads / tpc_)), (unsigned)a.B);
        kern<<<grid, kStepThreads, 0, stream>>>(a);
    };
    switch (tpc) {
        case 1: go(ssm_step_kernel<DT, SDT, 1>, 1); break;
        case 2: go(ssm_step_kernel<DT, SDT, 2>, 2); break;
        case 4: go(ssm_step_kernel<DT, SDT, 4>, 4); break;
        case 8: go(ssm_step_kernel<DT, SDT, 8>, 8); break;
        case 16: go(ssm_step_kernel<DT, SDT, 16>, 16); break;
        case 32: go(ssm_step_kernel<DT, SDT, 32>, 32); break;
        default: return fail(NT_ERR_ARG, "scan: d_state %lld > 256 unsupported", (long long)a.N);
    }
    return check_launch("ssm_step_kernel");
}

}  // namespace

template <int DT>
int launch_segmented(int state_dtype, const ScanArgs& a, int S, float* ws, cudaStream_t stream);

// Segments: for one or two rows, the largest power of two S with B*S <= 8, T
// divisible by S and at least 128 steps per segment (1: no segmentation).
// Measured on the small preset (T = 2048): B=1 2.79 ms per forward with 8
// segments (3.79 without), B=2 3.91 ms with 4 (4.56), B=4 slower with 2.
int scan_segments(int64_t B, int64_t T) {
    if (B > 2) return 1;
    int S = 1;
    while (B * S * 2 <= 8 && T % (S * 2) == 0 && T / (S * 2) >= 128) S *= 2;
    return S;
}

size_t selective_scan_segmented_workspace(int64_t B, int64_t T, int64_t d, int64_t N) {
    const int S = scan_segments(B, T);
    return S > 1 ? 3 * (size_t)(B * S) * (size_t)d * (size_t)N * sizeof(float) : 0;
}

int launch_selective_scan_segmented(int dtype, int state_dtype, const ScanArgs& a, void* ws, size_t ws_bytes,
                                    cudaStream_t stream) {
    const int S = scan_segments(a.B, a.T);
    if (S == 1 || !ws || ws_bytes < selective_scan_segmented_workspace(a.B, a.T, a.d, a.N))
        return launch_selective_scan(dtype, state_dtype, a, stream);
    if (dtype == NT_F32 && state_dtype == NT_F32) return launch_segmented<NT_F32>(state_dtype, a, S, static_cast<float*>(ws), stream);
    if (dtype == NT_BF16 && (state_dtype == NT_F32 || state_dtype == NT_BF16))
        return launch_segmented<NT_BF16>(state_dtype, a, S, static_cast<float*>(ws), stream);
    return fail(NT_ERR_DTYPE, "selective_scan: unsupported dtype %d / state dtype %d", dtype, state_dtype);
}

int launch_selective_scan(int dtype, int state_dtype, const ScanArgs& a, cudaStream_t stream) {
    if (a.T <= kStepMaxT && a.N <= 256 && a.B <= 65535) {
        if (dtype == NT_F32 && state_dtype == NT_F32) return launch_step<NT_F32, NT_F32>(a, stream);
        if (dtype == NT_BF16 && state_dtype == NT_F32) return launch_step<NT_BF16, NT_F32>(a, stream);
        if (dtype == NT_BF16 && state_dtype == NT_BF16) return launch_step<NT_BF16, NT_BF16>(a, stream);
    }
    FusedArgs f{};
    if (dtype == NT_F32 && state_dtype == NT_F32) return launch_mode<NT_F32, NT_F32, 0>(a, f, stream);
    if (dtype == NT_BF16 && state_dtype == NT_F32) return launch_mode<NT_BF16, NT_F32, 0>(a, f, stream);
    if (dtype == NT_BF16 && state_dtype == NT_BF16) return launch_mode<NT_BF16, NT_BF16, 0>(a, f, stream);
    return fail(NT_ERR_DTYPE, "selective_scan: unsupported dtype %d / state dtype %d", dtype, state_dtype);
}

// ---------------------------------------------------------------------------
// Time-segmented scan for small batches.  With B rows the plain scan has
// B*d/CPB CTAs, each walking all T steps; splitting T into S segments gives
// S times the CTAs and S times shorter serial chains:
//   A. state-only pass over every segment from a zero state: its end state
//      and its decay exp(A*sum(dt)) per state;
//   B. carry-in of segment s: h_in[0] = state_in,
//      h_in[s+1] = end[s] + decay[s] * h_in[s]  (the recurrence is linear in h);
//      h_in after the last segment is the returned state;
//   C. the ordinary scan of every segment from its h_in, writing the outputs.
// Segments are consecutive row ranges of one sequence, so a (row, segment)
// pair is handled as a "batch row" of length T/S at rows (b*S + s)*T/S.
// ---------------------------------------------------------------------------
constexpr int kMaxSegments = 8;   // scan_segments keeps B*S <= 8

__global__ void __launch_bounds__(256) scan_seg_combine_kernel(int64_t B, int S, int64_t dN, const float* h_end,
                                                              const float* decay, const void* state_in, int sin_bf16,
                                                              float* h_in, void* state_out, int sout_bf16) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < B * dN; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / dN, j = i % dN;
        float h = 0.f;
        if (state_in) h = sin_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(state_in)[i])
                                   : static_cast<const float*>(state_in)[i];
        // all segments' loads first (S <= kMaxSegments), then the chain
        float e[kMaxSegments], q[kMaxSegments];
#pragma unroll
        for (int s = 0; s < kMaxSegments; ++s) {
            if (s < S) {
                const int64_t v = (b * S + s) * dN + j;
                e[s] = h_end[v];
                q[s] = decay[v];
            }
        }
#pragma unroll
        for (int s = 0; s < kMaxSegments; ++s) {
            if (s < S) {
                h_in[(b * S + s) * dN + j] = h;
                h = fmaf(q[s], h, e[s]);
            }
        }
        if (state_out) {
            if (sout_bf16) static_cast<__nv_bfloat16*>(state_out)[i] = __float2bfloat16_rn(h);
            else static_cast<float*>(state_out)[i] = h;
        }
    }
}

template <int DT>
int launch_segmented(int state_dtype, const ScanArgs& a, int S, float* ws, cudaStream_t stream) {
    FusedArgs f{};
    const int64_t Ts = a.T / S, Bs = a.B * S, n_st = Bs * a.d * a.N;
    float* h_end = ws;
    float* decay = h_end + n_st;
    float* h_in = decay + n_st;
    ScanArgs pa = a;                               // A: state-only, zero start
    pa.B = Bs; pa.T = Ts; pa.state_in = nullptr; pa.state_out = h_end; pa.seg_decay = decay;
    pa.gate = nullptr; pa.y = nullptr; pa.row_pos = nullptr; pa.sparse_flag = nullptr;
    int rc = launch_mode<DT, NT_F32, 0, 0>(pa, f, stream);
    if (rc != NT_OK) return rc;
    const int64_t dN = a.d * a.N;                  // B: carry-in per segment, returned state
    const int64_t blocks = std::min<int64_t>((a.B * dN + 255) / 256, 148 * 8);
    scan_seg_combine_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a.B, S, dN, h_end, decay, a.state_in,
                                                                  state_dtype == NT_BF16, h_in, a.state_out,
                                                                  state_dtype == NT_BF16);
    rc = check_launch("scan_seg_combine_kernel");
    if (rc != NT_OK) return rc;
    ScanArgs pc = a;                               // C: outputs from the carry-in
    pc.B = Bs; pc.T = Ts; pc.state_in = h_in; pc.state_out = nullptr;
    return launch_mode<DT, NT_F32, 0, 1>(pc, f, stream);
}

int launch_lif_ssm_fused(const FusedArgs& f, cudaStream_t stream) {
    ScanArgs a{};
    return launch_mode<NT_BF16, NT_F32, 1>(a, f, stream);
}

}  // namespace nt
