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

// Shared-memory plan of one CTA: CPB channels of one batch row, 128 threads,
// TPC threads per channel holding NPT states each (NP = TPC*NPT >= d_state).
template <int TPC, int NPT, typename T>
struct ScanLayout {
    static constexpr int TCH = 32;                 // time steps per staged chunk
    static constexpr int CPB = 128 / TPC;          // channels per CTA
    static constexpr int NP = TPC * NPT;           // padded d_state
    // raw staging (double-buffered): u|x, dt, gate tiles [TCH][CPB]; B, C tiles [TCH][NP]
    static constexpr int RAW = 3 * TCH * CPB + 2 * TCH * NP;
    static constexpr int RAW_BYTES = ((RAW * (int)sizeof(T)) + 15) & ~15;
    // widened: (u, dt) [TCH][CPB] float2; B/(n+1) and C [TCH][NP] float each;
    // output tile [TCH][CPB] of T; row positions [TCH]; 1/(n+1) [NP]
    static constexpr int UD_BYTES = 8 * TCH * CPB;
    static constexpr int BC_BYTES = 4 * 2 * TCH * NP;
    static constexpr int YO_BYTES = ((TCH * CPB * (int)sizeof(T)) + 15) & ~15;
    static constexpr size_t BYTES = 2 * (size_t)RAW_BYTES + UD_BYTES + BC_BYTES + YO_BYTES + 4 * TCH + 4 * NP;
};

// Position of logical state n of a staged B or C row: the slices of the TPC
// threads are interleaved by groups of four states (group q of every thread's
// slice, then group q+1), so the 16-byte reads of one step by the threads of
// a warp fall on consecutive bank groups (one wavefront for up to 8 slices;
// threads of one slice read the same address, a broadcast).
template <int TPC, int NPT>
__device__ __forceinline__ int bc_pos(int n) {
    const int sub = n / NPT, q = (n % NPT) >> 2;
    return q * 4 * TPC + sub * 4 + (n & 3);
}

// Widen EPV = 16/sizeof(T) elements (one 16-byte vector) to float32.
__device__ __forceinline__ void widen16(const float* src, float* v) {
    const float4 q = *reinterpret_cast<const float4*>(src);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void widen16(const __nv_bfloat16* src, float* v) {
    const uint4 q = *reinterpret_cast<const uint4*>(src);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
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
// Thread (cl, sub) owns states [NPT*sub, NPT*sub + NPT) of channel c0 + cl.
// Per chunk of TCH steps:
//   1. cp.async stages the next chunk's raw inputs while this one computes;
//   2. one widening pass per CTA: (u, dt) per (step, channel) -- in MODE 1 one
//      thread per channel runs the LIF membrane through the chunk here --
//      and B/(n+1), C per (step, state), shared by every channel of the CTA;
//   3. each thread advances its states through the chunk from registers, in
//      groups of TPC steps whose partial C.h sums are combined by a register
//      butterfly (reduce_scatter); the lane that ends up with step j's sum
//      adds D*u, applies the gate and writes the output tile;
//   4. the output tile goes to global memory with 16-byte stores.
template <int DT, int SDT, int TPC, int NPT, int MODE, int OUT = 1>
__global__ void __launch_bounds__(128, NPT == 8 ? 4 : 5)
ssm_scan_kernel(ScanArgs a, FusedArgs f) {
    static_assert(OUT == 1 || MODE == 0, "state-only pass is a MODE 0 variant");
    static_assert(NPT == 4 || NPT == 8, "4 or 8 states per thread");
    using T = typename Elem<MODE == 0 ? DT : NT_BF16>::T;
    using L = ScanLayout<TPC, NPT, T>;
    constexpr int CPB = L::CPB, NP = L::NP, kTch = L::TCH, NPR = NPT / 2, NQ = NPT / 4;
    constexpr int EPV = 16 / (int)sizeof(T);
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float2* w_ud = reinterpret_cast<float2*>(smem_raw + 2 * L::RAW_BYTES);            // [kTch][CPB] (u, dt)
    float* w_B = reinterpret_cast<float*>(smem_raw + 2 * L::RAW_BYTES + L::UD_BYTES); // [kTch][NP] B/(n+1)
    float* w_C = w_B + kTch * NP;                                                    // [kTch][NP] C
    T* w_yo = reinterpret_cast<T*>(smem_raw + 2 * L::RAW_BYTES + L::UD_BYTES + L::BC_BYTES);  // [kTch][CPB]
    int* w_pos = reinterpret_cast<int*>(smem_raw + 2 * L::RAW_BYTES + L::UD_BYTES + L::BC_BYTES + L::YO_BYTES);
    float* w_rn = reinterpret_cast<float*>(w_pos + kTch);                            // [NP] 1/(n+1)

    const int64_t T_len = MODE ? f.L : a.T, d = MODE ? f.d : a.d, N = MODE ? f.N : a.N;
    const T* p_u = static_cast<const T*>(MODE ? f.x : a.u);
    const T* p_dt = static_cast<const T*>(MODE ? f.delta : a.dt);
    const T* p_B = static_cast<const T*>(MODE ? f.Bm : a.Bm);
    const T* p_C = static_cast<const T*>(MODE ? f.Cm : a.Cm);
    const T* p_g = MODE == 0 ? static_cast<const T*>(a.gate) : nullptr;
    const bool has_gate = p_g != nullptr;
    const int64_t ld_bc = (MODE == 0 && a.ld_bc > 0) ? a.ld_bc : N;

    const int tid = threadIdx.x, cl = tid / TPC, sub = tid % TPC, lane = tid & 31;
    const unsigned gmask = TPC >= 32 ? 0xffffffffu : (((1u << TPC) - 1u) << (lane & ~(TPC - 1)));
    const int64_t c0 = (int64_t)blockIdx.x * CPB, c = c0 + cl, b = blockIdx.y;
    const bool live = c < d;

    // ---- per-state constants -------------------------------------------------
    // A = -exp(log_A), rounded like the reference's own tensor op (ssm.py:121)
    auto load_logA = [&](int64_t n) -> float {
        if (MODE == 0) return Elem<DT>::load(static_cast<const typename Elem<DT>::T*>(a.log_A) + c * N + n);
        return f.log_A[c * N + n];
    };
    auto A_of = [&](float la) -> float { return MODE == 0 ? -Elem<DT>::rnd(expf(la)) : -expf(la); };
    // HiPPO structure test, per channel.  fp32 parameters: A[c,n] == (n+1)*A[c,0]
    // to 1e-6 relative.  bf16 parameters: log_A[c,n] == log(n+1) + log_A[c,0] to
    // one bf16 ulp of the stored value (the HiPPO init up to storage rounding).
    constexpr bool kBf16Params = (MODE == 0 && DT == NT_BF16);
    float A2[NPT], h[NPT];
    float2 ci2[NPR], lim2[NPR];
    bool hippo_ok = true;
    const float la0 = live ? load_logA(0) : 0.f;
    const float Abase = live ? A_of(la0) : -1.f;
    const void* sin = MODE ? (const void*)f.state_in : a.state_in;
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int64_t n = (int64_t)sub * NPT + j;
        float A = 0.f;
        h[j] = 0.f;
        const bool on = live && n < N;
        if (on) {
            const float la = load_logA(n);
            A = A_of(la);
            if (sin) {
                const int64_t si = (b * d + c) * N + n;
                if (MODE == 0 && SDT == NT_BF16) h[j] = __bfloat162float(static_cast<const __nv_bfloat16*>(sin)[si]);
                else h[j] = static_cast<const float*>(sin)[si];
            }
            if (kBf16Params) {
                int e2;
                frexpf(la, &e2);                                   // |la| in [2^(e2-1), 2^e2)
                const float ulp = la == 0.f ? 0.f : ldexpf(1.f, e2 - 8);
                if (fabsf(la - (logf((float)(n + 1)) + la0)) > ulp) hippo_ok = false;
            } else if (fabsf(A - (float)(n + 1) * Abase) > 1e-6f * fabsf(A)) {
                hippo_ok = false;
            }
        }
        const bool lim = on && fabsf(A) < 1e-6f;
        if (lim) hippo_ok = false;
        A2[j] = A * kLog2e;
        // general path on B' = B/(n+1): B_bar*u = (A_bar - 1) * ((n+1)/A) * B' * u,
        // or dt * (n+1) * B' * u for the |A| < 1e-6 states (ssm.py:129-137)
        const float np1 = (float)(n + 1);
        const float ci = (lim || A == 0.f) ? 0.f : np1 / A;
        if (j & 1) { ci2[j / 2].y = ci; lim2[j / 2].y = lim ? np1 : 0.f; }
        else { ci2[j / 2].x = ci; lim2[j / 2].x = lim ? np1 : 0.f; }
    }
    // one decision per channel: every state of the channel must qualify
    const unsigned okm = __ballot_sync(0xffffffffu, hippo_ok);
    const bool hippo = (okm & gmask) == gmask;
    // HiPPO constants: first-state exponent, ratio exponent, 1/A[c,0]
    const float a2first = (float)(sub * NPT + 1) * Abase * kLog2e;
    const float q2 = Abase * kLog2e;
    const float rA0 = 1.0f / Abase;
    float Dv = 0.f;
    if (live) Dv = MODE == 0 ? Elem<DT>::load(static_cast<const typename Elem<DT>::T*>(a.D) + c) : f.Dskip[c];

    float beta = 0.f, th = 0.f, mem = 0.f;          // MODE 1: thread tid < CPB runs channel c0 + tid's LIF
    const int64_t cm = c0 + tid;
    if (MODE == 1 && tid < CPB && cm < d) {
        beta = f.beta[cm];
        th = f.threshold[cm];
        if (f.mem_in) mem = f.mem_in[b * d + cm];
    }
    unsigned spike_local = 0;
    float dt_sum = 0.f;                             // state-only pass: sum of dt over the segment
    for (int i = tid; i < NP; i += 128) w_rn[i] = 1.0f / (float)(i + 1);
    const bool sparse_rows = (MODE == 0) && a.row_pos != nullptr && a.sparse_flag != nullptr && *a.sparse_flag != 0;

    // 16-byte staging is possible when every tile row starts 16-byte aligned
    const bool act_vec = (d % EPV == 0) && (c0 + CPB <= d) && (CPB % EPV == 0) &&
                         ((reinterpret_cast<uintptr_t>(p_u) | reinterpret_cast<uintptr_t>(p_dt) |
                           reinterpret_cast<uintptr_t>(p_g)) & 15) == 0;
    const bool bc_vec = (NP == N) && (ld_bc % EPV == 0) &&
                        ((reinterpret_cast<uintptr_t>(p_B) | reinterpret_cast<uintptr_t>(p_C)) & 15) == 0;
    const int64_t row0 = b * T_len;   // first (batch, time) row of this batch element

    auto raw_buf = [&](int k) { return reinterpret_cast<T*>(smem_raw + (k & 1) * L::RAW_BYTES); };
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

    // One step of this thread's NPT states.  Steps past the end of the
    // sequence see u = dt = B = 0, which leaves the state unchanged.
    auto step = [&](int tt, auto hip) -> float {
        constexpr bool HIP = decltype(hip)::value;
        float Bf[NPT], Cf[NPT];
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
            const int o = tt * NP + q * 4 * TPC + sub * 4;
            const float4 bq = *reinterpret_cast<const float4*>(w_B + o);
            Bf[4 * q] = bq.x; Bf[4 * q + 1] = bq.y; Bf[4 * q + 2] = bq.z; Bf[4 * q + 3] = bq.w;
            if (OUT) {
                const float4 cq = *reinterpret_cast<const float4*>(w_C + o);
                Cf[4 * q] = cq.x; Cf[4 * q + 1] = cq.y; Cf[4 * q + 2] = cq.z; Cf[4 * q + 3] = cq.w;
            }
        }
        const float2 ud = w_ud[tt * CPB + cl];
        const float u = ud.x, dtv = ud.y;
        float2 av[NPR], hv[NPR];
#pragma unroll
        for (int j = 0; j < NPR; ++j) hv[j] = make_float2(h[2 * j], h[2 * j + 1]);
        if (HIP) {
            // A[n] = (n+1) A0.  With e = A_bar - 1 = exp(dt A[n]) - 1 and
            // w = u B/((n+1) A0) = u B_bar / e, the update A_bar h + B_bar u is
            //     h' = h + e (h + w)      (two fmas: t = B' * u/A0 + h, h + e t)
            // and e follows the chain e[n+1] = e[n] q + (q - 1), q = exp(dt A0).
            const float e0 = ex2(dtv * a2first) - 1.0f;
            const float qv = ex2(dtv * q2);
            av[0] = make_float2(e0, __fmaf_rn(e0, qv, qv - 1.0f));
            const float qs = qv * qv;
            const float2 qq = make_float2(qs, qs);
            const float qm = __fmaf_rn(qv, qv, -1.0f);
            const float2 qqm = make_float2(qm, qm);
#pragma unroll
            for (int j = 1; j < NPR; ++j) av[j] = __ffma2_rn(av[j - 1], qq, qqm);
            const float sc = u * rA0;
            const float2 ss = make_float2(sc, sc);
#pragma unroll
            for (int j = 0; j < NPR; ++j) {
                const float2 t = __ffma2_rn(make_float2(Bf[2 * j], Bf[2 * j + 1]), ss, hv[j]);
                hv[j] = __ffma2_rn(av[j], t, hv[j]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < NPR; ++j) av[j] = make_float2(ex2(dtv * A2[2 * j]), ex2(dtv * A2[2 * j + 1]));
            const float2 uu = make_float2(u, u), dd = make_float2(dtv, dtv);
#pragma unroll
            for (int j = 0; j < NPR; ++j) {
                const float2 nci = make_float2(-ci2[j].x, -ci2[j].y);
                const float2 coef = __ffma2_rn(dd, lim2[j], __ffma2_rn(av[j], ci2[j], nci));
                const float2 bu = __fmul2_rn(coef, __fmul2_rn(make_float2(Bf[2 * j], Bf[2 * j + 1]), uu));
                hv[j] = __ffma2_rn(av[j], hv[j], bu);
            }
        }
#pragma unroll
        for (int j = 0; j < NPR; ++j) { h[2 * j] = hv[j].x; h[2 * j + 1] = hv[j].y; }
        if constexpr (OUT) {
            // C.h as one packed fma chain, then one add of the two lanes
            float2 y2 = __fmul2_rn(make_float2(Cf[0], Cf[1]), hv[0]);
#pragma unroll
            for (int j = 1; j < NPR; ++j) y2 = __ffma2_rn(make_float2(Cf[2 * j], Cf[2 * j + 1]), hv[j], y2);
            return y2.x + y2.y;
        } else {
            dt_sum += dtv;                         // the segment's total decay exponent
            return 0.f;
        }
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
        __syncthreads();
        const int nt = (T_len - t0 < kTch) ? (int)(T_len - t0) : kTch;
        // ---- widening pass --------------------------------------------------
        const T* rb = raw_buf(kc);
        const T* r_u = rb;
        const T* r_dt = r_u + kTch * CPB;
        const T* r_g = r_dt + kTch * CPB;
        const T* r_B = r_g + kTch * CPB;
        const T* r_C = r_B + kTch * NP;
        if (MODE == 0) {
            for (int i = tid * EPV; i < kTch * CPB; i += 128 * EPV) {
                float uv[EPV], dv[EPV];
                widen16(r_u + i, uv);
                widen16(r_dt + i, dv);
#pragma unroll
                for (int k = 0; k < EPV; k += 2)
                    *reinterpret_cast<float4*>(w_ud + i + k) = make_float4(uv[k], dv[k], uv[k + 1], dv[k + 1]);
            }
        } else if (tid < CPB) {
            // LIF (snn.py:177-181) in fp32 for channel c0 + tid through the chunk;
            // steps past the sequence end give u = 0 and leave the membrane alone
            const bool on = cm < d;
#pragma unroll 4
            for (int tt = 0; tt < kTch; ++tt) {
                const float xv = to_f(r_u[tt * CPB + tid]);
                const float m1 = __fadd_rn(__fmul_rn(beta, mem), xv);
                const float s1 = (m1 >= th) ? 1.f : 0.f;
                const bool in_seq = on && tt < nt;
                const float uu = in_seq ? s1 : 0.f;
                mem = in_seq ? __fsub_rn(m1, __fmul_rn(th, s1)) : mem;
                w_ud[tt * CPB + tid] = make_float2(uu, to_f(r_dt[tt * CPB + tid]));
                if (in_seq) {
                    spike_local += uu != 0.f;
                    if (f.spikes) {
                        const int64_t idx = (row0 + t0 + tt) * d + cm;
                        if (f.spike_dtype == NT_U8) static_cast<unsigned char*>(f.spikes)[idx] = (unsigned char)(uu != 0.f);
                        else static_cast<__nv_bfloat16*>(f.spikes)[idx] = __float2bfloat16_rn(uu);
                    }
                }
            }
        }
        for (int i = tid * EPV; i < kTch * NP; i += 128 * EPV) {
            float bv[EPV], cv[EPV];
            widen16(r_B + i, bv);
            if (OUT) widen16(r_C + i, cv);
#pragma unroll
            for (int k = 0; k < EPV; k += 4) {
                const int tt = (i + k) / NP, n = (i + k) % NP;     // four states of one row
                const int o = tt * NP + bc_pos<TPC, NPT>(n);
                const float4 r4 = *reinterpret_cast<const float4*>(w_rn + n);
                *reinterpret_cast<float4*>(w_B + o) =
                    make_float4(bv[k] * r4.x, bv[k + 1] * r4.y, bv[k + 2] * r4.z, bv[k + 3] * r4.w);
                if (OUT) *reinterpret_cast<float4*>(w_C + o) = make_float4(cv[k], cv[k + 1], cv[k + 2], cv[k + 3]);
            }
        }
        if (sparse_rows && tid < kTch) w_pos[tid] = (t0 + tid < T_len) ? a.row_pos[row0 + t0 + tid] : -1;
        __syncthreads();
        // ---- recurrence: groups of TPC steps, partial sums combined in registers
        auto run = [&](auto hip) {
            static_for<0, kTch / TPC>([&](auto grp) {
                constexpr int g0 = decltype(grp)::value * TPC;
                float yp[TPC];
                static_for<0, TPC>([&](auto j) { yp[decltype(j)::value] = step(g0 + decltype(j)::value, hip); });
                if constexpr (OUT) {
                    if constexpr (TPC > 1) reduce_scatter<TPC>(yp, sub, gmask);
                    const int tt = g0 + (TPC > 1 ? sub : 0);
                    const float uu = w_ud[tt * CPB + cl].x;
                    const float yv = __fadd_rn(yp[0], __fmul_rn(Dv, uu));
                    if (MODE == 0) {
                        using E = Elem<DT>;
                        float o = E::rnd(yv);
                        if (has_gate) {
                            const float gv = to_f(r_g[tt * CPB + cl]);
                            o = E::rnd(o * (a.gate_is_silu ? gv : E::rnd(silu_f(gv))));
                        }
                        w_yo[tt * CPB + cl] = E::from_f(o);
                    } else {
                        w_yo[tt * CPB + cl] = __float2bfloat16_rn(yv);
                    }
                }
            });
        };
        if (hippo) run(std::true_type{});
        else run(std::false_type{});
        if constexpr (OUT) {
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
        }
        __syncthreads();   // raw_buf(kc) and the tiles are refilled by the next chunk
    }
    // ---- carry-out -----------------------------------------------------------
    if constexpr (!OUT) {
        // end state of the segment (float32) and its decay exp(A*sum(dt)) per state
        if (live) {
#pragma unroll
            for (int j = 0; j < NPT; ++j) {
                const int64_t n = (int64_t)sub * NPT + j;
                if (n >= N) continue;
                const int64_t si = (b * d + c) * N + n;
                const float a2 = hippo ? (float)(n + 1) * Abase * kLog2e : A2[j];
                static_cast<float*>(a.state_out)[si] = h[j];
                a.seg_decay[si] = ex2(a2 * dt_sum);
            }
        }
        return;
    }
    void* sout = MODE ? (void*)f.state_out : a.state_out;
    if (live && sout) {
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int64_t n = (int64_t)sub * NPT + j;
            if (n >= N) continue;
            const int64_t si = (b * d + c) * N + n;
            if (MODE == 0 && SDT == NT_BF16) static_cast<__nv_bfloat16*>(sout)[si] = __float2bfloat16_rn(h[j]);
            else static_cast<float*>(sout)[si] = h[j];
        }
    }
    if (MODE == 1) {
        if (tid < CPB && cm < d && f.mem_out) f.mem_out[b * d + cm] = mem;
        if (f.spike_count) {
            const unsigned w = __reduce_add_sync(0xffffffffu, spike_local);
            if ((tid & 31) == 0 && w) atomicAdd(f.spike_count, (unsigned long long)w);
        }
    }
}

int pow2_at_least(int64_t x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

template <int DT, int SDT, int MODE, int TPC, int NPT, int OUT>
int launch_tpc(const ScanArgs& a, const FusedArgs& f, cudaStream_t stream) {
    using T = typename Elem<MODE == 0 ? DT : NT_BF16>::T;
    using L = ScanLayout<TPC, NPT, T>;
    auto kern = ssm_scan_kernel<DT, SDT, TPC, NPT, MODE, OUT>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::BYTES);
    if (e != cudaSuccess) return fail(NT_ERR_CUDA, "scan: smem attribute: %s", cudaGetErrorString(e));
    const int64_t d = MODE ? f.d : a.d, B = MODE ? f.B : a.B;
    dim3 grid((unsigned)((d + L::CPB - 1) / L::CPB), (unsigned)B);
    kern<<<grid, 128, L::BYTES, stream>>>(a, f);
    return check_launch("ssm_scan_kernel");
}

#ifndef NT_SCAN_NARROW_WARPS
#define NT_SCAN_NARROW_WARPS 3
#endif
// States per thread: 8, or 4 when 8 would give the GPU fewer than
// NT_SCAN_NARROW_WARPS warps per SM sub-partition: the recurrence of one warp
// is a serial chain over T, so a sub-partition with one warp more than its
// neighbours sets the kernel's time, and halving the slice doubles the warps.
template <int DT, int SDT, int MODE, int OUT = 1>
int launch_mode(const ScanArgs& a, const FusedArgs& f, cudaStream_t stream) {
    const int64_t N = MODE ? f.N : a.N, d = MODE ? f.d : a.d, B = MODE ? f.B : a.B;
    if (N > 256) return fail(NT_ERR_ARG, "scan: d_state %lld > 256 unsupported", (long long)N);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tpc8 = pow2_at_least((N + 7) / 8);
    const int64_t warps8 = B * ((d + 128 / tpc8 - 1) / (128 / tpc8)) * 4;
    const bool narrow = N > 4 && tpc8 <= 16 && warps8 < (int64_t)NT_SCAN_NARROW_WARPS * 4 * sms;
    if (narrow || N <= 4) {
        switch (pow2_at_least((N + 3) / 4)) {
            case 1: return launch_tpc<DT, SDT, MODE, 1, 4, OUT>(a, f, stream);
            case 2: return launch_tpc<DT, SDT, MODE, 2, 4, OUT>(a, f, stream);
            case 4: return launch_tpc<DT, SDT, MODE, 4, 4, OUT>(a, f, stream);
            case 8: return launch_tpc<DT, SDT, MODE, 8, 4, OUT>(a, f, stream);
            case 16: return launch_tpc<DT, SDT, MODE, 16, 4, OUT>(a, f, stream);
            case 32: return launch_tpc<DT, SDT, MODE, 32, 4, OUT>(a, f, stream);
            default: break;
        }
    }
    switch (tpc8) {
        case 1: return launch_tpc<DT, SDT, MODE, 1, 8, OUT>(a, f, stream);
        case 2: return launch_tpc<DT, SDT, MODE, 2, 8, OUT>(a, f, stream);
        case 4: return launch_tpc<DT, SDT, MODE, 4, 8, OUT>(a, f, stream);
        case 8: return launch_tpc<DT, SDT, MODE, 8, 8, OUT>(a, f, stream);
        case 16: return launch_tpc<DT, SDT, MODE, 16, 8, OUT>(a, f, stream);
        case 32: return launch_tpc<DT, SDT, MODE, 32, 8, OUT>(a, f, stream);
        default: return fail(NT_ERR_ARG, "scan: d_state %lld > 256 unsupported", (long long)N);
    }
}

// ---------------------------------------------------------------------------
// Short sequences (decode steps, T <= kStepMaxT): one warp per (batch row,
// channel), lane l holding states l, l+32, ... in registers, with no shared
// memory staging.  The chunked kernel above stages and steps through a whole
// 16-32-step chunk and pays its per-CTA set-up for every 8-16 channels, which
// for one step costs ~40x the step itself; this kernel is bounded by reading
// and writing the state.  Same arithmetic as the chunked kernel (A rounded
// like the reference's op, the HiPPO form h' = h + e (h + w) when log_A has the
// HiPPO structure -- tested per channel here, per CTA there -- and the general
// (A_bar - 1)/A form otherwise), but each state's exponential is taken
// directly instead of by the chunked kernel's product chain, and C.h is summed
// by a warp reduction: results agree with it to a few float32 ulps.
constexpr int kStepMaxT = 4;
constexpr int kStepWarps = 8;

template <int DT, int SDT, int NPT>
__global__ void __launch_bounds__(32 * kStepWarps)
ssm_step_kernel(ScanArgs a) {
    using E = Elem<DT>;
    using T = typename E::T;
    const int lane = threadIdx.x & 31;
    const int64_t c = (int64_t)blockIdx.x * kStepWarps + (threadIdx.x >> 5), b = blockIdx.y;
    const int64_t d = a.d, N = a.N, Tl = a.T;
    if (c >= d) return;                                   // whole warps leave together
    const int64_t ld_bc = a.ld_bc > 0 ? a.ld_bc : N;
    const T* logA = static_cast<const T*>(a.log_A) + c * N;
    const float la0 = E::load(logA);
    const float Abase = -E::rnd(expf(la0));
    float A2[NPT], ci[NPT], limf[NPT], h[NPT];
    bool ok = true;
#pragma unroll
    for (int j = 0; j < NPT; ++j) {
        const int64_t n = lane + 32 * j;
        const bool on = n < N;
        const float la = on ? E::load(logA + n) : 0.f;
        const float A = on ? -E::rnd(expf(la)) : 0.f;
        h[j] = 0.f;
        if (on && a.state_in) {
            const int64_t si = (b * d + c) * N + n;
            h[j] = SDT == NT_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.state_in)[si])
                                  : static_cast<const float*>(a.state_in)[si];
        }
        if (on) {
            if (DT == NT_BF16) {
                int e2;
                frexpf(la, &e2);
                const float ulp = la == 0.f ? 0.f : ldexpf(1.f, e2 - 8);
                if (fabsf(la - (logf((float)(n + 1)) + la0)) > ulp) ok = false;
            } else if (fabsf(A - (float)(n + 1) * Abase) > 1e-6f * fabsf(A)) {
                ok = false;
            }
        }
        const bool lim = on && fabsf(A) < 1e-6f;
        if (lim) ok = false;
        limf[j] = lim ? 1.f : 0.f;
        A2[j] = A * kLog2e;
        ci[j] = (lim || A == 0.f) ? 0.f : 1.0f / A;
    }
    const bool hippo = __all_sync(0xffffffffu, ok);
    const float rA0 = 1.0f / Abase;
    const float Dv = E::load(static_cast<const T*>(a.D) + c);
    const bool sparse_rows = a.row_pos != nullptr && a.sparse_flag != nullptr && *a.sparse_flag != 0;
    const T* p_u = static_cast<const T*>(a.u);
    const T* p_dt = static_cast<const T*>(a.dt);
    const T* p_B = static_cast<const T*>(a.Bm);
    const T* p_C = static_cast<const T*>(a.Cm);
    const T* p_g = static_cast<const T*>(a.gate);
    for (int64_t t = 0; t < Tl; ++t) {
        const int64_t row = b * Tl + t;
        const float u = E::to_f(p_u[row * d + c]);
        const float dtv = E::to_f(p_dt[row * d + c]);
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int64_t n = lane + 32 * j;
            if (n >= N) continue;
            const float Bn = E::to_f(p_B[row * ld_bc + n]);
            const float Cn = E::to_f(p_C[row * ld_bc + n]);
            if (hippo) {
                const float e = ex2(dtv * ((float)(n + 1) * Abase * kLog2e)) - 1.0f;
                const float tv = __fmaf_rn(Bn * (1.0f / (float)(n + 1)), u * rA0, h[j]);
                h[j] = __fmaf_rn(e, tv, h[j]);
            } else {
                const float av = ex2(dtv * A2[j]);
                const float coef = __fmaf_rn(dtv, limf[j], __fmaf_rn(av, ci[j], -ci[j]));
                h[j] = __fmaf_rn(av, h[j], coef * (Bn * u));
            }
            y = __fmaf_rn(Cn, h[j], y);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (lane == 0) {
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
    if (a.state_out) {
#pragma unroll
        for (int j = 0; j < NPT; ++j) {
            const int64_t n = lane + 32 * j;
            if (n >= N) continue;
            const int64_t si = (b * d + c) * N + n;
            if (SDT == NT_BF16) static_cast<__nv_bfloat16*>(a.state_out)[si] = __float2bfloat16_rn(h[j]);
            else static_cast<float*>(a.state_out)[si] = h[j];
        }
    }
}

template <int DT, int SDT>
int launch_step(const ScanArgs& a, cudaStream_t stream) {
    dim3 grid((unsigned)((a.d + kStepWarps - 1) / kStepWarps), (unsigned)a.B);
    const int npt = a.N <= 32 ? 1 : a.N <= 64 ? 2 : a.N <= 128 ? 4 : 8;
    switch (npt) {
        case 1: ssm_step_kernel<DT, SDT, 1><<<grid, 32 * kStepWarps, 0, stream>>>(a); break;
        case 2: ssm_step_kernel<DT, SDT, 2><<<grid, 32 * kStepWarps, 0, stream>>>(a); break;
        case 4: ssm_step_kernel<DT, SDT, 4><<<grid, 32 * kStepWarps, 0, stream>>>(a); break;
        default: ssm_step_kernel<DT, SDT, 8><<<grid, 32 * kStepWarps, 0, stream>>>(a); break;
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
