// Sliding-window causal attention with rotary embedding
// (neuratensor/core/model.py:148-182 SlidingWindowAttention.forward, RoPE
// model.py:88-126), bf16, head_dim 64 (small preset) or 128 (large preset).
//
// Query i attends to keys j with i - window <= j <= i (the reference's
// tril & |i - j| <= window mask; plain causal when T <= window).  One CTA
// owns 64 queries of one (batch, head); its four warps own 16 queries each.
// The CTA walks only the key tiles its window reaches (at most
// (window + 64) / 64 + 1 tiles of 64 keys) instead of all T keys.
//
// Inputs come straight from the qkv projection, row-major [B*T, 3*d_model]
// with columns [q | k | v], heads of HD contiguous columns.  RoPE is applied
// while Q and K tiles are copied to shared memory, rounding like the
// reference's three bf16 tensor ops: rnd(rnd(x*cos) + rnd(rot(x)*sin)), with
// rot(x) = [-x[HD/2:], x[:HD/2]] and the module's own bf16 cos/sin tables.
//
// Scores S = (Q K^T) / sqrt(HD) and the output O = softmax(S) V are computed with
// mma.sync m16n8k16 (bf16 operands, fp32 accumulation) and an online softmax
// in fp32 (the flash-attention recurrence); P is rounded to bf16 for the PV
// product.  O is written bf16 to out[b*T + i, h*HD + d], the layout o_proj
// reads ([B, T, d_model]).
#include "nt_kernels.cuh"

namespace nt {

namespace {

constexpr int kQB = 64;          // queries per CTA
constexpr int kKB = 64;          // keys per tile
constexpr int kAttnThreads = 128;

// Tiles are [64 rows][HD bf16] = HD/8 chunks of 16 bytes per row; chunk c of
// row r is stored at chunk c ^ (r & 7) so that ldmatrix's eight row reads
// (same chunk, eight consecutive rows) hit eight different bank groups.
template <int HD>
__device__ __forceinline__ int swz(int r, int c) { return r * (HD / 8) + (c ^ (r & 7)); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
// D += A * B, m16n8k16, bf16 inputs, fp32 accumulators
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&p);
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// out = rnd(rnd(x*c) + rnd(r*s)) for two bf16 lanes (x, r, c, s packed pairs)
__device__ __forceinline__ uint32_t rope2(uint32_t x, uint32_t r, uint32_t c, uint32_t s, bool neg) {
    float o[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const float xv = k ? bf_hi(x) : bf_lo(x);
        const float rv = (k ? bf_hi(r) : bf_lo(r)) * (neg ? -1.f : 1.f);
        const float cv = k ? bf_hi(c) : bf_lo(c);
        const float sv = k ? bf_hi(s) : bf_lo(s);
        o[k] = bf16_round(bf16_round(xv * cv) + bf16_round(rv * sv));
    }
    return pack_bf16(o[0], o[1]);
}

// Copy rows [r0, r0+64) of one head's HD columns (base points at row 0,
// column h*HD of q, k or v; ld in elements) into a swizzled tile; rows at or
// past T are zero.  With rope, chunks c and c+HC (dims d and d+HD/2, HC =
// HD/16) are rotated together: out[d] = x[d]*cos[d] - x[d+HD/2]*sin[d] for
// d < HD/2, out[d+HD/2] = x[d+HD/2]*cos[d+HD/2] + x[d]*sin[d+HD/2].
template <int HD, bool ROPE>
__device__ __forceinline__ void load_tile(uint4* tile, const __nv_bfloat16* base, int64_t ld, int r0, int T,
                                          const __nv_bfloat16* cosT, const __nv_bfloat16* sinT) {
    constexpr int HC = HD / 16;            // chunk pairs per row
    // 64 rows x HC chunk pairs
    for (int p = threadIdx.x; p < 64 * HC; p += kAttnThreads) {
        const int r = p / HC, c = p % HC, t = r0 + r;
        uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
        if (t < T) {
            const uint4* src = reinterpret_cast<const uint4*>(base + (int64_t)t * ld);
            lo = __ldg(src + c);
            hi = __ldg(src + c + HC);
            if (ROPE) {
                const uint4* cr = reinterpret_cast<const uint4*>(cosT + (int64_t)t * HD);
                const uint4* sr = reinterpret_cast<const uint4*>(sinT + (int64_t)t * HD);
                const uint4 clo = __ldg(cr + c), chi = __ldg(cr + c + HC);
                const uint4 slo = __ldg(sr + c), shi = __ldg(sr + c + HC);
                const uint4 x0 = lo, x1 = hi;
                lo.x = rope2(x0.x, x1.x, clo.x, slo.x, true);
                lo.y = rope2(x0.y, x1.y, clo.y, slo.y, true);
                lo.z = rope2(x0.z, x1.z, clo.z, slo.z, true);
                lo.w = rope2(x0.w, x1.w, clo.w, slo.w, true);
                hi.x = rope2(x1.x, x0.x, chi.x, shi.x, false);
                hi.y = rope2(x1.y, x0.y, chi.y, shi.y, false);
                hi.z = rope2(x1.z, x0.z, chi.z, shi.z, false);
                hi.w = rope2(x1.w, x0.w, chi.w, shi.w, false);
            }
        }
        tile[swz<HD>(r, c)] = lo;
        tile[swz<HD>(r, c + HC)] = hi;
    }
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads)
window_attention_kernel(int64_t T, int64_t window, int64_t dm, const __nv_bfloat16* qkv, int64_t ld_qkv,
                        const __nv_bfloat16* cosT, const __nv_bfloat16* sinT, __nv_bfloat16* out, int64_t ld_out) {
    constexpr int KS = HD / 16;            // 16-wide k-steps over head_dim (and 16-wide output column pairs)
    __shared__ __align__(128) uint4 sQ[kQB * HD / 8];
    __shared__ __align__(128) uint4 sK[kKB * HD / 8];
    __shared__ __align__(128) uint4 sV[kKB * HD / 8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kQB, h = blockIdx.y, b = blockIdx.z;
    const int Ti = (int)T;
    const __nv_bfloat16* rows = qkv + (int64_t)b * T * ld_qkv;
    const __nv_bfloat16* qbase = rows + (int64_t)h * HD;
    const __nv_bfloat16* kbase = rows + dm + (int64_t)h * HD;
    const __nv_bfloat16* vbase = rows + 2 * dm + (int64_t)h * HD;

    load_tile<HD, true>(sQ, qbase, ld_qkv, q0, Ti, cosT, sinT);
    __syncthreads();
    // this warp's 16 queries as A fragments for the KS 16-wide k-steps of head_dim
    uint32_t qa[KS][4];
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), c = 2 * kk + (lane >> 4);
        ldsm_x4(smem_addr(&sQ[swz<HD>(r, c)]), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
    }

    // 1/sqrt(HD) * log2(e)
    constexpr float kScaleLog2 = (HD == 64 ? 0.125f : 0.08838834764831845f) * 1.4426950408889634f;
    const int qa_row = q0 + warp * 16 + (lane >> 2), qb_row = qa_row + 8;
    float o[2 * KS][4];
#pragma unroll
    for (int j = 0; j < 2 * KS; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

    const int lo_key = q0 - (int)window > 0 ? q0 - (int)window : 0;
    const int hi_key = (q0 + kQB - 1 < Ti - 1) ? q0 + kQB - 1 : Ti - 1;
    for (int k0 = (lo_key / kKB) * kKB; k0 <= hi_key; k0 += kKB) {
        __syncthreads();                       // previous K/V tiles fully consumed
        load_tile<HD, true>(sK, kbase, ld_qkv, k0, Ti, cosT, sinT);
        load_tile<HD, false>(sV, vbase, ld_qkv, k0, Ti, nullptr, nullptr);
        __syncthreads();
        // S = Q K^T for 16 queries x 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                const int r = 16 * np + (lane & 7) + 8 * (lane >> 4), c = 2 * kk + ((lane >> 3) & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(smem_addr(&sK[swz<HD>(r, c)]), b0, b1, b2, b3);
                mma_bf16(s[2 * np], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
                mma_bf16(s[2 * np + 1], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b2, b3);
            }
        }
        // scale (log2 domain), window mask, running max
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = k0 + 8 * j + 2 * (lane & 3) + e;
                const bool ok_a = key <= qa_row && key >= qa_row - (int)window && key < Ti;
                const bool ok_b = key <= qb_row && key >= qb_row - (int)window && key < Ti;
                s[j][e] = ok_a ? s[j][e] * kScaleLog2 : -INFINITY;
                s[j][2 + e] = ok_b ? s[j][2 + e] * kScaleLog2 : -INFINITY;
                mx_a = fmaxf(mx_a, s[j][e]);
                mx_b = fmaxf(mx_b, s[j][2 + e]);
            }
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        // rows with no valid key yet keep a zero base (exp(-inf - 0) = 0)
        const float base_a = mn_a == -INFINITY ? 0.f : mn_a, base_b = mn_b == -INFINITY ? 0.f : mn_b;
        const float corr_a = m_a == -INFINITY ? 0.f : ex2(m_a - base_a);
        const float corr_b = m_b == -INFINITY ? 0.f : ex2(m_b - base_b);
        m_a = mn_a;
        m_b = mn_b;
        l_a *= corr_a;
        l_b *= corr_b;
#pragma unroll
        for (int j = 0; j < 2 * KS; ++j) {
            o[j][0] *= corr_a; o[j][1] *= corr_a;
            o[j][2] *= corr_b; o[j][3] *= corr_b;
        }
        // P = exp2(S - m) as bf16 A fragments; the row sums use the rounded values
        uint32_t pa[4][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t pa01 = pack_bf16(ex2(s[j][0] - base_a), ex2(s[j][1] - base_a));
            const uint32_t pb01 = pack_bf16(ex2(s[j][2] - base_b), ex2(s[j][3] - base_b));
            l_a += bf_lo(pa01) + bf_hi(pa01);
            l_b += bf_lo(pb01) + bf_hi(pb01);
            pa[j >> 1][(j & 1) * 2 + 0] = pa01;
            pa[j >> 1][(j & 1) * 2 + 1] = pb01;
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int dp = 0; dp < KS; ++dp) {
                const int r = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1), c = 2 * dp + (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(smem_addr(&sV[swz<HD>(r, c)]), b0, b1, b2, b3);
                mma_bf16(o[2 * dp], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
                mma_bf16(o[2 * dp + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
            }
        }
    }
    // normalise and store
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    const float ia = l_a > 0.f ? 1.f / l_a : 0.f, ib = l_b > 0.f ? 1.f / l_b : 0.f;
    __nv_bfloat16* orow = out + (int64_t)b * T * ld_out + (int64_t)h * HD + 2 * (lane & 3);
#pragma unroll
    for (int j = 0; j < 2 * KS; ++j) {
        if (qa_row < Ti)
            *reinterpret_cast<uint32_t*>(orow + (int64_t)qa_row * ld_out + 8 * j) = pack_bf16(o[j][0] * ia, o[j][1] * ia);
        if (qb_row < Ti)
            *reinterpret_cast<uint32_t*>(orow + (int64_t)qb_row * ld_out + 8 * j) = pack_bf16(o[j][2] * ib, o[j][3] * ib);
    }
}

}  // namespace

int launch_window_attention(int64_t B, int64_t T, int64_t H, int64_t head_dim, int64_t window, const void* qkv,
                            int64_t ld_qkv, const void* cos_t, const void* sin_t, void* out, int64_t ld_out,
                            cudaStream_t stream) {
    dim3 grid((unsigned)((T + kQB - 1) / kQB), (unsigned)H, (unsigned)B);
    const auto* q = static_cast<const __nv_bfloat16*>(qkv);
    const auto* c = static_cast<const __nv_bfloat16*>(cos_t);
    const auto* s = static_cast<const __nv_bfloat16*>(sin_t);
    auto* o = static_cast<__nv_bfloat16*>(out);
    if (head_dim == 64)
        window_attention_kernel<64><<<grid, kAttnThreads, 0, stream>>>(T, window, H * 64, q, ld_qkv, c, s, o, ld_out);
    else if (head_dim == 128)
        window_attention_kernel<128><<<grid, kAttnThreads, 0, stream>>>(T, window, H * 128, q, ld_qkv, c, s, o, ld_out);
    else
        return fail(NT_ERR_ARG, "window_attention: head_dim %lld (64 or 128 supported)", (long long)head_dim);
    return check_launch("window_attention_kernel");
}

}  // namespace nt
