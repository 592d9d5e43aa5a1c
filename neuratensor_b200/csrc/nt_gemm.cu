// GEMMs of the block: D[M,N] = A[M,K] * W[N,K]^T with fused epilogues.
//
//  * bf16: a persistent tcgen05 tensor-core kernel, one CTA per SM walking
//    128 x BN output tiles.  A TMA warp (cp.async.bulk.tensor, 128-byte
//    swizzle) streams A and W k-blocks into a STAGES-deep shared-memory ring;
//    one elected thread of the MMA warp issues tcgen05.mma (kind::f16, fp32
//    accumulation) into one of two TMEM accumulators; eight epilogue warps
//    drain the other accumulator with tcgen05.ld and apply the epilogue
//    (softplus for dt, out_scale + residual + row scatter for out_proj, ...),
//    so a tile's epilogue overlaps the next tile's MMAs.
//  * fp32: the reference's fp32 mode needs fp32 products; a tiled CUDA-core
//    kernel with the same epilogues.
//
// Every mbarrier wait is bounded: on expiry the kernel raises a bit in the
// device error word and winds down instead of spinning forever.
#include "nt_kernels.cuh"

#include <cuda.h>
#include <algorithm>
#include <mutex>

namespace nt {

// ---------------------------------------------------------------------------
// Epilogue (per element; rounding points follow the reference's tensor ops)
// ---------------------------------------------------------------------------

// softplus(v) = max(v, 0) + log1p(exp(-|v|)), identity above 20 (the
// reference's threshold, ssm.py:330).  exp and log on the MUFU pipe; log1p(z)
// for z < 1e-2 from its Taylor series z - z^2/2 + z^3/3, where log(1 + z)
// would lose the low bits of z.
__device__ __forceinline__ float softplus_f(float v) {
    if (v > 20.f) return v;
    const float z = __expf(-fabsf(v));
    const float l = z < 1e-2f ? z * (1.f - z * (0.5f - z * (1.f / 3.f))) : __logf(1.f + z);
    return fmaxf(v, 0.f) + l;
}
// Output row of accumulator row `row` for the scattering epilogues.
__device__ __forceinline__ int64_t out_row(const EpiArgs& e, int64_t row) {
    const bool mapped = e.row_idx && (!e.row_sparse || *e.row_sparse != 0);
    return mapped ? (int64_t)e.row_idx[row] : row;
}
// silu(g) = g * sigmoid(g)
__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }
template <int DT, int KIND>
__device__ __forceinline__ void epi_apply(const EpiArgs& e, int64_t row, int64_t col, float acc) {
    using E = Elem<DT>;
    using T = typename E::T;
    if (KIND == EPI_STORE) {
        static_cast<T*>(e.out)[row * e.ldo + col] = E::from_f(acc);
    } else if (KIND == EPI_SPLIT2) {
        if (col < e.split) static_cast<T*>(e.out)[row * e.ldo + col] = E::from_f(acc);
        else static_cast<T*>(e.out2)[row * e.ldo2 + (col - e.split)] = E::from_f(acc);
    } else if (KIND == EPI_SPLIT2_SILU) {
        // h as computed; gate -> rnd(silu(rnd(gate))) as the reference's F.silu (fused.py:130)
        if (col < e.split) {
            static_cast<T*>(e.out)[row * e.ldo + col] = E::from_f(acc);
        } else {
            const float g = E::rnd(acc);
            static_cast<T*>(e.out2)[row * e.ldo2 + (col - e.split)] = E::from_f(silu_fast(g));
        }
    } else if (KIND == EPI_SSM_PROJ) {
        if (col < e.split) {
            // dt = softplus(u W_dt^T + b_dt)  (ssm.py:330; threshold 20)
            const float v = E::rnd(acc + E::load(static_cast<const T*>(e.bias) + col));
            const float sp = softplus_f(v);
            static_cast<T*>(e.out)[row * e.ldo + col] = E::from_f(sp);
        } else {
            static_cast<T*>(e.out2)[row * e.ldo2 + (col - e.split)] = E::from_f(acc);
        }
    } else if (KIND == EPI_OUT_PROJ) {
        // out = out_proj(o) * out_scale + residual  (fused.py:138)
        const int64_t r = out_row(e, row);
        const float s = E::load(static_cast<const T*>(e.scale));
        float v = E::rnd(acc);
        v = E::rnd(v * s);
        v = E::rnd(v + E::load(static_cast<const T*>(e.resid) + r * e.ldr + col));
        static_cast<T*>(e.out)[r * e.ldo + col] = E::from_f(v);
    } else if (KIND == EPI_RESID) {
        // o_proj(o) + x  (model.py:181): the product rounded, then the sum
        const float v = E::rnd(E::rnd(acc) + E::load(static_cast<const T*>(e.resid) + row * e.ldr + col));
        static_cast<T*>(e.out)[row * e.ldo + col] = E::from_f(v);
    } else {  // EPI_SCATTER
        const int64_t r = out_row(e, row);
        static_cast<T*>(e.out)[r * e.ldo + col] = E::from_f(acc);
    }
}

// Eight consecutive columns [col, col+8) of one row.  Vector path: the eight
// outputs leave as one 16-byte store (bf16) when the host marked the output
// layout 16-byte compatible (e.vec) and the group lies inside [0, N) on one
// side of `split`; scalar fallback otherwise.
__device__ __forceinline__ uint4 pack_bf16x8(const float (&o)[8]) {
    uint4 r;
    uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 p = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&p);
    }
    return r;
}
__device__ __forceinline__ void unpack_bf16x8(uint4 q, float (&o)[8]) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        o[2 * i] = __uint_as_float(w[i] << 16);
        o[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

// Eight consecutive columns [col, col+8) of one row, in two phases so the
// epilogue can issue its global reads (bias, residual) before it waits for
// the accumulator: epi_pre8 loads them, epi_fin8 applies the epilogue and
// stores.  Vector path: the eight outputs leave as one 16-byte store when the
// host marked the layout 16-byte compatible (e.vec) and the group lies inside
// [0, N) on one side of `split`; scalar fallback otherwise.  `orow` is the
// output (and residual) row of accumulator row `row` (out_row()).
__device__ __forceinline__ bool epi_vec8(const EpiArgs& e, int64_t col, int64_t N) { return e.vec && col + 8 <= N; }

template <int KIND>
__device__ __forceinline__ uint4 epi_pre8(const EpiArgs& e, int64_t orow, int64_t col, int64_t N) {
    if (!epi_vec8(e, col, N)) return make_uint4(0, 0, 0, 0);
    if (KIND == EPI_SSM_PROJ && col < e.split)
        return __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(e.bias) + col));
    if (KIND == EPI_OUT_PROJ || KIND == EPI_RESID)
        return __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(e.resid) + orow * e.ldr + col));
    return make_uint4(0, 0, 0, 0);
}

template <int KIND>
__device__ __forceinline__ void epi_fin8(const EpiArgs& e, int64_t row, int64_t orow, int64_t col, int64_t N,
                                         const float (&acc)[8], uint4 pre) {
    using E = Elem<NT_BF16>;
    if (!epi_vec8(e, col, N)) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (col + j < N) epi_apply<NT_BF16, KIND>(e, row, col + j, acc[j]);
        return;
    }
    float o[8];
    __nv_bfloat16* dst;
    if (KIND == EPI_STORE) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = acc[j];
        dst = static_cast<__nv_bfloat16*>(e.out) + row * e.ldo + col;
    } else if (KIND == EPI_SPLIT2) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = acc[j];
        dst = col < e.split ? static_cast<__nv_bfloat16*>(e.out) + row * e.ldo + col
                            : static_cast<__nv_bfloat16*>(e.out2) + row * e.ldo2 + (col - e.split);
    } else if (KIND == EPI_SPLIT2_SILU) {
        if (col < e.split) {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = acc[j];
            dst = static_cast<__nv_bfloat16*>(e.out) + row * e.ldo + col;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = silu_fast(E::rnd(acc[j]));
            dst = static_cast<__nv_bfloat16*>(e.out2) + row * e.ldo2 + (col - e.split);
        }
    } else if (KIND == EPI_SSM_PROJ) {
        if (col < e.split) {
            float bias[8];
            unpack_bf16x8(pre, bias);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = softplus_f(E::rnd(acc[j] + bias[j]));
            dst = static_cast<__nv_bfloat16*>(e.out) + row * e.ldo + col;
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = acc[j];
            dst = static_cast<__nv_bfloat16*>(e.out2) + row * e.ldo2 + (col - e.split);
        }
    } else if (KIND == EPI_OUT_PROJ) {
        const float s = E::load(static_cast<const __nv_bfloat16*>(e.scale));
        float res[8];
        unpack_bf16x8(pre, res);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = E::rnd(E::rnd(E::rnd(acc[j]) * s) + res[j]);
        dst = static_cast<__nv_bfloat16*>(e.out) + orow * e.ldo + col;
    } else if (KIND == EPI_RESID) {
        float res[8];
        unpack_bf16x8(pre, res);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = E::rnd(E::rnd(acc[j]) + res[j]);
        dst = static_cast<__nv_bfloat16*>(e.out) + row * e.ldo + col;
    } else {  // EPI_SCATTER
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = acc[j];
        dst = static_cast<__nv_bfloat16*>(e.out) + orow * e.ldo + col;
    }
    *reinterpret_cast<uint4*>(dst) = pack_bf16x8(o);
}

// ---------------------------------------------------------------------------
// PTX wrappers (sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum) : "memory");
}
// 32 lanes x 16 columns of fp32 accumulator: thread i gets lane (row) i.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 64 bf16 (128 B), 8-row core-matrix groups 1024 B apart (SBO), version 1.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);        // start address
    d |= (uint64_t)1 << 16;                         // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;               // SBO
    d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                         // SWIZZLE_128B
    return d;
}

// Instruction descriptor: bf16 x bf16 -> f32, both K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4)                 // D format f32
         | (1u << 7)                 // A bf16
         | (1u << 10)                // B bf16
         | ((uint32_t)(N >> 3) << 17)
         | ((uint32_t)(M >> 4) << 24);
}

constexpr int kBM = 128, kBK = 64;
constexpr int kEpiWarps = 16;                      // four per TMEM lane quarter
constexpr int kTcThreads = 64 + 32 * kEpiWarps;    // TMA warp, MMA warp, epilogue warps
constexpr int kAccStride = 256;                    // TMEM columns between the two accumulators
constexpr uint32_t kTmemCols = 512;

template <int BN, int STAGES>
struct TcSmem {
    __nv_bfloat16 a[STAGES][kBM * kBK];
    __nv_bfloat16 b[STAGES][BN * kBK];
    uint64_t full[STAGES];       // TMA -> MMA: k-block landed
    uint64_t empty[STAGES];      // MMA -> TMA: k-block consumed
    uint64_t acc_full[2];        // MMA -> epilogue: accumulator complete
    uint64_t acc_empty[2];       // epilogue -> MMA: accumulator drained
    uint32_t tmem_base;
};

// Deepest ring that fits next to the tile of BN columns (<= 6 stages).
template <int BN> struct TcStages {
    static constexpr int bytes = (kBM + BN) * kBK * 2;
    static constexpr int value = (220 * 1024) / bytes > 6 ? 6 : (220 * 1024) / bytes;
};

// Tiles are numbered m-major in groups: tile t covers output rows
// (t / n_tiles) * 128 and columns (t % n_tiles) * BN, so the CTAs working at
// the same time share A row blocks through L2.
template <int KIND, int BN, int STAGES>
__global__ void __launch_bounds__(kTcThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               int64_t M, int64_t N, int64_t K, const int* m_count, EpiArgs epi, unsigned* err, int splits,
               float* partials) {
    static_assert(BN % 16 == 0 && BN >= 32 && BN <= kAccStride, "tile width");
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment for the swizzled tiles
    const uintptr_t base = (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023);
    auto& S = *reinterpret_cast<TcSmem<BN, STAGES>*>(base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m_eff = m_count ? (int64_t)*m_count : M;
    const int m_tiles = (int)((m_eff + kBM - 1) / kBM);
    const int n_tiles = (int)((N + BN - 1) / BN);
    const int total = m_tiles * n_tiles;
    const int nk = (int)((K + kBK - 1) / kBK);
    // work items: (tile, K split); split s covers k-blocks [s*nk/splits, (s+1)*nk/splits),
    // never empty (splits <= nk), and with splits > 1 the epilogue writes float32
    // partial sums for gemm_splitk_epi_kernel instead of the outputs
    const int items = total * splits;
    if ((int)blockIdx.x >= items) return;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&map_a);
        tma_prefetch_desc(&map_b);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&S.full[s]), 1);
            mbar_init(smem_u32(&S.empty[s]), 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_u32(&S.acc_full[i]), 1);
            mbar_init(smem_u32(&S.acc_empty[i]), kEpiWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&S.tmem_base)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            constexpr uint32_t bytes = (uint32_t)((kBM + BN) * kBK * sizeof(__nv_bfloat16));
            int it = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x) {
                const int tile = item / splits, sp = item % splits;
                const int kb0 = (int)((int64_t)sp * nk / splits), kb1 = (int)((int64_t)(sp + 1) * nk / splits);
                const int m0 = (tile / n_tiles) * kBM, n0 = (tile % n_tiles) * BN;
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait(smem_u32(&S.empty[s]), ((it / STAGES) - 1) & 1)) {
                        atomicOr(err, ERRF_TIMEOUT_PRODUCER);
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(smem_u32(&S.full[s]), bytes);
                    tma_load_2d(smem_u32(S.a[s]), &map_a, smem_u32(&S.full[s]), kb * kBK, m0);
                    tma_load_2d(smem_u32(S.b[s]), &map_b, smem_u32(&S.full[s]), kb * kBK, n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = idesc_bf16(kBM, BN);
            int it = 0, local = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < items && ok; item += gridDim.x, ++local) {
                const int sp = item % splits;
                const int kb0 = (int)((int64_t)sp * nk / splits), kb1 = (int)((int64_t)(sp + 1) * nk / splits);
                const int buf = local & 1;
                if (local >= 2 && !mbar_wait(smem_u32(&S.acc_empty[buf]), ((local >> 1) - 1) & 1)) {
                    atomicOr(err, ERRF_TIMEOUT_MMA);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(buf * kAccStride);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(smem_u32(&S.full[s]), (it / STAGES) & 1)) {
                        atomicOr(err, ERRF_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(S.a[s]), sb = smem_u32(S.b[s]);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k) {
                        // advance 16 bf16 (32 bytes) along K inside the swizzle atom
                        tc_mma(d, sw128_kmajor_desc(sa + k * 32), sw128_kmajor_desc(sb + k * 32), idesc,
                               (kb != kb0 || k) ? 1u : 0u);
                    }
                    tc_commit(smem_u32(&S.empty[s]));
                }
                if (ok) tc_commit(smem_u32(&S.acc_full[buf]));
            }
        }
    } else {
        // ---------------- epilogue: TMEM -> registers -> global ----------------
        constexpr int kParts = kEpiWarps / 4;      // warps sharing a lane quarter
        constexpr int kChunks = (BN / 16 + kParts - 1) / kParts;   // 16-column chunks per warp, at most
        const int q = warp & 3;                     // TMEM lane quarter this warp may access
        const int part = (warp - 2) >> 2;           // its 16-column chunks: part, part + kParts, ...
        int local = 0;
        for (int item = blockIdx.x; item < items; item += gridDim.x, ++local) {
            const int tile = item / splits, sp = item % splits;
            const int buf = local & 1;
            const int64_t m0 = (int64_t)(tile / n_tiles) * kBM, n0 = (int64_t)(tile % n_tiles) * BN;
            const int64_t row = m0 + q * 32 + lane;
            const bool row_ok = row < m_eff;
            const int64_t orow = (KIND == EPI_OUT_PROJ || KIND == EPI_SCATTER) && row_ok && splits == 1
                                     ? out_row(epi, row) : row;
            // the epilogue's global operands (residual rows, bias) do not depend on the
            // accumulator: they are requested before waiting for it, so their latency
            // overlaps the tile's MMAs
            uint4 pre[kChunks][2];
#pragma unroll
            for (int i = 0; i < kChunks; ++i) {
                const int c = 16 * (part + i * kParts);
                pre[i][0] = pre[i][1] = make_uint4(0, 0, 0, 0);
                if (row_ok && c < BN && splits == 1) {
                    pre[i][0] = epi_pre8<KIND>(epi, orow, n0 + c, N);
                    pre[i][1] = epi_pre8<KIND>(epi, orow, n0 + c + 8, N);
                }
            }
            const bool ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&S.acc_full[buf]), (local >> 1) & 1));
            __syncwarp();                           // tcgen05.ld is .sync.aligned: whole warp, converged
            if (!ok) {
                if (lane == 0) atomicOr(err, ERRF_TIMEOUT_EPILOGUE);
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int i = 0; i < kChunks; ++i) {
                const int c = 16 * (part + i * kParts);           // warp-uniform
                if (c >= BN) break;
                float v[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kAccStride + c), v);
                if (splits > 1) {
                    // this split's partial sums of the 16 columns, float32
                    if (row_ok) {
                        float* dst = partials + ((int64_t)sp * M + row) * N + n0 + c;
                        if ((N & 3) == 0 && n0 + c + 16 <= N) {
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                reinterpret_cast<float4*>(dst)[j] =
                                    make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (n0 + c + j < N) dst[j] = v[j];
                        }
                    }
                } else if (row_ok) {
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        const float (&v8)[8] = *reinterpret_cast<const float(*)[8]>(v + 8 * g);
                        epi_fin8<KIND>(epi, row, orow, n0 + c + 8 * g, N, v8, pre[i][g]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&S.acc_empty[buf]));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ---------------------------------------------------------------------------
// fp32 CUDA-core GEMM (64 x 64 tile, 256 threads, 4 x 4 outputs per thread)
// ---------------------------------------------------------------------------
template <int KIND>
__global__ void __launch_bounds__(256)
gemm_f32_kernel(int64_t M, int64_t N, int64_t K, const float* A, int64_t lda, const float* W, int64_t ldb,
                const int* m_count, EpiArgs epi) {
    __shared__ float As[16][64 + 4];
    __shared__ float Ws[16][64 + 4];
    const int64_t m_eff = m_count ? (int64_t)*m_count : M;
    const int64_t m0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
    if (m0 >= m_eff) return;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 16 * 64; i += 256) {
            const int kk = i % 16, rr = i / 16;
            const int64_t ra = m0 + rr, rb = n0 + rr, k = k0 + kk;
            As[kk][rr] = (ra < m_eff && k < K) ? A[ra * lda + k] : 0.f;
            Ws[kk][rr] = (rb < N && k < K) ? W[rb * ldb + k] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; b[i] = Ws[kk][tx * 4 + i]; }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t row = m0 + ty * 4 + i;
        if (row >= m_eff) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t col = n0 + tx * 4 + j;
            if (col < N) epi_apply<NT_F32, KIND>(epi, row, col, acc[i][j]);
        }
    }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps through the driver entry point (no libcuda link)
// ---------------------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode() {
    static PFN_encodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(p);
    });
    return fn;
}

// 2-D bf16 row-major [rows, cols] with leading dimension ld, box = box_rows x 64.
static int make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
    PFN_encodeTiled enc = get_encode();
    if (!enc) return fail(NT_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16)
        return fail(NT_ERR_ARG, "gemm: operand must be 16-byte aligned with a leading dimension multiple of 8");
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(NT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return NT_OK;
}

// Split-K: out = epilogue(sum over the splits' float32 partial sums), the sum in
// split order.
template <int KIND>
__global__ void __launch_bounds__(256) gemm_splitk_epi_kernel(int64_t M, int64_t N, const int* m_count, int splits,
                                                              const float* part, EpiArgs epi) {
    const int64_t m_eff = m_count ? (int64_t)*m_count : M;
    const int64_t total = m_eff * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / N, col = i % N;
        float acc = part[row * N + col];
        for (int s = 1; s < splits; ++s) acc += part[((int64_t)s * M + row) * N + col];
        epi_apply<NT_BF16, KIND>(epi, row, col, acc);
    }
}

template <int KIND, int BN>
static int launch_tc(const GemmArgs& g, cudaStream_t stream) {
    constexpr int STAGES = TcStages<BN>::value;
    CUtensorMap ma, mb;
    int rc = make_map(&ma, g.A, g.M, g.K, g.lda, kBM);
    if (rc) return rc;
    rc = make_map(&mb, g.Bw, g.N, g.K, g.ldb, BN);
    if (rc) return rc;
    const size_t smem = sizeof(TcSmem<BN, STAGES>) + 1024;
    auto kern = gemm_tc_kernel<KIND, BN, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(NT_ERR_CUDA, "gemm: smem attribute: %s", cudaGetErrorString(e));
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t tiles = ((g.M + kBM - 1) / kBM) * ((g.N + BN - 1) / BN);
    int splits = 1;
    if (g.part) {
        splits = gemm_split_k(g.M, g.N, g.K);
        if ((int64_t)splits * g.M * g.N > g.part_elems) splits = 1;
    }
    const int64_t items = tiles * splits;
    const unsigned grid = (unsigned)(items < sms ? items : sms);
    kern<<<grid, kTcThreads, smem, stream>>>(ma, mb, g.M, g.N, g.K, g.m_count, g.epi, device_error_word(dev), splits,
                                             g.part);
    int rc2 = check_launch("gemm_tc_kernel");
    if (rc2 != NT_OK || splits == 1) return rc2;
    const int64_t blocks = std::min<int64_t>((g.M * g.N + 255) / 256, (int64_t)sms * 8);
    gemm_splitk_epi_kernel<KIND><<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, stream>>>(
        g.M, g.N, g.m_count, splits, g.part, g.epi);
    return check_launch("gemm_splitk_epi_kernel");
}

#ifndef NT_GEMM_TILE_OVERHEAD
#define NT_GEMM_TILE_OVERHEAD 64
#endif
// Tile width for an M x N output on `sms` persistent CTAs.  First choice:
// the candidate that wastes the fewest columns of N (ties go to the wider
// tile, which re-reads A fewer times).  When that leaves fewer than two tiles
// per CTA (small M), the candidate with the smallest modelled time instead:
// waves * (BN + overhead), a wave being one tile per CTA and the overhead (in
// columns) a tile's fixed cost (pipeline fill, epilogue tail).
static int pick_bn(int64_t M, int64_t N, int sms) {
    static const int cand[] = {256, 224, 192, 160, 128, 96, 64};
    const int64_t m_tiles = (M + kBM - 1) / kBM;
    int pad_best = 128;
    int64_t best_pad = -1;
    for (int bn : cand) {
        if (bn < 128) continue;
        const int64_t pad = ((N + bn - 1) / bn) * bn - N;
        if (best_pad < 0 || pad < best_pad) { pad_best = bn; best_pad = pad; }
    }
    if (m_tiles * ((N + pad_best - 1) / pad_best) >= 2LL * sms) return pad_best;
    int best = pad_best;
    int64_t best_cost = -1;
    for (int bn : cand) {
        const int64_t tiles = m_tiles * ((N + bn - 1) / bn);
        const int64_t cost = ((tiles + sms - 1) / sms) * (bn + NT_GEMM_TILE_OVERHEAD);
        if (best_cost < 0 || cost < best_cost) { best = bn; best_cost = cost; }
    }
    return best;
}

#ifndef NT_GEMM_MAX_SPLITS
#define NT_GEMM_MAX_SPLITS 8
#endif
// Fewer output tiles than SMs: split K so that about one work item runs per
// SM, keeping at least 8 k-blocks (512 of K) per split for the TMA ring.
int gemm_split_k(int64_t M, int64_t N, int64_t K) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int bn = pick_bn(M, N, sms);
    const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
    const int64_t nk = (K + kBK - 1) / kBK;
    int64_t s = tiles > 0 ? sms / tiles : 1;
    s = std::min<int64_t>(s, nk / 8);
    s = std::min<int64_t>(s, NT_GEMM_MAX_SPLITS);
    return (int)std::max<int64_t>(s, 1);
}

template <int KIND>
static int launch_kind(int dtype, const GemmArgs& g, cudaStream_t stream) {
    if (dtype == NT_BF16) {
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        switch (pick_bn(g.M, g.N, sms)) {
            case 256: return launch_tc<KIND, 256>(g, stream);
            case 224: return launch_tc<KIND, 224>(g, stream);
            case 192: return launch_tc<KIND, 192>(g, stream);
            case 160: return launch_tc<KIND, 160>(g, stream);
            case 128: return launch_tc<KIND, 128>(g, stream);
            case 96: return launch_tc<KIND, 96>(g, stream);
            default: return launch_tc<KIND, 64>(g, stream);
        }
    }
    dim3 grid((unsigned)((g.N + 63) / 64), (unsigned)((g.M + 63) / 64));
    gemm_f32_kernel<KIND><<<grid, 256, 0, stream>>>(g.M, g.N, g.K, static_cast<const float*>(g.A), g.lda,
                                                     static_cast<const float*>(g.Bw), g.ldb, g.m_count, g.epi);
    return check_launch("gemm_f32_kernel");
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int launch_gemm(int dtype, const GemmArgs& g_in, cudaStream_t stream) {
    if (dtype != NT_F32 && dtype != NT_BF16) return fail(NT_ERR_DTYPE, "gemm: dtype %d", dtype);
    if (g_in.M <= 0 || g_in.N <= 0 || g_in.K <= 0) return NT_OK;
    GemmArgs g = g_in;
    {
        // 16-byte epilogue stores need every 8-column group of every output row aligned
        const EpiArgs& e = g.epi;
        bool v = dtype == NT_BF16 && al16(e.out) && e.ldo % 8 == 0;
        if (e.kind == EPI_SPLIT2 || e.kind == EPI_SSM_PROJ || e.kind == EPI_SPLIT2_SILU)
            v = v && e.split % 8 == 0 && al16(e.out2) && e.ldo2 % 8 == 0;
        if (e.kind == EPI_SSM_PROJ) v = v && al16(e.bias);
        if (e.kind == EPI_OUT_PROJ || e.kind == EPI_RESID) v = v && al16(e.resid) && e.ldr % 8 == 0;
        g.epi.vec = v ? 1 : 0;
    }
    switch (g.epi.kind) {
        case EPI_STORE: return launch_kind<EPI_STORE>(dtype, g, stream);
        case EPI_SPLIT2: return launch_kind<EPI_SPLIT2>(dtype, g, stream);
        case EPI_SSM_PROJ: return launch_kind<EPI_SSM_PROJ>(dtype, g, stream);
        case EPI_OUT_PROJ: return launch_kind<EPI_OUT_PROJ>(dtype, g, stream);
        case EPI_SCATTER: return launch_kind<EPI_SCATTER>(dtype, g, stream);
        case EPI_RESID: return launch_kind<EPI_RESID>(dtype, g, stream);
        case EPI_SPLIT2_SILU: return launch_kind<EPI_SPLIT2_SILU>(dtype, g, stream);
        default: return fail(NT_ERR_ARG, "gemm: epilogue kind %d", g.epi.kind);
    }
}

}  // namespace nt
