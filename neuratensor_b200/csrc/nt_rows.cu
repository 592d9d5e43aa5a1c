// Row-wise kernels: RMSNorm (neuratensor/core/fused.py:118, nn.RMSNorm with
// eps=None) and the spike-row compaction behind the sparse out_proj
// (neuratensor/core/fused.py:149-165).
//
// Compaction is a stream compaction over the per-row "any spike" flags:
// warp ballots + popc give each warp its active-row count, one CTA-wide
// exclusive scan turns counts into positions.  The whole decision of
// _sparse_out_proj (density = n_active/M, dense when density > 0.5) is made
// on the device, so the host never waits for it.
#include "nt_kernels.cuh"

#include <algorithm>

namespace nt {

// ---------------------------------------------------------------------------
// RMSNorm: y = rnd(rnd(x * 1/sqrt(mean(x^2) + eps)) * w), eps = FLT_EPSILON.
// torch computes rms_norm in float32 for bf16 inputs and rounds the
// normalised value to the input dtype before the weight multiply.
// One warp per row, 16-byte vectors per lane when rows allow.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) rmsnorm_kernel(int64_t M, int64_t D, const void* xv, const void* wv, void* yv) {
    using E = Elem<DT>;
    using T = typename E::T;
    constexpr int EPV = 16 / (int)sizeof(T);           // elements per 16-byte vector
    const T* x = static_cast<const T*>(xv);
    const T* w = static_cast<const T*>(wv);
    T* y = static_cast<T*>(yv);
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    // 16-byte vectors per lane when every row starts 16-byte aligned
    const bool vec = (D % EPV == 0) &&
                     ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
    auto widen = [](const T* p, float (&v)[EPV]) {
        if constexpr (sizeof(T) == 2) {
            const uint4 q = *reinterpret_cast<const uint4*>(p);
            const uint32_t qq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[2 * i] = __uint_as_float(qq[i] << 16);
                v[2 * i + 1] = __uint_as_float(qq[i] & 0xffff0000u);
            }
        } else {
            const float4 q = *reinterpret_cast<const float4*>(p);
            v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
        }
    };
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < M; r += warps) {
        const T* xr = x + r * D;
        T* yr = y + r * D;
        float ss = 0.f;
        if (vec) {
            // unrolled so that several 16-byte loads of the row are in flight at once
#pragma unroll 4
            for (int64_t i = (int64_t)lane * EPV; i < D; i += 32 * EPV) {
                float v[EPV];
                widen(xr + i, v);
#pragma unroll
                for (int k = 0; k < EPV; ++k) ss = fmaf(v[k], v[k], ss);
            }
        } else {
            for (int64_t i = lane; i < D; i += 32) {
                const float v = E::load(xr + i);
                ss = fmaf(v, v, ss);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float mean = ss / (float)D;
        const float rs = 1.0f / sqrtf(mean + 1.1920928955078125e-07f);
        if (vec) {
#pragma unroll 4
            for (int64_t i = (int64_t)lane * EPV; i < D; i += 32 * EPV) {
                float v[EPV], g[EPV];
                widen(xr + i, v);
                widen(w + i, g);
                T o[EPV];
#pragma unroll
                for (int k = 0; k < EPV; ++k) o[k] = E::from_f(E::rnd(v[k] * rs) * g[k]);
                *reinterpret_cast<uint4*>(yr + i) = *reinterpret_cast<const uint4*>(o);
            }
        } else {
            for (int64_t i = lane; i < D; i += 32) {
                const float v = E::rnd(E::load(xr + i) * rs);
                yr[i] = E::from_f(v * E::load(w + i));
            }
        }
    }
}

int launch_rmsnorm(int dtype, int64_t M, int64_t D, const void* x, const void* w, void* y, cudaStream_t stream) {
    const int64_t blocks = std::min<int64_t>((M + 7) / 8, 148 * 16);
    if (dtype == NT_F32) rmsnorm_kernel<NT_F32><<<(unsigned)blocks, 256, 0, stream>>>(M, D, x, w, y);
    else if (dtype == NT_BF16) rmsnorm_kernel<NT_BF16><<<(unsigned)blocks, 256, 0, stream>>>(M, D, x, w, y);
    else return fail(NT_ERR_DTYPE, "rmsnorm: dtype %d", dtype);
    return check_launch("rmsnorm_kernel");
}

// ---------------------------------------------------------------------------
// Embedding gather (model.py:258, nn.Embedding): out[r, :] = W[ids[r], :].
// One warp per row, 16-byte vectors when rows allow.  An id outside
// [0, vocab) writes a zero row and raises ERRF_BAD_ARG in the device error
// word (the reference raises IndexError; a kernel reports instead of trapping).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) embedding_kernel(int64_t M, int64_t D, int64_t vocab, const int64_t* ids,
                                                         const T* W, T* out, unsigned* err) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const bool vec = ((D * (int64_t)sizeof(T)) % 16 == 0) &&
                     ((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < M; r += warps) {
        const int64_t id = ids[r];
        const bool ok = id >= 0 && id < vocab;
        if (!ok && lane == 0 && err) atomicOr(err, ERRF_BAD_ARG);
        T* o = out + r * D;
        if (vec) {
            const int64_t nv = D * (int64_t)sizeof(T) / 16;
            const uint4* src = reinterpret_cast<const uint4*>(W + (ok ? id : 0) * D);
            uint4* dst = reinterpret_cast<uint4*>(o);
            for (int64_t i = lane; i < nv; i += 32) dst[i] = ok ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
        } else {
            for (int64_t i = lane; i < D; i += 32) o[i] = ok ? W[id * D + i] : T(0.f);
        }
    }
}

int launch_embedding(int dtype, int64_t M, int64_t D, int64_t vocab, const int64_t* ids, const void* W, void* out,
                     cudaStream_t stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    const int64_t blocks = std::min<int64_t>((M + 7) / 8, 148 * 16);
    if (dtype == NT_F32)
        embedding_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(M, D, vocab, ids, static_cast<const float*>(W),
                                                                      static_cast<float*>(out), device_error_word(dev));
    else if (dtype == NT_BF16)
        embedding_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
            M, D, vocab, ids, static_cast<const __nv_bfloat16*>(W), static_cast<__nv_bfloat16*>(out),
            device_error_word(dev));
    else return fail(NT_ERR_DTYPE, "embedding: dtype %d", dtype);
    return check_launch("embedding_kernel");
}

// ---------------------------------------------------------------------------
// Greedy token choice (model.py:344-359 with top_k = 1): the reference keeps
// every logit equal to the row maximum (`logits < topk(logits, 1)[-1]` ->
// -inf), softmaxes and samples, i.e. picks uniformly among the tied maxima.
// One CTA per row: the maximum and the number of positions holding it, then
// the floor(u * ties)-th of them in index order (u in [0, 1) per row, from the
// caller's generator).  NaN logits compare false, as in torch's `<`.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) greedy_kernel(int64_t V, const T* logits, int64_t ld, const float* u,
                                                      int64_t* out) {
    __shared__ float s_red[8];
    __shared__ int s_cnt[8];
    __shared__ int s_pick;
    const int64_t r = blockIdx.x;
    const T* row = logits + r * ld;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto at = [&](int64_t i) -> float {
        if constexpr (sizeof(T) == 2) return __bfloat162float(row[i]);
        else return row[i];
    };
    float m = -INFINITY;
    for (int64_t i = tid; i < V; i += 256) m = fmaxf(m, at(i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_red[warp] = m;
    __syncthreads();
    m = s_red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, s_red[w]);
    // ties, counted per thread over a contiguous slice so that the k-th tie in
    // index order can be located with one prefix over the 256 counts
    const int64_t per = (V + 255) / 256, lo = tid * per, hi = lo + per < V ? lo + per : V;
    int cnt = 0;
    for (int64_t i = lo; i < hi; ++i) cnt += at(i) == m;
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) s_cnt[warp] = incl;
    __syncthreads();
    int base = 0, total = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        if (w < warp) base += s_cnt[w];
        total += s_cnt[w];
    }
    const int excl = base + incl - cnt;
    if (tid == 0) s_pick = -1;
    __syncthreads();
    int k = total > 0 ? (int)(u[r] * (float)total) : 0;
    if (k >= total) k = total - 1;
    if (cnt > 0 && k >= excl && k < excl + cnt) {
        int seen = excl;
        for (int64_t i = lo; i < hi; ++i)
            if (at(i) == m) {
                if (seen == k) { out[r] = i; break; }
                ++seen;
            }
        s_pick = 1;
    }
    __syncthreads();
    if (tid == 0 && s_pick < 0) out[r] = 0;              // no comparable logit (all NaN)
}

int launch_greedy(int dtype, int64_t B, int64_t V, const void* logits, int64_t ld, const float* u, int64_t* out,
                  cudaStream_t stream) {
    if (dtype == NT_F32)
        greedy_kernel<float><<<(unsigned)B, 256, 0, stream>>>(V, static_cast<const float*>(logits), ld, u, out);
    else if (dtype == NT_BF16)
        greedy_kernel<__nv_bfloat16><<<(unsigned)B, 256, 0, stream>>>(V, static_cast<const __nv_bfloat16*>(logits),
                                                                       ld, u, out);
    else return fail(NT_ERR_DTYPE, "greedy: dtype %d", dtype);
    return check_launch("greedy_kernel");
}

// ---------------------------------------------------------------------------
// flags[r] = any(spikes[r, :] != 0).  One warp per row, 16-byte loads when
// the row is 16-byte aligned; a value is non-zero when its magnitude bits
// are (so -0.0 counts as zero, as in torch's `any`).
// Row activity as 32-row words: bit j of words[g] is set when row 32g + j has
// a non-zero value.  A 256-thread block owns one word; each warp tests four
// rows (16-byte loads when rows are 16-byte aligned), then warp 0 packs the
// 32 answers with a ballot.
template <int DT>
__global__ void __launch_bounds__(256) row_any_words_kernel(int64_t M, int64_t K, const void* sv, unsigned* words) {
    using T = typename Elem<DT>::T;
    __shared__ int any_row[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row_bytes = K * (int64_t)sizeof(T);
    const bool vec = (row_bytes % 16 == 0) && ((reinterpret_cast<uintptr_t>(sv) & 15) == 0);
    const uint32_t mag = sizeof(T) == 2 ? 0x7FFF7FFFu : 0x7FFFFFFFu;
    const int64_t n_words = (M + 31) / 32;
    for (int64_t g = blockIdx.x; g < n_words; g += gridDim.x) {
#pragma unroll 1
        for (int j = warp; j < 32; j += 8) {
            const int64_t r = 32 * g + j;
            uint32_t acc = 0;
            if (r < M) {
                if (vec) {
                    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const char*>(sv) + r * row_bytes);
                    for (int64_t i = lane; i < row_bytes / 16; i += 32) {
                        const uint4 q = __ldg(p + i);
                        acc |= (q.x | q.y | q.z | q.w) & mag;
                    }
                } else {
                    const T* p = static_cast<const T*>(sv) + r * K;
                    for (int64_t i = lane; i < K; i += 32) acc |= (Elem<DT>::load(p + i) != 0.f) ? 1u : 0u;
                }
            }
            const unsigned a = __ballot_sync(0xffffffffu, acc != 0);
            if (lane == 0) any_row[j] = a != 0;
        }
        __syncthreads();
        if (warp == 0) {
            const unsigned w = __ballot_sync(0xffffffffu, any_row[lane] != 0);
            if (lane == 0) words[g] = w;
        }
        __syncthreads();
    }
}

int launch_row_any_words(int dtype, int64_t M, int64_t K, const void* spikes, unsigned* words, cudaStream_t stream) {
    const int64_t blocks = std::min<int64_t>((M + 31) / 32, 148 * 16);
    if (dtype == NT_F32) row_any_words_kernel<NT_F32><<<(unsigned)blocks, 256, 0, stream>>>(M, K, spikes, words);
    else if (dtype == NT_BF16) row_any_words_kernel<NT_BF16><<<(unsigned)blocks, 256, 0, stream>>>(M, K, spikes, words);
    else return fail(NT_ERR_DTYPE, "row_any: dtype %d", dtype);
    return check_launch("row_any_words_kernel");
}


// ---------------------------------------------------------------------------
// Single-CTA stream compaction.  counters[0] = n_active, counters[1] = 1 when
// the sparse branch is taken, counters[2] = rows the out_proj GEMM processes
// (n_active when sparse, M when dense).  On the sparse branch row_idx lists
// those rows and row_pos maps a row to its compacted position (-1 when
// skipped); on the dense branch both stay unwritten and mean the identity.
// ---------------------------------------------------------------------------

// Inclusive scan of one int per thread across a 1024-thread CTA; *total gets the sum.
__device__ __forceinline__ int cta_scan_1024(int v, int* warp_tot, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += o;
    }
    if (lane == 31) warp_tot[warp] = v;
    __syncthreads();
    if (warp == 0) {
        int w = warp_tot[lane];
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int o = __shfl_up_sync(0xffffffffu, w, off);
            if (lane >= off) w += o;
        }
        warp_tot[lane] = w;
        if (lane == 31) *total = w;
    }
    __syncthreads();
    return v + (warp ? warp_tot[warp - 1] : 0);
}
// The same from row-activity words: word (b, w) covers rows b*T + 32w + j,
// j < min(32, T - 32w); a row is active when any channel block set its bit.
// Thread i owns a run of consecutive words.
__global__ void __launch_bounds__(1024) compact_row_bits_kernel(int64_t B, int64_t T, int64_t n_cblk,
                                                                const unsigned* bits, int* row_pos, int* row_idx,
                                                                int* counters, int sparse_enabled,
                                                                long long* n_active_out) {
    __shared__ int warp_tot[32];
    __shared__ int s_total;
    const int64_t n_words = (T + 31) / 32, words = B * n_words;
    const int64_t per = (words + 1023) / 1024;
    const int64_t w0 = threadIdx.x * per, w1 = (w0 + per < words) ? w0 + per : words;
    auto word_mask = [&](int64_t g) -> unsigned {
        const int64_t b = g / n_words, w = g % n_words;
        unsigned m = 0;
        for (int64_t k = 0; k < n_cblk; ++k) m |= bits[(k * B + b) * n_words + w];
        const int64_t valid = T - 32 * w;
        return valid >= 32 ? m : (m & ((1u << valid) - 1u));
    };
    int cnt = 0;
    for (int64_t g = w0; g < w1; ++g) cnt += __popc(word_mask(g));
    const int incl = cta_scan_1024(cnt, warp_tot, &s_total);
    const int64_t M = B * T;
    const int n_active = s_total;
    const bool sparse = sparse_enabled && (2LL * n_active <= M);
    if (sparse) {
        int pos = incl - cnt;
        for (int64_t g = w0; g < w1; ++g) {
            const unsigned m = word_mask(g);
            const int64_t b = g / n_words, w = g % n_words;
            const int64_t valid = T - 32 * w < 32 ? T - 32 * w : 32;
            for (int j = 0; j < valid; ++j) {
                const int64_t r = b * T + 32 * w + j;
                if ((m >> j) & 1u) { row_pos[r] = pos; row_idx[pos] = (int)r; ++pos; }
                else row_pos[r] = -1;
            }
        }
    }
    if (threadIdx.x == 0) {
        counters[0] = n_active;
        counters[1] = sparse ? 1 : 0;
        counters[2] = sparse ? n_active : (int)M;
        if (n_active_out) *n_active_out = n_active;
    }
}

int launch_compact_row_bits(int64_t B, int64_t T, int64_t n_cblk, const unsigned* row_bits, int* row_pos,
                            int* row_idx, int* counters, int sparse_enabled, cudaStream_t stream,
                            long long* n_active_out) {
    if (B * T > (int64_t)INT32_MAX) return fail(NT_ERR_ARG, "compact_row_bits: B*T too large");
    compact_row_bits_kernel<<<1, 1024, 0, stream>>>(B, T, n_cblk, row_bits, row_pos, row_idx, counters,
                                                    sparse_enabled, n_active_out);
    return check_launch("compact_row_bits_kernel");
}

// dst[i, :] = src[row_idx[i], :] for i < counters[2].  Rows of 16-byte chunks.
__global__ void __launch_bounds__(256) gather_rows_kernel(int64_t M, int64_t row_bytes, const char* src,
                                                          const int* row_idx, const int* counters, char* dst) {
    const int64_t m = counters[2];
    const bool mapped = counters[1] != 0;
    const int64_t chunks = row_bytes / 16;
    const int64_t total = m * chunks;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / chunks, k = i % chunks;
        const int64_t sr = mapped ? row_idx[r] : r;
        reinterpret_cast<uint4*>(dst + r * row_bytes)[k] = __ldg(reinterpret_cast<const uint4*>(src + sr * row_bytes) + k);
    }
}

int launch_gather_rows(int dtype, int64_t M, int64_t K, const void* src, const int* row_idx, const int* counters,
                       void* dst, cudaStream_t stream) {
    const int64_t es = dtype == NT_F32 ? 4 : 2;
    const int64_t row_bytes = K * es;
    if (row_bytes % 16) return fail(NT_ERR_ARG, "gather_rows: row bytes %lld not a multiple of 16", (long long)row_bytes);
    const int64_t blocks = std::min<int64_t>((M * (row_bytes / 16) + 255) / 256, 148 * 16);
    gather_rows_kernel<<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, stream>>>(
        M, row_bytes, static_cast<const char*>(src), row_idx, counters, static_cast<char*>(dst));
    return check_launch("gather_rows_kernel");
}

// For rows skipped by the sparse branch (row_pos[r] < 0 and counters[1] != 0):
// dst[r, :] = src ? src[r, :] : 0.  One warp per row; active rows are skipped
// whole; 16-byte accesses when the rows allow them.
template <typename T>
__global__ void __launch_bounds__(256) fill_inactive_kernel(int64_t M, int64_t N, const int* row_pos,
                                                            const int* counters, const T* src, T* dst, int vec) {
    if (counters[1] == 0) return;
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < M; r += warps) {
        if (row_pos[r] >= 0) continue;
        if (vec) {
            constexpr int EPV = 16 / (int)sizeof(T);
            uint4* d = reinterpret_cast<uint4*>(dst + r * N);
            const uint4* sp = src ? reinterpret_cast<const uint4*>(src + r * N) : nullptr;
            for (int64_t i = lane; i < N / EPV; i += 32) d[i] = sp ? __ldg(sp + i) : make_uint4(0, 0, 0, 0);
        } else {
            for (int64_t i = lane; i < N; i += 32) dst[r * N + i] = src ? src[r * N + i] : T(0.f);
        }
    }
}

int launch_fill_inactive(int dtype, int64_t M, int64_t N, const int* row_pos, const int* counters,
                         const void* src, void* dst, cudaStream_t stream) {
    const int64_t es = dtype == NT_F32 ? 4 : 2;
    const int vec = (N * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(src) & 15) == 0;
    const int64_t blocks = std::max<int64_t>(std::min<int64_t>((M + 7) / 8, 148 * 16), 1);
    if (dtype == NT_F32)
        fill_inactive_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(
            M, N, row_pos, counters, static_cast<const float*>(src), static_cast<float*>(dst), vec);
    else
        fill_inactive_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
            M, N, row_pos, counters, static_cast<const __nv_bfloat16*>(src), static_cast<__nv_bfloat16*>(dst), vec);
    return check_launch("fill_inactive_kernel");
}

}  // namespace nt
