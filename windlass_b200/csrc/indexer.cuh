// indexer.cuh — DSA lightning-indexer scoring on the tensor cores.
//
// Computes, for query row r and key t < len(r),
//     index[r][t] = sum_h w[r][h] * relu(qk_scale * scale[t] * (q[r][h] . e4m3(k[t])))
// which is the reference's indexer_scores_relu + indexer_combine
// (src/glm_kernels.cuh:308-340; numpy: tools/ref_glm_chain.py:482-501) with
// the key cache in fp8-e4m3 plus a per-key fp32 scale. The [H,T] score array
// the reference writes to global memory and reads back never leaves TMEM here.
//
// Prefill form (many query rows over one cache; one CTA = 4 warps = one 128-key tile):
//   * the TMA engine streams the tile's 16 KB of fp8 keys into shared memory
//     (cp.async.bulk, one contiguous copy: rows are packed 128-byte lines);
//   * each thread widens one key row e4m3 -> bf16 (exact) into a 128B-swizzled
//     K-major tile — tcgen05 kind::f16 needs A and B of one type;
//   * one thread issues tcgen05.mma with M = 128 keys, N = 32 heads x G query
//     rows, K = 128, fp32 accumulators in TMEM;
//   * each thread reads its key's N accumulators back with tcgen05.ld and
//     applies scale, relu and the head-weighted sum in registers.
// Bytes per key: 128 (fp8) + 4 (scale); the kernel is HBM-bound at decode.
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int IDX_H = 32;
constexpr int IDX_D = 128;
constexpr int IDX_TILE = 128;

struct IdxParams {
    const uint8_t* keys;
    long long keys_seq;   // bytes between sequences
    const float* scale;
    long long scale_seq;  // floats between sequences
    int T;
    int n_rows, rows_per_seq, len0, len_step;
    const __nv_bfloat16* q;  // [n_rows][32][128]
    const float* w;          // [n_rows][32]
    float* out;
    long long out_stride;
    float qk_scale;
    int groups_per_cta;
};

__device__ __forceinline__ int rows_len(int r, int rows_per_seq, int len0, int len_step, int T) {
    const long long l = (long long)len0 + (long long)(r % rows_per_seq) * len_step;
    return (int)(l < T ? l : T);
}

template <int G>
struct IdxLayout {
    static constexpr int N = 32 * G;
    static constexpr uint32_t A_BYTES = IDX_TILE * IDX_D * 2;  // bf16 keys, 2 K-chunks
    static constexpr uint32_t A_CHUNK = IDX_TILE * 128;
    static constexpr uint32_t Q_CHUNK = N * 128;
    static constexpr uint32_t Q_BYTES = 2 * Q_CHUNK;
    static constexpr uint32_t K8_BYTES = IDX_TILE * IDX_D;
    static constexpr uint32_t OFF_A = 0;
    static constexpr uint32_t OFF_Q = OFF_A + A_BYTES;
    static constexpr uint32_t OFF_K8 = OFF_Q + Q_BYTES;
    static constexpr uint32_t OFF_W = OFF_K8 + K8_BYTES;
    static constexpr uint32_t OFF_BAR = OFF_W + N * 4;
    static constexpr uint32_t OFF_SLOT = OFF_BAR + 16;
    static constexpr uint32_t BYTES = OFF_SLOT + 16 + 1024;  // + alignment slack
    static constexpr uint32_t TMEM_COLS = N;                   // 32..256, power of two
    static constexpr uint32_t IDESC = idesc_bf16(128, N, 0, 0);
};

template <int G>
__global__ void __launch_bounds__(128) indexer_scores_kernel(IdxParams p) {
    using L = IdxLayout<G>;
    static_assert(G == 1 || G == 2 || G == 4 || G == 8, "G must be a power of two <= 8");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sA = smem_u32(smem + L::OFF_A);
    const uint32_t sQ = smem_u32(smem + L::OFF_Q);
    uint8_t* k8 = smem + L::OFF_K8;
    float* sW = reinterpret_cast<float*>(smem + L::OFF_W);
    uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* bar_mma = bar_tma + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_SLOT);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int t0 = blockIdx.x * IDX_TILE;
    const int nk = min(IDX_TILE, p.T - t0);
    const int n_groups = (p.n_rows + G - 1) / G;
    const int g_begin = blockIdx.y * p.groups_per_cta;
    const int g_end = min(g_begin + p.groups_per_cta, n_groups);
    if (g_begin >= g_end || nk <= 0) return;
    // Rows of one CTA share one sequence (host guarantees it).
    const int seq = (g_begin * G) / p.rows_per_seq;
    // Causal skip: nothing to do if the tile starts past every row's length.
    // (len_step >= 0, so the last row of the CTA is the longest.)
    {
        const int last_row = min(g_end * G, p.n_rows) - 1;
        if (t0 >= rows_len(last_row, p.rows_per_seq, p.len0, p.len_step, p.T)) return;
    }

    if (tid == 0) {
        mbar_init(bar_tma, 1);
        mbar_init(bar_mma, 1);
        fence_mbar_init();
        mbar_expect_tx(bar_tma, (uint32_t)nk * IDX_D);
        bulk_g2s(k8, p.keys + (long long)seq * p.keys_seq + (long long)t0 * IDX_D, (uint32_t)nk * IDX_D,
                 bar_tma);
    }
    if (warp == 0) tmem_alloc(tmem_slot, L::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

    const float sc = (tid < nk) ? __ldg(p.scale + (long long)seq * p.scale_seq + t0 + tid) * p.qk_scale : 0.f;

    // Widen key row `tid` e4m3 -> bf16 into the swizzled K-major A tile.
    bool ok = mbar_wait(bar_tma, 0, 1);
    if (__syncthreads_and(ok)) {
        const uint32_t src = smem_u32(k8) + tid * 128u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t p8 = (uint32_t)(j + tid) & 7u;  // rotate: spread banks
            uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
            if (tid < nk) {
                const uint4 v = lds_v4(src + p8 * 16u);
                lo.x = e4m3x2_to_bf16x2((uint16_t)(v.x & 0xffff));
                lo.y = e4m3x2_to_bf16x2((uint16_t)(v.x >> 16));
                lo.z = e4m3x2_to_bf16x2((uint16_t)(v.y & 0xffff));
                lo.w = e4m3x2_to_bf16x2((uint16_t)(v.y >> 16));
                hi.x = e4m3x2_to_bf16x2((uint16_t)(v.z & 0xffff));
                hi.y = e4m3x2_to_bf16x2((uint16_t)(v.z >> 16));
                hi.z = e4m3x2_to_bf16x2((uint16_t)(v.w & 0xffff));
                hi.w = e4m3x2_to_bf16x2((uint16_t)(v.w >> 16));
            }
            const uint32_t chunk = p8 >> 2, c16 = (p8 & 3u) * 2u;
            sts_v4(sA + chunk * L::A_CHUNK + sw128_off(tid, c16), lo);
            sts_v4(sA + chunk * L::A_CHUNK + sw128_off(tid, c16 + 1), hi);
        }

        uint32_t phase = 0;
        for (int g = g_begin; g < g_end; ++g) {
            const int r0 = g * G;
            // Query rows r0..r0+G-1 (32 heads each) -> swizzled K-major B tile.
            for (int pid = tid; pid < L::N * 16; pid += 128) {
                const int row = pid >> 4, pc = pid & 15;
                const int qr = r0 + row / IDX_H;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (qr < p.n_rows)
                    v = ldg_nc_v4(p.q + ((long long)qr * IDX_H + (row % IDX_H)) * IDX_D + pc * 8);
                sts_v4(sQ + (uint32_t)(pc >> 3) * L::Q_CHUNK + sw128_off(row, pc & 7), v);
            }
            for (int i = tid; i < L::N; i += 128) {
                const int qr = r0 + i / IDX_H;
                sW[i] = (qr < p.n_rows) ? __ldg(p.w + (long long)qr * IDX_H + (i % IDX_H)) : 0.f;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
#pragma unroll
                for (int kk = 0; kk < IDX_D / 16; ++kk) {
                    const uint32_t c = kk >> 2, ko = (kk & 3) * 32;
                    const uint64_t ad = desc_sw128(sA + c * L::A_CHUNK + ko, 16, 1024);
                    const uint64_t bd = desc_sw128(sQ + c * L::Q_CHUNK + ko, 16, 1024);
                    mma_bf16(tmem, ad, bd, L::IDESC, kk > 0 ? 1u : 0u);
                }
                mma_commit(bar_mma);
            }
            ok = mbar_wait(bar_mma, phase, 2);
            phase ^= 1;
            if (!__syncthreads_and(ok)) break;
            tc_fence_after();

            const int t = t0 + tid;
#pragma unroll 1
            for (int gg = 0; gg < G; ++gg) {
                const int row = r0 + gg;
                if (row >= p.n_rows) break;  // uniform across the CTA
                float acc[32];
                tmem_ld32(tmem + lane_base + (uint32_t)(gg * 32), acc);
                tmem_wait_ld();
                float v = 0.f;
#pragma unroll
                for (int h = 0; h < 32; ++h) v = fmaf(sW[gg * 32 + h], fmaxf(acc[h] * sc, 0.f), v);
                const int len = rows_len(row, p.rows_per_seq, p.len0, p.len_step, p.T);
                if (tid < nk) p.out[(long long)row * p.out_stride + t] = (t < len) ? v : -INFINITY;
            }
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

}  // namespace wl

namespace wl {

// ---- decode form: persistent, warp-specialised, fp8 tensor cores ---------------------------
// One CTA per SM streams a contiguous range of 128-key tiles of one row's
// cache. Roles (10 warps), connected by mbarriers only:
//   warp 0      TMA producer: the tile's fp8 keys as one 128 x 128-byte box with
//               128B swizzle (a tensor-map load; rows past the cache end read as
//               zero) into ring stage i % IDX_NS
//   warp 1      MMA issuer:   tcgen05.mma kind::f8f6f4 straight on the fp8 keys
//               (M = 128 keys, K = 32 per instruction), one chain of 4
//               per tile: N = 64 = the query's hi and lo e4m3 terms side by side
//   warps 2-9   epilogue:     tcgen05.ld both halves for one key, combine, scale,
//               relu, head-weighted sum, store (+ fused top-k histogram); two
//               groups of 4 warps take alternate tiles
//
// The query in e4m3: per head, q * s_h (s_h a power of two putting the head's
// largest element in [128, 256)) = hi + lo / 32 with hi = e4m3(q s_h) and
// lo = e4m3((q s_h - hi) * 32). Every bf16 element is reproduced to within
// 2^-22 of the head's largest element (exactly for all but elements more than
// ~2^-14 below it), far inside fp32 rounding of the 128-term dot product. The
// head weight absorbs 1/s_h: w_h relu(x / s_h) = (w_h / s_h) relu(x), s_h > 0.
//
// The epilogue can also accumulate, per row, the histogram of the top
// TOPK_HIST_BITS bits of the order-preserving score keys — the first radix pass
// of the top-k, fused here so that no kernel re-reads the scores for it. Each
// CTA counts into shared memory and adds its nonzero bins to the row's global
// histogram at the end (warp-aggregating global atomics with __match_any_sync
// measured slower).
constexpr int IDX_NS = 8;    // TMA stages of fp8 keys
constexpr int IDX_CTAS_PER_SM = 1;
constexpr int IDX_NACC = 4;  // accumulator sets (hi, lo) in flight
constexpr int IDX_EPI_GROUPS = 2;  // epilogue groups of 4 warps, alternating tiles
constexpr int IDX_STREAM_THREADS = 64 + 128 * IDX_EPI_GROUPS;
constexpr int TOPK_HIST_BITS = 13;
constexpr int TOPK_HIST_BINS = 1 << TOPK_HIST_BITS;

struct IdxStreamLayout {
    static constexpr uint32_t K8_TILE = IDX_TILE * IDX_D;  // 16 KB, 128B-swizzled (1024-aligned)
    static constexpr uint32_t QT = IDX_H * IDX_D;          // one e4m3 query term, 4 KB
    static constexpr uint32_t OFF_K8 = 0;
    static constexpr uint32_t OFF_Q = OFF_K8 + IDX_NS * K8_TILE;  // hi, lo
    static constexpr uint32_t OFF_W = OFF_Q + 2 * QT;
    static constexpr uint32_t OFF_HIST = OFF_W + IDX_H * 4;  // this CTA's share of the row histogram
    static constexpr uint32_t OFF_QRAW = OFF_HIST + TOPK_HIST_BINS * 4;  // the row's bf16 query, as copied
    static constexpr uint32_t OFF_BAR = OFF_QRAW + IDX_H * IDX_D * 2;
    static constexpr int N_BARS = 2 * IDX_NS + 2 * IDX_NACC + 1;  // full, empty, acc_full, acc_empty, query
    static constexpr uint32_t OFF_SLOT = OFF_BAR + N_BARS * 8;
    static constexpr uint32_t BYTES = OFF_SLOT + 16 + 1024;
    static constexpr uint32_t TMEM_COLS = 64 * IDX_NACC;  // 256
    // kind::f8f6f4: E4M3 A and B (format 0), fp32 D; M = 128, N = 64 (hi ‖ lo)
    static constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(2 * IDX_H >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
};

__device__ __forceinline__ uint32_t score_key(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u << 1) == 0u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tma_load3d(void* dst, const CUtensorMap* tm, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// The key cache as a uint8 tensor {128 bytes, T keys, sequences} (strides
// 128 and keys_seq bytes), loaded in {128, 128, 1} boxes with 128B swizzle:
// key rows at or past T read as zero.
struct IdxStreamParams {
    CUtensorMap tm_keys;
};

#ifdef WL_TRACE
__device__ long long* g_trace;
#define WL_TRB(slot)                                                                                    \
    do {                                                                                                \
        if (g_trace && threadIdx.x == 0) {                                                              \
            unsigned long long t_;                                                                      \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                      \
            g_trace[512 + 2 * (blockIdx.y * gridDim.x + blockIdx.x) + (slot)] = (long long)t_;          \
        }                                                                                               \
    } while (0)
#define WL_TRP(slot)                                                                                    \
    do {                                                                                                \
        if (g_trace && blockIdx.x == 0 && blockIdx.y == 0) {                                            \
            unsigned long long t_;                                                                      \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                      \
            g_trace[900 + (slot)] = (long long)t_;                                                      \
        }                                                                                               \
    } while (0)
#define WL_TR(slot, i)                                                                                  \
    do {                                                                                                \
        if (g_trace && blockIdx.x == 0 && blockIdx.y == 0 && (i) < 64) g_trace[(i) * 8 + (slot)] = clock64(); \
    } while (0)
#else
#define WL_TR(slot, i) \
    do {               \
    } while (0)
#define WL_TRB(slot) \
    do {             \
    } while (0)
#define WL_TRP(slot) \
    do {             \
    } while (0)
#endif

__global__ void __launch_bounds__(IDX_STREAM_THREADS, IDX_CTAS_PER_SM)
    indexer_stream_kernel(IdxParams p, const __grid_constant__ IdxStreamParams sp, unsigned* hist, int tiles_per_cta) {
    using L = IdxStreamLayout;
    WL_KT_BEGIN(0);
    WL_TRB(0);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* k8 = smem + L::OFF_K8;
    uint8_t* sQ = smem + L::OFF_Q;
    float* sW = reinterpret_cast<float*>(smem + L::OFF_W);
    unsigned* sHist = reinterpret_cast<unsigned*>(smem + L::OFF_HIST);
    const __nv_bfloat16* sQraw = reinterpret_cast<const __nv_bfloat16*>(smem + L::OFF_QRAW);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* empty = full + IDX_NS;
    uint64_t* acc_full = empty + IDX_NS;
    uint64_t* acc_empty = acc_full + IDX_NACC;
    uint64_t* qbar = acc_empty + IDX_NACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_SLOT);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = blockIdx.y;
    const int seq = r / p.rows_per_seq;
    const int len = rows_len(r, p.rows_per_seq, p.len0, p.len_step, p.T);
    const int ntiles = (len + IDX_TILE - 1) / IDX_TILE;
    const int tb = blockIdx.x * tiles_per_cta;
    const int n = min(tb + tiles_per_cta, ntiles) - tb;
    if (n <= 0) {
        pdl_wait();
        return;
    }
    const float* scale = p.scale + (long long)seq * p.scale_seq;
    float* out = p.out + (long long)r * p.out_stride;
    unsigned* hrow = hist ? hist + (long long)r * TOPK_HIST_BINS : nullptr;

    if (tid == 0) {
        for (int s = 0; s < IDX_NS; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);  // the MMA's commit
        }
        for (int b = 0; b < IDX_NACC; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 128);
        }
        mbar_init(qbar, 1);
        fence_mbar_init();
        // The producer (this thread) copies the row's query (8 KB) at once, so
        // that it lands during the setup below, ahead of the key stream; every
        // other warp converts it from shared memory. (Loading it with per-warp
        // global loads queued behind the key stream, and issuing the first key
        // tiles together with it let them overtake it: both delayed the first
        // MMA by microseconds.)
        pdl_wait();
        mbar_expect_tx(qbar, IDX_H * IDX_D * 2);
        bulk_g2s(smem + L::OFF_QRAW, p.q + (long long)r * IDX_H * IDX_D, IDX_H * IDX_D * 2, qbar);
    }
    if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);  // warp 1 allocates and frees
    if (hist)
        for (int b = tid; b < TOPK_HIST_BINS; b += IDX_STREAM_THREADS) sHist[b] = 0;
    tc_fence_before();
    __syncthreads();  // barriers initialised, TMEM address published
    tc_fence_after();
    if (tid == 0) WL_TRP(0);
    pdl_wait();  // everything above overlaps the previous kernel; global data below
    pdl_trigger();
    const uint32_t tmem = *tmem_slot;
    const bool producer = warp == 0;
    // Query -> two e4m3 terms per head, by every warp but the producer; a named
    // barrier joins them.
    constexpr int CONV_WARPS = IDX_STREAM_THREADS / 32 - 1;
    float wv[(IDX_H + CONV_WARPS - 1) / CONV_WARPS];  // head weights, loaded while the query lands
    if (!producer) {
#pragma unroll
        for (int k2 = 0; k2 < (IDX_H + CONV_WARPS - 1) / CONV_WARPS; ++k2) {
            const int h = warp - 1 + k2 * CONV_WARPS;
            wv[k2] = (lane == 0 && h < IDX_H) ? __ldg(p.w + (long long)r * IDX_H + h) : 0.f;
        }
        mbar_wait(qbar, 0, 9);
    }
#pragma unroll
    for (int k2 = 0; k2 < (IDX_H + CONV_WARPS - 1) / CONV_WARPS; ++k2) {
        const int h = warp - 1 + k2 * CONV_WARPS;
        if (producer || h >= IDX_H) break;
        const uint2 raw = *reinterpret_cast<const uint2*>(sQraw + h * IDX_D + lane * 4);
        const __nv_bfloat162 q01 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
        const __nv_bfloat162 q23 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
        float x[4] = {__low2float(q01), __high2float(q01), __low2float(q23), __high2float(q23)};
        float mx = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) mx = fmaxf(mx, fabsf(x[e]));
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // s_h = 2^(7 - floor(log2 mx)): the largest element lands in [128, 256).
        const int ex = mx > 0.f ? max(((__float_as_int(mx) >> 23) & 0xff) - 127, -100) : 0;
        const float s_h = __int_as_float((127 + 7 - ex) << 23);
        uint32_t hi4 = 0, lo4 = 0;
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
            const float a0 = x[e] * s_h, a1 = x[e + 1] * s_h;
            const __nv_fp8x2_storage_t h2 = __nv_cvt_float2_to_fp8x2(make_float2(a0, a1), __NV_SATFINITE, __NV_E4M3);
            const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(h2, __NV_E4M3);
            const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hr));
            const __nv_fp8x2_storage_t l2 =
                __nv_cvt_float2_to_fp8x2(make_float2((a0 - hf.x) * 32.f, (a1 - hf.y) * 32.f), __NV_SATFINITE, __NV_E4M3);
            hi4 |= (uint32_t)h2 << (8 * e);
            lo4 |= (uint32_t)l2 << (8 * e);
        }
        // 4 codes = 4 bytes at byte lane*4 of the 128-byte row h, 128B-swizzled
        const uint32_t byte = (uint32_t)lane * 4u;
        const uint32_t off = (uint32_t)h * 128u + ((((byte >> 4) ^ (uint32_t)h) & 7u) << 4) + (byte & 15u);
        *reinterpret_cast<uint32_t*>(sQ + off) = hi4;
        *reinterpret_cast<uint32_t*>(sQ + L::QT + off) = lo4;
        if (lane == 0) sW[h] = wv[k2] / s_h;
    }
    if (tid == 32) WL_TRP(1);
    if (!producer) {
        fence_proxy_async_smem();  // the query tile is read by the tensor cores
        asm volatile("bar.sync 1, %0;" ::"n"(IDX_STREAM_THREADS - 32) : "memory");
    }

    if (producer) {
        // ---------------- TMA producer (whole warp loops, lane 0 issues) ----------------
        for (int i = 0; i < n; ++i) {
            const int s = i % IDX_NS;
            if (i >= IDX_NS && !mbar_wait(empty + s, (uint32_t)(i / IDX_NS - 1) & 1u, 10)) break;
            if (lane == 0) {
                WL_TR(0, i);
                if (i == 0) WL_TRP(2);
                const int t0 = (tb + i) * IDX_TILE;
                mbar_expect_tx(full + s, L::K8_TILE);
                tma_load3d(k8 + s * L::K8_TILE, &sp.tm_keys, 0, t0, seq, full + s);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (whole warp loops, lane 0 issues) ----------------
        const uint32_t sQa = smem_u32(sQ);
        for (int i = 0; i < n; ++i) {
            const int s = i % IDX_NS, a = i % IDX_NACC;
            if (!mbar_wait(full + s, (uint32_t)(i / IDX_NS) & 1u, 11)) break;
            if (i >= IDX_NACC && !mbar_wait(acc_empty + a, (uint32_t)(i / IDX_NACC - 1) & 1u, 12)) break;
            tc_fence_after();
            if (lane == 0) {
                WL_TR(3, i);
                if (i == 0) WL_TRP(3);
                if (i == n - 1) WL_TRP(4);
                const uint32_t sA = smem_u32(k8 + s * L::K8_TILE);
                const uint32_t d = tmem + (uint32_t)(a * 64);
#pragma unroll
                for (int kk = 0; kk < IDX_D / 32; ++kk) {
                    // B = the 64 rows hi[0..31] ‖ lo[0..31], one swizzled block
                    mma_f8(d, desc_sw128(sA + kk * 32, 16, 1024), desc_sw128(sQa + kk * 32, 16, 1024), L::IDESC,
                           kk > 0 ? 1u : 0u);
                }
                mma_commit(acc_full + a);
                mma_commit(empty + s);  // keys consumed
                WL_TR(4, i);
            }
            __syncwarp();
        }
    } else {
        // ------- epilogue (warps 2..9 -> TMEM lane quarters 2,3,0,1; group g takes tiles i = g mod 2) -------
        const int quarter = warp & 3;
        const int key = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        auto load_scale = [&](int i) {
            const int t = (tb + i) * IDX_TILE + key;
            return (i < n && t < len) ? __ldg(scale + t) : 0.f;
        };
        // Scales by plain loads one tile of this group ahead (a TMA copy per
        // tile this small would cost the copy engine as much time as the 16 KB
        // key tile).
        float sc_next = load_scale((warp - 2) >> 2);
        for (int i = (warp - 2) >> 2; i < n; i += IDX_EPI_GROUPS) {
            const int a = i % IDX_NACC;
            const int t0 = (tb + i) * IDX_TILE;
            const float sc_raw = sc_next;
            sc_next = load_scale(i + IDX_EPI_GROUPS);
            if (!mbar_wait(acc_full + a, (uint32_t)(i / IDX_NACC) & 1u, 15)) break;
            if (key == 0) WL_TR(5, i);
            tc_fence_after();
            const float sc = sc_raw * p.qk_scale;
            float acc[64];  // [0, 32): hi terms, [32, 64): lo terms
            tmem_ld64(tmem + lane_base + (uint32_t)(a * 64), acc);
            tc_fence_before();
            mbar_arrive(acc_empty + a);
            float v = 0.f;
#pragma unroll
            for (int h = 0; h < 32; ++h) v = fmaf(sW[h], fmaxf(fmaf(acc[32 + h], 0.03125f, acc[h]) * sc, 0.f), v);
            const int t = t0 + key;
            const bool valid = t < len;
#ifndef WL_EXP_NOSTORE
            if (valid) out[t] = v;
#endif
            if (key == 0) WL_TR(6, i);
            if (key == 0 && i == n - 1) WL_TRP(5);
            if (hrow && valid) atomicAdd(&sHist[score_key(v) >> (32 - TOPK_HIST_BITS)], 1u);
        }
    }
    tc_fence_before();
    if (tid == 0) WL_TRP(6);
    __syncthreads();
    if (tid == 0) WL_TRP(7);
    if (hrow) {  // this CTA's counts into the row's histogram: nonzero bins only
        for (int b4 = tid; b4 < TOPK_HIST_BINS / 4; b4 += IDX_STREAM_THREADS) {
            const uint4 c = reinterpret_cast<const uint4*>(sHist)[b4];
            if (c.x) atomicAdd(hrow + 4 * b4, c.x);
            if (c.y) atomicAdd(hrow + 4 * b4 + 1, c.y);
            if (c.z) atomicAdd(hrow + 4 * b4 + 2, c.z);
            if (c.w) atomicAdd(hrow + 4 * b4 + 3, c.w);
        }
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
    WL_KT_END(0);
    WL_TRB(1);
    if (tid == 0) WL_TRP(8);
}

}  // namespace wl
