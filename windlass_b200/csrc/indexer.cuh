// indexer.cuh — DSA lightning-indexer scoring on the tensor cores.
//
// Computes, for query row r and key t < len(r),
//     index[r][t] = sum_h w[r][h] * relu(qk_scale * scale[t] * (q[r][h] . e4m3(k[t])))
// which is the reference's indexer_scores_relu + indexer_combine
// (src/glm_kernels.cuh:308-340; numpy: tools/ref_glm_chain.py:482-501) with
// the key cache in fp8-e4m3 plus a per-key fp32 scale. The [H,T] score array
// the reference writes to global memory and reads back never leaves TMEM here.
//
// Layout of the work (one CTA = 4 warps = one 128-key tile):
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
    int scale_bulk;  // scale rows may be fetched by the TMA engine (16-byte aligned)
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

// ---- decode form: persistent, warp-specialised ------------------------------------------
// One CTA per SM streams a contiguous range of 128-key tiles of one row's
// cache. Roles (14 warps), connected by mbarriers only — no block-wide barrier
// in the tile loop, so each role runs at its own rate:
//   warp 0       TMA producer: fp8 keys + scales of tile i into ring stage i % IDX_NS
//   warp 1       MMA issuer:   tcgen05.mma (M = 128 keys, N = 32 heads, K = 128) into
//                              accumulator set i % IDX_NACC; the 8 K-steps go to
//                              IDX_KSPLIT independent accumulators so the tensor pipe
//                              overlaps them instead of chaining them on one
//   warps 2-9    converters:   e4m3 -> fp16 into A tile i % IDX_NA (128B-swizzled, K-major)
//   warps 10-13  epilogue:     sum the partial accumulators of one key, scale, relu,
//                              head-weighted sum, store (+ fused histogram)
//
// Operand types: tcgen05 kind::f16 with fp16 A and B. A key is widened to fp16
// holding e4m3 * 2^-8 by bit placement alone (exact for every finite code; the
// 2^8 goes into the per-key scale). The bf16 query is scaled per head by a power
// of two (its largest element lands in [2^14, 2^15)) and converted to fp16 —
// exact for every element the scale keeps in fp16's normal range, i.e. all but
// those below 2^-28 of the head's largest, whose contribution is far below fp32
// rounding of the dot product. The scale is undone in the head weight:
// w_h * relu(x / s_h) = (w_h / s_h) * relu(x) for s_h > 0, exact for a power of two.
//
// The epilogue can also accumulate, per row, the histogram of the top
// TOPK_HIST_BITS bits of the order-preserving score keys (warp-aggregated
// global atomics) — the first radix pass of the top-k, fused here so that no
// kernel re-reads the scores for it.
constexpr int IDX_NS = 4;      // TMA stages
constexpr int IDX_NA = 2;      // fp16 A tiles
constexpr int IDX_NACC = 4;    // accumulator sets in flight
constexpr int IDX_KSPLIT = 4;  // independent partial accumulators per tile
constexpr int IDX_STREAM_THREADS = 448;
constexpr int IDX_CONV = 256;  // converter threads
// Scale rows in flight between a converter writing tile i and the epilogue of
// tile i reading it: converters lead the MMA by at most IDX_NA tiles and the
// MMA leads the epilogue by at most IDX_NACC.
constexpr int IDX_NSC = IDX_NA + IDX_NACC + 1;
constexpr int TOPK_HIST_BITS = 13;
constexpr int TOPK_HIST_BINS = 1 << TOPK_HIST_BITS;

struct IdxStreamLayout {
    static constexpr uint32_t A_TILE = IDX_TILE * IDX_D * 2;   // 32 KB
    static constexpr uint32_t A_CHUNK = IDX_TILE * 128;
    static constexpr uint32_t Q_CHUNK = IDX_H * 128;           // 4 KB
    static constexpr uint32_t K8_TILE = IDX_TILE * IDX_D;      // 16 KB
    static constexpr uint32_t STAGE = K8_TILE + IDX_TILE * 4;  // + the tile's scales
    static constexpr uint32_t OFF_A = 0;
    static constexpr uint32_t OFF_Q = OFF_A + IDX_NA * A_TILE;
    static constexpr uint32_t OFF_K8 = OFF_Q + 2 * Q_CHUNK;
    static constexpr uint32_t OFF_W = OFF_K8 + IDX_NS * STAGE;
    static constexpr uint32_t OFF_SC = OFF_W + IDX_H * 4;  // [IDX_NSC][128] scale * qk_scale * 2^8
    static constexpr uint32_t OFF_BAR = OFF_SC + IDX_NSC * IDX_TILE * 4;
    static constexpr int N_BARS = 2 * IDX_NS + 2 * IDX_NA + 2 * IDX_NACC;
    static constexpr uint32_t OFF_SLOT = OFF_BAR + N_BARS * 8;
    static constexpr uint32_t BYTES = OFF_SLOT + 16 + 1024;
    static constexpr uint32_t TMEM_COLS = 32 * IDX_KSPLIT * IDX_NACC;  // 512
    static constexpr uint32_t IDESC = idesc_f16(128, IDX_H);
};

__device__ __forceinline__ uint32_t score_key(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u << 1) == 0u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Four e4m3 codes (one word) -> four fp16 (two words) holding e4m3 * 2^-8,
// exactly, by bit placement alone: the fp16 pattern (b & 0x80) << 8 |
// (b & 0x7F) << 7 puts e4m3's sign, 4 exponent and 3 mantissa bits into
// fp16's fields, which is the e4m3 value times 2^(7-15) for normal codes and,
// because 2^-8 also maps e4m3 subnormals (m * 2^-9) onto fp16 subnormals
// ((m << 7) * 2^-24), for every finite code. NaN codes are not valid keys.
__device__ __forceinline__ void e4m3x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t x01 = __byte_perm(w, 0u, 0x4140);  // [b0, 0, b1, 0]
    const uint32_t x23 = __byte_perm(w, 0u, 0x4342);  // [b2, 0, b3, 0]
    lo = ((x01 << 7) & 0x3F803F80u) | ((x01 << 8) & 0x80008000u);
    hi = ((x23 << 7) & 0x3F803F80u) | ((x23 << 8) & 0x80008000u);
}

#ifdef WL_TRACE
__device__ long long* g_trace;
#define WL_TR(slot, i)                                                                                  \
    do {                                                                                                \
        if (g_trace && blockIdx.x == 0 && blockIdx.y == 0 && (i) < 64) g_trace[(i) * 8 + (slot)] = clock64(); \
    } while (0)
#else
#define WL_TR(slot, i) \
    do {               \
    } while (0)
#endif

__global__ void __launch_bounds__(IDX_STREAM_THREADS, 1)
    indexer_stream_kernel(IdxParams p, unsigned* hist, int tiles_per_cta) {
    using L = IdxStreamLayout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sA = smem_u32(smem + L::OFF_A);
    const uint32_t sQ = smem_u32(smem + L::OFF_Q);
    uint8_t* k8 = smem + L::OFF_K8;
    float* sW = reinterpret_cast<float*>(smem + L::OFF_W);
    float* sc_s = reinterpret_cast<float*>(smem + L::OFF_SC);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* empty = full + IDX_NS;
    uint64_t* a_full = empty + IDX_NS;     // converters -> MMA       (per A tile)
    uint64_t* a_free = a_full + IDX_NA;    // MMA commit -> converters (per A tile)
    uint64_t* acc_full = a_free + IDX_NA;  // MMA commit -> epilogue   (per accumulator set)
    uint64_t* acc_empty = acc_full + IDX_NACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_SLOT);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = blockIdx.y;
    const int seq = r / p.rows_per_seq;
    const int len = rows_len(r, p.rows_per_seq, p.len0, p.len_step, p.T);
    const int ntiles = (len + IDX_TILE - 1) / IDX_TILE;
    const int tb = blockIdx.x * tiles_per_cta;
    const int n = min(tb + tiles_per_cta, ntiles) - tb;
    if (n <= 0) return;
    const uint8_t* keys = p.keys + (long long)seq * p.keys_seq;
    const float* scale = p.scale + (long long)seq * p.scale_seq;
    float* out = p.out + (long long)r * p.out_stride;
    unsigned* hrow = hist ? hist + (long long)r * TOPK_HIST_BINS : nullptr;

    if (tid == 0) {
        for (int s = 0; s < IDX_NS; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, IDX_CONV);
        }
        for (int b = 0; b < IDX_NA; ++b) {
            mbar_init(a_full + b, IDX_CONV);
            mbar_init(a_free + b, 1);
        }
        for (int b = 0; b < IDX_NACC; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 128);
        }
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);  // warp 1 allocates and frees
    // Query -> fp16 with a per-head power-of-two scale; 14 warps over 32 heads.
    for (int h = warp; h < IDX_H; h += IDX_STREAM_THREADS / 32) {
        const __nv_bfloat16* qh = p.q + ((long long)r * IDX_H + h) * IDX_D;
        float x[4];
        float mx = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            x[e] = __bfloat162float(qh[lane * 4 + e]);
            mx = fmaxf(mx, fabsf(x[e]));
        }
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        // 2^(14 - floor(log2 mx)): the largest element lands in [2^14, 2^15).
        const int ex = mx > 0.f ? max(((__float_as_int(mx) >> 23) & 0xff) - 127, -100) : 0;
        const float s_h = __int_as_float((127 + 14 - ex) << 23);
        const __half2 a = __floats2half2_rn(x[0] * s_h, x[1] * s_h), b = __floats2half2_rn(x[2] * s_h, x[3] * s_h);
        const uint32_t e0 = (uint32_t)lane * 4u, chunk = e0 >> 6, byte = (e0 & 63u) * 2u;
        const uint32_t addr = sQ + chunk * L::Q_CHUNK + (uint32_t)h * 128u + ((((byte >> 4) ^ (uint32_t)h) & 7u) << 4) +
                              (byte & 15u);
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(*reinterpret_cast<const uint32_t*>(&a)),
                     "r"(*reinterpret_cast<const uint32_t*>(&b))
                     : "memory");
        if (lane == 0) sW[h] = __ldg(p.w + (long long)r * IDX_H + h) / s_h;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool sc_bulk_all = p.scale_bulk != 0;

    if (warp == 0) {
        // ---------------- TMA producer (whole warp loops, lane 0 issues) ----------------
        for (int i = 0; i < n; ++i) {
            const int s = i % IDX_NS;
            if (i >= IDX_NS && !mbar_wait(empty + s, (uint32_t)(i / IDX_NS - 1) & 1u, 10)) break;
            if (lane == 0) {
                WL_TR(0, i);
                const int t0 = (tb + i) * IDX_TILE;
                const int nk = min(IDX_TILE, len - t0);
                const bool sc_bulk = sc_bulk_all && (nk & 3) == 0;
                mbar_expect_tx(full + s, (uint32_t)nk * IDX_D + (sc_bulk ? (uint32_t)nk * 4u : 0u));
                bulk_g2s(k8 + s * L::STAGE, keys + (long long)t0 * IDX_D, (uint32_t)nk * IDX_D, full + s);
                if (sc_bulk) bulk_g2s(k8 + s * L::STAGE + L::K8_TILE, scale + t0, (uint32_t)nk * 4u, full + s);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (whole warp loops, lane 0 issues) ----------------
        for (int i = 0; i < n; ++i) {
            const int b = i % IDX_NA, a = i % IDX_NACC;
            if (!mbar_wait(a_full + b, (uint32_t)(i / IDX_NA) & 1u, 11)) break;
            if (i >= IDX_NACC && !mbar_wait(acc_empty + a, (uint32_t)(i / IDX_NACC - 1) & 1u, 12)) break;
            tc_fence_after();
            if (lane == 0) {
                WL_TR(3, i);
                const uint32_t d0 = tmem + (uint32_t)(a * 32 * IDX_KSPLIT);
#pragma unroll
                for (int kk = 0; kk < IDX_D / 16; ++kk) {
                    const uint32_t c = kk >> 2, ko = (kk & 3) * 32;
                    const uint64_t ad = desc_sw128(sA + (uint32_t)b * L::A_TILE + c * L::A_CHUNK + ko, 16, 1024);
                    const uint64_t bd = desc_sw128(sQ + c * L::Q_CHUNK + ko, 16, 1024);
                    const int part = kk % IDX_KSPLIT;
                    mma_bf16(d0 + (uint32_t)(part * 32), ad, bd, L::IDESC, kk >= IDX_KSPLIT ? 1u : 0u);
                }
                mma_commit(a_free + b);
                mma_commit(acc_full + a);
                WL_TR(4, i);
            }
            __syncwarp();
        }
    } else if (warp < 10) {
        // ---------------- converters ----------------
        const int ct = tid - 64;  // 0..255
        const int piece = ct & 7, rbase = ct >> 3;  // 8 threads per 128-byte key row, 32 rows per pass
        for (int i = 0; i < n; ++i) {
            const int s = i % IDX_NS, b = i % IDX_NA;
            const int t0 = (tb + i) * IDX_TILE;
            const int nk = min(IDX_TILE, len - t0);
            if (!mbar_wait(full + s, (uint32_t)(i / IDX_NS) & 1u, 13)) break;
            if (i >= IDX_NA && !mbar_wait(a_free + b, (uint32_t)(i / IDX_NA - 1) & 1u, 14)) break;
            if (ct == 0) WL_TR(1, i);
            if (ct < IDX_TILE) {
                float sv = 0.f;
                if (ct < nk)
                    sv = (sc_bulk_all && (nk & 3) == 0)
                             ? reinterpret_cast<const float*>(k8 + s * L::STAGE + L::K8_TILE)[ct]
                             : __ldg(scale + t0 + ct);
                sc_s[(i % IDX_NSC) * IDX_TILE + ct] = sv * p.qk_scale * 256.f;  // undo the 2^-8 of the keys
            }
            const uint4* src = reinterpret_cast<const uint4*>(k8 + s * L::STAGE) + piece;
            uint4 v[4];
#pragma unroll
            for (int ps = 0; ps < 4; ++ps) v[ps] = src[(ps * 32 + rbase) * 8];  // all loads first
            uint8_t* dA = smem + L::OFF_A + b * L::A_TILE;
            const uint32_t chunk = (uint32_t)piece >> 2, c16 = ((uint32_t)piece & 3u) * 2u;
            const bool sw = piece >= 4;  // pieces 4..7 store hi first: 8 distinct bank groups per row
#pragma unroll
            for (int ps = 0; ps < 4; ++ps) {
                const int row = ps * 32 + rbase;
                uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
                if (row < nk) {
                    e4m3x4_to_f16x4(v[ps].x, lo.x, lo.y);
                    e4m3x4_to_f16x4(v[ps].y, lo.z, lo.w);
                    e4m3x4_to_f16x4(v[ps].z, hi.x, hi.y);
                    e4m3x4_to_f16x4(v[ps].w, hi.z, hi.w);
                }
                uint8_t* base = dA + chunk * L::A_CHUNK;
                *reinterpret_cast<uint4*>(base + sw128_off(row, c16 + (sw ? 1u : 0u))) = sw ? hi : lo;
                *reinterpret_cast<uint4*>(base + sw128_off(row, c16 + (sw ? 0u : 1u))) = sw ? lo : hi;
            }
            mbar_arrive(empty + s);  // stage read (its loads were consumed above)
            fence_proxy_async_smem();
            mbar_arrive(a_full + b);
            if (ct == 0) WL_TR(2, i);
        }
    } else {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3;  // warps 10..13 cover TMEM lane quarters 2,3,0,1
        const int key = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        for (int i = 0; i < n; ++i) {
            const int a = i % IDX_NACC;
            if (!mbar_wait(acc_full + a, (uint32_t)(i / IDX_NACC) & 1u, 15)) break;
            if (key == 0) WL_TR(5, i);
            tc_fence_after();
            const float sc = sc_s[(i % IDX_NSC) * IDX_TILE + key];  // read before releasing the set
            float acc[32], part[32];
            const uint32_t d0 = tmem + lane_base + (uint32_t)(a * 32 * IDX_KSPLIT);
            tmem_ld32(d0, acc);
#pragma unroll
            for (int k = 1; k < IDX_KSPLIT; ++k) {
                tmem_ld32(d0 + (uint32_t)(k * 32), part);
#pragma unroll
                for (int h = 0; h < 32; ++h) acc[h] += part[h];
            }
            tc_fence_before();
            mbar_arrive(acc_empty + a);
            float v = 0.f;
#pragma unroll
            for (int h = 0; h < 32; ++h) v = fmaf(sW[h], fmaxf(acc[h] * sc, 0.f), v);
            const int t = (tb + i) * IDX_TILE + key;
            const bool valid = t < len;
            if (valid) out[t] = v;
            if (key == 0) WL_TR(6, i);
            if (hrow) {
                const uint32_t bb = valid ? score_key(v) >> (32 - TOPK_HIST_BITS) : 0xFFFFFFFFu;
                const unsigned peers = __match_any_sync(0xffffffffu, bb);
                if (valid && lane == __ffs(peers) - 1) atomicAdd(hrow + bb, (unsigned)__popc(peers));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

}  // namespace wl
