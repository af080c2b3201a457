// indexer.cuh — DSA lightning-indexer scoring on the tensor cores.
//
// Computes, for query row r and key t < len(r),
//     index[r][t] = sum_h w[r][h] * relu(qk_scale * scale[t] * (q[r][h] . e4m3(k[t])))
// which is the reference's indexer_scores_relu + indexer_combine
// (src/glm_kernels.cuh:308-340; numpy: tools/ref_glm_chain.py:482-501) with
// the key cache in fp8-e4m3 plus a per-key fp32 scale. The [H,T] score array
// the reference writes to global memory and reads back never leaves TMEM here.
//
// One kernel, indexer_stream_kernel<R>: R query rows share each 128-key tile
// (R = 1 at decode, where every row streams its own cache; R = 4 at prefill,
// where consecutive rows of one sequence read the same keys). The fp8 keys go
// to the tensor cores as they are (kind::f8f6f4); details below.
// Bytes per key: 128 (fp8) + 4 (scale); the decode form is HBM-bound.
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
};

__device__ __forceinline__ int rows_len(int r, int rows_per_seq, int len0, int len_step, int T) {
    const long long l = (long long)len0 + (long long)(r % rows_per_seq) * len_step;
    return (int)(l < T ? l : T);
}

// ---- warp-specialised, fp8 tensor cores ------------------------------------------------
// A CTA streams a contiguous range of 128-key tiles of one cache for R query
// rows (decode: one row, one CTA per SM across all rows; prefill: groups of 4
// consecutive rows, one CTA per group). Roles (18 warps at decode, 10 at
// prefill), connected by mbarriers only:
//   warp 0      TMA producer: the rows' bf16 queries (bulk copy during setup),
//               then each tile's fp8 keys as one 128 x 128-byte box with 128B
//               swizzle (a tensor-map load; rows past the cache end read as
//               zero) into ring stage i % IDX_NS (128 KB of keys in flight)
//   warp 1      MMA issuer:   tcgen05.mma kind::f8f6f4 straight on the fp8 keys
//               (M = 128 keys, K = 32 per instruction), one chain of 4 per
//               tile: N = 64 R = each row's hi and lo e4m3 query terms
//   warps 2..   epilogue:     tcgen05.ld both halves for one (key, row), combine,
//               scale, relu, head-weighted sum, store (+ fused top-k histogram
//               at decode); groups of 4 warps (four groups at decode, two at
//               prefill) take the tiles in turn
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
constexpr int TOPK_HIST_BITS = 13;
constexpr int TOPK_HIST_BINS = 1 << TOPK_HIST_BITS;

// R query rows per MMA (N = 64 R: each row's hi ‖ lo terms): R = 1 at decode
// (each row streams its own cache), R = 4 at prefill (4 consecutive rows of one
// sequence share every key tile).
template <int R>
struct IdxStream {
    static_assert(R == 1 || R == 2 || R == 4, "N = 64 R <= 256");
    static constexpr int NACC = R == 1 ? 4 : 2;            // accumulator sets in flight
    static constexpr int EPI_GROUPS = R == 1 ? 4 : 2;      // epilogue groups of 4 warps, alternating tiles
    // Each accumulator set must always be drained by the same group (tiles a,
    // a + NACC, ...), or a group could wait on a set's next phase while its
    // current one is still open (a parity wait two phases ahead passes at once).
    static_assert(NACC % EPI_GROUPS == 0, "epilogue groups must divide the accumulator sets");
    static constexpr int THREADS = 64 + 128 * EPI_GROUPS;  // producer + MMA warps + epilogue
    static constexpr bool HIST = R == 1;                   // fused top-k histogram (decode)
    static constexpr uint32_t K8_TILE = IDX_TILE * IDX_D;  // 16 KB, 128B-swizzled (1024-aligned)
    static constexpr uint32_t QROWS = 64 * R;              // B operand rows: per query row hi[32] ‖ lo[32]
    static constexpr uint32_t OFF_K8 = 0;
    static constexpr uint32_t OFF_Q = OFF_K8 + IDX_NS * K8_TILE;
    static constexpr uint32_t OFF_W = OFF_Q + QROWS * 128;
    static constexpr uint32_t OFF_HIST = OFF_W + R * IDX_H * 4;  // this CTA's share of the row histogram
    static constexpr uint32_t OFF_QRAW = OFF_HIST + (HIST ? TOPK_HIST_BINS * 4 : 0);  // bf16 queries, as copied
    static constexpr uint32_t OFF_BAR = OFF_QRAW + R * IDX_H * IDX_D * 2;
    static constexpr int N_BARS = 2 * IDX_NS + 2 * NACC + 1;  // full, empty, acc_full, acc_empty, query
    static constexpr uint32_t OFF_SLOT = OFF_BAR + N_BARS * 8;
    static constexpr uint32_t BYTES = OFF_SLOT + 16 + 1024;
    static constexpr uint32_t TMEM_COLS = QROWS * NACC;  // 256 or 512
    // kind::f8f6f4: E4M3 A and B (format 0), fp32 D; M = 128, N = 64 R
    static constexpr uint32_t IDESC = (1u << 4) | ((QROWS >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
};

static_assert(IdxStream<1>::BYTES <= 232448 && IdxStream<4>::BYTES <= 232448, "one CTA per SM");

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


// grid (CTAs per group, row groups): a CTA takes R consecutive rows (one key
// cache) and a contiguous range of `tiles_per_cta` tiles of their keys.
template <int R>
__global__ void __launch_bounds__(IdxStream<R>::THREADS, IDX_CTAS_PER_SM)
    indexer_stream_kernel(IdxParams p, const __grid_constant__ IdxStreamParams sp, unsigned* hist, int tiles_per_cta) {
    using L = IdxStream<R>;
    constexpr int NT = L::THREADS, NACC = L::NACC;
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
    uint64_t* acc_empty = acc_full + NACC;
    uint64_t* qbar = acc_empty + NACC;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_SLOT);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r0 = blockIdx.y * R;                      // first row of the group
    const int nrows = min(R, p.n_rows - r0);            // rows of the group that exist
    const int seq = r0 / p.rows_per_seq;                // all R rows read this cache
    int len_max = 0;
    for (int j = 0; j < nrows; ++j) len_max = max(len_max, rows_len(r0 + j, p.rows_per_seq, p.len0, p.len_step, p.T));
    const int ntiles = (len_max + IDX_TILE - 1) / IDX_TILE;
    const int tb = blockIdx.x * tiles_per_cta;
    const int n = min(tb + tiles_per_cta, ntiles) - tb;
    if (n <= 0 || nrows <= 0) {
        pdl_wait();
        return;
    }
    const float* scale = p.scale + (long long)seq * p.scale_seq;
    unsigned* hrow = (L::HIST && hist) ? hist + (long long)r0 * TOPK_HIST_BINS : nullptr;

    if (tid == 0) {
        for (int s = 0; s < IDX_NS; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);  // the MMA's commit
        }
        for (int b = 0; b < NACC; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_empty + b, 128);
        }
        mbar_init(qbar, 1);
        fence_mbar_init();
        // The producer (this thread) copies the group's queries (8 KB a row) at
        // once, so that they land during the setup below, ahead of the key
        // stream; every other warp converts them from shared memory. (Loading
        // them with per-warp global loads queued behind the key stream, and
        // issuing the first key tiles together with them let those overtake
        // them: both delayed the first MMA by microseconds.)
        pdl_wait();
        mbar_expect_tx(qbar, (uint32_t)nrows * IDX_H * IDX_D * 2);
        bulk_g2s(smem + L::OFF_QRAW, p.q + (long long)r0 * IDX_H * IDX_D, (uint32_t)nrows * IDX_H * IDX_D * 2, qbar);
    }
    if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);  // warp 1 allocates and frees
    if (hrow)
        for (int b = tid; b < TOPK_HIST_BINS; b += NT) sHist[b] = 0;
    tc_fence_before();
    __syncthreads();  // barriers initialised, TMEM address published
    tc_fence_after();
    pdl_wait();  // everything above overlaps the previous kernel; global data below
    pdl_trigger();
    const uint32_t tmem = *tmem_slot;
    const bool producer = warp == 0;
    // Queries -> two e4m3 terms per (row, head), by every warp but the
    // producer; a named barrier joins them. B row (j, term, h) = j*64 + term*32 + h.
    constexpr int CONV_WARPS = NT / 32 - 1;
    constexpr int PER_WARP = (R * IDX_H + CONV_WARPS - 1) / CONV_WARPS;
    float wv[PER_WARP];  // head weights, loaded while the queries land
    if (!producer) {
#pragma unroll
        for (int k2 = 0; k2 < PER_WARP; ++k2) {
            const int hr = warp - 1 + k2 * CONV_WARPS;  // (row j, head h) = (hr / 32, hr % 32)
            wv[k2] = (lane == 0 && hr < nrows * IDX_H) ? __ldg(p.w + (long long)r0 * IDX_H + hr) : 0.f;
        }
        mbar_wait(qbar, 0, 9);
    }
#pragma unroll
    for (int k2 = 0; k2 < PER_WARP; ++k2) {
        const int hr = warp - 1 + k2 * CONV_WARPS;
        if (producer || hr >= R * IDX_H) break;
        const int j = hr / IDX_H, h = hr % IDX_H;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        if (j < nrows) {
            const uint2 raw = *reinterpret_cast<const uint2*>(sQraw + hr * IDX_D + lane * 4);
            const __nv_bfloat162 q01 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
            const __nv_bfloat162 q23 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
            x[0] = __low2float(q01);
            x[1] = __high2float(q01);
            x[2] = __low2float(q23);
            x[3] = __high2float(q23);
        }
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
            const __half2_raw hr2 = __nv_cvt_fp8x2_to_halfraw2(h2, __NV_E4M3);
            const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hr2));
            const __nv_fp8x2_storage_t l2 =
                __nv_cvt_float2_to_fp8x2(make_float2((a0 - hf.x) * 32.f, (a1 - hf.y) * 32.f), __NV_SATFINITE, __NV_E4M3);
            hi4 |= (uint32_t)h2 << (8 * e);
            lo4 |= (uint32_t)l2 << (8 * e);
        }
        // 4 codes = 4 bytes at byte lane*4 of a 128-byte B row, 128B-swizzled
        const uint32_t byte = (uint32_t)lane * 4u;
        const uint32_t rh = (uint32_t)(j * 64 + h), rl = rh + 32;
        *reinterpret_cast<uint32_t*>(sQ + rh * 128u + ((((byte >> 4) ^ rh) & 7u) << 4) + (byte & 15u)) = hi4;
        *reinterpret_cast<uint32_t*>(sQ + rl * 128u + ((((byte >> 4) ^ rl) & 7u) << 4) + (byte & 15u)) = lo4;
        if (lane == 0) sW[hr] = j < nrows ? wv[k2] / s_h : 0.f;
    }
    if (!producer) {
        fence_proxy_async_smem();  // the query tiles are read by the tensor cores
        asm volatile("bar.sync 1, %0;" ::"n"(NT - 32) : "memory");
    }

    if (producer) {
        // ---------------- TMA producer (whole warp loops, lane 0 issues) ----------------
        for (int i = 0; i < n; ++i) {
            const int s = i % IDX_NS;
            if (i >= IDX_NS && !mbar_wait(empty + s, (uint32_t)(i / IDX_NS - 1) & 1u, 10)) break;
            if (lane == 0) {
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
            const int s = i % IDX_NS, a = i % NACC;
            if (!mbar_wait(full + s, (uint32_t)(i / IDX_NS) & 1u, 11)) break;
            if (i >= NACC && !mbar_wait(acc_empty + a, (uint32_t)(i / NACC - 1) & 1u, 12)) break;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t sA = smem_u32(k8 + s * L::K8_TILE);
                const uint32_t d = tmem + (uint32_t)(a * L::QROWS);
#pragma unroll
                for (int kk = 0; kk < IDX_D / 32; ++kk) {
                    // B = the 64 R query rows, one swizzled block
                    mma_f8(d, desc_sw128(sA + kk * 32, 16, 1024), desc_sw128(sQa + kk * 32, 16, 1024), L::IDESC,
                           kk > 0 ? 1u : 0u);
                }
                mma_commit(acc_full + a);
                mma_commit(empty + s);  // keys consumed
            }
            __syncwarp();
        }
    } else {
        // ------- epilogue (warps 2.. -> TMEM lane quarters by warp % 4; group g takes tiles i = g mod EPI_GROUPS) -------
        const int quarter = warp & 3;
        const int key = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        auto load_scale = [&](int i) {
            const int t = (tb + i) * IDX_TILE + key;
            return (i < n && t < len_max) ? __ldg(scale + t) : 0.f;
        };
        // Scales by plain loads one tile of this group ahead (a TMA copy per
        // tile this small would cost the copy engine as much time as the 16 KB
        // key tile).
        const int g0 = (warp - 2) >> 2;
        float sc_next = load_scale(g0);
        for (int i = g0; i < n; i += L::EPI_GROUPS) {
            const int a = i % NACC;
            const int t = (tb + i) * IDX_TILE + key;
            const float sc_raw = sc_next;
            sc_next = load_scale(i + L::EPI_GROUPS);
            if (!mbar_wait(acc_full + a, (uint32_t)(i / NACC) & 1u, 15)) break;
            tc_fence_after();
            const float sc = sc_raw * p.qk_scale;
#pragma unroll 1
            for (int j = 0; j < nrows; ++j) {
                float acc[64];  // [0, 32): hi terms, [32, 64): lo terms
                tmem_ld64(tmem + lane_base + (uint32_t)(a * L::QROWS + j * 64), acc);
                float v = 0.f;
#pragma unroll
                for (int h = 0; h < 32; ++h)
                    v = fmaf(sW[j * IDX_H + h], fmaxf(fmaf(acc[32 + h], 0.03125f, acc[h]) * sc, 0.f), v);
                const int r = r0 + j;
                const bool valid = t < rows_len(r, p.rows_per_seq, p.len0, p.len_step, p.T);
                if (valid) p.out[(long long)r * p.out_stride + t] = v;
                if constexpr (L::HIST)
                    if (hrow && valid) atomicAdd(&sHist[score_key(v) >> (32 - TOPK_HIST_BITS)], 1u);
            }
            tc_fence_before();
            mbar_arrive(acc_empty + a);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (hrow) {  // this CTA's counts into the row's histogram: nonzero bins only
        for (int b4 = tid; b4 < TOPK_HIST_BINS / 4; b4 += NT) {
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
}

}  // namespace wl
