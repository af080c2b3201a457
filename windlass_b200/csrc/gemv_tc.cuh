// gemv_tc.cuh — the weight-streaming products around the attention substep on
// the tensor cores (tcgen05): the indexer's query projection and the MLA
// absorption before and after the attention.
//
//   GV_IDXQ  q_idx[r][o] = RoPE(sum_k wq_b[o][k] q_resid[r][k])         o < 4096, k < 2048
//            (launch_indexer_query's matvec + rope_interleave_slice,
//            src/glm_kernels.cuh:469-472, 137-160)
//   GV_PROJV out[r][h][v] = sum_c ctx[r][h][c] kv_b[h*448 + 192 + v][c]  v < 256, c < 512
//            (mla_project_v, src/glm_layer_runner.cuh:217-234)
//   GV_ABSQ  q_abs[r][h][c] = sum_d q[r][h][d] kv_b[h*448 + d][c]        c < 512, d < 192
//            (mla_absorb_q, src/glm_layer_runner.cuh:196-215), plus the
//            query's roped part copied to q_abs[r][h][512 ...]
//
// At a decode batch these read each bf16 weight once (29-46 MB) for a few
// query rows: HBM-bound. A CTA owns 128 output rows of the weight (the MMA's
// M) and pulls its whole weight slice into shared memory with TMA (128B
// swizzle; K-major tiles of wq_b and W_UV, M-major tiles of W_UK, whose output
// index is the contiguous one). The fp32 activations enter the MMA as bf16
// terms: x = hi + mid + lo, each the bf16 rounding of what the previous terms
// leave (24 significant bits in all), as three consecutive N columns per query
// row; bf16 x bf16 products are exact in the fp32 accumulator, and the
// epilogue adds a row's three columns. Query rows go through in chunks of
// GV_RC (N = 3 GV_RC) while the weight slice stays in shared memory.
// wq_b's K = 2048 is split over a 4-CTA cluster (512 each); the partial sums
// meet in distributed shared memory and are added in rank order.
#pragma once
#include "mla_attn64.cuh"

namespace wl {

// kv_b_proj per head: qk_nope 192 W_UK rows, then v_head 256 W_UV rows, 512 wide
constexpr int PJ_H = 64, PJ_NOPE = 192, PJ_ROPE = 64, PJ_QK = PJ_NOPE + PJ_ROPE, PJ_V = 256, PJ_L = 512;
constexpr int PJ_KVB_ROWS = PJ_NOPE + PJ_V;

enum { GV_IDXQ = 0, GV_PROJV = 1, GV_ABSQ = 2 };
constexpr int GV_M = 128;       // weight rows per CTA
constexpr int GV_RC = 16;       // query rows per chunk
constexpr int GV_N = 3 * GV_RC; // MMA N: three bf16 terms per row
constexpr int GV_THREADS = 128;
constexpr int GV_CL = 4;        // GV_IDXQ: CTAs per cluster along K

template <int MODE>
struct GvShape {
    static constexpr int K = MODE == GV_IDXQ ? 512 : MODE == GV_PROJV ? 512 : 192;  // per CTA
    static constexpr int KCH = K / 64;                                              // 64-wide K chunks
    static constexpr bool A_MN = MODE == GV_ABSQ;
    // A: K-major 128 x 64 boxes (16 KB each), or two M-major 64 (m) x 192 (k) boxes
    static constexpr uint32_t A_BYTES = GV_M * K * 2;
    static constexpr uint32_t A_CHUNK = A_MN ? 64 * K * 2 : GV_M * 128;
    static constexpr int A_LOADS = A_MN ? 2 : KCH;
    static constexpr uint32_t B_CHUNK = GV_N * 128;  // N rows x 64 bf16 of K
    static constexpr uint32_t OFF_A = 0;
    static constexpr uint32_t OFF_B = OFF_A + A_BYTES;
    static constexpr uint32_t OFF_PART = OFF_B + KCH * B_CHUNK;  // GV_IDXQ: [GV_RC][128] fp32
    static constexpr uint32_t OFF_BAR = OFF_PART + (MODE == GV_IDXQ ? GV_RC * GV_M * 4 : 0);
    static constexpr uint32_t BYTES = OFF_BAR + 8 * (A_LOADS + 1) + 16 + 1024;
    static constexpr uint32_t IDESC = idesc_bf16(GV_M, GV_N, A_MN ? 1 : 0, 0);
};
static_assert(GvShape<GV_IDXQ>::BYTES <= 232448 && GvShape<GV_PROJV>::BYTES <= 232448, "fits one SM");
static_assert((GvShape<GV_IDXQ>::B_CHUNK % 1024) == 0, "B chunks on swizzle-atom boundaries");

struct GvParams {
    CUtensorMap tm_w;   // the weight, box {64, 128} (K-major) or {64, 192} (M-major)
    int n;              // query rows
    const float* x;     // activations (row stride x_row floats)
    long long x_row;
    void* out;          // q_idx bf16 / out fp32 / q_abs bf16 (row stride out_row elements)
    long long out_row;
    const float* cos;   // GV_IDXQ: the rows' RoPE tables [n][32]
    const float* sin;
};

__device__ __forceinline__ void tmem_ld32x32b_x16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Three bf16 terms of 8 consecutive fp32 values: hi, mid, lo (x = hi + mid + lo
// to 24 significant bits), each packed as 8 bf16 in a uint4.
__device__ __forceinline__ void gv_split8(const float* x, uint4& hi, uint4& mid, uint4& lo) {
    uint32_t h[4], m[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float a = x[2 * e], b = x[2 * e + 1];
        const __nv_bfloat162 ha = __floats2bfloat162_rn(a, b);
        const float ra = a - __low2float(ha), rb = b - __high2float(ha);
        const __nv_bfloat162 ma = __floats2bfloat162_rn(ra, rb);
        const __nv_bfloat162 la = __floats2bfloat162_rn(ra - __low2float(ma), rb - __high2float(ma));
        h[e] = *reinterpret_cast<const uint32_t*>(&ha);
        m[e] = *reinterpret_cast<const uint32_t*>(&ma);
        l[e] = *reinterpret_cast<const uint32_t*>(&la);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    mid = make_uint4(m[0], m[1], m[2], m[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

// GV_IDXQ: grid (GV_CL, 32 output tiles), cluster (GV_CL): CTA k sums K range
//          [512 k, 512 k + 512) of output rows [128 y, 128 y + 128) (one head).
// GV_PROJV: grid (2, 64 heads): CTA x owns v in [128 x, 128 x + 128).
// GV_ABSQ: grid (4, 64 heads): CTA x owns c in [128 x, 128 x + 128).
template <int MODE>
__global__ void __launch_bounds__(GV_THREADS, 1) gemv_tc_kernel(const __grid_constant__ GvParams p) {
    using S = GvShape<MODE>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sA = smem_u32(smem + S::OFF_A), sB = smem_u32(smem + S::OFF_B);
    uint64_t* afull = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* mdone = afull + S::A_LOADS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t crank = MODE == GV_IDXQ ? cluster_ctarank() : 0u;
    const int h = blockIdx.y;
    if (tid == 0) {
        for (int i = 0; i < S::A_LOADS; ++i) mbar_init(afull + i, 1);
        mbar_init(mdone, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, 64);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) {
        // The CTA's whole weight slice, one TMA box per chunk, fetched before the
        // programmatic wait so that it streams while the previous kernel
        // finishes. No kernel of this library writes the weights, and a
        // caller's kernel that does precedes this one as an ordinary stream
        // predecessor (it signals no early launch), so it has finished first.
        for (int i = 0; i < S::A_LOADS; ++i) {
            mbar_expect_tx(afull + i, S::A_CHUNK);
            if (MODE == GV_IDXQ)
                tma_load2d(sA + i * S::A_CHUNK, &p.tm_w, (int)crank * S::K + 64 * i, h * GV_M, afull + i);
            else if (MODE == GV_PROJV)
                tma_load2d(sA + i * S::A_CHUNK, &p.tm_w, 64 * i, h * 448 + 192 + (int)blockIdx.x * GV_M, afull + i);
            else
                tma_load2d(sA + i * S::A_CHUNK, &p.tm_w, (int)blockIdx.x * GV_M + 64 * i, h * 448, afull + i);
        }
    }
    pdl_wait();  // the activations below may come from the previous kernel
    pdl_trigger();
    // activation row r, element k of this CTA's K range
    auto xrow = [&](int r) -> const float* {
        if (MODE == GV_IDXQ) return p.x + (long long)r * p.x_row + crank * S::K;
        if (MODE == GV_PROJV) return p.x + (long long)r * p.x_row + h * 512;
        return p.x + (long long)r * p.x_row + h * 256;
    };
    bool ok = true;
    int it = 0;
    for (int r0 = 0; r0 < p.n; r0 += GV_RC, ++it) {
        const int nr = min(GV_RC, p.n - r0);
        // ---- B: the chunk's rows as three bf16 terms, K-major, 128B-swizzled ----
        for (int i = tid; i < GV_RC * (S::K / 8); i += GV_THREADS) {
            const int r = i / (S::K / 8), k8 = i % (S::K / 8);
            float xv[8];
            if (r < nr) {
                const float4 a = *reinterpret_cast<const float4*>(xrow(r0 + r) + 8 * k8);
                const float4 b = *reinterpret_cast<const float4*>(xrow(r0 + r) + 8 * k8 + 4);
                xv[0] = a.x, xv[1] = a.y, xv[2] = a.z, xv[3] = a.w, xv[4] = b.x, xv[5] = b.y, xv[6] = b.z,
                xv[7] = b.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) xv[e] = 0.f;
            }
            uint4 t0, t1, t2;
            gv_split8(xv, t0, t1, t2);
            const uint32_t chunk = sB + (uint32_t)(k8 >> 3) * S::B_CHUNK;
            const uint32_t c16 = (uint32_t)(k8 & 7);
            sts_v4(chunk + sw128_off(3 * r, c16), t0);
            sts_v4(chunk + sw128_off(3 * r + 1, c16), t1);
            sts_v4(chunk + sw128_off(3 * r + 2, c16), t2);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // ---- MMA: D[128 x N] = A[128 x K] . B[N x K]^T ----
        if (tid == 0) {
            for (int c = 0; c < S::KCH && ok; ++c) {
                if (it == 0 && (!S::A_MN || c == 0)) {
                    if (S::A_MN) {
                        for (int j = 0; j < S::A_LOADS && ok; ++j) ok = mbar_wait_fast(afull + j, 0, 60);
                    } else {
                        ok = mbar_wait_fast(afull + c, 0, 60);
                    }
                    tc_fence_after();
                }
                if (!ok) break;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    uint64_t ad;
                    if (S::A_MN)  // two 64-row M blocks LBO apart; 16 K rows = 2048 bytes
                        ad = desc_sw128(sA + (uint32_t)(c * 4 + kk) * 2048u, S::A_CHUNK, 1024);
                    else
                        ad = desc_sw128(sA + (uint32_t)c * S::A_CHUNK + kk * 32, 16, 1024);
                    const uint64_t bd = desc_sw128(sB + (uint32_t)c * S::B_CHUNK + kk * 32, 16, 1024);
                    mma_bf16(tmem, ad, bd, S::IDESC, (c | kk) != 0 ? 1u : 0u);
                }
            }
            mma_commit(mdone);  // arrives also when nothing was issued
        }
        __syncwarp();
        ok = mbar_wait_fast(mdone, (uint32_t)it & 1u, 61) && ok;
        tc_fence_after();
        // ---- epilogue: thread = weight row m (TMEM lane), three columns per query row ----
        const int m = 32 * warp + lane;
        float acc[GV_N];
#pragma unroll
        for (int j = 0; j < GV_N / 16; ++j) tmem_ld32x32b_x16(tmem + ((uint32_t)(32 * warp) << 16) + 16 * j, acc + 16 * j);
        float y[GV_RC];
#pragma unroll
        for (int r = 0; r < GV_RC; ++r) y[r] = (acc[3 * r] + acc[3 * r + 1]) + acc[3 * r + 2];
        if (MODE == GV_PROJV) {
            float* out = static_cast<float*>(p.out);
#pragma unroll
            for (int r = 0; r < GV_RC; ++r)
                if (r < nr && ok) out[(long long)(r0 + r) * p.out_row + h * 256 + blockIdx.x * GV_M + m] = y[r];
        } else if (MODE == GV_ABSQ) {
            __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
            for (int r = 0; r < GV_RC; ++r)
                if (r < nr && ok)
                    out[(long long)(r0 + r) * p.out_row + h * 576 + blockIdx.x * GV_M + m] = __float2bfloat16_rn(y[r]);
            if (blockIdx.x == 0)  // the roped part rides along
                for (int i = tid; i < nr * 64; i += GV_THREADS) {
                    const int r = i >> 6, j = i & 63;
                    out[(long long)(r0 + r) * p.out_row + h * 576 + 512 + j] =
                        __float2bfloat16_rn(p.x[(long long)(r0 + r) * p.x_row + h * 256 + 192 + j]);
                }
        } else {
            // partial sums of this K quarter into shared memory, then CTA k of the
            // cluster adds the 4 quarters of rows [32 k, 32 k + 32) in rank order
            float* part = reinterpret_cast<float*>(smem + S::OFF_PART);
#pragma unroll
            for (int r = 0; r < GV_RC; ++r) part[r * GV_M + m] = y[r];
            cluster_sync_all();
            const int mm = 32 * (int)crank + lane;  // this thread's output row of the tile (one head: 128 dims)
            __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
            for (int rr = 0; rr < GV_RC / 4; ++rr) {
                const int r = warp * (GV_RC / 4) + rr;
                float s = 0.f;
#pragma unroll
                for (uint32_t k = 0; k < GV_CL; ++k) {
                    const uint32_t ra = dsmem_addr(part + r * GV_M + mm, k);
                    float v;
                    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
                    s += v;
                }
                const float other = __shfl_xor_sync(0xffffffffu, s, 1);  // RoPE partner (dims 2i, 2i + 1)
                if (r < nr && ok) {
                    __nv_bfloat16* qo = out + (long long)(r0 + r) * p.out_row + h * 128;
                    if (mm < 64) {
                        const int i = mm >> 1;
                        const float c = p.cos[(long long)(r0 + r) * 32 + i], sn = p.sin[(long long)(r0 + r) * 32 + i];
                        if ((mm & 1) == 0)
                            qo[i] = __float2bfloat16_rn(s * c - other * sn);
                        else
                            qo[32 + i] = __float2bfloat16_rn(s * c + other * sn);
                    } else {
                        qo[mm] = __float2bfloat16_rn(s);
                    }
                }
            }
            cluster_sync_all();  // remote reads done before part is rewritten or the CTA exits
        }
        tc_fence_before();
        __syncthreads();  // TMEM and B are rewritten by the next chunk
        tc_fence_after();
        // After a timed-out wait (recorded in the error word) the loop still runs
        // to the end without MMAs or stores, so that every CTA of a cluster
        // reaches the same cluster barriers.
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 64);
    }
}

}  // namespace wl
