// mla_proj.cuh — the MLA absorption around the attention: the query's no-RoPE
// part through W_UK (into the absorbed query the attention reads) and the
// attention output through W_UV.
//
// Reference (src/glm_layer_runner.cuh):
//   mla_absorb_q  :196-215  q_abs[h][c] = sum_{d < 192} q[h][d] * kv_b[h*448 + d][c]
//   mla_project_v :217-234  out[h][v]   = sum_{c < 512} ctx[h][c] * kv_b[h*448 + 192 + v][c]
// with kv_b = kv_b_proj [64 * (192 + 256), 512] bf16 (qk_nope 192, v_head 256)
// and fp32 queries / context. absorb_q also appends the query's roped part,
// giving the attention's input row [absorbed 512 | q_rot 64] in bf16.
//
// At decode these are matrix-vector products over 29 MB of bf16 weights (12.6
// MB of W_UK, 16.8 MB of W_UV): HBM-bound. Each CTA pulls its weight slice —
// contiguous rows of kv_b — into shared memory with one bulk copy (the TMA
// engine, no per-thread loads), keeps it there, and streams the query rows
// through in chunks of PJ_ROWS; fp32 accumulation; every sum that spans
// threads or CTAs runs in a fixed order, so results do not depend on
// scheduling.
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int PJ_H = 64, PJ_NOPE = 192, PJ_ROPE = 64, PJ_QK = PJ_NOPE + PJ_ROPE, PJ_V = 256, PJ_L = 512;
constexpr int PJ_KVB_ROWS = PJ_NOPE + PJ_V;  // kv_b rows per head
constexpr int PJ_ROWS = 8;                   // query rows per chunk
constexpr int PJ_THREADS = 256;

// ---- absorb_q: a cluster of AQ_SPLIT CTAs per head, each over 48 of the 192 d ----
constexpr int AQ_SPLIT = 4, AQ_D = PJ_NOPE / AQ_SPLIT;
struct AqLayout {
    static constexpr uint32_t OFF_W = 0;                                  // [48][512] bf16
    static constexpr uint32_t OFF_PART = OFF_W + AQ_D * PJ_L * 2;         // [8][512] fp32 partial sums
    static constexpr uint32_t OFF_Q = OFF_PART + PJ_ROWS * PJ_L * 4;      // [8][48] fp32
    static constexpr uint32_t OFF_BAR = OFF_Q + PJ_ROWS * AQ_D * 4;
    static constexpr uint32_t BYTES = OFF_BAR + 16;
};

// grid (AQ_SPLIT, 64 heads), cluster (AQ_SPLIT): CTA k of head h holds W_UK rows
// [48 k, 48 k + 48). Thread t owns columns [8 (t % 64), + 8) and chunk rows
// 2 (t / 64), + 1, summing its CTA's 48 d (one 16-byte weight load and one
// 8-byte query load per 16 FMAs); then CTA k adds the AQ_SPLIT partials of
// columns [128 k, 128 k + 128) over distributed shared memory in rank order.
__global__ void __cluster_dims__(AQ_SPLIT, 1, 1) __launch_bounds__(PJ_THREADS, 2)
    mla_absorb_q_kernel(int n, const float* __restrict__ q, long long q_row, const __nv_bfloat16* __restrict__ kvb,
                        __nv_bfloat16* __restrict__ q_abs, long long o_row) {
    using L = AqLayout;
    extern __shared__ __align__(128) uint8_t smem[];
    const __nv_bfloat16* ws = reinterpret_cast<const __nv_bfloat16*>(smem + L::OFF_W);
    float* part = reinterpret_cast<float*>(smem + L::OFF_PART);
    float* qs = reinterpret_cast<float*>(smem + L::OFF_Q);  // [48 d][8 rows]
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    const int h = blockIdx.y, tid = threadIdx.x;
    const int cg = tid & 63, rg = tid >> 6;
    const uint32_t rank = cluster_ctarank();
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    if (tid == 0) {
        mbar_expect_tx(bar, AQ_D * PJ_L * 2);
        bulk_g2s(smem + L::OFF_W, kvb + ((long long)h * PJ_KVB_ROWS + rank * AQ_D) * PJ_L, AQ_D * PJ_L * 2, bar);
    }
    for (int r0 = 0; r0 < n; r0 += PJ_ROWS) {
        const int nr = min(PJ_ROWS, n - r0);
        for (int i = tid; i < PJ_ROWS * AQ_D; i += PJ_THREADS) {
            const int r = i / AQ_D, d = i % AQ_D;
            qs[d * PJ_ROWS + r] = r < nr ? q[(long long)(r0 + r) * q_row + h * PJ_QK + rank * AQ_D + d] : 0.f;
        }
        __syncthreads();
        if (r0 == 0) mbar_wait_fast(bar, 0, 41);  // bounded; a timeout is recorded and the sums run on
        float acc[2][8];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[r][c] = 0.f;
#pragma unroll 4
        for (int d = 0; d < AQ_D; ++d) {
            const uint4 wq = *reinterpret_cast<const uint4*>(ws + d * PJ_L + 8 * cg);
            const float2 x = *reinterpret_cast<const float2*>(qs + d * PJ_ROWS + 2 * rg);
            const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wq);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(w2[e]);
                acc[0][2 * e] = fmaf(x.x, f.x, acc[0][2 * e]);
                acc[0][2 * e + 1] = fmaf(x.x, f.y, acc[0][2 * e + 1]);
                acc[1][2 * e] = fmaf(x.y, f.x, acc[1][2 * e]);
                acc[1][2 * e + 1] = fmaf(x.y, f.y, acc[1][2 * e + 1]);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float4* pr = reinterpret_cast<float4*>(part + (2 * rg + r) * PJ_L + 8 * cg);
            pr[0] = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
            pr[1] = make_float4(acc[r][4], acc[r][5], acc[r][6], acc[r][7]);
        }
        cluster_sync_all();  // every CTA's partials visible to the cluster
        {
            const int r = tid >> 5, c = (int)rank * 128 + 4 * (tid & 31);
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (uint32_t k = 0; k < AQ_SPLIT; ++k) {
                const float4 v = dsmem_ld_f32x4(dsmem_addr(part + r * PJ_L + c, k));
                s.x += v.x;
                s.y += v.y;
                s.z += v.z;
                s.w += v.w;
            }
            if (r < nr) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(s.x, s.y), hi = __floats2bfloat162_rn(s.z, s.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&lo);
                u.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(q_abs + (long long)(r0 + r) * o_row + h * (PJ_L + PJ_ROPE) + c) = u;
            }
        }
        if (rank == 0)  // the roped part rides along
            for (int i = tid; i < nr * PJ_ROPE; i += PJ_THREADS) {
                const int r = i / PJ_ROPE, j = i % PJ_ROPE;
                q_abs[(long long)(r0 + r) * o_row + h * (PJ_L + PJ_ROPE) + PJ_L + j] =
                    __float2bfloat16_rn(q[(long long)(r0 + r) * q_row + h * PJ_QK + PJ_NOPE + j]);
            }
        cluster_sync_all();  // remote reads done before partials are rewritten or the CTA exits
    }
}

// ---- project_v: PV_SPLIT CTAs per head, each over 64 of the 256 v ----
constexpr int PV_SPLIT = 4, PV_V = PJ_V / PV_SPLIT;
struct PvLayout {
    static constexpr uint32_t OFF_W = 0;                              // [64][512] bf16
    static constexpr uint32_t OFF_C = OFF_W + PV_V * PJ_L * 2;        // [8][512] fp32
    static constexpr uint32_t OFF_BAR = OFF_C + PJ_ROWS * PJ_L * 4;
    static constexpr uint32_t BYTES = OFF_BAR + 16;
};

// grid (PV_SPLIT, 64 heads). Warp w computes v = 64 k + 8 w .. + 7: lane l dots
// columns [8 l, 8 l + 8) and [256 + 8 l, 256 + 8 l + 8) of those 8 weight rows
// with each context row; the 8 lane-partials are
// then summed across the warp by a fixed butterfly that halves the values
// each lane carries at every step (9 shuffles for 8 outputs).
__global__ void __launch_bounds__(PJ_THREADS, 2) mla_project_v_kernel(int n, const float* __restrict__ ctx,
                                                                      long long c_row,
                                                                      const __nv_bfloat16* __restrict__ kvb,
                                                                      float* __restrict__ out, long long o_row) {
    using L = PvLayout;
    extern __shared__ __align__(128) uint8_t smem[];
    const __nv_bfloat16* ws = reinterpret_cast<const __nv_bfloat16*>(smem + L::OFF_W);
    float* cs = reinterpret_cast<float*>(smem + L::OFF_C);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    const int h = blockIdx.y, k = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    if (tid == 0) {
        mbar_expect_tx(bar, PV_V * PJ_L * 2);
        bulk_g2s(smem + L::OFF_W, kvb + ((long long)h * PJ_KVB_ROWS + PJ_NOPE + k * PV_V) * PJ_L, PV_V * PJ_L * 2,
                 bar);
    }
    // the output this lane ends up holding: v index within the warp's 8
    const int vi = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
    for (int r0 = 0; r0 < n; r0 += PJ_ROWS) {
        const int nr = min(PJ_ROWS, n - r0);
        for (int i = tid; i < PJ_ROWS * PJ_L / 4; i += PJ_THREADS) {
            const int r = i / (PJ_L / 4), c4 = i % (PJ_L / 4);
            reinterpret_cast<float4*>(cs)[i] =
                r < nr ? *reinterpret_cast<const float4*>(ctx + (long long)(r0 + r) * c_row + h * PJ_L + 4 * c4)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
        if (r0 == 0) mbar_wait_fast(bar, 0, 42);  // bounded; a timeout is recorded
        for (int r = 0; r < nr; ++r) {
            float s[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) s[j] = 0.f;
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                const float4 a = *reinterpret_cast<const float4*>(cs + r * PJ_L + 256 * half + 8 * lane);
                const float4 b = *reinterpret_cast<const float4*>(cs + r * PJ_L + 256 * half + 8 * lane + 4);
                const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 wq = *reinterpret_cast<const uint4*>(ws + (warp * 8 + j) * PJ_L + 256 * half + 8 * lane);
                    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&wq);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __bfloat1622float2(p[e]);
                        s[j] = fmaf(x[2 * e], f.x, s[j]);
                        s[j] = fmaf(x[2 * e + 1], f.y, s[j]);
                    }
                }
            }
            // butterfly: keep half, send half, at lane distances 16, 8, 4; then 2, 1
            const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
            float t[4], u[2];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float keep = b16 ? s[4 + j] : s[j], send = b16 ? s[j] : s[4 + j];
                t[j] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float keep = b8 ? t[2 + j] : t[j], send = b8 ? t[j] : t[2 + j];
                u[j] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
            }
            float v;
            {
                const float keep = b4 ? u[1] : u[0], send = b4 ? u[0] : u[1];
                v = keep + __shfl_xor_sync(0xffffffffu, send, 4);
            }
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            if ((lane & 3) == 0) out[(long long)(r0 + r) * o_row + h * PJ_V + k * PV_V + warp * 8 + vi] = v;
        }
        __syncthreads();  // cs is rewritten by the next chunk
    }
}

}  // namespace wl
