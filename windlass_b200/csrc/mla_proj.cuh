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
// MB for W_UK, 16.8 MB for W_UV): HBM-bound, so each CTA streams its weight
// tile once, coalesced, and applies it to a chunk of up to PJ_ROWS query rows
// held in shared memory; fp32 accumulation; every cross-warp sum in a fixed
// order (the results do not depend on scheduling).
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int PJ_H = 64, PJ_NOPE = 192, PJ_ROPE = 64, PJ_QK = PJ_NOPE + PJ_ROPE, PJ_V = 256, PJ_L = 512;
constexpr int PJ_KVB_ROWS = PJ_NOPE + PJ_V;  // kv_b rows per head
constexpr int PJ_ROWS = 8;                   // query rows per chunk
constexpr int PJ_THREADS = 256;

// grid (512 / 64 column blocks, 64 heads). Warp w sums d in [24 w, 24 w + 24)
// for the block's 64 columns (two per lane, one 128-byte weight row segment
// per d); the 8 warps' partials are added in warp order.
__global__ void __launch_bounds__(PJ_THREADS) mla_absorb_q_kernel(int n, const float* __restrict__ q,
                                                                  long long q_row, const __nv_bfloat16* __restrict__ kvb,
                                                                  __nv_bfloat16* __restrict__ q_abs, long long o_row) {
    pdl_wait();
    pdl_trigger();
    __shared__ float qs[PJ_ROWS][PJ_NOPE];
    __shared__ float part[8][PJ_ROWS][64];
    const int h = blockIdx.y, c0 = blockIdx.x * 64;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const __nv_bfloat16* w = kvb + (long long)h * PJ_KVB_ROWS * PJ_L + c0 + 2 * lane;
    constexpr int DW = PJ_NOPE / 8;  // d per warp
    __nv_bfloat162 wv[DW];           // this lane's weights, read once
#pragma unroll
    for (int j = 0; j < DW; ++j)
        wv[j] = *reinterpret_cast<const __nv_bfloat162*>(w + (long long)(warp * DW + j) * PJ_L);
    for (int r0 = 0; r0 < n; r0 += PJ_ROWS) {
        const int nr = min(PJ_ROWS, n - r0);
        for (int i = tid; i < PJ_ROWS * PJ_NOPE; i += PJ_THREADS) {
            const int r = i / PJ_NOPE, d = i % PJ_NOPE;
            qs[r][d] = r < nr ? q[(long long)(r0 + r) * q_row + h * PJ_QK + d] : 0.f;
        }
        __syncthreads();
        float acc[PJ_ROWS][2];
#pragma unroll
        for (int r = 0; r < PJ_ROWS; ++r) acc[r][0] = acc[r][1] = 0.f;
#pragma unroll
        for (int j = 0; j < DW; ++j) {
            const float2 f = __bfloat1622float2(wv[j]);
#pragma unroll
            for (int r = 0; r < PJ_ROWS; ++r) {
                const float x = qs[r][warp * DW + j];
                acc[r][0] = fmaf(x, f.x, acc[r][0]);
                acc[r][1] = fmaf(x, f.y, acc[r][1]);
            }
        }
#pragma unroll
        for (int r = 0; r < PJ_ROWS; ++r) {
            part[warp][r][2 * lane] = acc[r][0];
            part[warp][r][2 * lane + 1] = acc[r][1];
        }
        __syncthreads();
        for (int i = tid; i < PJ_ROWS * 64; i += PJ_THREADS) {
            const int r = i / 64, c = i % 64;
            if (r >= nr) continue;
            float s = part[0][r][c];
#pragma unroll
            for (int k = 1; k < 8; ++k) s += part[k][r][c];
            q_abs[(long long)(r0 + r) * o_row + h * (PJ_L + PJ_ROPE) + c0 + c] = __float2bfloat16_rn(s);
        }
        if (blockIdx.x == 0)  // the roped part rides along
            for (int i = tid; i < nr * PJ_ROPE; i += PJ_THREADS) {
                const int r = i / PJ_ROPE, j = i % PJ_ROPE;
                q_abs[(long long)(r0 + r) * o_row + h * (PJ_L + PJ_ROPE) + PJ_L + j] =
                    __float2bfloat16_rn(q[(long long)(r0 + r) * q_row + h * PJ_QK + PJ_NOPE + j]);
            }
        __syncthreads();  // qs / part are reused by the next chunk
    }
}

// grid (256 / 32 v blocks, 64 heads). Warp w computes v = v0 + 4 w .. + 3: lane
// l dots columns [8 l, 8 l + 8) and [256 + 8 l, 256 + 8 l + 8) of the weight
// row with the context, then a fixed-order tree over the lanes.
__global__ void __launch_bounds__(PJ_THREADS) mla_project_v_kernel(int n, const float* __restrict__ ctx,
                                                                   long long c_row,
                                                                   const __nv_bfloat16* __restrict__ kvb,
                                                                   float* __restrict__ out, long long o_row) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) float cs[PJ_ROWS][PJ_L];
    const int h = blockIdx.y, v0 = blockIdx.x * 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint4 wv[4][2];  // the warp's 4 weight rows, this lane's 2 x 8 columns
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __nv_bfloat16* wr = kvb + ((long long)h * PJ_KVB_ROWS + PJ_NOPE + v0 + 4 * warp + k) * PJ_L;
        wv[k][0] = *reinterpret_cast<const uint4*>(wr + 8 * lane);
        wv[k][1] = *reinterpret_cast<const uint4*>(wr + 256 + 8 * lane);
    }
    for (int r0 = 0; r0 < n; r0 += PJ_ROWS) {
        const int nr = min(PJ_ROWS, n - r0);
        for (int i = tid; i < PJ_ROWS * PJ_L / 4; i += PJ_THREADS) {
            const int r = i / (PJ_L / 4), c4 = i % (PJ_L / 4);
            reinterpret_cast<float4*>(cs[r])[c4] =
                r < nr ? *reinterpret_cast<const float4*>(ctx + (long long)(r0 + r) * c_row + h * PJ_L + 4 * c4)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
        for (int r = 0; r < nr; ++r) {
            float x[16];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const float4 a = *reinterpret_cast<const float4*>(&cs[r][256 * half + 8 * lane]);
                const float4 b = *reinterpret_cast<const float4*>(&cs[r][256 * half + 8 * lane + 4]);
                x[8 * half + 0] = a.x;
                x[8 * half + 1] = a.y;
                x[8 * half + 2] = a.z;
                x[8 * half + 3] = a.w;
                x[8 * half + 4] = b.x;
                x[8 * half + 5] = b.y;
                x[8 * half + 6] = b.z;
                x[8 * half + 7] = b.w;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float s = 0.f;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&wv[k][half]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __bfloat1622float2(p[e]);
                        s = fmaf(x[8 * half + 2 * e], f.x, s);
                        s = fmaf(x[8 * half + 2 * e + 1], f.y, s);
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
                if (lane == 0) out[(long long)(r0 + r) * o_row + h * PJ_V + v0 + 4 * warp + k] = s;
            }
        }
        __syncthreads();  // cs is reused by the next chunk
    }
}

}  // namespace wl
