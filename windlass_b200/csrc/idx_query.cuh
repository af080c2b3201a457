// idx_query.cuh — the indexer's query side before the scoring: the query
// projection from the shared q-LoRA residual with RoPE on the leading 64 dims
// of each head, and the per-head weights.
//
// Reference: launch_indexer_query (src/glm_kernels.cuh:453-472):
//   q = wq_b @ q_resid (launch_matvec_bf16; wq_b [32*128, 2048] bf16), then
//   rope_interleave_slice on dims [0, 64) of every head (:137-160, interleaved
//   pairs in, halves out), and
//   w[h] = (weights_proj @ x)[h] * 32^-0.5 (indexer_head_weights, :290-303;
//   weights_proj [32, hidden] fp32, x the input_layernorm output).
// numpy: tools/ref_glm_chain.py:482-501 (indexer_scores, its q and w).
// Output: the scoring kernels' inputs, q_idx bf16 [n][32][128] and w_idx fp32
// [n][32]. Decode-shaped (n rows of a batch or a prefill chunk, in chunks of
// IQ_ROWS); fp32 accumulation; sums across lanes and warps in a fixed order.
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int IQ_H = 32, IQ_D = 128, IQ_ROT = 64, IQ_QL = 2048;
constexpr int IQ_ROWS = 8;        // query rows per chunk
constexpr int IQ_DIMS = 8;        // output dims per CTA, one per warp
constexpr int IQ_THREADS = 32 * IQ_DIMS;
constexpr uint32_t IQ_SMEM = IQ_ROWS * IQ_QL * 4 + IQ_ROWS * IQ_DIMS * 4;  // q_resid rows + dot products

// grid (32 * 128 / IQ_DIMS). Warp w owns output dim o = IQ_DIMS b + w with its weight
// row in registers (lane l: columns 8 l + 256 j, j < 8); per query row the
// lane partials are summed by a xor butterfly into shared memory, then the
// CTA applies RoPE to the pairs (o, o + 1) with o % 128 < 64 and stores bf16.
__global__ void __launch_bounds__(IQ_THREADS, 2) idx_query_kernel(int n, const float* __restrict__ q_resid,
                                                                  long long qr_row,
                                                                  const __nv_bfloat16* __restrict__ wq_b,
                                                                  const float* __restrict__ cos,
                                                                  const float* __restrict__ sin,
                                                                  __nv_bfloat16* __restrict__ q_idx,
                                                                  long long q_row) {
    extern __shared__ __align__(16) float xs[];  // [IQ_ROWS][2048], then dots [IQ_ROWS][IQ_DIMS]
    float* dots = xs + IQ_ROWS * IQ_QL;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ob = blockIdx.x * IQ_DIMS;
    pdl_wait();
    pdl_trigger();
    uint4 w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        w[j] = *reinterpret_cast<const uint4*>(wq_b + (long long)(ob + warp) * IQ_QL + 256 * j + 8 * lane);
    for (int r0 = 0; r0 < n; r0 += IQ_ROWS) {
        const int nr = min(IQ_ROWS, n - r0);
        for (int i = tid; i < IQ_ROWS * IQ_QL / 4; i += IQ_THREADS) {
            const int r = i / (IQ_QL / 4), c4 = i % (IQ_QL / 4);
            reinterpret_cast<float4*>(xs)[i] =
                r < nr ? *reinterpret_cast<const float4*>(q_resid + (long long)(r0 + r) * qr_row + 4 * c4)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
        for (int r = 0; r < nr; ++r) {
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 a = *reinterpret_cast<const float4*>(xs + r * IQ_QL + 256 * j + 8 * lane);
                const float4 b = *reinterpret_cast<const float4*>(xs + r * IQ_QL + 256 * j + 8 * lane + 4);
                const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&w[j]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(p[e]);
                    s = fmaf(x[2 * e], f.x, s);
                    s = fmaf(x[2 * e + 1], f.y, s);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) dots[r * IQ_DIMS + warp] = s;
        }
        __syncthreads();
        if (tid < nr * IQ_DIMS / 2) {  // one thread per (row, dim pair)
            const int r = tid / (IQ_DIMS / 2), pr = tid % (IQ_DIMS / 2);
            const int o = ob + 2 * pr, h = o / IQ_D, dd = o % IQ_D;
            const float a = dots[r * IQ_DIMS + 2 * pr], b = dots[r * IQ_DIMS + 2 * pr + 1];
            __nv_bfloat16* qo = q_idx + (long long)(r0 + r) * q_row + h * IQ_D;
            if (dd < IQ_ROT) {
                const int i = dd >> 1;
                const float c = cos[(long long)(r0 + r) * (IQ_ROT / 2) + i];
                const float sn = sin[(long long)(r0 + r) * (IQ_ROT / 2) + i];
                qo[i] = __float2bfloat16_rn(a * c - b * sn);
                qo[IQ_ROT / 2 + i] = __float2bfloat16_rn(b * c + a * sn);
            } else {
                qo[dd] = __float2bfloat16_rn(a);
                qo[dd + 1] = __float2bfloat16_rn(b);
            }
        }
        __syncthreads();  // xs and dots are rewritten by the next chunk
    }
}

// grid (32 heads, n rows): w[r][h] = scale * sum_k weights_proj[h][k] * x[r][k].
// Warp w sums k in [w * hidden / 8, (w + 1) * hidden / 8) with float4 loads;
// the 8 warp partials are added in warp order.
__global__ void __launch_bounds__(256) idx_head_weights_kernel(int n, const float* __restrict__ x, long long x_row,
                                                               const float* __restrict__ wp, int hidden, float scale,
                                                               float* __restrict__ w_idx, long long w_row) {
    __shared__ float part[8];
    const int h = blockIdx.x, r = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait();
    pdl_trigger();
    if (r >= n) return;
    const int span = hidden / 8;  // a multiple of 128
    const float* wr = wp + (long long)h * hidden + warp * span;
    const float* xr = x + (long long)r * x_row + warp * span;
    float s = 0.f;
    for (int k = 4 * lane; k < span; k += 128) {
        const float4 a = *reinterpret_cast<const float4*>(wr + k);
        const float4 b = *reinterpret_cast<const float4*>(xr + k);
        s = fmaf(a.x, b.x, s);
        s = fmaf(a.y, b.y, s);
        s = fmaf(a.z, b.z, s);
        s = fmaf(a.w, b.w, s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) part[warp] = s;
    __syncthreads();
    if (tid == 0) {
        float t = part[0];
#pragma unroll
        for (int k = 1; k < 8; ++k) t += part[k];
        w_idx[(long long)r * w_row + h] = t * scale;
    }
}

}  // namespace wl
