// idx_query.cuh — the indexer's query side before the scoring: shapes and the
// per-head weights (the query projection itself, with its RoPE, runs on the
// tensor cores: gemv_tc.cuh, GV_IDXQ).
//
// Reference: launch_indexer_query (src/glm_kernels.cuh:453-472):
//   q = wq_b @ q_resid (launch_matvec_bf16; wq_b [32*128, 2048] bf16), then
//   rope_interleave_slice on dims [0, 64) of every head (:137-160, interleaved
//   pairs in, halves out), and
//   w[h] = (weights_proj @ x)[h] * 32^-0.5 (indexer_head_weights, :290-303;
//   weights_proj [32, hidden] fp32, x the input_layernorm output).
// numpy: tools/ref_glm_chain.py:482-501 (indexer_scores, its q and w).
// Output: the scoring kernels' inputs, q_idx bf16 [n][32][128] and w_idx fp32
// [n][32]; fp32 accumulation; sums across lanes and warps in a fixed order.
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int IQ_H = 32, IQ_D = 128, IQ_ROT = 64, IQ_QL = 2048;
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
