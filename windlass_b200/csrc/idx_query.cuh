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
constexpr int IQ_THREADS = 256;   // 8 warps, 2 output dims each
constexpr int IQ_DIMS = 16;       // output dims per CTA
constexpr uint32_t IQ_SMEM = IQ_ROWS * IQ_QL * 4;  // the chunk's q_resid rows

// grid (32 * 128 / 16). Warp w owns output dims o = 16 b + 2 w, + 1 — a RoPE
// pair when o % 128 < 64 — with their two weight rows in registers (lane l:
// columns 8 l + 256 j, j < 8); per query row, lane partials are summed by a
// xor butterfly and lane 0 applies the rotation and stores bf16.
__global__ void __launch_bounds__(IQ_THREADS, 2) idx_query_kernel(int n, const float* __restrict__ q_resid,
                                                                  long long qr_row,
                                                                  const __nv_bfloat16* __restrict__ wq_b,
                                                                  const float* __restrict__ cos,
                                                                  const float* __restrict__ sin,
                                                                  __nv_bfloat16* __restrict__ q_idx,
                                                                  long long q_row) {
    extern __shared__ __align__(16) float xs[];  // [IQ_ROWS][2048]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int o0 = blockIdx.x * IQ_DIMS + 2 * warp;  // even
    const int h = o0 / IQ_D, dd = o0 % IQ_D;
    pdl_wait();
    pdl_trigger();
    uint4 w0[8], w1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        w0[j] = *reinterpret_cast<const uint4*>(wq_b + (long long)o0 * IQ_QL + 256 * j + 8 * lane);
        w1[j] = *reinterpret_cast<const uint4*>(wq_b + (long long)(o0 + 1) * IQ_QL + 256 * j + 8 * lane);
    }
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
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 a = *reinterpret_cast<const float4*>(xs + r * IQ_QL + 256 * j + 8 * lane);
                const float4 b = *reinterpret_cast<const float4*>(xs + r * IQ_QL + 256 * j + 8 * lane + 4);
                const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                const __nv_bfloat162* p0 = reinterpret_cast<const __nv_bfloat162*>(&w0[j]);
                const __nv_bfloat162* p1 = reinterpret_cast<const __nv_bfloat162*>(&w1[j]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f0 = __bfloat1622float2(p0[e]), f1 = __bfloat1622float2(p1[e]);
                    s0 = fmaf(x[2 * e], f0.x, s0);
                    s0 = fmaf(x[2 * e + 1], f0.y, s0);
                    s1 = fmaf(x[2 * e], f1.x, s1);
                    s1 = fmaf(x[2 * e + 1], f1.y, s1);
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                s0 += __shfl_xor_sync(0xffffffffu, s0, o);
                s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            }
            if (lane == 0) {
                __nv_bfloat16* qo = q_idx + (long long)(r0 + r) * q_row + h * IQ_D;
                if (dd < IQ_ROT) {
                    const int i = dd >> 1;
                    const float c = cos[(long long)(r0 + r) * (IQ_ROT / 2) + i];
                    const float sn = sin[(long long)(r0 + r) * (IQ_ROT / 2) + i];
                    qo[i] = __float2bfloat16_rn(s0 * c - s1 * sn);
                    qo[IQ_ROT / 2 + i] = __float2bfloat16_rn(s1 * c + s0 * sn);
                } else {
                    qo[dd] = __float2bfloat16_rn(s0);
                    qo[dd + 1] = __float2bfloat16_rn(s1);
                }
            }
        }
        __syncthreads();  // xs is rewritten by the next chunk
    }
}

// grid (32 heads): w[r][h] = scale * sum_k weights_proj[h][k] * x[r][k]. Warp w
// sums k in [w * hidden / 8, (w + 1) * hidden / 8) with float4 loads; the 8
// warp partials are added in warp order.
__global__ void __launch_bounds__(256) idx_head_weights_kernel(int n, const float* __restrict__ x, long long x_row,
                                                               const float* __restrict__ wp, int hidden, float scale,
                                                               float* __restrict__ w_idx, long long w_row) {
    __shared__ float part[8];
    const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait();
    pdl_trigger();
    const int span = hidden / 8;  // a multiple of 128
    const float* wr = wp + (long long)h * hidden + warp * span;
    for (int r = 0; r < n; ++r) {
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
        __syncthreads();
    }
}

}  // namespace wl
