// cache_append.cuh — the cache write path: each new token's indexer key and
// latent row, from the projections' outputs to the formats the indexer and the
// attention read.
//
// Reference: launch_indexer_key (src/glm_kernels.cuh:432-448) = LayerNorm
// (indexer_k_layernorm, :255-278; eps 1e-6) -> RoPE on the leading 64 of the
// 128 dims (rope_interleave_slice with rope_off 0, :137-160) -> bf16 store
// (indexer_store_k_bf16, :280-285); and the latent row write of run_attention
// (src/glm_layer_runner.cuh:544-570): RMSNorm of the first 512 of
// kv_a_proj_with_mqa(x) with the kv_a_layernorm weight (eps 1e-6, rms_norm_bf16),
// the trailing 64 not normalised but roped at the token's position. numpy:
// tools/ref_glm_chain.py:63-121 (rms_norm, rope_interleave, layer_norm) and
// :465-480 (indexer_keys).
//
// Formats written: the index key as fp8-e4m3 of its bf16 value (the value the
// reference caches) with one fp32 scale per key = amax / 448; c_kv and k_rot
// as bf16 rows.
//
// One warp per token. Sums run in one fixed order — lane l accumulates its
// own elements in order, then a tree over lanes (offsets 16, 8, 4, 2, 1) ends
// in lane 0 — and every product and sum is rounded on its own (no fused
// multiply-add), so a CPU restatement reproduces every output bit. The
// reference's own block reductions add in another order; the two agree to
// fp32 rounding.
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int CA_WARPS = 4;  // tokens per CTA

struct AppendParams {
    int n;                      // tokens
    const int* pos;             // [n] cache row of each token
    const int* seq;             // [n] sequence of each token, or null (all 0)
    int n_seq;                  // sequences the caches hold (seq[i] must be below it)
    int T_max;                  // rows each sequence's caches hold
    const float* cos;           // [n][32] the token's RoPE table row
    const float* sin;
    // indexer key (skipped when k_raw is null)
    const float* k_raw;         // [n][128] wk(x)
    const __nv_bfloat16* k_w;   // [128] LayerNorm weight
    const __nv_bfloat16* k_b;   // [128] LayerNorm bias
    float ln_eps;
    uint8_t* keys;              // [seq][T_max][128] e4m3
    long long keys_seq;         // bytes
    float* scale;               // [seq][T_max]
    long long scale_seq;        // floats
    // latent row (skipped when kv_raw is null)
    const float* kv_raw;        // [n][576] kv_a_proj_with_mqa(x)
    const __nv_bfloat16* kv_w;  // [512] RMSNorm weight
    float rms_eps;
    __nv_bfloat16* c_kv;
    long long ckv_row, ckv_seq;  // elements
    __nv_bfloat16* k_rot;
    long long krot_row, krot_seq;
};

// Sum over the warp in the fixed order: tree into lane 0, then broadcast.
__device__ __forceinline__ float ca_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
    return __shfl_sync(0xffffffffu, v, 0);
}
__device__ __forceinline__ float ca_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(32 * CA_WARPS) cache_append_kernel(AppendParams p) {
    pdl_wait();
    pdl_trigger();
    __shared__ float kbuf[CA_WARPS][128];
    __shared__ __nv_bfloat16 rbuf[CA_WARPS][64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tok = blockIdx.x * CA_WARPS + warp;
    if (tok >= p.n) return;
    const int row = p.pos[tok];
    const int sq = p.seq ? p.seq[tok] : 0;
    if (row < 0 || row >= p.T_max || sq < 0 || sq >= p.n_seq) {
        if (lane == 0) set_error(ERRC_BOUNDS, 40);
        return;
    }
    const float* cs = p.cos + (long long)tok * 32;
    const float* sn = p.sin + (long long)tok * 32;

    if (p.k_raw) {
        // ---- indexer key: LayerNorm, RoPE on dims [0, 64), bf16, e4m3 + scale ----
        const float4 v4 = *reinterpret_cast<const float4*>(p.k_raw + (long long)tok * 128 + 4 * lane);
        const float v[4] = {v4.x, v4.y, v4.z, v4.w};
        const float mean = __fdiv_rn(ca_warp_sum(__fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), v[2]), v[3])), 128.f);
        float d[4], q = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            d[e] = __fsub_rn(v[e], mean);
            q = __fadd_rn(q, __fmul_rn(d[e], d[e]));
        }
        const float var = __fdiv_rn(ca_warp_sum(q), 128.f);
        const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, p.ln_eps)));
        float y[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
            y[e] = __fadd_rn(__fmul_rn(__fmul_rn(d[e], inv), __bfloat162float(p.k_w[4 * lane + e])),
                             __bfloat162float(p.k_b[4 * lane + e]));
        float* kb = kbuf[warp];
        if (lane < 16) {
            // adjacent pairs (4l, 4l+1) and (4l+2, 4l+3) are rotation pairs 2l and
            // 2l+1; the output takes the halves layout [a c - b s | b c + a s]
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 2 * lane + h;
                const float a = y[2 * h], b = y[2 * h + 1], c = cs[i], s = sn[i];
                kb[i] = ca_bf16(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)));
                kb[32 + i] = ca_bf16(__fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s)));
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) kb[4 * lane + e] = ca_bf16(y[e]);
        }
        __syncwarp();
        float k[4], amax = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            k[e] = kb[4 * lane + e];
            amax = fmaxf(amax, fabsf(k[e]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float sc = amax > 0.f ? __fdiv_rn(amax, 448.f) : 1.f;
        uint32_t codes = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
            codes |= (uint32_t)__nv_cvt_float_to_fp8(__fdiv_rn(k[e], sc), __NV_SATFINITE, __NV_E4M3) << (8 * e);
        *reinterpret_cast<uint32_t*>(p.keys + sq * p.keys_seq + (long long)row * 128 + 4 * lane) = codes;
        if (lane == 0) p.scale[sq * p.scale_seq + row] = sc;
    }

    if (p.kv_raw) {
        // ---- c_kv: RMSNorm of the first 512 (elements j*128 + 4l + e of lane l) ----
        const float* x = p.kv_raw + (long long)tok * 576;
        float4 c4[4];
        float q = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            c4[j] = *reinterpret_cast<const float4*>(x + j * 128 + 4 * lane);
            q = __fadd_rn(q, __fmul_rn(c4[j].x, c4[j].x));
            q = __fadd_rn(q, __fmul_rn(c4[j].y, c4[j].y));
            q = __fadd_rn(q, __fmul_rn(c4[j].z, c4[j].z));
            q = __fadd_rn(q, __fmul_rn(c4[j].w, c4[j].w));
        }
        const float ms = __fdiv_rn(ca_warp_sum(q), 512.f);
        const float inv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(ms, p.rms_eps)));
        __nv_bfloat16* out = p.c_kv + sq * p.ckv_seq + (long long)row * p.ckv_row;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c0 = j * 128 + 4 * lane;
            const float e0 = __fmul_rn(__fmul_rn(c4[j].x, inv), __bfloat162float(p.kv_w[c0]));
            const float e1 = __fmul_rn(__fmul_rn(c4[j].y, inv), __bfloat162float(p.kv_w[c0 + 1]));
            const float e2 = __fmul_rn(__fmul_rn(c4[j].z, inv), __bfloat162float(p.kv_w[c0 + 2]));
            const float e3 = __fmul_rn(__fmul_rn(c4[j].w, inv), __bfloat162float(p.kv_w[c0 + 3]));
            __nv_bfloat162 lo = __floats2bfloat162_rn(e0, e1), hi = __floats2bfloat162_rn(e2, e3);
            uint2 w;
            w.x = *reinterpret_cast<uint32_t*>(&lo);
            w.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(out + c0) = w;
        }
        // ---- k_rot: RoPE of the trailing 64, not normalised ----
        __nv_bfloat16* rb = rbuf[warp];
        if (lane < 16) {
            const float4 r4 = *reinterpret_cast<const float4*>(x + 512 + 4 * lane);
            const float r[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 2 * lane + h;
                const float a = r[2 * h], b = r[2 * h + 1], c = cs[i], s = sn[i];
                rb[i] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)));
                rb[32 + i] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s)));
            }
        }
        __syncwarp();
        __nv_bfloat16* kr = p.k_rot + sq * p.krot_seq + (long long)row * p.krot_row;
        reinterpret_cast<uint32_t*>(kr)[lane] = reinterpret_cast<const uint32_t*>(rb)[lane];
    }
}

}  // namespace wl
