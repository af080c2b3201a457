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
