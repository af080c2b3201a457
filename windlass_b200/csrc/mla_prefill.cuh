// mla_prefill.cuh — sparse absorbed-MLA attention for many query rows
// (chunked prefill): the 64 heads of one query row form the M dimension.
//
// Same computation as mla_sparse_attn_kernel (src/glm_layer_runner.cuh:251-298
// with the index mask of src/glm_kernels.cuh:526-545), organised for rows that
// each attend over up to thousands of keys:
//   S[h, j]  = q_abs[h] . [c_kv | k_rot][key j]        (M = 64 heads, N = 64 keys, K = 576)
//   O[h, :] += P[h, j] . c_kv[key j]                   (M = 64, N = 2 x 256 latent, K = 64 keys)
// One CTA per query row; warp roles, connected by mbarriers:
//   warps 4-11 gather:  the next 64 selected rows with 16-byte cp.async into one
//              of two 72 KB key tiles (9 128B-swizzled chunks of 64 rows),
//              while the tensor cores work on the other;
//   warp 12    MMA:     P.V of tile i into O, then QK of tile i + 1 into one of
//              two S accumulators;
//   warps 0-3  softmax: per head, its 64 scores of a tile (TMEM lanes 16-31 of
//              the warp's quarter, two threads per head), running max and sum,
//              P (bf16) into shared memory as the A operand of P.V; rescale of
//              O (TMEM lanes 0-15) when needed; the final O / l and lse.
// TMEM (512 columns): an M = 64 accumulator occupies lanes 0-15 of each 32-lane
// quarter (row m at lane 32 (m / 16) + m % 16); O sits there in all 512 columns,
// the two S tiles at lane offset 16, each as PF_KSPLIT partial accumulators
// (columns [64 (3 b + q), + 64)) that the softmax adds. Threads
// reach one 16-lane half with the 16x32bx2 access shape, so the softmax and
// the O accesses never touch each other's lanes.
// Rescaling is lazy: a head's running max moves only when a tile's maximum
// exceeds it by more than 2^8 (P <= 256 stays exact in bf16's relative
// precision and fp32 sums), so O is rarely rescaled; P and l always use the
// same max, and O / l is the same quotient.
#pragma once
#include "mla_attn.cuh"

namespace wl {

#ifdef WL_TRACE
__device__ long long* g_trace_pf;
#define WL_TPF(slot, i)                                                                              \
    do {                                                                                             \
        if (g_trace_pf && blockIdx.x == 100 && (i) < 64) g_trace_pf[(i) * 8 + (slot)] = clock64();  \
    } while (0)
#else
#define WL_TPF(slot, i) \
    do {                \
    } while (0)
#endif

constexpr int PF_TILE = 64;      // keys per tile
constexpr int PF_KSPLIT = 3;     // independent QK accumulators per tile (3 K-chunks each)
constexpr int PF_GATHER = 256;   // gather threads (warps 4-11)
constexpr int PF_THREADS = 128 + PF_GATHER + 32;  // softmax warps, gather warps, one MMA warp
constexpr int PF_MMA_WARP = (128 + PF_GATHER) / 32;
constexpr float PF_RESCALE_LOG2 = 8.f;

struct PfLayout {
    static constexpr uint32_t CHUNK = PF_TILE * 128;                     // 8 KB: 64 rows x 64 bf16
    static constexpr uint32_t Q_CHUNK = AT_H * 128;                      // 8 KB
    static constexpr uint32_t OFF_Q = 0;                                 // 9 chunks
    static constexpr uint32_t OFF_K = OFF_Q + AT_CHUNKS * Q_CHUNK;       // 2 tiles x 9 chunks
    static constexpr uint32_t OFF_P = OFF_K + 2 * AT_CHUNKS * CHUNK;     // 64 heads x 64 keys bf16
    static constexpr uint32_t OFF_ROWS = OFF_P + AT_H * 128;             // 2 x 64 row indices
    static constexpr uint32_t OFF_INVL = OFF_ROWS + 2 * PF_TILE * 4;  // [64] 1 / l per head
    static constexpr uint32_t OFF_BAR = OFF_INVL + AT_H * 4;
    static constexpr int N_BARS = 2 + 2 + 2 + 2 + 1 + 1 + 1;  // kfull, kfree, sfull, sfree, pready, pvdone, q
    static constexpr uint32_t OFF_MISC = OFF_BAR + N_BARS * 8;
    static constexpr uint32_t BYTES = OFF_MISC + 32 + 1024;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t IDESC_QK = idesc_bf16(64, PF_TILE, 0, 0);
    static constexpr uint32_t IDESC_PV = idesc_bf16(64, 256, 0, 1);
};
static_assert(PfLayout::BYTES <= 232448, "one CTA per SM");

// The absorbed queries as a bf16 tensor {576, 64 rows}: 64 x 64 boxes with
// 128B swizzle land exactly as the K-major chunks the MMA reads.
struct PfParams {
    CUtensorMap tm_q;  // {AT_D, 64 * n_rows}, box {64, 64}
};

__device__ __forceinline__ void tma_load2d(uint32_t dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__global__ void __launch_bounds__(PF_THREADS, 1)
    mla_prefill_kernel(AttnParams p, const __grid_constant__ PfParams pp) {
    using L = PfLayout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sQ = smem_u32(smem + L::OFF_Q);
    const uint32_t sK = smem_u32(smem + L::OFF_K);
    const uint32_t sP = smem_u32(smem + L::OFF_P);
    int* rows_sh = reinterpret_cast<int*>(smem + L::OFF_ROWS);
    float* inv_l_sh = reinterpret_cast<float*>(smem + L::OFF_INVL);
    uint64_t* kfull = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* kfree = kfull + 2;
    uint64_t* sfull = kfree + 2;
    uint64_t* sfree = sfull + 2;
    uint64_t* pready = sfree + 2;
    uint64_t* pvdone = pready + 1;
    uint64_t* qbar = pvdone + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) WL_TPF(7, 0);
    const int r = blockIdx.x;
    const int seq = r / p.rows_per_seq;
    const long long lraw = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    const int len = (int)(lraw < p.len_T ? lraw : p.len_T);
    const int* list = p.sel ? p.sel + (long long)r * p.sel_stride : nullptr;
    pdl_wait();
    pdl_trigger();
    const int n_keys = list ? (p.sel_n_dev ? __ldg(p.sel_n_dev + r) : p.sel_n) : len;
    float* ctx = p.o_part + (long long)r * (AT_H * AT_DV);
    float* lse_out = p.lse_part + (long long)r * AT_H;
    if (n_keys <= 0) {
        for (int i = tid; i < AT_H * AT_DV / 4; i += PF_THREADS)
            reinterpret_cast<float4*>(ctx)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tid < AT_H) lse_out[tid] = -INFINITY;
        return;
    }
    const int n_tiles = (n_keys + PF_TILE - 1) / PF_TILE;

    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(kfull + b, PF_GATHER);  // the gather threads
            mbar_init(kfree + b, 1);    // the P.V commit
            mbar_init(sfull + b, 1);    // the QK commit
            mbar_init(sfree + b, 128);  // the softmax threads
        }
        mbar_init(pready, 128);
        mbar_init(pvdone, 1);
        mbar_init(qbar, 1);
        fence_mbar_init();
        // the row's absorbed query [64][576]: 9 TMA boxes (the MMA waits on qbar)
        mbar_expect_tx(qbar, AT_CHUNKS * L::Q_CHUNK);
        for (int c = 0; c < AT_CHUNKS; ++c) tma_load2d(sQ + (uint32_t)c * L::Q_CHUNK, &pp.tm_q, c * 64, r * AT_H, qbar);
    }
    if (warp == PF_MMA_WARP) tmem_alloc(tmem_slot, L::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) WL_TPF(7, 4);
    const uint32_t tmem = *tmem_slot;
    const __nv_bfloat16* ckv = p.c_kv + (long long)seq * p.ckv_seq;
    const __nv_bfloat16* krt = p.k_rot + (long long)seq * p.krot_seq;

    if (warp >= 4 && warp < PF_MMA_WARP) {
        // ---------------- gather ----------------
        const int g = tid - 128;
        volatile int* go = reinterpret_cast<volatile int*>(tmem_slot + 1);
        auto key_of = [&](int i) -> int {  // this thread's row index of tile i (g < PF_TILE), -1 past the list
            const int e = i * PF_TILE + g;
            if (g >= PF_TILE || i >= n_tiles || e >= n_keys) return -1;
            const long long key = list ? (long long)__ldg(list + e) : (long long)e;
            if (key < 0 || key >= p.T) {
                set_error(ERRC_BOUNDS, 31);
                return -1;
            }
            return (int)key;
        };
        int key_next = key_of(0);  // indices one tile ahead: their load latency hides behind a tile
        for (int i = 0; i < n_tiles; ++i) {
            const int b = i & 1;
            // one thread waits for the buffer and tells the others, so that all
            // gather threads leave together on a timeout (the named barriers need all)
            if (g == 0) *go = (i < 2 || mbar_wait_fast(kfree + b, (uint32_t)((i >> 1) - 1) & 1u, 30)) ? 1 : 0;
            if (g < PF_TILE) rows_sh[b * PF_TILE + g] = key_next;
            asm volatile("bar.sync 2, %0;" ::"n"(PF_GATHER) : "memory");
            if (!*go) break;
            key_next = key_of(i + 1);
            const uint32_t tile = sK + (uint32_t)b * AT_CHUNKS * L::CHUNK;
#pragma unroll 3
            for (int k2 = 0; k2 < AT_CHUNKS * PF_TILE * 8 / PF_GATHER; ++k2) {  // 18 pieces of 16 B per thread
                const int pid = k2 * PF_GATHER + g;
                const int c = pid / (PF_TILE * 8), rem = pid % (PF_TILE * 8);
                const int j = rem >> 3, seg = rem & 7;
                const int row = rows_sh[b * PF_TILE + j];
                const __nv_bfloat16* src = (c < 8) ? ckv + (long long)(row < 0 ? 0 : row) * p.ckv_row + c * 64 + seg * 8
                                                   : krt + (long long)(row < 0 ? 0 : row) * p.krot_row + seg * 8;
                cp_async16(tile + (uint32_t)c * L::CHUNK + sw128_off(j, seg), src, row < 0 ? 0u : 16u);
            }
            cp_async_commit();
            if (g == 0) WL_TPF(0, i);
            cp_async_wait_all();
            fence_proxy_async_smem();
            mbar_arrive(kfull + b);
            if (g == 0) WL_TPF(1, i);
            asm volatile("bar.sync 2, %0;" ::"n"(PF_GATHER) : "memory");  // rows_sh[b] is rewritten two tiles on
        }
    } else if (warp == PF_MMA_WARP) {
        // ---------------- MMA ----------------
        // PV(i) goes before QK(i + 1): it frees tile i's buffer early, so the
        // gather of tile i + 2 hides behind QK(i + 1) and the softmax.
        auto issue_qk = [&](int i) -> bool {
            const int b = i & 1;
            if (!mbar_wait_fast(kfull + b, (uint32_t)(i >> 1) & 1u, 32)) return false;
            if (i >= 2 && !mbar_wait_fast(sfree + b, (uint32_t)((i >> 1) - 1) & 1u, 33)) return false;
            tc_fence_after();
            if (lane == 0) {
                WL_TPF(2, i);
                const uint32_t tile = sK + (uint32_t)b * AT_CHUNKS * L::CHUNK;
                // K split over PF_KSPLIT accumulators, interleaved so consecutive
                // MMAs never wait on each other (one accumulator chains them)
#pragma unroll 1
                for (int c0 = 0; c0 < AT_CHUNKS / PF_KSPLIT; ++c0) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                        for (int q = 0; q < PF_KSPLIT; ++q) {
                            const int c = q * (AT_CHUNKS / PF_KSPLIT) + c0;
                            const uint32_t d = tmem + (16u << 16) + (uint32_t)((b * PF_KSPLIT + q) * PF_TILE);
                            mma_bf16(d, desc_sw128(sQ + (uint32_t)c * L::Q_CHUNK + kk * 32, 16, 1024),
                                     desc_sw128(tile + (uint32_t)c * L::CHUNK + kk * 32, 16, 1024), L::IDESC_QK,
                                     (c0 | kk) != 0 ? 1u : 0u);
                        }
                    }
                }
                mma_commit(sfull + b);
            }
            __syncwarp();
            return true;
        };
        auto issue_pv = [&](int i) -> bool {
            const int b = i & 1;
            if (!mbar_wait_fast(pready, (uint32_t)i & 1u, 34)) return false;
            tc_fence_after();
            if (lane == 0) {
                WL_TPF(3, i);
                const uint32_t tile = sK + (uint32_t)b * AT_CHUNKS * L::CHUNK;
#pragma unroll
                for (int ks = 0; ks < PF_TILE / 16; ++ks) {
#pragma unroll
                    for (int half = 0; half < 2; ++half)
                        mma_bf16(tmem + (uint32_t)(half * 256), desc_sw128(sP + ks * 32, 16, 1024),
                                 desc_sw128(tile + (uint32_t)(4 * half) * L::CHUNK + ks * 2048, L::CHUNK, 1024),
                                 L::IDESC_PV, (i > 0 || ks > 0) ? 1u : 0u);
                }
                mma_commit(kfree + b);
                mma_commit(pvdone);
            }
            __syncwarp();
            return true;
        };
        bool ok = mbar_wait_fast(qbar, 0, 38);
        ok = ok && issue_qk(0);
        for (int i = 0; ok && i < n_tiles; ++i) {
            ok = issue_pv(i);
            if (ok && i + 1 < n_tiles) ok = issue_qk(i + 1);
        }
    } else {
        // ---------------- softmax (warps 0-3) ----------------
        // Thread t < 16 of warp w: head 16 w + t, keys [0, 32) of a tile and O
        // columns [c, c + 32); thread t + 16: the same head, keys [32, 64), O
        // columns [c + 256, c + 288).
        const int h = 16 * warp + (lane & 15);
        const bool hi_half = lane >= 16;
        const uint32_t lane_o = (uint32_t)(32 * warp) << 16, lane_s = (uint32_t)(32 * warp + 16) << 16;
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int i = 0; i < n_tiles && ok; ++i) {
            const int b = i & 1;
            const int nv = min(PF_TILE, n_keys - i * PF_TILE);
            if (!(ok = mbar_wait_fast(sfull + b, (uint32_t)(i >> 1) & 1u, 35))) break;
            if (tid == 0) WL_TPF(4, i);
            tc_fence_after();
            float sv[32];
            tmem_ld16x2_32<32>(tmem + lane_s + (uint32_t)(b * PF_KSPLIT * PF_TILE), sv);
#pragma unroll
            for (int q = 1; q < PF_KSPLIT; ++q) {
                float sq[32];
                tmem_ld16x2_32<32>(tmem + lane_s + (uint32_t)((b * PF_KSPLIT + q) * PF_TILE), sq);
#pragma unroll
                for (int j = 0; j < 32; ++j) sv[j] += sq[j];
            }
            tc_fence_before();
            mbar_arrive(sfree + b);
            const int j0 = hi_half ? 32 : 0;
            float tmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                sv[j] = (j0 + j < nv) ? sv[j] * p.scale_log2 : -INFINITY;
                tmax = fmaxf(tmax, sv[j]);
            }
            tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
            // lazy max: move only on a large increase (or the first tile)
            const float m_new = (m_run == -INFINITY || tmax > m_run + PF_RESCALE_LOG2) ? tmax : m_run;
            const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
            // P of the previous tile must be consumed (and O complete) first
            if (i >= 1 && !(ok = mbar_wait_fast(pvdone, (uint32_t)(i - 1) & 1u, 36))) break;
            if (tid == 0) WL_TPF(5, i);
            tc_fence_after();
            float sum = 0.f;
            const uint32_t prow = sP + (uint32_t)h * 128u;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {  // 8 keys = one 16-byte chunk per step
                uint32_t w4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = c4 * 8 + e * 2;
                    const __nv_bfloat162 b2 = __floats2bfloat162_rn(exp2f(sv[j] - m_new), exp2f(sv[j + 1] - m_new));
                    w4[e] = *reinterpret_cast<const uint32_t*>(&b2);
                    sum += __low2float(b2) + __high2float(b2);
                }
                const uint32_t chunk = (uint32_t)((hi_half ? 4 : 0) + c4);
                sts_v4(prow + (((chunk ^ (uint32_t)h) & 7u) << 4), make_uint4(w4[0], w4[1], w4[2], w4[3]));
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 16);
            l_run = l_run * alpha + sum;
            // Rescale this head's O row when its max moved after the first tile.
            const bool resc = i > 0 && m_new != m_run;
            m_run = m_new;
            if (__any_sync(0xffffffffu, resc)) {
#pragma unroll 1
                for (int c = 0; c < 256; c += 32) {
                    float ov[32];
                    tmem_ld16x2_32<256>(tmem + lane_o + (uint32_t)c, ov);
                    const float f = resc ? alpha : 1.f;
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] *= f;
                    tmem_st16x2_32<256>(tmem + lane_o + (uint32_t)c, ov);
                }
                tmem_wait_st();
            }
            fence_proxy_async_smem();  // P is read by the tensor cores
            tc_fence_before();
            mbar_arrive(pready);
            if (tid == 0) WL_TPF(6, i);
        }
        // ---- 1 / l and lse per head, for the epilogue warps ----
        if (!hi_half) {
            inv_l_sh[h] = (ok && l_run > 0.f) ? 1.f / l_run : 0.f;
            lse_out[h] = (ok && l_run > 0.f) ? (m_run + log2f(l_run)) * 0.69314718055994531f : -INFINITY;
        }
    }
    // ---- O / l -> ctx, by the softmax and gather warps (warp % 4 = TMEM quarter) ----
    __syncthreads();  // every role is past its loop; inv_l_sh is written
    if (warp < PF_MMA_WARP) {
        const int grp = warp >> 2, ngrp = PF_MMA_WARP / 4;  // 3 groups of 4 warps
        const int q4 = warp & 3, hq = 16 * q4 + (lane & 15);
        const bool hi = lane >= 16;
        const uint32_t lane_o = (uint32_t)(32 * q4) << 16;
        bool done = mbar_wait_fast(pvdone, (uint32_t)(n_tiles - 1) & 1u, 37);
        tc_fence_after();
        if (done) {
            const float inv = inv_l_sh[hq];
            float* crow = ctx + (long long)hq * AT_DV + (hi ? 256 : 0);
#pragma unroll 1
            for (int c = grp * 32; c < 256; c += 32 * ngrp) {
                float ov[32];
                tmem_ld16x2_32<256>(tmem + lane_o + (uint32_t)c, ov);
#pragma unroll
                for (int e = 0; e < 32; e += 4)
                    *reinterpret_cast<float4*>(crow + c + e) =
                        make_float4(ov[e] * inv, ov[e + 1] * inv, ov[e + 2] * inv, ov[e + 3] * inv);
            }
        }
    }
    if (tid == 0) WL_TPF(7, 1);
    tc_fence_before();
    __syncthreads();
    if (tid == 0) WL_TPF(7, 2);
    if (warp == PF_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
    if (tid == 0) WL_TPF(7, 3);
}

}  // namespace wl
