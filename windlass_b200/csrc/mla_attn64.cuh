// mla_attn64.cuh — sparse absorbed-MLA attention with the 64 heads of one
// query row as the M dimension (chunked prefill and split-K decode).
//
// Same computation as mla_sparse_attn_kernel (src/glm_layer_runner.cuh:251-298
// with the index mask of src/glm_kernels.cuh:526-545), organised as a pipeline
// over 64-key tiles of one row's selection (or of a split of it):
//   S[h, j]  = q_abs[h] . [c_kv | k_rot][key j]        (M = 64 heads, N = 64 keys, K = 576)
//   O[h, :] += P[h, j] . c_kv[key j]                   (M = 64, N = 2 x 256 latent, K = 64 keys)
// grid (splits, rows): one CTA per (query row, range of its list inside the key
// window), writing that range's normalised o and lse (one partial, merged by
// lse_merge_kernel when a row has several). Warp roles, connected by mbarriers:
//   warps 4-11 gather:  the next 64 selected rows with 16-byte cp.async into one
//              of three 72 KB key tiles (9 128B-swizzled chunks of 64 rows), the
//              row indices prefetched a tile ahead;
//   warp 12    MMA:     QK of tile i + 1 into one of two S accumulators, then P.V
//              of tile i into O — the softmax of tile i overlaps QK(i + 1);
//   warps 0-3  softmax: per head, its 64 scores of a tile (two threads per
//              head), running max and sum, P (bf16) into shared memory as the A
//              operand of P.V; rescale of O when needed; 1 / l and lse.
// Tensor memory (512 columns x 128 lanes). An M = 64 accumulator occupies
// lanes 0-15 of each 32-lane quarter (row m at lane 32 (m / 16) + m % 16), or
// lanes 16-31 with a lane offset of 16:
//   lanes 0-15:   O [64 x 512] fp32, all columns;
//   lanes 16-31:  S tiles (columns [0, 64), [64, 128)) and the query as the QK
//                 A operand (columns [128, 416): two bf16 per column) — an A
//                 operand in tensor memory sits in its accumulator's lanes.
// Threads reach one 16-lane half with the 16x32bx2 access shape, so the
// softmax's and O's accesses never touch each other's lanes. The query passes
// through the third key tile's space once, on its way into tensor memory.
// Rescaling is lazy: a head's running max moves only when a tile's maximum
// exceeds it by more than 2^8 (P <= 256 stays exact in bf16's relative
// precision and fp32 sums), so O is rarely rescaled; P and l always use the
// same max, and O / l is the same quotient.
#pragma once
#include "mla_attn.cuh"

namespace wl {


constexpr int PF_TILE = 64;       // keys per tile
constexpr int PF_NBUF = 3;        // key tiles in shared memory
constexpr int PF_GATHER = 256;    // gather threads (warps 4-11)
constexpr int PF_THREADS = 128 + PF_GATHER + 32;  // softmax warps, gather warps, one MMA warp
constexpr int PF_MMA_WARP = (128 + PF_GATHER) / 32;
constexpr float PF_RESCALE_LOG2 = 8.f;
constexpr uint32_t PF_TM_Q = 128;  // query columns in tensor memory (lanes 16-31)

struct PfLayout {
    static constexpr uint32_t CHUNK = PF_TILE * 128;                     // 8 KB: 64 rows x 64 bf16
    static constexpr uint32_t TILE = AT_CHUNKS * CHUNK;                  // 72 KB
    static constexpr uint32_t OFF_K = 0;                                 // PF_NBUF tiles
    static constexpr uint32_t OFF_P = OFF_K + PF_NBUF * TILE;            // 64 heads x 64 keys bf16
    static constexpr uint32_t OFF_ROWS = OFF_P + AT_H * 128;             // PF_NBUF x 64 row indices
    static constexpr uint32_t OFF_INVL = OFF_ROWS + PF_NBUF * PF_TILE * 4;  // [64] 1 / l per head
    static constexpr uint32_t OFF_BAR = OFF_INVL + AT_H * 4;
    // kfull, kfree (per tile buffer), sfull, sfree (per S buffer), pready, pvdone, qload, qtmem
    static constexpr int N_BARS = 2 * PF_NBUF + 2 * 2 + 4;
    static constexpr uint32_t OFF_MISC = OFF_BAR + N_BARS * 8;
    static constexpr uint32_t BYTES = OFF_MISC + 32 + 1024;  // misc: TMEM slot, gather flag, e0, e1
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t IDESC_QK = idesc_bf16(64, PF_TILE, 0, 0);
    static constexpr uint32_t IDESC_PV = idesc_bf16(64, 256, 0, 1);
};
static_assert(PfLayout::BYTES <= 232448, "one CTA per SM");
static_assert(PF_TM_Q + AT_D / 2 <= 512, "query columns fit beside the S tiles");

// The absorbed queries as a bf16 tensor {576, 64 rows}: 64 x 64 boxes with
// 128B swizzle land as the K-major chunks the MMA reads.
struct PfParams {
    CUtensorMap tm_q;  // {AT_D, 64 * n_rows}, box {64, 64}
    // The (o) partials [rows][splits][64][512] fp32 as {512, 64 * rows * splits},
    // 32 x 64 boxes with 128B swizzle: O leaves through shared memory and TMA
    // stores (o_tma), else with plain stores.
    CUtensorMap tm_o;
    int o_tma;
};

__device__ __forceinline__ void tma_store2d(const CUtensorMap* tm, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(x), "r"(y), "r"(src)
                 : "memory");
}

__device__ __forceinline__ void tma_load2d(uint32_t dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__global__ void __launch_bounds__(PF_THREADS, 1)
    mla_attn64_kernel(AttnParams p, const __grid_constant__ PfParams pp) {
    using L = PfLayout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sK = smem_u32(smem + L::OFF_K);
    const uint32_t sP = smem_u32(smem + L::OFF_P);
    const uint32_t sQstage = sK + (PF_NBUF - 1) * L::TILE;  // the query's way in (last tile's space)
    int* rows_sh = reinterpret_cast<int*>(smem + L::OFF_ROWS);
    float* inv_l_sh = reinterpret_cast<float*>(smem + L::OFF_INVL);
    uint64_t* kfull = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* kfree = kfull + PF_NBUF;
    uint64_t* sfull = kfree + PF_NBUF;
    uint64_t* sfree = sfull + 2;
    uint64_t* pready = sfree + 2;
    uint64_t* pvdone = pready + 1;
    uint64_t* qload = pvdone + 1;
    uint64_t* qtmem = qload + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_MISC);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int r = blockIdx.y, split = blockIdx.x;
    const int seq = r / p.rows_per_seq;
    const long long lraw = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    const long long len = lraw < p.len_T ? lraw : p.len_T;
    const int* list = p.sel ? p.sel + (long long)r * p.sel_stride : nullptr;
    // Set-up that touches no global memory runs before the wait on the
    // previous kernel (under programmatic launch it overlaps that kernel's
    // tail): the barriers and the tensor memory (see pdl_wait in ptx.cuh for
    // why allocating here cannot deadlock).
    if (tid == 0) {
        for (int b = 0; b < PF_NBUF; ++b) {
            mbar_init(kfull + b, PF_GATHER);  // the gather threads
            mbar_init(kfree + b, 1);          // the P.V commit
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(sfull + b, 1);    // the QK commit
            mbar_init(sfree + b, 128);  // the softmax threads
        }
        mbar_init(pready, 128);
        mbar_init(pvdone, 1);
        mbar_init(qload, 1);
        mbar_init(qtmem, 128);  // the softmax threads, once the query is in tensor memory
        fence_mbar_init();
    }
    if (warp == PF_MMA_WARP) tmem_alloc(tmem_slot, L::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    pdl_trigger();
    if (tid == 0) {
        // the row's absorbed query [64][576]: 9 TMA boxes into the staging tile,
        // issued before the split's range is known (it overlaps that search)
        mbar_expect_tx(qload, AT_CHUNKS * L::CHUNK);
        for (int c = 0; c < AT_CHUNKS; ++c) tma_load2d(sQstage + (uint32_t)c * L::CHUNK, &pp.tm_q, c * 64, r * AT_H, qload);
    }
    // Entry range [e0, e1) of the list (or key range) inside the key window
    // [win_lo, win_hi) — a 32-ary lower-bound search on the ascending list by
    // warps 0 and 1 when the window cuts the row — then this CTA's split of it.
    int* misc = reinterpret_cast<int*>(smem + L::OFF_MISC) + 2;  // [0] e0, [1] e1
    {
        const long long lo_key = p.win_lo > 0 ? p.win_lo : 0;
        const long long hi_key = p.win_hi < len ? p.win_hi : len;
        if (!list) {
            if (tid == 0) {
                misc[0] = (int)lo_key;
                misc[1] = (int)(hi_key > lo_key ? hi_key : lo_key);
            }
        } else {
            const int n = p.sel_n_dev ? __ldg(p.sel_n_dev + r) : p.sel_n;
            if (p.win_lo <= 0 && p.win_hi >= len) {
                if (tid == 0) {
                    misc[0] = 0;
                    misc[1] = n;
                }
            } else if (warp < 2) {
                const long long key = warp == 0 ? lo_key : hi_key;
                int lo = 0, hi = n;  // first position whose key is >= `key` (or n)
                while (hi > lo) {
                    const int step = (hi - lo + 31) / 32;
                    const int pos = lo + lane * step;
                    const bool less = pos < hi && (long long)__ldg(list + pos) < key;
                    const int cnt = __popc(__ballot_sync(0xffffffffu, less));
                    if (cnt == 0) break;
                    const int nlo = lo + (cnt - 1) * step + 1;
                    hi = min(hi, lo + cnt * step);
                    lo = nlo;
                }
                if (lane == 0) misc[warp] = lo;
            }
        }
    }
    __syncthreads();
    int cb, ce;
    {
        const int e0 = misc[0], e1 = max(misc[1], misc[0]);
        if (p.dyn_split) {
            // the entries this rank's window holds, evenly over the row's CTAs
            const int per = (((e1 - e0) + p.max_splits - 1) / p.max_splits + PF_TILE - 1) / PF_TILE * PF_TILE;
            cb = min(e0 + split * per, e1);
            ce = min(cb + per, e1);
        } else if (p.split_keys > 0) {
            cb = e0 + split * p.split_keys;
            ce = min(cb + p.split_keys, e1);
        } else {
            cb = e0;
            ce = split == 0 ? e1 : e0;
        }
        ce = max(ce, cb);
    }
    __syncthreads();  // misc is reused below
    const int n_keys = ce - cb;
    float* ctx = p.o_part + ((long long)r * p.max_splits + split) * (AT_H * AT_DV);
    float* lse_out = p.lse_part + ((long long)r * p.max_splits + split) * AT_H;
    if (n_keys <= 0) {
        // An empty split: lse = -inf marks it; its o is never read (the merge
        // skips parts of weight zero), so it is not written.
        if (tid < AT_H) lse_out[tid] = -INFINITY;
        if (tid == 0) mbar_wait_fast(qload, 0, 39);  // the query copy lands before the CTA leaves
        if (warp == PF_MMA_WARP) {
            tc_fence_after();
            tmem_dealloc(tmem, L::TMEM_COLS);
        }
        return;
    }
    const int n_tiles = (n_keys + PF_TILE - 1) / PF_TILE;
    const __nv_bfloat16* ckv = p.c_kv + (long long)seq * p.ckv_seq;
    const __nv_bfloat16* krt = p.k_rot + (long long)seq * p.krot_seq;

    if (warp >= 4 && warp < PF_MMA_WARP) {
        // ---------------- gather ----------------
        const int g = tid - 128;
        volatile int* go = reinterpret_cast<volatile int*>(tmem_slot + 1);
        auto key_of = [&](int i) -> int {  // this thread's cache row of tile i (g < PF_TILE), -1 past the range
            const int e = i * PF_TILE + g;
            if (g >= PF_TILE || i >= n_tiles || e >= n_keys) return -1;
            const long long key = list ? (long long)__ldg(list + cb + e) : (long long)(cb + e);
            const long long row = key - p.win_lo;  // the cache holds the window's keys
            if (row < 0 || row >= p.T) {
                set_error(ERRC_BOUNDS, 31);
                return -1;
            }
            return (int)row;
        };
        int key_next = key_of(0);  // indices one tile ahead: their load latency hides behind a tile
        for (int i = 0; i < n_tiles; ++i) {
            const int b = i % PF_NBUF;
            // One thread waits for the buffer (and, for the staging tile's first
            // use, for the query to have left it) and tells the others, so that
            // all gather threads leave together on a timeout.
            if (g == 0) {
                bool ok = true;
                if (i >= PF_NBUF) ok = mbar_wait_fast(kfree + b, (uint32_t)(i / PF_NBUF - 1) & 1u, 30);
                else if (b == PF_NBUF - 1) ok = mbar_wait_fast(qtmem, 0, 29);
                *go = ok ? 1 : 0;
            }
            if (g < PF_TILE) rows_sh[b * PF_TILE + g] = key_next;
            asm volatile("bar.sync 2, %0;" ::"n"(PF_GATHER) : "memory");
            if (!*go) break;
            key_next = key_of(i + 1);
            const uint32_t tile = sK + (uint32_t)b * L::TILE;
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
            cp_async_wait_all();
            fence_proxy_async_smem();
            mbar_arrive(kfull + b);
            asm volatile("bar.sync 2, %0;" ::"n"(PF_GATHER) : "memory");  // rows_sh[b] is rewritten PF_NBUF tiles on
        }
    } else if (warp == PF_MMA_WARP) {
        // ---------------- MMA ----------------
        const uint32_t tq = tmem + (16u << 16) + PF_TM_Q;  // the query, A operand of QK
        auto issue_qk = [&](int i) -> bool {
            const int b = i % PF_NBUF, s = i & 1;
            if (!mbar_wait_fast(kfull + b, (uint32_t)(i / PF_NBUF) & 1u, 32)) return false;
            if (i >= 2 && !mbar_wait_fast(sfree + s, (uint32_t)((i >> 1) - 1) & 1u, 33)) return false;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t tile = sK + (uint32_t)b * L::TILE;
                const uint32_t d = tmem + (16u << 16) + (uint32_t)(s * PF_TILE);
#pragma unroll 1
                for (int c = 0; c < AT_CHUNKS; ++c) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)  // K = 16: 8 columns of the query per step
                        mma_bf16_ts(d, tq + (uint32_t)(c * 32 + kk * 8),
                                    desc_sw128(tile + (uint32_t)c * L::CHUNK + kk * 32, 16, 1024), L::IDESC_QK,
                                    (c | kk) != 0 ? 1u : 0u);
                }
                mma_commit(sfull + s);
            }
            __syncwarp();
            return true;
        };
        auto issue_pv = [&](int i) -> bool {
            const int b = i % PF_NBUF;
            if (!mbar_wait_fast(pready, (uint32_t)i & 1u, 34)) return false;
            tc_fence_after();
            if (lane == 0) {
                const uint32_t tile = sK + (uint32_t)b * L::TILE;
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
        bool ok = mbar_wait_fast(qtmem, 0, 38) && issue_qk(0);
        for (int i = 0; ok && i < n_tiles; ++i) {
            if (i + 1 < n_tiles) ok = issue_qk(i + 1);
            if (ok) ok = issue_pv(i);
        }
    } else {
        // ---------------- softmax (warps 0-3) ----------------
        // Thread t < 16 of warp w: head 16 w + t, keys [0, 32) of a tile and O
        // columns [c, c + 32); thread t + 16: the same head, keys [32, 64), O
        // columns [c + 256, c + 288).
        const int h = 16 * warp + (lane & 15);
        const bool hi_half = lane >= 16;
        const uint32_t lane_o = (uint32_t)(32 * warp) << 16, lane_s = (uint32_t)(32 * warp + 16) << 16;
        // The query into tensor memory, lanes 16-31, columns PF_TM_Q + [0, 288):
        // column c = elements (2c, 2c + 1) of the row; thread t < 16 writes
        // columns [16 k, 16 k + 16), thread t + 16 columns 144 + [16 k, 16 k + 16).
        bool ok = mbar_wait_fast(qload, 0, 39);
        if (ok) {
#pragma unroll 1
            for (int k = 0; k < 9; ++k) {
                const int e0 = 32 * k + (hi_half ? 288 : 0);  // first element of this thread's 16 columns
                const uint32_t src = sQstage + (uint32_t)(e0 >> 6) * L::CHUNK + (uint32_t)h * 128u;
                const int seg0 = (e0 & 63) >> 3;             // 16-byte pieces: 8 elements each
                uint32_t v[16];
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 x = lds_v4(src + ((((uint32_t)(seg0 + q)) ^ (uint32_t)h) & 7u) * 16u);
                    v[4 * q] = x.x;
                    v[4 * q + 1] = x.y;
                    v[4 * q + 2] = x.z;
                    v[4 * q + 3] = x.w;
                }
                tmem_st16x2_16u<144>(tmem + lane_s + PF_TM_Q + (uint32_t)(16 * k), v);
            }
            tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(qtmem);  // the MMA may read the query; the staging tile is free for keys
        float m_run = -INFINITY, l_run = 0.f;
        for (int i = 0; i < n_tiles && ok; ++i) {
            const int s = i & 1;
            const int nv = min(PF_TILE, n_keys - i * PF_TILE);
            if (!(ok = mbar_wait_fast(sfull + s, (uint32_t)(i >> 1) & 1u, 35))) break;
            tc_fence_after();
            float sv[32];
            tmem_ld16x2_32<32>(tmem + lane_s + (uint32_t)(s * PF_TILE), sv);
            tc_fence_before();
            mbar_arrive(sfree + s);
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
        const bool done = mbar_wait_fast(pvdone, (uint32_t)(n_tiles - 1) & 1u, 37);
        tc_fence_after();
        if (done && pp.o_tma) {
            // stage: box k = columns [32 k, 32 k + 32), row hq, 16-byte chunks
            // swizzled by the row (every key tile is consumed by now)
            const float inv = inv_l_sh[hq];
#pragma unroll 1
            for (int c = grp * 32; c < 256; c += 32 * ngrp) {
                float ov[32];
                tmem_ld16x2_32<256>(tmem + lane_o + (uint32_t)c, ov);
                const int k = (c >> 5) + (hi ? 8 : 0);
                const uint32_t row = sK + (uint32_t)k * (AT_H * 128) + (uint32_t)hq * 128u;
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    sts_v4(row + ((((uint32_t)j) ^ (uint32_t)hq) & 7u) * 16u,
                           make_uint4(__float_as_uint(ov[4 * j] * inv), __float_as_uint(ov[4 * j + 1] * inv),
                                      __float_as_uint(ov[4 * j + 2] * inv), __float_as_uint(ov[4 * j + 3] * inv)));
            }
            fence_proxy_async_smem();
        } else if (done) {
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
        if (pp.o_tma) {
            asm volatile("bar.sync 3, %0;" ::"n"(PF_MMA_WARP * 32) : "memory");  // the staged boxes are complete
            if (tid == 0 && done) {
                const int row0 = (r * p.max_splits + split) * AT_H;
                for (int k = 0; k < AT_DV / 32; ++k)
                    tma_store2d(&pp.tm_o, 32 * k, row0, sK + (uint32_t)k * (AT_H * 128));
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                // the staging buffer must stay until the copies have read it; the
                // writes themselves complete with the grid
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == PF_MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
}

}  // namespace wl
