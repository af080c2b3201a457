// mla_attn.cuh — sparse absorbed-MLA attention over gathered latent rows.
//
// For query row r, head h and the selected keys t (a canonical ascending list,
// or every key):
//     s[h,t] = (q_abs[h] . c_kv[t] + q_rot[h] . k_rot[t]) * softmax_scale
//     ctx[h] = sum_t softmax_t(s[h,t]) * c_kv[t]
// — the reference's mla_decode_absorbed (src/glm_layer_runner.cuh:251-298)
// with its index mask (src/glm_kernels.cuh:526-545 -> masked keys contribute
// exactly zero), computed only over the selected keys instead of over all T.
//
// One CTA (8 warps) walks a contiguous range of the selection list in tiles of
// 128 keys:
//   gather  — each key's 1152-byte [c_kv | k_rot] bf16 row is copied with
//             16-byte cp.async straight into a 128B-swizzled tile, one commit
//             group per 64-column chunk, so the QK MMAs of chunk c overlap the
//             loads of chunks c+1..8;
//   QK^T    — tcgen05.mma M = 128 keys x N = 64 heads x K = 576, A = the row
//             tile (K-major), B = the absorbed query (K-major), fp32 in TMEM;
//   softmax — two threads own key j's 64 scores (32 heads each, tcgen05.ld), per-head max and
//             sum are warp transpose-reductions, online rescaling across tiles;
//             P (bf16) is written over the consumed k_rot chunk;
//   P.V     — O^T[c,h] += V^T[c,j] P^T[j,h]: M = 128 latent columns (x4),
//             N = 64 heads, K = 128 keys; both operands MN-major views of
//             tiles already in shared memory (the row tile serves as K and V).
// The range's normalised output o[h][c] and lse[h] (natural log) are written
// as one partial; a split-K launch merges partials with lse_merge_kernel.
#pragma once
#include "p2p.cuh"

namespace wl {

constexpr int AT_TILE = 128;
constexpr int AT_H = 64;
constexpr int AT_D = 576;
constexpr int AT_DV = 512;
constexpr int AT_CHUNKS = 9;
constexpr int AT_THREADS = 256;  // 8 warps: two per TMEM lane quarter, splitting the heads

struct AttnLayout {
    static constexpr uint32_t ROW_CHUNK = AT_TILE * 128;  // 16 KB
    static constexpr uint32_t Q_CHUNK = AT_H * 128;       // 8 KB
    static constexpr uint32_t OFF_ROWS = 0;
    static constexpr uint32_t OFF_Q = OFF_ROWS + AT_CHUNKS * ROW_CHUNK;  // 147456
    static constexpr uint32_t OFF_RED = OFF_Q + AT_CHUNKS * Q_CHUNK;     // + 73728
    static constexpr uint32_t OFF_M = OFF_RED + 4 * AT_H * 4;
    static constexpr uint32_t OFF_L = OFF_M + AT_H * 4;
    static constexpr uint32_t OFF_ALPHA = OFF_L + AT_H * 4;
    static constexpr uint32_t OFF_ROWIDX = OFF_ALPHA + AT_H * 4;
    static constexpr uint32_t OFF_BAR = OFF_ROWIDX + AT_TILE * 4;
    static constexpr uint32_t OFF_MISC = OFF_BAR + 16;
    static constexpr uint32_t BYTES = OFF_MISC + 64 + 1024;
    static constexpr uint32_t TMEM_COLS = 512;  // S: [0,64)  O^T: [64, 320)
    static constexpr uint32_t IDESC_QK = idesc_bf16(128, 64, 0, 0);
    static constexpr uint32_t IDESC_PV = idesc_bf16(128, 64, 1, 1);
};

struct AttnParams {
    const __nv_bfloat16* c_kv;
    long long ckv_row, ckv_seq;
    const __nv_bfloat16* k_rot;
    long long krot_row, krot_seq;
    int T;  // cache rows present (this rank's window)
    int n_rows, rows_per_seq, len0, len_step, len_T;  // row lengths clamp to len_T
    const __nv_bfloat16* q_abs;  // [n_rows][64][576]
    const int* sel;              // null: identity
    long long sel_stride;
    const int* sel_n_dev;
    int sel_n;
    long long win_lo, win_hi;
    int split_keys;  // 0: one CTA covers the whole list
    int max_splits;
    float* o_part;
    float* lse_part;
    float scale_log2;
};

// Reduce 64 per-lane values across the warp; lane l ends with heads 2l, 2l+1.
template <bool IS_MAX>
__device__ __forceinline__ void warp_transpose_reduce64(float* v, float& out0, float& out1) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int step = 0; step < 5; ++step) {
        const int half = 32 >> step;  // values kept after this step
        const int off = 16 >> step;
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float a = v[i], b = v[i + half];
            const float send = upper ? a : b;
            const float keep = upper ? b : a;
            const float recv = __shfl_xor_sync(0xffffffffu, send, off);
            v[i] = IS_MAX ? fmaxf(keep, recv) : keep + recv;
        }
    }
    out0 = v[0];
    out1 = v[1];
}

// Reduce 32 per-lane values across the warp; lane l ends with value l.
template <bool IS_MAX>
__device__ __forceinline__ float warp_transpose_reduce32(float* v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int step = 0; step < 5; ++step) {
        const int half = 16 >> step;
        const int off = 16 >> step;
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float a = v[i], b = v[i + half];
            const float send = upper ? a : b;
            const float keep = upper ? b : a;
            const float recv = __shfl_xor_sync(0xffffffffu, send, off);
            v[i] = IS_MAX ? fmaxf(keep, recv) : keep + recv;
        }
    }
    return v[0];
}

__global__ void __launch_bounds__(AT_THREADS, 1) mla_sparse_attn_kernel(AttnParams p) {
    WL_KT_BEGIN(2);
    WL_TA(0);
    pdl_wait();
    pdl_trigger();
    using L = AttnLayout;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sRows = smem_u32(smem + L::OFF_ROWS);
    const uint32_t sQ = smem_u32(smem + L::OFF_Q);
    const uint32_t sP = sRows + 8 * L::ROW_CHUNK;  // P^T over the consumed k_rot chunk
    float* red = reinterpret_cast<float*>(smem + L::OFF_RED);
    float* m_run = reinterpret_cast<float*>(smem + L::OFF_M);
    float* l_run = reinterpret_cast<float*>(smem + L::OFF_L);
    float* alpha = reinterpret_cast<float*>(smem + L::OFF_ALPHA);
    int* row_idx = reinterpret_cast<int*>(smem + L::OFF_ROWIDX);
    uint64_t* bar_mma = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    int* misc = reinterpret_cast<int*>(smem + L::OFF_MISC);  // [0]=cb [1]=ce [2]=tmem [3]=rescale [4,5]=e0,e1

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, hh = warp >> 2;  // TMEM lane quarter; which 32 heads
    const int r = blockIdx.y, s = blockIdx.x;
    const int seq = r / p.rows_per_seq;
    const long long lraw = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    const long long len = lraw < p.len_T ? lraw : p.len_T;
    const int* list = p.sel ? p.sel + (long long)r * p.sel_stride : nullptr;

    // Entry range [e0, e1) of the list inside the key window. A window that
    // covers the whole row needs no search (canonical lists lie in [0, len));
    // otherwise warps 0 and 1 each run a 32-ary lower-bound search.
    {
        const long long lo_key = p.win_lo > 0 ? p.win_lo : 0;
        const long long hi_key = p.win_hi < len ? p.win_hi : len;
        if (!list) {
            if (tid == 0) {
                misc[4] = (int)lo_key;
                misc[5] = (int)(hi_key > lo_key ? hi_key : lo_key);
            }
        } else {
            const int n = p.sel_n_dev ? __ldg(p.sel_n_dev + r) : p.sel_n;
            if (p.win_lo <= 0 && p.win_hi >= len) {
                if (tid == 0) {
                    misc[4] = 0;
                    misc[5] = n;
                }
            } else if (warp < 2) {
                const long long key = warp == 0 ? lo_key : hi_key;
                // lower bound: first position whose key is >= `key` (or n)
                int lo = 0, hi = n;
                while (hi > lo) {
                    const int step = (hi - lo + 31) / 32;
                    const int pos = lo + lane * step;
                    const bool less = pos < hi && (long long)__ldg(list + pos) < key;
                    const int cnt = __popc(__ballot_sync(0xffffffffu, less));  // ascending list
                    if (cnt == 0) break;
                    const int nlo = lo + (cnt - 1) * step + 1;
                    hi = min(hi, lo + cnt * step);
                    lo = nlo;
                }
                if (lane == 0) misc[4 + warp] = lo;
            }
        }
        __syncthreads();
        if (tid == 0) {
            const long long e0 = misc[4];
            long long e1 = misc[5];
            if (e1 < e0) e1 = e0;
            long long cb, ce;
            if (p.split_keys > 0) {
                cb = e0 + (long long)s * p.split_keys;
                ce = cb + p.split_keys < e1 ? cb + p.split_keys : e1;
            } else {
                cb = e0;
                ce = (s == 0) ? e1 : e0;
            }
            misc[0] = (int)cb;
            misc[1] = (int)(ce > cb ? ce : cb);
        }
    }
    __syncthreads();
    const int cb = misc[0], ce = misc[1];
    WL_TA(1);
    float* o_out = p.o_part + ((long long)r * p.max_splits + s) * (AT_H * AT_DV);
    float* lse_out = p.lse_part + ((long long)r * p.max_splits + s) * AT_H;
    if (cb >= ce) {  // empty range: a zero partial with weight e^-inf
        for (int i = tid; i < AT_H * AT_DV / 4; i += AT_THREADS)
            reinterpret_cast<float4*>(o_out)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tid < AT_H) lse_out[tid] = -INFINITY;
        return;
    }

    if (tid == 0) {
        mbar_init(bar_mma, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(reinterpret_cast<uint32_t*>(misc + 2), L::TMEM_COLS);
    if (tid < AT_H) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.f;
    }
    // Absorbed query [64][576] -> 9 swizzled K-major chunks (commit group 0).
    {
        const __nv_bfloat16* q = p.q_abs + (long long)r * AT_H * AT_D;
        for (int pid = tid; pid < AT_H * 72; pid += AT_THREADS) {
            const int h = pid / 72, pp = pid % 72;
            cp_async16(sQ + (uint32_t)(pp >> 3) * L::Q_CHUNK + sw128_off(h, pp & 7),
                       q + (long long)h * AT_D + pp * 8, 16);
        }
        cp_async_commit();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    WL_TA(2);
    const uint32_t tmem = (uint32_t)misc[2];
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem, tO = tmem + 64;

    const __nv_bfloat16* ckv = p.c_kv + (long long)seq * p.ckv_seq;
    const __nv_bfloat16* krt = p.k_rot + (long long)seq * p.krot_seq;
    uint32_t phase = 0;
    bool ok = true;
    const int n_tiles = (ce - cb + AT_TILE - 1) / AT_TILE;

#pragma unroll 1
    for (int it = 0; it < n_tiles; ++it) {
        const int tb = cb + it * AT_TILE;
        const int nv = min(AT_TILE, ce - tb);
        if (tid < AT_TILE) {
            int row = -1;
            if (tid < nv) {
                const long long key = list ? (long long)list[tb + tid] : (long long)(tb + tid);
                const long long rr = key - p.win_lo;
                if (rr < 0 || rr >= p.T) set_error(ERRC_BOUNDS, 3);
                else row = (int)rr;
            }
            row_idx[tid] = row;
        }
        __syncthreads();
        // Gather: chunk c of row j = 8 pieces of 16 B; zero-fill rows past nv.
#pragma unroll 1
        for (int c = 0; c < AT_CHUNKS; ++c) {
#pragma unroll
            for (int k2 = 0; k2 < AT_TILE * 8 / AT_THREADS; ++k2) {
                const int pid = k2 * AT_THREADS + tid;
                const int j = pid >> 3, seg = pid & 7;
                const int row = row_idx[j];
                const __nv_bfloat16* src =
                    (c < 8) ? ckv + (long long)(row < 0 ? 0 : row) * p.ckv_row + c * 64 + seg * 8
                            : krt + (long long)(row < 0 ? 0 : row) * p.krot_row + seg * 8;
                cp_async16(sRows + (uint32_t)c * L::ROW_CHUNK + sw128_off(j, seg), src, row < 0 ? 0u : 16u);
            }
            cp_async_commit();
        }
        WL_TA(3);
        // QK^T chunk by chunk as the loads land.
#pragma unroll 1
        for (int c = 0; c < AT_CHUNKS; ++c) {
            switch (c) {
                case 0: cp_async_wait<8>(); break;
                case 1: cp_async_wait<7>(); break;
                case 2: cp_async_wait<6>(); break;
                case 3: cp_async_wait<5>(); break;
                case 4: cp_async_wait<4>(); break;
                case 5: cp_async_wait<3>(); break;
                case 6: cp_async_wait<2>(); break;
                case 7: cp_async_wait<1>(); break;
                default: cp_async_wait<0>(); break;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid == 0) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t ad = desc_sw128(sRows + (uint32_t)c * L::ROW_CHUNK + kk * 32, 16, 1024);
                    const uint64_t bd = desc_sw128(sQ + (uint32_t)c * L::Q_CHUNK + kk * 32, 16, 1024);
                    mma_bf16(tS, ad, bd, L::IDESC_QK, (c | kk) != 0 ? 1u : 0u);
                }
                if (c == AT_CHUNKS - 1) mma_commit(bar_mma);
            }
        }
        ok = mbar_wait(bar_mma, phase, 4);
        phase ^= 1;
        if (!__syncthreads_and(ok)) break;
        tc_fence_after();
        WL_TA(4);

        // ---- softmax over this tile (log2 domain) ----
        // Thread: key j = quarter * 32 + lane, heads [32 hh, 32 hh + 32).
        const int j = quarter * 32 + lane;
        float sv[32];
        tmem_ld32(tS + lane_base + (uint32_t)(hh * 32), sv);
        const bool valid = j < nv;
#pragma unroll
        for (int h = 0; h < 32; ++h) sv[h] = valid ? sv[h] * p.scale_log2 : -INFINITY;
        {
            float tmp[32];
#pragma unroll
            for (int h = 0; h < 32; ++h) tmp[h] = sv[h];
            red[quarter * 64 + hh * 32 + lane] = warp_transpose_reduce32<true>(tmp);
        }
        __syncthreads();
        if (tid < AT_H) {
            const float mt = fmaxf(fmaxf(red[tid], red[64 + tid]), fmaxf(red[128 + tid], red[192 + tid]));
            const float mo = m_run[tid];
            const float mn = fmaxf(mo, mt);
            alpha[tid] = exp2f(mo - mn);  // 0 on the first tile
            m_run[tid] = mn;
        }
        if (tid == 0) misc[3] = 0;
        __syncthreads();
        if (tid < AT_H && it > 0 && alpha[tid] != 1.f) misc[3] = 1;
        // P = exp2(s - m), rounded to bf16; row j = this thread's key.
        {
            float ps[32];
#pragma unroll
            for (int pc = 0; pc < 4; ++pc) {
                uint32_t w4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int hl = pc * 8 + e * 2, h = hh * 32 + hl;
                    const __nv_bfloat162 b2 =
                        __floats2bfloat162_rn(exp2f(sv[hl] - m_run[h]), exp2f(sv[hl + 1] - m_run[h + 1]));
                    w4[e] = *reinterpret_cast<const uint32_t*>(&b2);
                    ps[hl] = __low2float(b2);
                    ps[hl + 1] = __high2float(b2);
                }
                sts_v4(sP + sw128_off(j, hh * 4 + pc), make_uint4(w4[0], w4[1], w4[2], w4[3]));
            }
            // red[] was last read (the max) before the barrier above
            red[quarter * 64 + hh * 32 + lane] = warp_transpose_reduce32<false>(ps);
        }
        __syncthreads();
        if (tid < AT_H)
            l_run[tid] = alpha[tid] * l_run[tid] + ((red[tid] + red[64 + tid]) + (red[128 + tid] + red[192 + tid]));
        // Rescale the running O^T (lane = latent column, column = head).
        if (misc[3]) {
#pragma unroll 1
            for (int q = 2 * hh; q < 2 * hh + 2; ++q) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    float ov[32];
                    const uint32_t ta = tO + lane_base + (uint32_t)(q * 64 + hf * 32);
                    tmem_ld32(ta, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] *= alpha[hf * 32 + i];
                    tmem_st32(ta, ov);
                }
            }
            tmem_wait_st();
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        WL_TA(5);
        if (tid == 0) {
#pragma unroll 1
            for (int q = 0; q < 4; ++q) {
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint64_t ad = desc_sw128(sRows + (uint32_t)(2 * q) * L::ROW_CHUNK + ks * 2048,
                                                   L::ROW_CHUNK, 1024);
                    const uint64_t bd = desc_sw128(sP + ks * 2048, 0, 1024);
                    mma_bf16(tO + q * 64, ad, bd, L::IDESC_PV, (it > 0 || ks > 0) ? 1u : 0u);
                }
            }
            mma_commit(bar_mma);
        }
        ok = mbar_wait(bar_mma, phase, 5);
        phase ^= 1;
        if (!__syncthreads_and(ok)) break;
        tc_fence_after();
        WL_TA(6);
    }

    if (ok) {
        if (tid < AT_H) alpha[tid] = 1.f / l_run[tid];  // reuse: 1/l per head
        __syncthreads();
        // o[h][c] = O^T[c][h] / l[h], staged in shared memory over the (consumed)
        // row tile in the partial's own [h][c] layout, then copied out with
        // coalesced 16-byte stores. Lane = latent column c within chunk q.
        float* stage = reinterpret_cast<float*>(smem + L::OFF_ROWS);
#pragma unroll 1
        for (int q = 2 * hh; q < 2 * hh + 2; ++q) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                float ov[32];
                tmem_ld32(tO + lane_base + (uint32_t)(q * 64 + hf * 32), ov);
                const int c = q * 128 + quarter * 32 + lane;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const int h = hf * 32 + i;
                    stage[h * AT_DV + c] = ov[i] * alpha[h];
                }
            }
        }
        __syncthreads();
        const float4* st4 = reinterpret_cast<const float4*>(stage);
        float4* o4 = reinterpret_cast<float4*>(o_out);
#pragma unroll 4
        for (int i = tid; i < AT_H * AT_DV / 4; i += AT_THREADS) o4[i] = st4[i];
        if (tid < AT_H) lse_out[tid] = (m_run[tid] + log2f(l_run[tid])) * 0.69314718055994531f;
        WL_TA(7);
    } else {
        cp_async_wait_all();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, L::TMEM_COLS);
    }
    WL_KT_END(2);
}

// ---- (o, lse) merge ---------------------------------------------------------------
struct MergeParams {
    const float* o_part;
    const float* lse_part;
    int n_rows, n_parts;
    long long row_stride, part_stride, lse_row_stride, lse_part_stride;
    int n_heads, dv;
    float* ctx;
    float* lse;
    long long ctx_row_stride;  // floats between rows of ctx (n_heads * dv when dense)
    long long lse_out_row_stride;  // floats between rows of lse (n_heads when dense)
    // Parts arriving through the peer exchange (ll.base set): o_part / lse_part
    // are unused; part s's o words start at slot s, its lse words ll_lse_off on.
    P2PRecv ll;
    long long ll_lse_off;
};

// grid (n_heads, dv / 128, n_rows), 32 threads: lane l owns 4 latent columns.
// Up to 32 parts: lane s holds part s's lse; all parts' columns load at once.
template <bool LL>
__global__ void __launch_bounds__(32) lse_merge_kernel(MergeParams p) {
    WL_KT_BEGIN(3);
    pdl_wait();
    pdl_trigger();
    const int h = blockIdx.x, q = blockIdx.y, r = blockIdx.z, lane = threadIdx.x;
    const int c = q * 128 + lane * 4;
    constexpr bool ll = LL;  // parts arrive through the peer exchange (p.ll)
    const uint32_t epoch = ll ? p2p_epoch(p.ll) : 0u;
    const uint64_t* lb = ll ? p2p_slot(p.ll, epoch, 0) : nullptr;
    float ls = -INFINITY;
    if (lane < p.n_parts) {
        const long long li = (long long)r * p.lse_row_stride + h + (long long)lane * p.lse_part_stride;
        ls = ll ? __uint_as_float(ll_wait1(lb + p.ll_lse_off + li, epoch, ll_load1_raw(lb + p.ll_lse_off + li), 21))
                : p.lse_part[li];
    }
    float M = ls;
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float wl = (M == -INFINITY || ls == -INFINITY) ? 0.f : exp2f((ls - M) * 1.4426950408889634f);
    float W = wl;
    for (int o = 16; o > 0; o >>= 1) W += __shfl_xor_sync(0xffffffffu, W, o);
    const float inv = W > 0.f ? 1.f / W : 0.f;
    const long long oi = (long long)r * p.row_stride + (long long)h * p.dv + c;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // Parts in groups of 8: all loads of a group are issued before any use.
    for (int s0 = 0; s0 < p.n_parts; s0 += 8) {
        float4 v[8];
        float wv[8];
        uint64_t raw[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int s = s0 + j;
            wv[j] = __shfl_sync(0xffffffffu, wl, s & 31) * inv;
            const bool use = s < p.n_parts && wv[j] != 0.f;  // empty parts are never read
            if (!use) wv[j] = 0.f;
            v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (use) {
                const long long si = oi + (long long)s * p.part_stride;
                if constexpr (LL) {  // raw words now (all loads in flight), tags checked below
                    uint64_t w0, w1, w2, w3;
                    ll_load2_raw(lb + si, w0, w1);
                    ll_load2_raw(lb + si + 2, w2, w3);
                    raw[j][0] = w0;
                    raw[j][1] = w1;
                    raw[j][2] = w2;
                    raw[j][3] = w3;
                } else {
                    v[j] = *reinterpret_cast<const float4*>(p.o_part + si);
                }
            }
        }
        if constexpr (LL) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (wv[j] == 0.f) continue;
                const uint64_t* w = lb + oi + (long long)(s0 + j) * p.part_stride;
                v[j] = make_float4(__uint_as_float(ll_wait1(w, epoch, raw[j][0], 21)),
                                   __uint_as_float(ll_wait1(w + 1, epoch, raw[j][1], 21)),
                                   __uint_as_float(ll_wait1(w + 2, epoch, raw[j][2], 21)),
                                   __uint_as_float(ll_wait1(w + 3, epoch, raw[j][3], 21)));
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            acc.x = fmaf(wv[j], v[j].x, acc.x);
            acc.y = fmaf(wv[j], v[j].y, acc.y);
            acc.z = fmaf(wv[j], v[j].z, acc.z);
            acc.w = fmaf(wv[j], v[j].w, acc.w);
        }
    }
    *reinterpret_cast<float4*>(p.ctx + (long long)r * p.ctx_row_stride + (long long)h * p.dv + c) = acc;
    if (q == 0 && lane == 0 && p.lse)
        p.lse[(long long)r * p.lse_out_row_stride + h] = (W > 0.f) ? M + logf(W) : -INFINITY;
    WL_KT_END(3);
}

}  // namespace wl
