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
// This file holds what the attention kernels share — shapes, AttnParams — and
// the split-K (o, lse) merge; the attention itself is mla_attn64_kernel
// (mla_attn64.cuh): the 64 heads of a query row as the MMA's M dimension,
// pipelined over 64-key tiles of the row's selection or of a split of it.
#pragma once
#include "p2p.cuh"

namespace wl {

constexpr int AT_TILE = 64;  // split-K ranges are multiples of this many keys (one tile)
constexpr int AT_H = 64;
constexpr int AT_D = 576;
constexpr int AT_DV = 512;
constexpr int AT_CHUNKS = 9;

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
    int dyn_split;   // 1: split_keys ignored; the window's entries spread evenly over the
                     //    max_splits CTAs of the row, in multiples of 64 keys
    int max_splits;
    float* o_part;
    float* lse_part;
    float scale_log2;
};

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
    // Parts in groups of G (16 plain, 8 in the exchange format): all loads of a
    // group are issued before any use, so a row of up to 16 splits costs one
    // round of L2 latency.
    constexpr int G = LL ? 8 : 16;
    for (int s0 = 0; s0 < p.n_parts; s0 += G) {
        float4 v[G];
        float wv[G];
        uint64_t raw[LL ? G : 1][4];
#pragma unroll
        for (int j = 0; j < G; ++j) {
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
            for (int j = 0; j < G; ++j) {
                if (wv[j] == 0.f) continue;
                const uint64_t* w = lb + oi + (long long)(s0 + j) * p.part_stride;
                v[j] = make_float4(__uint_as_float(ll_wait1(w, epoch, raw[j][0], 21)),
                                   __uint_as_float(ll_wait1(w + 1, epoch, raw[j][1], 21)),
                                   __uint_as_float(ll_wait1(w + 2, epoch, raw[j][2], 21)),
                                   __uint_as_float(ll_wait1(w + 3, epoch, raw[j][3], 21)));
            }
        }
#pragma unroll
        for (int j = 0; j < G; ++j) {
            acc.x = fmaf(wv[j], v[j].x, acc.x);
            acc.y = fmaf(wv[j], v[j].y, acc.y);
            acc.z = fmaf(wv[j], v[j].z, acc.z);
            acc.w = fmaf(wv[j], v[j].w, acc.w);
        }
    }
    *reinterpret_cast<float4*>(p.ctx + (long long)r * p.ctx_row_stride + (long long)h * p.dv + c) = acc;
    if (q == 0 && lane == 0 && p.lse)
        p.lse[(long long)r * p.lse_out_row_stride + h] = (W > 0.f) ? M + logf(W) : -INFINITY;
}

// The same merge for parts in plain memory with four warps per (row, head,
// 128 columns): warp w loads and weighs parts w, w + 4, ... (at most 8, all in
// flight at once), then warp 0 adds the four partial sums in warp order. A
// row's partials cost one round of load latency on four times the threads.
constexpr int MG_WARPS = 4;
__global__ void __launch_bounds__(32 * MG_WARPS) lse_merge4_kernel(MergeParams p) {
    pdl_wait();
    pdl_trigger();
    __shared__ float4 part[MG_WARPS - 1][32];
    const int h = blockIdx.x, q = blockIdx.y, r = blockIdx.z, lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
    const int c = q * 128 + lane * 4;
    float ls = -INFINITY;
    if (lane < p.n_parts) ls = p.lse_part[(long long)r * p.lse_row_stride + h + (long long)lane * p.lse_part_stride];
    float M = ls;
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float wl = (M == -INFINITY || ls == -INFINITY) ? 0.f : exp2f((ls - M) * 1.4426950408889634f);
    float W = wl;
    for (int o = 16; o > 0; o >>= 1) W += __shfl_xor_sync(0xffffffffu, W, o);
    const float inv = W > 0.f ? 1.f / W : 0.f;
    const long long oi = (long long)r * p.row_stride + (long long)h * p.dv + c;
    constexpr int G = 32 / MG_WARPS;
    float4 v[G];
    float wv[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        const int s = wi + MG_WARPS * j;
        wv[j] = __shfl_sync(0xffffffffu, wl, s) * inv;
        if (s >= p.n_parts) wv[j] = 0.f;
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (wv[j] != 0.f) v[j] = *reinterpret_cast<const float4*>(p.o_part + oi + (long long)s * p.part_stride);
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < G; ++j) {
        acc.x = fmaf(wv[j], v[j].x, acc.x);
        acc.y = fmaf(wv[j], v[j].y, acc.y);
        acc.z = fmaf(wv[j], v[j].z, acc.z);
        acc.w = fmaf(wv[j], v[j].w, acc.w);
    }
    if (wi > 0) part[wi - 1][lane] = acc;
    __syncthreads();
    if (wi == 0) {
#pragma unroll
        for (int w = 0; w < MG_WARPS - 1; ++w) {
            const float4 o = part[w][lane];
            acc.x += o.x;
            acc.y += o.y;
            acc.z += o.z;
            acc.w += o.w;
        }
        *reinterpret_cast<float4*>(p.ctx + (long long)r * p.ctx_row_stride + (long long)h * p.dv + c) = acc;
        if (q == 0 && lane == 0 && p.lse)
            p.lse[(long long)r * p.lse_out_row_stride + h] = (W > 0.f) ? M + logf(W) : -INFINITY;
    }
}

}  // namespace wl
