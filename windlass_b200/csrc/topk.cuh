// topk.cuh — exact per-row top-k key selection and index-list normalisation.
//
// Semantics (the reference's indexer_topk, src/glm_kernels.cuh:344-414, and
// numpy's argsort(-index, kind="stable")[:k], tools/ref_glm_chain.py:504-515):
//   * k' = min(k, len); k' >= len returns every key 0..len-1;
//   * otherwise the k' largest scores, ties at the k-th value broken toward
//     the LOWEST key index (the stable argsort's rule and the reference
//     kernel's serial tie fill);
//   * -0.0 and +0.0 compare equal (as they do for numpy).
// The selected SET is what the reference specifies (it scatters the list into
// a mask, glm_kernels.cuh:526-537); this kernel writes it in ascending key
// order, which is the order the sparse attention consumes.
//
// Algorithm: MSD radix select on an order-preserving 32-bit key of each score
// (11 + 11 + 10 bits, shared-memory histograms), giving the exact k-th key
// `thr` and how many elements equal to it are needed; then one ordered pass
// emits, in index order, every element above thr and the first `need` equal
// to it, positions from a block-wide exclusive scan. No sort.
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int TOPK_THREADS = 1024;

__device__ __forceinline__ uint32_t ordered_key(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u << 1) == 0u) u = 0u;  // -0 == +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive scan over the block (blockDim.x == 1024). Returns the exclusive
// prefix of `v`; *total gets the block sum. `sh` holds >= 33 words.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* sh, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = sh[lane];
        uint32_t z = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, z, o);
            if (lane >= o) z += y;
        }
        sh[lane] = z - w;  // exclusive prefix of warp sums
        if (lane == 31) sh[32] = z;
    }
    __syncthreads();
    const uint32_t r = sh[warp] + x - v;
    *total = sh[32];
    __syncthreads();
    return r;
}

struct TopkParams {
    const float* in;
    long long in_stride;
    int n_rows, rows_per_seq, len0, len_step, T;
    int k;
    const int* cand_idx;  // optional; same layout as `in`
    int* out;
    long long out_stride;
    int* n_out;  // optional [n_rows]
};

__global__ void __launch_bounds__(TOPK_THREADS) topk_kernel(TopkParams p) {
    __shared__ uint32_t hist[2048];
    __shared__ uint32_t scan_sh[33];
    __shared__ uint32_t sel_bin, sel_above;

    const int r = blockIdx.x, tid = threadIdx.x;
    const long long lraw = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    const int len = (int)(lraw < p.T ? lraw : p.T);
    const int kk = min(p.k, len);
    const float* in = p.in + (long long)r * p.in_stride;
    const int* cidx = p.cand_idx ? p.cand_idx + (long long)r * p.in_stride : nullptr;
    int* out = p.out + (long long)r * p.out_stride;
    if (p.n_out && tid == 0) p.n_out[r] = kk;
    if (kk <= 0) return;
    if (kk >= len) {
        for (int i = tid; i < len; i += TOPK_THREADS) out[i] = cidx ? cidx[i] : i;
        return;
    }

    // ---- radix select: 3 passes, 11/11/10 bits ----
    uint32_t prefix = 0, mask_hi = 0, remaining = (uint32_t)kk;
#pragma unroll 1
    for (int pass = 0; pass < 3; ++pass) {
        const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
        const int nb = pass == 2 ? 1024 : 2048;
        for (int i = tid; i < nb; i += TOPK_THREADS) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < len; i += TOPK_THREADS) {
            const uint32_t u = ordered_key(in[i]);
            if ((u & mask_hi) == prefix) atomicAdd(&hist[(u >> shift) & (uint32_t)(nb - 1)], 1u);
        }
        __syncthreads();
        // Bins from the top: thread t owns bins nb-1-t*per .. (per bins).
        const int per = nb / TOPK_THREADS;
        uint32_t mine = 0;
        for (int j = 0; j < per; ++j) mine += hist[nb - 1 - tid * per - j];
        uint32_t tot;
        uint32_t above = block_excl_scan(mine, scan_sh, &tot);
        for (int j = 0; j < per; ++j) {
            const int b = nb - 1 - tid * per - j;
            const uint32_t c = hist[b];
            if (above < remaining && remaining <= above + c) {
                sel_bin = (uint32_t)b;
                sel_above = above;
            }
            above += c;
        }
        __syncthreads();
        prefix |= sel_bin << shift;
        mask_hi |= (uint32_t)(nb - 1) << shift;
        remaining -= sel_above;
        __syncthreads();
    }
    const uint32_t thr = prefix;
    const uint32_t need = remaining;  // >= 1 elements equal to thr to take
    const uint32_t total_gt = (uint32_t)kk - need;

    // ---- ordered emission: 4 consecutive elements per thread per round ----
    uint32_t carry_gt = 0, carry_eq = 0;
#pragma unroll 1
    for (int base = 0; base < len; base += 4 * TOPK_THREADS) {
        const int i0 = base + tid * 4;
        uint32_t flags = 0;  // bit 2j: gt, bit 2j+1: eq
        uint32_t ngt = 0, neq = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = i0 + j;
            if (i < len) {
                const uint32_t u = ordered_key(in[i]);
                if (u > thr) { flags |= 1u << (2 * j); ++ngt; }
                else if (u == thr) { flags |= 2u << (2 * j); ++neq; }
            }
        }
        uint32_t tot;
        const uint32_t ex = block_excl_scan((neq << 16) | ngt, scan_sh, &tot);
        uint32_t gt_b = carry_gt + (ex & 0xffffu);
        uint32_t eq_b = carry_eq + (ex >> 16);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = i0 + j;
            if (flags & (1u << (2 * j))) {
                out[gt_b + min(eq_b, need)] = cidx ? cidx[i] : i;
                ++gt_b;
            } else if (flags & (2u << (2 * j))) {
                if (eq_b < need) out[gt_b + eq_b] = cidx ? cidx[i] : i;
                ++eq_b;
            }
        }
        carry_gt += tot & 0xffffu;
        carry_eq += tot >> 16;
        if (carry_gt >= total_gt && carry_eq >= need) break;  // uniform
    }
}

// ---- normalisation of an arbitrary index list ---------------------------------
// Keeps key t in [0, len) iff some entry equals t: the mask the reference builds
// (index_mask_fill + index_mask_scatter, glm_kernels.cuh:526-537) read back as a
// list. Bitmap in dynamic shared memory: ceil(len/32) words.
struct NormParams {
    const int* in;
    long long in_stride;
    const int* n_in_dev;
    int n_in;
    int n_rows, rows_per_seq, len0, len_step, T;
    int* out;
    long long out_stride;
    int* n_out;
};

__global__ void __launch_bounds__(TOPK_THREADS) sel_normalize_kernel(NormParams p) {
    extern __shared__ uint32_t bm[];
    __shared__ uint32_t scan_sh[33];
    const int r = blockIdx.x, tid = threadIdx.x;
    const long long lraw = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    const int len = (int)(lraw < p.T ? lraw : p.T);
    const int nw = (len + 31) >> 5;
    const int n = p.n_in_dev ? p.n_in_dev[r] : p.n_in;
    const int* in = p.in + (long long)r * p.in_stride;
    int* out = p.out + (long long)r * p.out_stride;
    for (int i = tid; i < nw; i += TOPK_THREADS) bm[i] = 0;
    __syncthreads();
    for (int e = tid; e < n; e += TOPK_THREADS) {
        const int v = in[e];
        if (v >= 0 && v < len) atomicOr(&bm[v >> 5], 1u << (v & 31));
    }
    __syncthreads();
    uint32_t carry = 0;
    for (int base = 0; base < nw; base += TOPK_THREADS) {
        const int wi = base + tid;
        uint32_t word = wi < nw ? bm[wi] : 0u;
        uint32_t tot;
        uint32_t pos = carry + block_excl_scan((uint32_t)__popc(word), scan_sh, &tot);
        while (word) {
            const int b = __ffs(word) - 1;
            out[pos++] = wi * 32 + b;
            word &= word - 1;
        }
        carry += tot;
    }
    if (tid == 0 && p.n_out) p.n_out[r] = (int)carry;
}

}  // namespace wl
