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
#include "p2p.cuh"

namespace wl {

constexpr int TOPK_THREADS = 1024;

__device__ __forceinline__ uint32_t ordered_key(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u << 1) == 0u) u = 0u;  // -0 == +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive scan over the block (blockDim.x a multiple of 32, <= 1024).
// Returns the exclusive prefix of `v`; *total gets the block sum. `sh` holds
// >= 33 words.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* sh, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) sh[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = lane < nw ? sh[lane] : 0u;
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

// Find the bin b (scanning from the top) where the running count crosses
// `need`: count(bins > b) < need <= count(bins >= b). Every thread returns
// (b, count(bins > b)). Two levels, bank-conflict free: warps sum groups of 32
// bins (coalesced reads; `h` may be global or shared), warp 0 scans the group
// sums from the top and then the 32 bins of the crossing group.
// nb a multiple of 32 and <= 32 * 1024; `coarse` holds nb / 32 words.
__device__ __forceinline__ void find_bin_from_top(const uint32_t* h, int nb, uint32_t need, uint32_t* coarse,
                                                  uint32_t* sel, uint32_t* out_bin, uint32_t* out_above) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int ng = nb >> 5;
    for (int g = warp; g < ng; g += nw) {
        uint32_t v = h[g * 32 + lane];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) coarse[g] = v;
    }
    __syncthreads();
    if (warp == 0) {
        const int per = (ng + 31) >> 5;  // consecutive groups (from the top) per lane
        uint32_t mine = 0;
        for (int j = 0; j < per; ++j) {
            const int jj = (j + lane) % per;  // rotated reads
            const int g = ng - 1 - (lane * per + jj);
            if (g >= 0) mine += coarse[g];
        }
        uint32_t incl = mine;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const uint32_t excl = incl - mine;
        const unsigned who = __ballot_sync(0xffffffffu, excl < need && need <= incl);
        const int src = __ffs(who) - 1;
        int gsel = 0;
        uint32_t above_g = 0;
        if (lane == src) {
            uint32_t run = excl;
            for (int j = 0; j < per; ++j) {
                const int g = ng - 1 - (lane * per + j);
                if (g < 0) break;
                const uint32_t c = coarse[g];
                if (run < need && need <= run + c) {
                    gsel = g;
                    above_g = run;
                    break;
                }
                run += c;
            }
        }
        gsel = __shfl_sync(0xffffffffu, gsel, src);
        above_g = __shfl_sync(0xffffffffu, above_g, src);
        // bins of the group from the top: lane l holds bin gsel*32 + 31 - l
        const uint32_t c = h[gsel * 32 + 31 - lane];
        uint32_t inc = c;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        const uint32_t ex = above_g + inc - c;
        const unsigned hit = __ballot_sync(0xffffffffu, ex < need && need <= ex + c);
        const int l = __ffs(hit) - 1;
        if (lane == l) {
            sel[0] = (uint32_t)(gsel * 32 + 31 - l);
            sel[1] = ex;
        }
    }
    __syncthreads();
    *out_bin = sel[0];
    *out_above = sel[1];
    __syncthreads();
}

// Writes the selected elements of one row segment in index order: `gt_b0` /
// `eq_b0` are the counts of keys > thr / == thr before the segment; output
// position = (#gt before) + min(#eq before, need).
template <int NT>
__device__ __forceinline__ void emit_segment(const float* in, const int* cidx, int lo, int hi, uint32_t thr,
                                             uint32_t need, uint32_t gt_b0, uint32_t eq_b0, uint32_t total_gt,
                                             int* out, uint32_t* scan_sh) {
    const int tid = threadIdx.x;
#pragma unroll 1
    for (int base = lo; base < hi; base += 4 * NT) {
        const int i0 = base + tid * 4;
        uint32_t flags = 0, ngt = 0, neq = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = i0 + j;
            if (i < hi) {
                const uint32_t u = ordered_key(in[i]);
                if (u > thr) { flags |= 1u << (2 * j); ++ngt; }
                else if (u == thr) { flags |= 2u << (2 * j); ++neq; }
            }
        }
        uint32_t tot;
        const uint32_t ex = block_excl_scan((neq << 16) | ngt, scan_sh, &tot);
        uint32_t gt_b = gt_b0 + (ex & 0xffffu);
        uint32_t eq_b = eq_b0 + (ex >> 16);
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
        gt_b0 += tot & 0xffffu;
        eq_b0 += tot >> 16;
        if (gt_b0 >= total_gt && eq_b0 >= need) break;  // uniform: nothing left to emit
    }
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
    // Segmented rows (topk_reg_kernel only): seg_len > 0 places element i of a
    // row at row_base + (i / seg_len) * seg_stride + i % seg_len — e.g. the
    // [rank][row][k] result of an all-gather read as rows of rank * k entries.
    int seg_len;
    long long seg_stride;
    // Rows arriving through the peer exchange (topk_reg_kernel only; ll.base
    // set): `in` / `cand_idx` are unused, row r's score words start at slot 0
    // + r * in_stride (segments = slots), its index words ll_idx_off further on.
    P2PRecv ll;
    long long ll_idx_off;
};

// Optional candidate outputs of a selection (the sharded decode's exchange
// format): output position pos of row r also gets score[r * stride + pos] (the
// selected score) and gidx[r * stride + pos] = base + key index; positions
// [k', k) are padded with (-inf, INT_MAX).
struct CandOut {
    float* score;
    int* gidx;
    long long stride;
    int k;
    long long base;
};

// Inverse of ordered_key (-0 comes back as +0).
__device__ __forceinline__ float key_to_float(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

__device__ __forceinline__ void cand_pad(const CandOut& co, int r, int from, int tid, int nt) {
    if (!co.score) return;
    for (int pos = from + tid; pos < co.k; pos += nt) {
        co.score[(long long)r * co.stride + pos] = -INFINITY;
        co.gidx[(long long)r * co.stride + pos] = 0x7fffffff;
    }
}

// One CTA per row. Rows of up to TOPK_SMEM_MAX elements are staged once in
// shared memory and every pass reads them from there.
constexpr int TOPK_SMEM_MAX = 40960;

__global__ void __launch_bounds__(TOPK_THREADS) topk_kernel(TopkParams p) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float srow[];
    __shared__ uint32_t hist[2048];
    __shared__ uint32_t scan_sh[33];
    __shared__ uint32_t coarse[64], sel2[2];

    const int r = blockIdx.x, tid = threadIdx.x;
    const long long lraw = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    const int len = (int)(lraw < p.T ? lraw : p.T);
    const int kk = min(p.k, len);
    const float* gin = p.in + (long long)r * p.in_stride;
    const int* cidx = p.cand_idx ? p.cand_idx + (long long)r * p.in_stride : nullptr;
    int* out = p.out + (long long)r * p.out_stride;
    if (p.n_out && tid == 0) p.n_out[r] = kk;
    if (kk <= 0) return;
    if (kk >= len) {
        for (int i = tid; i < len; i += TOPK_THREADS) out[i] = cidx ? cidx[i] : i;
        return;
    }
    const bool staged = len <= TOPK_SMEM_MAX;
    if (staged) {
        for (int i = tid; i < len; i += TOPK_THREADS) srow[i] = gin[i];
        __syncthreads();
    }
    const float* in = staged ? srow : gin;

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
        uint32_t b, above;
        find_bin_from_top(hist, nb, remaining, coarse, sel2, &b, &above);
        prefix |= b << shift;
        mask_hi |= (uint32_t)(nb - 1) << shift;
        remaining -= above;
    }
    // `prefix` is the k-th key; `remaining` (>= 1) keys equal to it are taken.
    emit_segment<TOPK_THREADS>(in, cidx, 0, len, prefix, remaining, 0, 0, (uint32_t)kk - remaining, out, scan_sh);
}

// ---- multi-CTA top-k for long rows (decode) -------------------------------------------
// The first-level histogram (top HBITS bits of every score key) arrives from
// the indexer's epilogue (or topk_hist_kernel). Then:
//   partition (C CTAs / row): find the bin b1 that holds the k-th key; count
//             the keys above it per chunk; append the keys in b1 to a per-row
//             candidate list (buffered in shared memory, one global
//             reservation per buffer);
//   threshold (1 CTA / row):  finish the radix select on the candidates
//             (remaining 19 bits) -> exact k-th key `thr` and how many keys
//             equal to it are taken; per-chunk output offsets of the keys
//             > thr and == thr (exclusive scans over chunks);
//   emit      (C CTAs / row): rescan each chunk and write its selected keys at
//             their final positions, ascending.
constexpr int HBITS = 13;  // first-level histogram: bits 31..19 of the key
constexpr int HB = 1 << HBITS;
constexpr int TOPKM_THREADS = 256;
constexpr int TOPKM_CHUNK_MAX = 4096;   // candidates a partition CTA buffers in shared memory
constexpr int TOPKM_PART_SMEM = 2 * TOPKM_CHUNK_MAX * 4;
constexpr int TOPKM_CAND_SMEM = 16384;  // candidates the threshold kernel stages in shared memory
constexpr int TOPKM_THR_SMEM = (1024 + 2 * TOPKM_CAND_SMEM) * 4;

struct TopkMParams {
    const float* in;
    long long in_stride;
    int n_rows, rows_per_seq, len0, len_step, T, k;
    int* out;
    long long out_stride;
    int* n_out;
    const unsigned* hist;  // [rows][HB]
    int chunk, n_chunks;
    unsigned* cand_key;
    int* cand_pos;
    long long cand_stride;
    unsigned* cand_n;  // [rows], zero on entry
    unsigned* cnt_gt;  // [rows][n_chunks]
    unsigned* cnt_eq;  // [rows][n_chunks]
    unsigned* thr;     // [rows][2]: threshold key, need
};

__device__ __forceinline__ int topk_row_len(const TopkMParams& p, int r) {
    const long long l = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    return (int)(l < p.T ? l : p.T);
}

__global__ void __launch_bounds__(TOPKM_THREADS) topk_partition_kernel(TopkMParams p) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ uint32_t dyn[];  // candidate buffer: keys, positions
    uint32_t* ckey = dyn;
    int* cpos = reinterpret_cast<int*>(ckey + TOPKM_CHUNK_MAX);
    __shared__ uint32_t coarse[HB / 32], sel2[2];
    __shared__ uint32_t warp_gt[TOPKM_THREADS / 32], n_loc, g_base;
    const int c = blockIdx.x, r = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int len = topk_row_len(p, r);
    const int kk = min(p.k, len);
    if (kk >= len) return;
    if (tid == 0) n_loc = 0;
    uint32_t b1, above;
    find_bin_from_top(p.hist + (long long)r * HB, HB, (uint32_t)kk, coarse, sel2, &b1, &above);
    const float* in = p.in + (long long)r * p.in_stride;
    const int lo = c * p.chunk, hi = min(len, lo + p.chunk);
    unsigned* gk = p.cand_key + (long long)r * p.cand_stride;
    int* gp = p.cand_pos + (long long)r * p.cand_stride;
    uint32_t gt = 0;
    // Rounds of TOPKM_CHUNK_MAX elements: 16 independent loads per thread
    // first, then classification and candidate appends; a round can fill the
    // shared buffer at most once, so each round ends with one flush.
    constexpr int PER = TOPKM_CHUNK_MAX / TOPKM_THREADS;
#pragma unroll 1
    for (int base = lo; base < hi; base += TOPKM_CHUNK_MAX) {
        float x[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = base + j * TOPKM_THREADS + tid;
            x[j] = i < hi ? in[i] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = base + j * TOPKM_THREADS + tid;
            uint32_t key = 0;
            bool cand = false;
            if (i < hi) {
                key = ordered_key(x[j]);
                const uint32_t bin = key >> (32 - HBITS);
                gt += bin > b1;
                cand = bin == b1;
            }
            const unsigned m = __ballot_sync(0xffffffffu, cand);
            if (m) {
                unsigned wbase = 0;
                if (lane == 0) wbase = atomicAdd(&n_loc, (unsigned)__popc(m));
                wbase = __shfl_sync(0xffffffffu, wbase, 0);
                if (cand) {
                    const unsigned slot = wbase + __popc(m & ((1u << lane) - 1u));
                    ckey[slot] = key;
                    cpos[slot] = i;
                }
            }
        }
        __syncthreads();
        const unsigned nl = n_loc;
        if (tid == 0 && nl) g_base = atomicAdd(p.cand_n + r, nl);
        __syncthreads();
        for (unsigned j = tid; j < nl; j += TOPKM_THREADS) {
            gk[g_base + j] = ckey[j];
            gp[g_base + j] = cpos[j];
        }
        __syncthreads();
        if (tid == 0) n_loc = 0;
        __syncthreads();
    }
    for (int o = 16; o > 0; o >>= 1) gt += __shfl_xor_sync(0xffffffffu, gt, o);
    if (lane == 0) warp_gt[tid >> 5] = gt;
    __syncthreads();
    if (tid == 0) {
        uint32_t t = 0;
        for (int w = 0; w < TOPKM_THREADS / 32; ++w) t += warp_gt[w];
        p.cnt_gt[(long long)r * p.n_chunks + c] = t;
    }
}

__global__ void __launch_bounds__(TOPK_THREADS) topk_threshold_kernel(TopkMParams p) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ uint32_t dyn[];  // 1024-bin histogram, then staged candidates
    uint32_t* h = dyn;
    uint32_t* sk = dyn + 1024;
    int* spos = reinterpret_cast<int*>(sk + TOPKM_CAND_SMEM);
    __shared__ uint32_t scan_sh[33];
    __shared__ uint32_t coarse[HB / 32], sel2[2];
    __shared__ uint32_t cg[TOPK_THREADS], ce[TOPK_THREADS];
    const int r = blockIdx.x, tid = threadIdx.x;
    const int len = topk_row_len(p, r);
    const int kk = min(p.k, len);
    if (kk >= len) return;
    uint32_t b1, above1;
    find_bin_from_top(p.hist + (long long)r * HB, HB, (uint32_t)kk, coarse, sel2, &b1, &above1);
    const unsigned m = p.cand_n[r];
    const bool staged = m <= (unsigned)TOPKM_CAND_SMEM;
    const unsigned* ck = staged ? sk : p.cand_key + (long long)r * p.cand_stride;
    const int* cp = staged ? spos : p.cand_pos + (long long)r * p.cand_stride;
    if (staged) {
        const unsigned* gk = p.cand_key + (long long)r * p.cand_stride;
        const int* gp = p.cand_pos + (long long)r * p.cand_stride;
        for (unsigned i = tid; i < m; i += TOPK_THREADS) {
            sk[i] = gk[i];
            spos[i] = gp[i];
        }
        __syncthreads();
    }
    // Remaining 19 bits in two passes (10 + 9) over the candidates.
    uint32_t prefix = b1 << (32 - HBITS), mask_hi = ~0u << (32 - HBITS), remaining = (uint32_t)kk - above1;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
        const int shift = pass == 0 ? 9 : 0;
        const int nb = pass == 0 ? 1024 : 512;
        for (int i = tid; i < 1024; i += TOPK_THREADS) h[i] = 0;
        __syncthreads();
        for (unsigned i = tid; i < m; i += TOPK_THREADS) {
            const uint32_t u = ck[i];
            if ((u & mask_hi) == prefix) atomicAdd(&h[(u >> shift) & (uint32_t)(nb - 1)], 1u);
        }
        __syncthreads();
        uint32_t b, above;
        find_bin_from_top(h, 1024, remaining, coarse, sel2, &b, &above);
        prefix |= b << shift;
        mask_hi |= (uint32_t)(nb - 1) << shift;
        remaining -= above;
    }
    const uint32_t thr = prefix, need = remaining;
    // Per-chunk counts of candidate keys > thr and == thr.
    for (int i = tid; i < p.n_chunks; i += TOPK_THREADS) {
        cg[i] = 0;
        ce[i] = 0;
    }
    __syncthreads();
    for (unsigned base = 0; base < m; base += TOPK_THREADS) {
        const unsigned i = base + tid;
        int c = -1;
        uint32_t u = 0;
        if (i < m) {
            u = ck[i];
            c = cp[i] / p.chunk;
        }
        // lanes grouped by (chunk, class): one shared atomic per group
        const int cls = (i < m) ? (u > thr ? 1 : (u == thr ? 2 : 0)) : 0;
        const unsigned peers = __match_any_sync(0xffffffffu, (c << 2) | cls);
        if (cls && (tid & 31) == __ffs(peers) - 1) atomicAdd(cls == 1 ? &cg[c] : &ce[c], (unsigned)__popc(peers));
    }
    __syncthreads();
    const int c = tid;
    const uint32_t g = c < p.n_chunks ? p.cnt_gt[(long long)r * p.n_chunks + c] + cg[c] : 0u;
    const uint32_t e = c < p.n_chunks ? ce[c] : 0u;
    uint32_t tot;
    const uint32_t bg = block_excl_scan(g, scan_sh, &tot);
    const uint32_t be = block_excl_scan(e, scan_sh, &tot);
    if (c < p.n_chunks) {
        p.cnt_gt[(long long)r * p.n_chunks + c] = bg;
        p.cnt_eq[(long long)r * p.n_chunks + c] = be;
    }
    if (tid == 0) {
        p.thr[2 * r] = thr;
        p.thr[2 * r + 1] = need;
    }
}

__global__ void __launch_bounds__(TOPKM_THREADS) topk_emit_kernel(TopkMParams p) {
    pdl_wait();
    pdl_trigger();
    __shared__ uint32_t scan_sh[33];
    const int c = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
    const int len = topk_row_len(p, r);
    const int kk = min(p.k, len);
    int* out = p.out + (long long)r * p.out_stride;
    if (c == 0 && tid == 0 && p.n_out) p.n_out[r] = kk;
    const int lo = c * p.chunk, hi = min(len, lo + p.chunk);
    if (kk >= len) {
        for (int i = lo + tid; i < hi; i += TOPKM_THREADS) out[i] = i;
        return;
    }
    if (lo >= hi) return;
    const float* in = p.in + (long long)r * p.in_stride;
    const uint32_t thr = p.thr[2 * r], need = p.thr[2 * r + 1];
    emit_segment<TOPKM_THREADS>(in, nullptr, lo, hi, thr, need, p.cnt_gt[(long long)r * p.n_chunks + c],
                                p.cnt_eq[(long long)r * p.n_chunks + c], 0xFFFFFFFFu, out, scan_sh);
}

// Zeroes the fused histograms before the indexer adds to them. A kernel rather
// than a memset node so that the launch chain stays programmatic: the
// indexer's setup overlaps this kernel, this kernel overlaps the launch of the
// previous kernel's tail.
__global__ void __launch_bounds__(256) hist_zero_kernel(unsigned* h, long long n) {
    pdl_wait();
    pdl_trigger();
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += (long long)gridDim.x * 256) h[i] = 0u;
}

// ---- cluster top-k for decode rows ----------------------------------------------------
// One thread-block cluster of TOPKC_CL CTAs per row; CTA `rank` holds the
// scores [rank * 1024 * PER, (rank + 1) * 1024 * PER) of the row in registers
// (PER consecutive keys per thread), read once. With the first-level histogram
// (top HBITS bits) from the indexer's epilogue:
//   1. every CTA finds the bin b1 holding the k-th key from that histogram;
//   2. two refinement passes (10 + 9 bits) over the keys in b1, giving the
//      exact k-th key `thr` and how many keys equal to it are taken (`need`).
//      When b1 holds at most TOPKC_GCAP keys, every warp stores its keys of b1
//      into CTA 0's shared memory (slots reserved by one distributed-shared-
//      memory atomic per warp); CTA 0 refines over them, counts every CTA's
//      keys > thr and == thr, and writes each CTA its thr, need and output
//      bases (two cluster barriers). Otherwise each CTA builds its shared-
//      memory histogram, a cluster barrier publishes them, every CTA sums the
//      TOPKC_CL histograms over distributed shared memory and finds the next
//      bin, and the CTAs exchange their totals of > thr and == thr;
//   3. each CTA's block scan gives every thread its offsets, and every thread
//      writes its selected keys at their final, ascending positions.
// One launch, no global scratch beyond the histogram.
constexpr int TOPKC_CL = 8;
constexpr int TOPKC_THREADS = 1024;
constexpr int TOPKC_GCAP = 4096;  // keys of the crossing bin CTA 0 gathers (else the distributed refinement)


// Block-wide search from the top over bins held by threads: thread t owns the
// consecutive bins [t * PERB, (t + 1) * PERB) with counts c[0..PERB) (higher t
// and higher j = higher bins). Every thread returns the bin b where the running
// count from the top crosses `need` (count(bins > b) < need <= count(bins >= b))
// and count(bins > b), and with `out_count` the count of bin b. `sh` holds >= 35
// words (36 with `out_count`). Requires need <= total.
template <int PERB>
__device__ __forceinline__ void block_find_from_top(const uint32_t (&c)[PERB], uint32_t need, uint32_t* sh,
                                                    uint32_t* out_bin, uint32_t* out_above,
                                                    uint32_t* out_count = nullptr) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint32_t s = 0;
#pragma unroll
    for (int j = 0; j < PERB; ++j) s += c[j];
    uint32_t suf = s;  // inclusive suffix sum within the warp (lanes >= this one)
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += y;
    }
    if (lane == 0) sh[warp] = suf;  // warp total
    __syncthreads();
    // every warp: the sum of the totals of the warps above it
    const uint32_t wt = lane < nw && lane > warp ? sh[lane] : 0u;
    uint32_t above_w = wt;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) above_w += __shfl_xor_sync(0xffffffffu, above_w, o);
    uint32_t above = above_w + suf - s;  // count in the bins above this thread's segment
    if (s > 0 && above < need && need <= above + s) {
        uint32_t b = 0;
#pragma unroll
        for (int j = PERB - 1; j >= 0; --j) {
            if (above < need && need <= above + c[j]) {
                b = (uint32_t)(threadIdx.x * PERB + j);
                if (out_count) sh[35] = c[j];
                break;
            }
            above += c[j];
        }
        sh[33] = b;
        sh[34] = above;
    }
    __syncthreads();
    *out_bin = sh[33];
    *out_above = sh[34];
    if (out_count) *out_count = sh[35];
    __syncthreads();
}

template <int PER>
__global__ void __cluster_dims__(TOPKC_CL, 1, 1) __launch_bounds__(TOPKC_THREADS, 1)
    topk_cluster_kernel(TopkMParams p, int vec4, CandOut co) {
    pdl_wait();
    pdl_trigger();
    static_assert(PER % 4 == 0 && PER <= 32, "PER: whole float4s, one bit each in a 32-bit mask");
    __shared__ uint32_t hloc[2][1024];  // this CTA's refinement histograms (read by the cluster)
    __shared__ uint32_t scan_sh[36];
    __shared__ uint32_t tot[2];  // this CTA's count of keys > thr, == thr (read by the cluster)
    __shared__ uint2 gcand[TOPKC_GCAP];  // CTA 0: the crossing bin's (key, position) from every CTA
    // CTA 0: [0] candidates gathered; [1 + c] CTA c's keys above the crossing bin;
    // [1 + CL + c], [1 + 2 CL + c] CTA c's candidates > thr, == thr
    __shared__ uint32_t gctl[1 + 3 * TOPKC_CL];
    // written by CTA 0 (one 16-byte store): thr, need, this CTA's output bases (> thr, == thr)
    __shared__ __align__(16) uint32_t res[4];
    const int tid = threadIdx.x, r = blockIdx.y;
    const uint32_t rank = cluster_ctarank();
    const int len = topk_row_len(p, r);
    const int kk = min(p.k, len);
    int* out = p.out + (long long)r * p.out_stride;
    const int lo = (int)rank * TOPKC_THREADS * PER, hi = min(len, lo + TOPKC_THREADS * PER);
    if (rank == 0 && tid == 0 && p.n_out) p.n_out[r] = kk > 0 ? kk : 0;
    if (rank == 0) cand_pad(co, r, max(kk, 0), tid, TOPKC_THREADS);
    if (kk <= 0) return;  // uniform over the cluster
    if (kk >= len) {
        for (int i = lo + tid; i < hi; i += TOPKC_THREADS) {
            out[i] = i;
            if (co.score) {
                co.score[(long long)r * co.stride + i] = p.in[(long long)r * p.in_stride + i];
                co.gidx[(long long)r * co.stride + i] = (int)(co.base + i);
            }
        }
        return;
    }
    // ---- loads: the first-level histogram (8 consecutive bins per thread) and
    // the row's scores (PER consecutive per thread), all in flight together ----
    static_assert(HB == 8 * TOPKC_THREADS, "level-1 bins per thread");
    const uint4* hg = reinterpret_cast<const uint4*>(p.hist + (long long)r * HB) + 2 * tid;
    const uint4 hx = hg[0], hy = hg[1];
    const float* in = p.in + (long long)r * p.in_stride;
    const int i0 = lo + tid * PER;
    const int nvalid = max(0, min(PER, hi - i0));
    const uint32_t valid = nvalid >= 32 ? 0xffffffffu : (1u << nvalid) - 1u;
    float f[PER];
    if (vec4 && nvalid == PER) {
#pragma unroll
        for (int j = 0; j < PER; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(in + i0 + j);
            f[j] = v.x;
            f[j + 1] = v.y;
            f[j + 2] = v.z;
            f[j + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < PER; ++j) f[j] = j < nvalid ? in[i0 + j] : 0.f;
    }
    for (int i = tid; i < 2 * 1024; i += TOPKC_THREADS) (&hloc[0][0])[i] = 0;
    if (tid < 1 + 3 * TOPKC_CL) gctl[tid] = 0;
    // Every CTA of the cluster has started and CTA 0's counters are zero
    // before any remote access (the wait follows level 1).
    cluster_arrive();
    // ---- level 1: the bin b1 of the indexer's histogram holding the k-th key ----
    uint32_t b1, above1, bcount;
    {
        const uint32_t c8[8] = {hx.x, hx.y, hx.z, hx.w, hy.x, hy.y, hy.z, hy.w};
        block_find_from_top<8>(c8, (uint32_t)kk, scan_sh, &b1, &above1, &bcount);
    }
    uint32_t u[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) u[j] = ordered_key(f[j]);
    // One pass over the keys: those in bins above b1 are selected outright, those
    // in b1 are the candidates; every later step walks the candidate bits only.
    uint32_t mabove = 0, mcand = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const uint32_t bin = u[j] >> (32 - HBITS);
        mabove |= (bin > b1 ? 1u : 0u) << j;
        mcand |= (bin == b1 ? 1u : 0u) << j;
    }
    mabove &= valid;
    mcand &= valid;
    cluster_wait();
    if (bcount <= (uint32_t)TOPKC_GCAP) {  // uniform: the row's histogram
        // ---- the crossing bin's keys gathered into CTA 0, one slot range per warp ----
        const int lane = tid & 31, warp = tid >> 5;
        const uint32_t nc = __popc(mcand);
        uint32_t incl = nc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const uint32_t wtot = __shfl_sync(0xffffffffu, incl, 31);
        const uint32_t na = __reduce_add_sync(0xffffffffu, (uint32_t)__popc(mabove));
        uint32_t wbase = 0;
        if (lane == 0) {
            if (wtot) wbase = dsmem_atom_add(dsmem_addr(&gctl[0], 0), wtot);
            if (na) dsmem_atom_add(dsmem_addr(&gctl[1 + rank], 0), na);
        }
        uint32_t slot = __shfl_sync(0xffffffffu, wbase, 0) + incl - nc;
        const uint32_t gc0 = dsmem_addr(gcand, 0);
        for (uint32_t m = mcand; m; m &= m - 1, ++slot) {
            const int j = __ffs(m) - 1;
            if (slot < (uint32_t)TOPKC_GCAP) dsmem_st_v2(gc0 + slot * 8u, u[j], (uint32_t)(i0 + j));
        }
        cluster_sync_all();  // the candidates and counts are in CTA 0
        if (rank == 0) {
            // ---- levels 2, 3 (10 + 9 bits) over the gathered keys ----
            const uint32_t n = min(gctl[0], (uint32_t)TOPKC_GCAP);
            uint32_t prefix = b1 << (32 - HBITS), mask_hi = ~0u << (32 - HBITS), remaining = (uint32_t)kk - above1;
#pragma unroll 1
            for (int pass = 0; pass < 2; ++pass) {
                const int shift = pass == 0 ? 9 : 0;
                const uint32_t nb = pass == 0 ? 1024u : 512u;
                uint32_t* h = hloc[pass];
                for (uint32_t i = tid; i < n; i += TOPKC_THREADS) {
                    const uint32_t x = gcand[i].x;
                    if ((x & mask_hi) == prefix) atomicAdd(&h[(x >> shift) & (nb - 1)], 1u);
                }
                __syncthreads();
                uint32_t c1[1] = {tid < (int)nb ? h[tid] : 0u};
                uint32_t b, above;
                block_find_from_top<1>(c1, remaining, scan_sh, &b, &above);
                prefix |= b << shift;
                mask_hi |= (nb - 1) << shift;
                remaining -= above;
            }
            const uint32_t thr = prefix;
            // per source CTA: its candidates > thr and == thr
            for (uint32_t b0 = (uint32_t)warp * 32u; b0 < n; b0 += TOPKC_THREADS) {
                const uint32_t i = b0 + lane;
                const uint2 g = i < n ? gcand[i] : make_uint2(0u, 0u);
                const uint32_t src = g.y / (uint32_t)(TOPKC_THREADS * PER);
                const bool gt = i < n && g.x > thr, eq = i < n && g.x == thr;
#pragma unroll
                for (int c = 0; c < TOPKC_CL; ++c) {
                    const uint32_t bg = __ballot_sync(0xffffffffu, gt && src == (uint32_t)c);
                    const uint32_t be = __ballot_sync(0xffffffffu, eq && src == (uint32_t)c);
                    if (lane == 0 && bg) atomicAdd(&gctl[1 + TOPKC_CL + c], (uint32_t)__popc(bg));
                    if (lane == 0 && be) atomicAdd(&gctl[1 + 2 * TOPKC_CL + c], (uint32_t)__popc(be));
                }
            }
            __syncthreads();
            if (tid < TOPKC_CL) {
                uint32_t gb = 0, eb = 0;
                for (int c = 0; c < tid; ++c) {
                    gb += gctl[1 + c] + gctl[1 + TOPKC_CL + c];
                    eb += gctl[1 + 2 * TOPKC_CL + c];
                }
                dsmem_st_v4(dsmem_addr(res, (uint32_t)tid), thr, remaining, gb, eb);
            }
        }
        cluster_sync_all();  // every CTA's thr, need and output bases written; no remote access after this
        const uint32_t thr = res[0], need = res[1];
        uint32_t mgt = mabove, meq = 0;
        for (uint32_t m = mcand; m; m &= m - 1) {
            const int j = __ffs(m) - 1;
            const uint32_t x = u[j];
            mgt |= (x > thr ? 1u : 0u) << j;
            meq |= (x == thr ? 1u : 0u) << j;
        }
        uint32_t total;
        const uint32_t ex =
            block_excl_scan(((uint32_t)__popc(meq) << 16) | (uint32_t)__popc(mgt), scan_sh, &total);
        uint32_t gt_b = res[2] + (ex & 0xffffu), eq_b = res[3] + (ex >> 16);
        for (uint32_t m = mgt | meq; m; m &= m - 1) {
            const int j = __ffs(m) - 1;
            int pos = -1;
            if ((mgt >> j) & 1u) {
                pos = (int)(gt_b + min(eq_b, need));
                ++gt_b;
            } else {
                if (eq_b < need) pos = (int)(gt_b + eq_b);
                ++eq_b;
            }
            if (pos >= 0) {
                out[pos] = i0 + j;
                if (co.score) {
                    co.score[(long long)r * co.stride + pos] = key_to_float(u[j]);
                    co.gidx[(long long)r * co.stride + pos] = (int)(co.base + i0 + j);
                }
            }
        }
        return;
    }
    // ---- levels 2, 3 over the cluster: bin `tid` of each pass summed over the CTAs ----
    uint32_t prefix = b1 << (32 - HBITS), mask_hi = ~0u << (32 - HBITS), remaining = (uint32_t)kk - above1;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
        const int shift = pass == 0 ? 9 : 0;
        const uint32_t nb = pass == 0 ? 1024u : 512u;
        uint32_t* h = hloc[pass];
        for (uint32_t m = mcand; m; m &= m - 1) {
            const uint32_t x = u[__ffs(m) - 1];  // dynamic index: local memory only for this rare walk
            if ((x & mask_hi) == prefix) atomicAdd(&h[(x >> shift) & (nb - 1)], 1u);
        }
        cluster_sync_all();  // every CTA's histogram complete and visible
        uint32_t c1[1] = {0u};
        if (tid < (int)nb) {
#pragma unroll
            for (int c = 0; c < TOPKC_CL; ++c) c1[0] += dsmem_ld_u32(&h[tid], (uint32_t)c);
        }
        uint32_t b, above;
        block_find_from_top<1>(c1, remaining, scan_sh, &b, &above);
        prefix |= b << shift;
        mask_hi |= (nb - 1) << shift;
        remaining -= above;
    }
    const uint32_t thr = prefix, need = remaining;
    // ---- ordered emission ----
    uint32_t mgt = mabove, meq = 0;
    for (uint32_t m = mcand; m; m &= m - 1) {
        const int j = __ffs(m) - 1;
        const uint32_t x = u[j];
        mgt |= (x > thr ? 1u : 0u) << j;
        meq |= (x == thr ? 1u : 0u) << j;
    }
    uint32_t total;
    const uint32_t ex = block_excl_scan(((uint32_t)__popc(meq) << 16) | (uint32_t)__popc(mgt), scan_sh, &total);
    if (tid == 0) {
        tot[0] = total & 0xffffu;
        tot[1] = total >> 16;
    }
    cluster_sync_all();  // totals visible; also orders every remote histogram read before exit
    uint32_t gt_b = 0, eq_b = 0;
    for (uint32_t c = 0; c < rank; ++c) {
        gt_b += dsmem_ld_u32(&tot[0], c);
        eq_b += dsmem_ld_u32(&tot[1], c);
    }
    cluster_arrive();  // this CTA's remote reads are done
    gt_b += ex & 0xffffu;
    eq_b += ex >> 16;
    for (uint32_t m = mgt | meq; m; m &= m - 1) {
        const int j = __ffs(m) - 1;
        int pos = -1;
        if ((mgt >> j) & 1u) {
            pos = (int)(gt_b + min(eq_b, need));
            ++gt_b;
        } else {
            if (eq_b < need) pos = (int)(gt_b + eq_b);
            ++eq_b;
        }
        if (pos >= 0) {
            out[pos] = i0 + j;
            if (co.score) {
                co.score[(long long)r * co.stride + pos] = key_to_float(u[j]);
                co.gidx[(long long)r * co.stride + pos] = (int)(co.base + i0 + j);
            }
        }
    }
    cluster_wait();  // no CTA leaves while another may still read its totals
}

// ---- single-CTA top-k with the row in registers --------------------------------------
// Rows of up to TOPK_THREADS * PER keys (PER consecutive per thread, read once):
// the block's key range, then three radix levels over the offset from its
// minimum (up to 11 + 11 + 10 bits, shared-memory histograms) — a range-adaptive
// first level keeps crowded score distributions from piling onto a few bins
// (fixed bit fields put most of a row into one or two exponent bins, and the
// contended shared-memory atomics dominated) — then the ordered emission.
// (Aggregating a warp's lanes by bin with __match_any_sync measured several
// times slower than letting the shared-memory unit serialise.)
// Supports candidate-index mapping (`cand_idx`), segmented rows and candidate
// outputs.
template <int PER, bool LL>
__global__ void __launch_bounds__(TOPK_THREADS, 1) topk_reg_kernel(TopkParams p, int vec4, CandOut co) {
    static_assert(PER % 4 == 0 && PER <= 32, "PER: whole float4s, one bit each in a 32-bit mask");
    pdl_wait();
    pdl_trigger();
    __shared__ uint32_t hist[2048];
    __shared__ uint32_t scan_sh[36];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = blockIdx.x;
    const long long lraw = (long long)p.len0 + (long long)(r % p.rows_per_seq) * p.len_step;
    const int len = (int)(lraw < p.T ? lraw : p.T);
    const int kk = min(p.k, len);
    int* out = p.out + (long long)r * p.out_stride;
    if (tid == 0 && p.n_out) p.n_out[r] = kk > 0 ? kk : 0;
    cand_pad(co, r, max(kk, 0), tid, TOPK_THREADS);
    if (kk <= 0) return;
    const float* row = p.in + (long long)r * p.in_stride;
    const int* crow = p.cand_idx ? p.cand_idx + (long long)r * p.in_stride : nullptr;
    auto off = [&](int i) -> long long {
        return p.seg_len > 0 ? (long long)(i / p.seg_len) * p.seg_stride + i % p.seg_len : (long long)i;
    };
    constexpr bool ll = LL;  // rows arrive through the peer exchange (p.ll)
    const uint32_t epoch = ll ? p2p_epoch(p.ll) : 0u;
    const uint64_t* lrow = ll ? p2p_slot(p.ll, epoch, 0) + (long long)r * p.in_stride : nullptr;
    auto score_at = [&](int i) -> float {
        if constexpr (!LL) return row[off(i)];
        const uint64_t* w = lrow + off(i);
        return __uint_as_float(ll_wait1(w, epoch, ll_load1_raw(w), 22));
    };
    auto key_at = [&](int i) -> int {
        if constexpr (LL) {
            const uint64_t* w = lrow + p.ll_idx_off + off(i);
            return (int)ll_wait1(w, epoch, ll_load1_raw(w), 22);
        }
        return crow ? crow[off(i)] : i;
    };
    if (kk >= len) {
        for (int i = tid; i < len; i += TOPK_THREADS) {
            const int key = key_at(i);
            out[i] = key;
            if (co.score) {
                co.score[(long long)r * co.stride + i] = score_at(i);
                co.gidx[(long long)r * co.stride + i] = (int)(co.base + key);
            }
        }
        return;
    }
    const int i0 = tid * PER;
    const int nvalid = max(0, min(PER, len - i0));
    const uint32_t valid = nvalid >= 32 ? 0xffffffffu : (1u << nvalid) - 1u;
    uint32_t u[PER];
    {
        float f[PER];
        const long long o0 = nvalid > 0 ? off(i0) : 0;  // PER divides seg_len: one segment per thread
        if constexpr (LL) {
            uint64_t w[PER];
            if (nvalid == PER) {
#pragma unroll
                for (int j = 0; j < PER; j += 2) ll_load2_raw(lrow + o0 + j, w[j], w[j + 1]);
            } else {
#pragma unroll
                for (int j = 0; j < PER; ++j) w[j] = j < nvalid ? ll_load1_raw(lrow + o0 + j) : 0ull;
            }
#pragma unroll
            for (int j = 0; j < PER; ++j)
                f[j] = j < nvalid ? __uint_as_float(ll_wait1(lrow + o0 + j, epoch, w[j], 22)) : 0.f;
        } else if (vec4 && nvalid == PER) {
#pragma unroll
            for (int j = 0; j < PER; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(row + o0 + j);
                f[j] = v.x;
                f[j + 1] = v.y;
                f[j + 2] = v.z;
                f[j + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < PER; ++j) f[j] = j < nvalid ? row[o0 + j] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < PER; ++j) u[j] = ordered_key(f[j]);
    }
    // ---- the row's key range: levels bin the offset d = key - lo ----
    uint32_t lo = 0xffffffffu, hi = 0u;
#pragma unroll
    for (int j = 0; j < PER; ++j)
        if ((valid >> j) & 1u) {
            lo = min(lo, u[j]);
            hi = max(hi, u[j]);
        }
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    if (lane == 0) {
        scan_sh[warp] = lo;
        hist[warp] = hi;  // hist is zeroed below, after this is read
    }
    __syncthreads();
    if (warp == 0) {
        uint32_t l = scan_sh[lane], h = hist[lane];
        l = __reduce_min_sync(0xffffffffu, l);
        h = __reduce_max_sync(0xffffffffu, h);
        if (lane == 0) {
            scan_sh[34] = l;
            scan_sh[35] = h;
        }
    }
    __syncthreads();
    lo = scan_sh[34];
    const uint32_t span = scan_sh[35] - lo;
    // Level 1 takes the span's top (up to) 11 significant bits, level 2 the next
    // 11, level 3 the rest (at most 10): the bins follow the data, so a row whose
    // scores sit in a few binades still spreads over every bin of a level.
    const int nbits = span ? 32 - __clz(span) : 0;
    const int s1 = max(0, nbits - 11), s2 = max(0, s1 - 11);
    for (int i = tid; i < 2048; i += TOPK_THREADS) hist[i] = 0;
    __syncthreads();
    // ---- level 1 ----
#pragma unroll
    for (int j = 0; j < PER; ++j)
        if ((valid >> j) & 1u) atomicAdd(&hist[(u[j] - lo) >> s1], 1u);
    __syncthreads();
    uint32_t b1, above1;
    {
        uint32_t c2[2] = {hist[2 * tid], hist[2 * tid + 1]};
        block_find_from_top<2>(c2, (uint32_t)kk, scan_sh, &b1, &above1);
    }
    // ---- levels 2 and 3 over the crossing bin's keys ----
    uint32_t prefix = b1 << s1, mask_hi = s1 >= 32 ? 0u : (0xffffffffu << s1), remaining = (uint32_t)kk - above1;
    int shift_hi = s1;
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
        const int shift = pass == 0 ? s2 : 0;
        const int nb_bits = shift_hi - shift;
        if (nb_bits <= 0) continue;  // uniform: this level has no bits left
        const uint32_t nb = 1u << nb_bits;
        for (int i = tid; i < 2048; i += TOPK_THREADS) hist[i] = 0;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const uint32_t d = u[j] - lo;
            if (((valid >> j) & 1u) && (d & mask_hi) == prefix) atomicAdd(&hist[(d >> shift) & (nb - 1u)], 1u);
        }
        __syncthreads();
        uint32_t c2[2] = {2u * tid < nb ? hist[2 * tid] : 0u, 2u * tid + 1 < nb ? hist[2 * tid + 1] : 0u}, b, above;
        block_find_from_top<2>(c2, remaining, scan_sh, &b, &above);
        prefix |= b << shift;
        mask_hi |= (nb - 1u) << shift;
        remaining -= above;
        shift_hi = shift;
    }
    prefix += lo;  // back from the offset to the key
    const uint32_t thr = prefix, need = remaining;
    // ---- ordered emission ----
    uint32_t mgt = 0, meq = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const bool v = (valid >> j) & 1u;
        mgt |= (v && u[j] > thr ? 1u : 0u) << j;
        meq |= (v && u[j] == thr ? 1u : 0u) << j;
    }
    uint32_t total;
    const uint32_t ex = block_excl_scan(((uint32_t)__popc(meq) << 16) | (uint32_t)__popc(mgt), scan_sh, &total);
    uint32_t gt_b = ex & 0xffffu, eq_b = ex >> 16;
    for (uint32_t m = mgt | meq; m; m &= m - 1) {
        const int j = __ffs(m) - 1;
        int pos = -1;
        if ((mgt >> j) & 1u) {
            pos = (int)(gt_b + min(eq_b, need));
            ++gt_b;
        } else {
            if (eq_b < need) pos = (int)(gt_b + eq_b);
            ++eq_b;
        }
        if (pos >= 0) {
            const int key = key_at(i0 + j);
            out[pos] = key;
            if (co.score) {
                co.score[(long long)r * co.stride + pos] = key_to_float(u[j]);
                co.gidx[(long long)r * co.stride + pos] = (int)(co.base + key);
            }
        }
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
    pdl_wait();
    pdl_trigger();
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
