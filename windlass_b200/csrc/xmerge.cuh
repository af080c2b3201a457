// xmerge.cuh — the sharded decode's (o, lse) combination over NVLink peer
// memory as a reduce-scatter followed by an all-gather.
//
// After its attention, rank r holds split-K partials of every (row, head) over
// the selected keys in its shard. Every rank must end with the full merged
// ctx [B][64][512] and lse [B][64] (the single-GPU result). Heads are dealt
// out to ranks in contiguous slices of hs = 64 / N:
//   xscatter (rank r): merges its split partials of each (row, head) and
//            stores the merged partial into the PART slot r of the rank that
//            owns the head;
//   xgather  (rank q): merges the N partials of each of its (row, head) pairs
//            and stores the final row into the GATH slot q of every rank;
//   xunpack  (every rank): copies the N slices of its GATH slots into ctx/lse
//            (fused into xgather's CTAs in the decode path).
// Per rank, NVLink carries about 2 x (N - 1) / N x B x 64 x 513 words (in the
// wire format of p2p.cuh, 8 bytes per 4-byte word), instead of N x B x 64 x 513
// words for an all-gather of every rank's partials.
//
// Slot layout (words), for B rows and hs heads: o of (b, hl) at
// (b * hs + hl) * 512, its lse at B * hs * 512 + b * hs + hl.
//
// Reuse of the slots across calls needs no second copy: rank r writes PART
// slot r of rank q for step i + 1 only after its own xunpack of step i, which
// waited for q's GATH words of step i, which q stored after reading its PART
// slots of step i; and r writes GATH slot r of q for step i + 1 only after q's
// PART words of step i + 1, which q stores after its xunpack of step i. Stale
// words carry an older epoch and never pass for new ones.
//
// The lse combination is the standard one for disjoint key sets (as
// lse_merge_kernel): L = M + log sum_s e^(lse_s - M), o = sum_s e^(lse_s - L) o_s.
#pragma once
#include "mla_attn.cuh"

namespace wl {

struct XMergeParams {
    P2PArgs a;
    int B;             // rows (sequences) of the call
    int hs;            // heads per rank (64 / nranks)
    int nsplit;        // xscatter: split partials per row
    const float* o_part;    // xscatter: [B][nsplit][64][512]
    const float* lse_part;  // xscatter: [B][nsplit][64]
    long long part_off, part_slot;  // bytes: PART slots in every region
    long long gath_off, gath_slot;  // bytes: GATH slots in every region
    float* ctx;        // xunpack: [B][64][512]
    float* lse;        // xunpack: [B][64] (may be null)
};

__device__ __forceinline__ void ll_store1(uint64_t* dst, uint32_t a, uint32_t epoch) {
    const uint64_t x = ((uint64_t)epoch << 32) | a;
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst), "l"(x) : "memory");
}

// Epoch of a put kernel of `type`: one more than the rank's counter; the last
// CTA to finish advances the counter (every CTA has read it by then).
__device__ __forceinline__ uint32_t xput_epoch(const P2PArgs& a, int type) {
    return *reinterpret_cast<volatile unsigned*>(a.ctr + type) + 1u;
}
__device__ __forceinline__ void xput_done(const P2PArgs& a, int type, uint32_t epoch) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned nblk = gridDim.x * gridDim.y * gridDim.z;
        const unsigned prev = atomicAdd(a.ctr + XCH_TYPES + type, 1u);
        if (prev == nblk - 1) {
            a.ctr[XCH_TYPES + type] = 0;
            a.ctr[type] = epoch;
        }
    }
}

// The merged row of one (row, head) and 128 columns (4 per lane) into the
// slot words at `dst` (o) and `dst_lse` (lse, lane 0 of column quarter 0).
__device__ __forceinline__ void xstore_row(uint64_t* dst, uint64_t* dst_lse, const float4& v, float L,
                                           uint32_t epoch, bool with_lse) {
    ll_store2(dst, __float_as_uint(v.x), __float_as_uint(v.y), epoch);
    ll_store2(dst + 2, __float_as_uint(v.z), __float_as_uint(v.w), epoch);
    if (with_lse) ll_store1(dst_lse, __float_as_uint(L), epoch);
}

// grid (64 / XS_HEADS, 4 column quarters, B), 32 XS_HEADS threads: warp w
// takes head XS_HEADS x + w, lane l 4 columns. (Fewer, larger CTAs: every CTA
// ends with one atomic on the epoch counter, and 2048 single-warp CTAs spent
// microseconds queueing on it.)
constexpr int XS_HEADS = 8;
__global__ void __launch_bounds__(32 * XS_HEADS) xscatter_kernel(XMergeParams p) {
    pdl_wait();
    pdl_trigger();
    const int h = blockIdx.x * XS_HEADS + (threadIdx.x >> 5), q = blockIdx.y, b = blockIdx.z, lane = threadIdx.x & 31;
    const int c = q * 128 + lane * 4;
    const uint32_t epoch = xput_epoch(p.a, XCH_PART);
    float ls = -INFINITY;
    if (lane < p.nsplit) ls = p.lse_part[((long long)b * p.nsplit + lane) * AT_H + h];
    float M = ls;
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float wl = (M == -INFINITY || ls == -INFINITY) ? 0.f : exp2f((ls - M) * 1.4426950408889634f);
    float W = wl;
    for (int o = 16; o > 0; o >>= 1) W += __shfl_xor_sync(0xffffffffu, W, o);
    const float inv = W > 0.f ? 1.f / W : 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // splits in groups of 16: all loads of a group in flight before any use
    for (int s0 = 0; s0 < p.nsplit; s0 += 16) {
        float4 v[16];
        float w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int s = s0 + j;
            w[j] = __shfl_sync(0xffffffffu, wl, s & 31) * inv;
            if (s >= p.nsplit) w[j] = 0.f;
            v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (w[j] != 0.f)  // empty splits are never read
                v[j] = *reinterpret_cast<const float4*>(p.o_part + (((long long)b * p.nsplit + s) * AT_H + h) * AT_DV + c);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            acc.x = fmaf(w[j], v[j].x, acc.x);
            acc.y = fmaf(w[j], v[j].y, acc.y);
            acc.z = fmaf(w[j], v[j].z, acc.z);
            acc.w = fmaf(w[j], v[j].w, acc.w);
        }
    }
    const float L = (W > 0.f) ? M + logf(W) : -INFINITY;
    const int owner = h / p.hs, hl = h % p.hs;
    uint64_t* slot = reinterpret_cast<uint64_t*>(p.a.region[owner] + p.part_off + (long long)p.a.rank * p.part_slot);
    const long long row = (long long)b * p.hs + hl;
    xstore_row(slot + row * AT_DV + c, slot + (long long)p.B * p.hs * AT_DV + row, acc, L, epoch,
               q == 0 && lane == 0);
    xput_done(p.a, XCH_PART, epoch);
}

// The final rows of heads {r hs + hl : r < N} (each owned by rank r) from this
// rank's GATH slots into ctx / lse: what CTA (hl, q, b) of the gather unpacks.
__device__ __forceinline__ void xunpack_head(const XMergeParams& p, int h, int q, int b, int lane, uint32_t eg) {
    const int c = q * 128 + lane * 4;
    const int owner = h / p.hs, hl = h % p.hs;
    const uint64_t* slot =
        reinterpret_cast<const uint64_t*>(p.a.region[p.a.rank] + p.gath_off + (long long)owner * p.gath_slot);
    const long long row = (long long)b * p.hs + hl;
    const uint64_t* w = slot + row * AT_DV + c;
    uint64_t r0, r1, r2, r3;
    ll_load2_raw(w, r0, r1);
    ll_load2_raw(w + 2, r2, r3);
    float4 v;
    v.x = __uint_as_float(ll_wait1(w, eg, r0, 52));
    v.y = __uint_as_float(ll_wait1(w + 1, eg, r1, 52));
    v.z = __uint_as_float(ll_wait1(w + 2, eg, r2, 52));
    v.w = __uint_as_float(ll_wait1(w + 3, eg, r3, 52));
    *reinterpret_cast<float4*>(p.ctx + ((long long)b * AT_H + h) * AT_DV + c) = v;
    if (q == 0 && lane == 0 && p.lse) {
        const uint64_t* wl = slot + (long long)p.B * p.hs * AT_DV + row;
        p.lse[(long long)b * AT_H + h] = __uint_as_float(ll_wait1(wl, eg, ll_load1_raw(wl), 53));
    }
}

// grid (hs heads, 4 column quarters, B), 32 N threads: every warp merges the
// N partials of position (hl, q, b) (the same words, from this GPU's memory),
// then warp w stores the result into rank (rank + w) % N and — UNPACK — copies
// that rank's final slice of the position into ctx / lse (the all-gather's
// receive side), so the N destinations and the N waits proceed in parallel
// and no third kernel is needed.
template <bool UNPACK>
__global__ void __launch_bounds__(32 * P2P_MAX_RANKS) xgather_kernel(XMergeParams p) {
    pdl_wait();
    pdl_trigger();
    const int hl = blockIdx.x, q = blockIdx.y, b = blockIdx.z, lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
    const int c = q * 128 + lane * 4;
    const int N = p.a.nranks;
    const uint32_t ep = *reinterpret_cast<volatile unsigned*>(p.a.ctr + XCH_PART);  // this step's PART epoch
    const uint32_t eg = xput_epoch(p.a, XCH_GATH);
    const uint64_t* mine = reinterpret_cast<const uint64_t*>(p.a.region[p.a.rank] + p.part_off);
    const long long slot_words = p.part_slot / 8, row = (long long)b * p.hs + hl;
    const long long lse_w = (long long)p.B * p.hs * AT_DV + row;
    float ls = -INFINITY;
    if (lane < N) {
        const uint64_t* w = mine + lane * slot_words + lse_w;
        ls = __uint_as_float(ll_wait1(w, ep, ll_load1_raw(w), 50));
    }
    float M = ls;
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float wl = (M == -INFINITY || ls == -INFINITY) ? 0.f : exp2f((ls - M) * 1.4426950408889634f);
    float W = wl;
    for (int o = 16; o > 0; o >>= 1) W += __shfl_xor_sync(0xffffffffu, W, o);
    const float inv = W > 0.f ? 1.f / W : 0.f;
    // all parts' words in flight at once, tags checked after
    uint64_t raw[P2P_MAX_RANKS][4];
    float wv[P2P_MAX_RANKS];
#pragma unroll
    for (int s = 0; s < P2P_MAX_RANKS; ++s) {
        wv[s] = __shfl_sync(0xffffffffu, wl, s) * inv;
        if (s < N && wv[s] != 0.f) {
            const uint64_t* w = mine + s * slot_words + row * AT_DV + c;
            ll_load2_raw(w, raw[s][0], raw[s][1]);
            ll_load2_raw(w + 2, raw[s][2], raw[s][3]);
        }
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < P2P_MAX_RANKS; ++s) {
        if (s >= N || wv[s] == 0.f) continue;
        const uint64_t* w = mine + s * slot_words + row * AT_DV + c;
        acc.x = fmaf(wv[s], __uint_as_float(ll_wait1(w, ep, raw[s][0], 51)), acc.x);
        acc.y = fmaf(wv[s], __uint_as_float(ll_wait1(w + 1, ep, raw[s][1], 51)), acc.y);
        acc.z = fmaf(wv[s], __uint_as_float(ll_wait1(w + 2, ep, raw[s][2], 51)), acc.z);
        acc.w = fmaf(wv[s], __uint_as_float(ll_wait1(w + 3, ep, raw[s][3], 51)), acc.w);
    }
    const float L = (W > 0.f) ? M + logf(W) : -INFINITY;
    if (wi < N) {
        // ranks start on different destinations; warp 0 stores to this rank's
        // own region and then reads those words back (same threads)
        const int d = (p.a.rank + wi) % N;
        uint64_t* slot = reinterpret_cast<uint64_t*>(p.a.region[d] + p.gath_off + (long long)p.a.rank * p.gath_slot);
        xstore_row(slot + row * AT_DV + c, slot + (long long)p.B * p.hs * AT_DV + row, acc, L, eg,
                   q == 0 && lane == 0);
        if constexpr (UNPACK) xunpack_head(p, d * p.hs + hl, q, b, lane, eg);
    }
    xput_done(p.a, XCH_GATH, eg);
}

// grid (64 heads, 4 column quarters, B), 32 threads: the receive side on its
// own (the emulated-rank test hook runs it as a separate stage).
__global__ void __launch_bounds__(32) xunpack_kernel(XMergeParams p) {
    pdl_wait();
    pdl_trigger();
    xunpack_head(p, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x,
                 *reinterpret_cast<volatile unsigned*>(p.a.ctr + XCH_GATH));
}

}  // namespace wl
