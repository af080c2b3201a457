// p2p.cuh — the sharded decode's two exchanges over NVLink peer memory.
//
// Every rank owns one exchange region in its HBM that every other rank has
// mapped (CUDA IPC); layout:
//   [P2P_OFF_CAND, ...)            candidates, slot s = rank s's block
//   [P2P_OFF_CAND + N * cand_slot) partials, two copies (by epoch parity) of N slots
// An exchange is one put kernel per rank: it writes the rank's local block into
// slot `rank` of every region (its own included) in a self-validating wire
// format (below), tagged with the exchange's epoch — the count of exchanges of
// that type so far, identical on every rank. A consumer reads the slots of its
// local region, waiting (bounded) on each word until its tag matches.
//
// Reuse. Candidate slots are written once per owner step, and a rank only
// starts its next candidate put after its previous partial exchange, which
// needed every peer's partials — so every peer has finished reading the
// previous candidates. Partials use two copies (by epoch parity): a
// consumer-only step has no other exchange, and a fast rank may put step i + 1
// while a slow one still merges step i; it cannot reach step i + 2 before the
// slow rank's step i + 1 partials exist. A stale word carries an older epoch,
// so it never passes for new data.
//
// No TMA and no multicast: plain loads and stores, peer stores included.
#pragma once
#include "ptx.cuh"

namespace wl {

constexpr int P2P_MAX_RANKS = 8;
constexpr int XCH_CAND = 0, XCH_PART = 1, XCH_GATH = 2, XCH_TYPES = 3;
constexpr long long P2P_OFF_CAND = 0;

struct P2PArgs {
    uint8_t* region[P2P_MAX_RANKS];  // every rank's region in this process's address space
    int nranks, rank;
    unsigned* ctr;  // this rank's counters: [type] epoch, [XCH_TYPES + type] put CTAs done
};

// ---- the wire format: one aligned 8-byte store per 4-byte payload word ----
// {low: payload, high: epoch}. An aligned 64-bit store is single-copy atomic, so
// a receiver that reads a word whose epoch matches has that word's payload — no
// fence and no separate flag are needed (system-scope fences and release stores
// cost several microseconds each on this platform).
__device__ __forceinline__ void ll_store2(uint64_t* dst, uint32_t a, uint32_t b, uint32_t epoch) {
    const uint64_t x = ((uint64_t)epoch << 32) | a, y = ((uint64_t)epoch << 32) | b;
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(x), "l"(y) : "memory");
}
__device__ __forceinline__ void ll_load2_raw(const uint64_t* src, uint64_t& x, uint64_t& y) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(src) : "memory");
}
__device__ __forceinline__ uint64_t ll_load1_raw(const uint64_t* src) {
    uint64_t x;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(x) : "l"(src) : "memory");
    return x;
}
// Payload of one word once its epoch matches; bounded (error recorded, 0 returned).
__device__ __forceinline__ uint32_t ll_wait1(const uint64_t* src, uint32_t epoch, uint64_t first, unsigned site) {
    uint64_t x = first;
    if ((uint32_t)(x >> 32) == epoch) return (uint32_t)x;
    const long long t0 = clock64(), lim = g_wait_cycles;
    while (true) {
        x = ll_load1_raw(src);
        if ((uint32_t)(x >> 32) == epoch) return (uint32_t)x;
        if (clock64() - t0 > lim) {
            set_error(ERRC_TIMEOUT, site);
            return 0u;
        }
        __nanosleep(128);
    }
}
// Two consecutive words (16-byte aligned).
__device__ __forceinline__ void ll_load2(const uint64_t* src, uint32_t epoch, unsigned site, uint32_t& a,
                                         uint32_t& b) {
    uint64_t x, y;
    ll_load2_raw(src, x, y);
    a = ll_wait1(src, epoch, x, site);
    b = ll_wait1(src + 1, epoch, y, site);
}

// Copies n32 (even) payload words from `src` into slot `rank` of every rank's
// region in the wire format, at byte offset
//   dst_off + rank * slot_bytes (+ parity_bytes when the new epoch is even);
// then the last CTA advances this rank's epoch of `type`.
__global__ void __launch_bounds__(256) p2p_put_kernel(P2PArgs a, int type, const uint32_t* src, long long n32,
                                                      long long dst_off, long long slot_bytes,
                                                      long long parity_bytes) {
    pdl_wait();
    pdl_trigger();
    const uint32_t epoch = *reinterpret_cast<volatile unsigned*>(a.ctr + type) + 1u;
    const long long off = dst_off + (long long)a.rank * slot_bytes + ((epoch & 1u) ? 0 : parity_bytes);
    const long long n2 = n32 / 2, stride = (long long)gridDim.x * blockDim.x;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n2; i += stride) {
        const uint2 v = reinterpret_cast<const uint2*>(src)[i];
        for (int q = 0; q < a.nranks; ++q) {
            const int pr = (a.rank + q) % a.nranks;  // ranks start on different destinations
            ll_store2(reinterpret_cast<uint64_t*>(a.region[pr] + off) + 2 * i, v.x, v.y, epoch);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(a.ctr + XCH_TYPES + type, 1u);
        if (prev == gridDim.x - 1) {
            a.ctr[XCH_TYPES + type] = 0;
            a.ctr[type] = epoch;  // every CTA has read the old value by now
        }
    }
}

// Where a consumer finds one exchange in its region: the words of slot s start
// at base + s * slot_words (+ parity_words for the even-epoch copy).
struct P2PRecv {
    const uint64_t* base;  // null: not an exchange
    long long slot_words;
    long long parity_words;
    const unsigned* epoch_ctr;  // this rank's epoch counter of the type
};

__device__ __forceinline__ uint32_t p2p_epoch(const P2PRecv& r) {
    return *reinterpret_cast<const volatile unsigned*>(r.epoch_ctr);
}
__device__ __forceinline__ const uint64_t* p2p_slot(const P2PRecv& r, uint32_t epoch, int s) {
    return r.base + (long long)s * r.slot_words + ((epoch & 1u) ? 0 : r.parity_words);
}

}  // namespace wl
