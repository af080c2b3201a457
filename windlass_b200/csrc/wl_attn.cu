// wl_attn.cu — host side of the C ABI declared in include/wl_attn.h, plus the
// single translation unit that holds every kernel of the library (so the
// device error word is one symbol).
//
// The orchestration mirrors the hot block of the reference's run_attention
// (src/glm_layer_runner.cuh:582-644):
//   owner    -> indexer scores -> top-k -> (publish) -> sparse attention
//   consumer -> (require) -> [normalise list] -> sparse attention
//   dense    -> attention over every key
// followed by the split-K (o, lse) merge. All launches go on the caller's
// stream, with programmatic dependent launch between the library's kernels;
// no call allocates (a communicator allocates its peer-exchange region once,
// at creation); every failure is a status code.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <vector>
#include <mutex>
#include <nccl.h>

#include "../../include/wl_attn.h"
#include "cache_append.cuh"
#include "idx_query.cuh"
#include "indexer.cuh"
#include "mla_attn.cuh"
#include "mla_attn64.cuh"
#include "p2p.cuh"
#include "topk.cuh"
#include "xmerge.cuh"
#include "gemv_tc.cuh"

namespace {

// Phase timeline of the sharded decode (diagnostics, off by default): when a
// caller has set a stamp buffer with wl_diag_phase_stamps, a one-thread kernel
// writes the global timer at each phase boundary of wl_attn_decode_sharded.
// It works inside CUDA graphs (the buffer pointer is baked into the captured
// launches). The extra launches break the programmatic overlap between the
// phases, so a stamped step runs somewhat slower than an unstamped one.
__global__ void phase_stamp_kernel(unsigned long long* buf, int i) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    buf[i] = t;
}
std::mutex g_ph_mu;
unsigned long long* g_ph_buf = nullptr;
int g_ph_cap = 0;
int g_ph_n = 0;
void phase_stamp(cudaStream_t st) {
    std::lock_guard<std::mutex> lk(g_ph_mu);
    if (!g_ph_buf || g_ph_n >= g_ph_cap) return;
    phase_stamp_kernel<<<1, 1, 0, st>>>(g_ph_buf, g_ph_n++);
}
#define WL_PHASE(st) phase_stamp(st)

constexpr int kMaxSplits = 32;   // split-K CTAs per decode row (the merge takes up to 32 parts)
constexpr int kMaxDevices = 64;

#define WL_CUDA_TRY(expr)                                           \
    do {                                                            \
        cudaError_t e_ = (expr);                                    \
        if (e_ != cudaSuccess) {                                    \
            std::fprintf(stderr, "wl_attn: %s failed: %s\n", #expr, \
                         cudaGetErrorString(e_));                   \
            return WL_ERR_CUDA;                                     \
        }                                                           \
    } while (0)

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
inline long long ceil_div(long long a, long long b) { return (a + b - 1) / b; }

bool cfg_supported(const wl_attn_cfg* c) {
    return c && c->n_heads == wl::AT_H && c->kv_lora == wl::AT_DV && c->rope_dim == wl::AT_D - wl::AT_DV &&
           c->idx_heads == wl::IDX_H && c->idx_dim == wl::IDX_D && c->index_topk > 0 && c->T_max > 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per-device one-time kernel attributes (dynamic shared memory opt-in) and SM count.
std::mutex g_attr_mu;
bool g_attr_done[kMaxDevices];
int g_sm_count[kMaxDevices];

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    return g_sm_count[dev] > 0 ? g_sm_count[dev] : 148;
}

int ensure_attrs() {
    int dev = 0;
    WL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return WL_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    if (g_attr_done[dev]) return WL_OK;
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::mla_attn64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::PfLayout::BYTES));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::sel_normalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::TOPK_SMEM_MAX * 4));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::indexer_stream_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::IdxStream<1>::BYTES));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::indexer_stream_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::IdxStream<4>::BYTES));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::topk_partition_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::TOPKM_PART_SMEM));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::topk_threshold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::TOPKM_THR_SMEM));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::gemv_tc_kernel<wl::GV_IDXQ>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::GvShape<wl::GV_IDXQ>::BYTES));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::gemv_tc_kernel<wl::GV_PROJV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::GvShape<wl::GV_PROJV>::BYTES));
    WL_CUDA_TRY(cudaFuncSetAttribute(wl::gemv_tc_kernel<wl::GV_ABSQ>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     wl::GvShape<wl::GV_ABSQ>::BYTES));
    int sms = 0;
    WL_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    g_sm_count[dev] = sms;
    g_attr_done[dev] = true;
    return WL_OK;
}

// cuTensorMapEncodeTiled, fetched once from the driver through the runtime
// (the library links only the CUDA runtime).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// The fp8 key cache as {128 bytes, T keys, n_seq sequences}, 128x128-byte boxes,
// 128B swizzle, zero fill past T.
int encode_keys_map(CUtensorMap* tm, const void* keys, int32_t T, int n_seq, int64_t seq_stride) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return WL_ERR_CUDA;
    if (n_seq > 1 && (seq_stride < (int64_t)T * 128 || (seq_stride & 15))) return WL_ERR_ARG;
    const cuuint64_t dims[3] = {128, (cuuint64_t)T, (cuuint64_t)n_seq};
    const cuuint64_t strides[2] = {128, (cuuint64_t)(n_seq > 1 ? seq_stride : (int64_t)T * 128)};
    const cuuint32_t box[3] = {128, 128, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(keys), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::fprintf(stderr, "wl_attn: cuTensorMapEncodeTiled failed (%d)\n", (int)r);
        return WL_ERR_CUDA;
    }
    return WL_OK;
}

// Launches a kernel of the decode chain with programmatic stream
// serialisation, so that its launch and prologue overlap the previous kernel
// (each such kernel calls pdl_wait() before touching global data). WL_NO_PDL=1
// in the environment turns this off.
bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("WL_NO_PDL");
        return !(e && e[0] == '1');
    }();
    return on;
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// A bf16 matrix [outer][inner] (row stride `row_elems`) as a 2D tensor map with
// {box_inner, box_outer} boxes, 128B swizzle (box_inner = 64: 128-byte rows).
int encode_bf16_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer, uint64_t row_elems,
                   uint32_t box_inner, uint32_t box_outer) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return WL_ERR_CUDA;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)row_elems * 2};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::fprintf(stderr, "wl_attn: cuTensorMapEncodeTiled (weights) failed (%d)\n", (int)r);
        return WL_ERR_CUDA;
    }
    return WL_OK;
}

// One of the tensor-core weight products (gemv_tc.cuh), programmatic launch;
// the query projection as 4-CTA clusters along K.
template <int MODE>
int launch_gemv(const wl::GvParams& p, dim3 grid, cudaStream_t st) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(wl::GV_THREADS);
    cfg.dynamicSmemBytes = wl::GvShape<MODE>::BYTES;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl_enabled()) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (MODE == wl::GV_IDXQ) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = wl::GV_CL;
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    WL_CUDA_TRY(cudaLaunchKernelEx(&cfg, wl::gemv_tc_kernel<MODE>, p));
    return WL_OK;
}

// Zeroes n_rows fused top-k histograms (HB + 1 words each) in the launch chain.
cudaError_t hist_zero(unsigned* hist, int32_t n_rows, cudaStream_t st) {
    const long long n = (long long)n_rows * (wl::HB + 1);
    const int blocks = (int)std::min<long long>(148, (n + 2047) / 2048);
    return launch_pdl(wl::hist_zero_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0, st, hist, n);
}

// The absorbed queries [n_rows][64][576] bf16 as a 2D tensor {576, 64 n_rows},
// 64 x 64 boxes, 128B swizzle (the prefill attention's query tiles).
int encode_q_map(CUtensorMap* tm, const void* q_abs, int32_t n_rows) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return WL_ERR_CUDA;
    const cuuint64_t dims[2] = {(cuuint64_t)wl::AT_D, (cuuint64_t)wl::AT_H * n_rows};
    const cuuint64_t strides[1] = {(cuuint64_t)wl::AT_D * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)wl::AT_H};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(q_abs), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        std::fprintf(stderr, "wl_attn: cuTensorMapEncodeTiled (queries) failed (%d)\n", (int)r);
        return WL_ERR_CUDA;
    }
    return WL_OK;
}

// The (o) partials [rows * splits][64][512] fp32 as {512, 64 rows * splits},
// 32 x 64 boxes, 128B swizzle (the attention's staged output).
int encode_o_map(CUtensorMap* tm, void* o_part, int64_t n_parts) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return WL_ERR_CUDA;
    const cuuint64_t dims[2] = {(cuuint64_t)wl::AT_DV, (cuuint64_t)(wl::AT_H * n_parts)};
    const cuuint64_t strides[1] = {(cuuint64_t)wl::AT_DV * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)wl::AT_H};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, o_part, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? WL_OK : WL_ERR_CUDA;
}

int rows_ok(const wl_rows* r, int32_t T) {
    if (!r || r->n_rows <= 0 || r->rows_per_seq <= 0 || r->len0 < 0 || r->len_step < 0 || T <= 0)
        return WL_ERR_ARG;
    return WL_OK;
}

// Split-K CTAs per decode row: about one wave of CTAs over all rows (the
// attention is latency-bound at decode batches), at most `cap`, and no more
// than one per 64-key tile of the longest list. The kernel spreads each row's
// entries (inside its key window) evenly over these CTAs.
// WL_ATTN_SPLITS=n in the environment caps it further (a tuning knob).
int splits_env_cap() {
    static const int v = [] {
        const char* e = std::getenv("WL_ATTN_SPLITS");
        const int n = e ? std::atoi(e) : 0;
        return n > 0 ? n : 1 << 30;
    }();
    return v;
}
int splits_for(int32_t rows, long long n_max, int cap) {
    if (cap > splits_env_cap()) cap = splits_env_cap();
    long long s = sm_count() / (rows > 0 ? rows : 1);
    s = s < 1 ? 1 : s;
    s = s > cap ? cap : s;
    const long long n = n_max > 0 ? n_max : 1;
    const long long tiles = ceil_div(n, wl::AT_TILE);
    if (s > tiles) s = tiles;
    // no CTA left without work when the list is full: as many splits as whole
    // shares of ceil(n / s) rounded up to tiles need
    const long long per = ceil_div(ceil_div(n, s), wl::AT_TILE) * wl::AT_TILE;
    return (int)ceil_div(n, per);
}

// ---- kernel launchers ----------------------------------------------------------
int launch_indexer(const wl_attn_cfg* cfg, const wl_index_cache* cache, int32_t T, const wl_rows* rows,
                   const void* q_idx, const float* w_idx, float* out, int64_t out_stride,
                   cudaStream_t st, unsigned* hist = nullptr) {
    if (!cache || !cache->keys || !cache->scale || !q_idx || !w_idx || !out) return WL_ERR_ARG;
    if (!aligned16(cache->keys) || !aligned16(q_idx) || (cache->keys_seq_stride & 15)) return WL_ERR_ARG;
    if (out_stride < T) return WL_ERR_ARG;
    wl::IdxParams p{};
    p.keys = static_cast<const uint8_t*>(cache->keys);
    p.keys_seq = cache->keys_seq_stride;
    p.scale = cache->scale;
    p.scale_seq = cache->scale_seq_stride;
    p.T = T;
    p.n_rows = rows->n_rows;
    p.rows_per_seq = rows->rows_per_seq;
    p.len0 = rows->len0;
    p.len_step = rows->len_step;
    p.q = static_cast<const __nv_bfloat16*>(q_idx);
    p.w = w_idx;
    p.out = out;
    p.out_stride = out_stride;
    p.qk_scale = cfg->idx_qk_scale;
    const int ntiles = (int)ceil_div(T, wl::IDX_TILE);
    wl::IdxStreamParams sp{};
    const int n_seq = (int)ceil_div(rows->n_rows, rows->rows_per_seq);
    if (int e = encode_keys_map(&sp.tm_keys, cache->keys, T, n_seq, cache->keys_seq_stride)) return e;
    if (rows->n_rows >= 8 && (rows->rows_per_seq % 4 == 0 || rows->rows_per_seq >= rows->n_rows)) {
        // Many rows over shared caches (prefill): 4 consecutive rows of one
        // sequence per MMA (N = 256), one CTA per group over all its tiles.
        const int groups = (int)ceil_div(rows->n_rows, 4);
        if (groups > 65535) return WL_ERR_ARG;
        WL_CUDA_TRY(launch_pdl(wl::indexer_stream_kernel<4>, dim3(1, groups), dim3(wl::IdxStream<4>::THREADS),
                               wl::IdxStream<4>::BYTES, st, p, sp, (unsigned*)nullptr, ntiles));
    } else {
        // Decode: each row streams its own cache; at most one CTA per SM in
        // total, each over a contiguous range of tiles.
        if (rows->n_rows > 65535) return WL_ERR_ARG;
        int cpr = wl::IDX_CTAS_PER_SM * sm_count() / rows->n_rows;
        if (cpr < 1) cpr = 1;
        if (cpr > ntiles) cpr = ntiles;
        const int tpc = (int)ceil_div(ntiles, cpr);
        dim3 grid((unsigned)ceil_div(ntiles, tpc), rows->n_rows);
        WL_CUDA_TRY(launch_pdl(wl::indexer_stream_kernel<1>, grid, dim3(wl::IdxStream<1>::THREADS),
                               wl::IdxStream<1>::BYTES, st, p, sp, hist, tpc));
    }
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
}

// Rows longer than this use the multi-CTA top-k (which needs a workspace).
constexpr int kTopkMultiMin = wl::TOPK_SMEM_MAX + 1;
// Rows in (kTopkClusterMin, kTopkClusterMax] use the one-launch cluster top-k
// (with a workspace for its first-level histogram).
constexpr int kTopkClusterMin = 8192;
constexpr int kTopkClusterMax = wl::TOPKC_CL * wl::TOPKC_THREADS * 24;
// Whether a decode row of length T selects through a first-level histogram
// (which the indexer's epilogue can then accumulate for free).
inline bool topk_wants_hist(int32_t T, int32_t k) { return T > kTopkClusterMin && k < T; }
constexpr int kTopkMaxChunks = 1024;
// Rows up to this length (without the cluster path) select in one CTA with the
// row in registers.
constexpr int kTopkRegMax = wl::TOPK_THREADS * 32;
static_assert(wl::TOPK_HIST_BITS == wl::HBITS, "indexer-fused histogram and top-k agree on bits");

struct TopkWs {
    unsigned* hist;  // [rows][HB] then cand_n [rows] (one contiguous block, zeroed per call)
    unsigned* cand_n;
    unsigned* cand_key;
    int* cand_pos;
    unsigned* cnt_gt;
    unsigned* cnt_eq;
    unsigned* thr;
    long long cand_stride;
};

size_t topk_ws_bytes(int32_t rows, int32_t T) {
    return align256((size_t)rows * (wl::HB + 1) * 4) + 2 * align256((size_t)rows * T * 4) +
           2 * align256((size_t)rows * kTopkMaxChunks * 4) + align256((size_t)rows * 8) + 256;
}

TopkWs topk_ws_carve(void* base, int32_t rows, int32_t T) {
    TopkWs w{};
    char* b = static_cast<char*>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        void* p = b + off;
        off += align256(bytes);
        return p;
    };
    w.hist = static_cast<unsigned*>(take((size_t)rows * (wl::HB + 1) * 4));
    w.cand_n = w.hist + (size_t)rows * wl::HB;
    w.cand_key = static_cast<unsigned*>(take((size_t)rows * T * 4));
    w.cand_pos = static_cast<int*>(take((size_t)rows * T * 4));
    w.cnt_gt = static_cast<unsigned*>(take((size_t)rows * kTopkMaxChunks * 4));
    w.cnt_eq = static_cast<unsigned*>(take((size_t)rows * kTopkMaxChunks * 4));
    w.thr = static_cast<unsigned*>(take((size_t)rows * 8));
    w.cand_stride = T;
    return w;
}

// First-level histogram (top HBITS bits of the score keys) when the indexer
// did not fuse it.
__global__ void topk_hist_kernel(const float* in, long long in_stride, int len0, int len_step, int rows_per_seq,
                                 int T, unsigned* hist) {
    wl::pdl_wait();
    wl::pdl_trigger();
    const int r = blockIdx.y;
    const long long l = (long long)len0 + (long long)(r % rows_per_seq) * len_step;
    const int len = (int)(l < T ? l : T);
    const float* row = in + (long long)r * in_stride;
    unsigned* hrow = hist + (long long)r * wl::HB;
    for (long long base = blockIdx.x * (long long)blockDim.x; base < len; base += (long long)gridDim.x * blockDim.x) {
        const long long i = base + threadIdx.x;
        const bool valid = i < len;
        const uint32_t b = valid ? wl::ordered_key(row[i]) >> (32 - wl::HBITS) : 0xFFFFFFFFu;
        const unsigned peers = __match_any_sync(0xffffffffu, b);
        if (valid && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(hrow + b, (unsigned)__popc(peers));
    }
}

int max_row_len(const wl_rows* rows, int32_t T) {
    const int last = (rows->rows_per_seq < rows->n_rows ? rows->rows_per_seq : rows->n_rows) - 1;
    const long long l = (long long)rows->len0 + (long long)last * rows->len_step;
    return (int)(l < T ? l : T);
}

// hist_ready: the histogram block of `ws` already holds this call's
// first-level histogram (fused into the indexer) and cand_n is zero.
bool lmax_le_reg(const wl_rows* rows, int32_t T) { return max_row_len(rows, T) <= kTopkRegMax; }

// `co` (optional) also writes each selection as (score, base + key) candidates;
// seg_len > 0 reads segmented rows (single-CTA register path only).
int launch_topk(const float* index, int64_t index_stride, const wl_rows* rows, int32_t T, int32_t k,
                const int32_t* cand_idx, int32_t* sel_out, int64_t sel_stride, int32_t* sel_n_out,
                cudaStream_t st, const TopkWs* ws = nullptr, bool hist_ready = false,
                const wl::CandOut* co = nullptr, int32_t seg_len = 0, int64_t seg_stride = 0,
                const wl::P2PRecv* ll = nullptr, int64_t ll_idx_off = 0) {
    const wl::CandOut cout = co ? *co : wl::CandOut{};
    if (ll && !(lmax_le_reg(rows, T))) return WL_ERR_ARG;
    if ((!index && !ll) || !sel_out || k <= 0) return WL_ERR_ARG;
    if (sel_stride < (k < T ? k : T)) return WL_ERR_ARG;
    const int lmax = max_row_len(rows, T);
    const bool cluster = lmax > kTopkClusterMin && lmax <= kTopkClusterMax;
    if (seg_len > 0 && (lmax > kTopkRegMax || (seg_len % 32))) return WL_ERR_ARG;
    if (co && !(seg_len > 0 || (ws && !cand_idx && cluster) || lmax <= kTopkRegMax)) return WL_ERR_ARG;
    if (seg_len == 0 && ws && !cand_idx && (cluster || lmax >= kTopkMultiMin) && rows->n_rows <= 65535) {
        wl::TopkMParams p{};
        p.in = index;
        p.in_stride = index_stride;
        p.n_rows = rows->n_rows;
        p.rows_per_seq = rows->rows_per_seq;
        p.len0 = rows->len0;
        p.len_step = rows->len_step;
        p.T = T;
        p.k = k;
        p.out = sel_out;
        p.out_stride = sel_stride;
        p.n_out = sel_n_out;
        p.hist = ws->hist;
        // ~2 waves of 256-thread CTAs over all rows, chunks a multiple of 1024.
        long long chunk = ceil_div(ceil_div((long long)lmax * rows->n_rows, 2LL * sm_count()), 1024) * 1024;
        if (chunk < 2048) chunk = 2048;
        if (ceil_div(lmax, chunk) > kTopkMaxChunks) chunk = ceil_div(ceil_div(lmax, kTopkMaxChunks), 1024) * 1024;
        p.chunk = (int)chunk;
        p.n_chunks = (int)ceil_div(lmax, chunk);
        p.cand_key = ws->cand_key;
        p.cand_pos = ws->cand_pos;
        p.cand_stride = ws->cand_stride;
        p.cand_n = ws->cand_n;
        p.cnt_gt = ws->cnt_gt;
        p.cnt_eq = ws->cnt_eq;
        p.thr = ws->thr;
        if (!hist_ready) {
            WL_CUDA_TRY(hist_zero(ws->hist, rows->n_rows, st));
            topk_hist_kernel<<<dim3((unsigned)ceil_div(lmax, 8192), rows->n_rows), 256, 0, st>>>(
                index, index_stride, rows->len0, rows->len_step, rows->rows_per_seq, T, ws->hist);
            WL_CUDA_TRY(cudaGetLastError());
        }
        if (cluster) {
            const dim3 gc(wl::TOPKC_CL, rows->n_rows);
            const int vec4 = aligned16(index) && (index_stride & 3) == 0;
            if (lmax <= wl::TOPKC_CL * wl::TOPKC_THREADS * 4)
                WL_CUDA_TRY(launch_pdl(wl::topk_cluster_kernel<4>, gc, dim3(wl::TOPKC_THREADS), 0, st, p, vec4, cout));
            else if (lmax <= wl::TOPKC_CL * wl::TOPKC_THREADS * 8)
                WL_CUDA_TRY(launch_pdl(wl::topk_cluster_kernel<8>, gc, dim3(wl::TOPKC_THREADS), 0, st, p, vec4, cout));
            else if (lmax <= wl::TOPKC_CL * wl::TOPKC_THREADS * 16)
                WL_CUDA_TRY(launch_pdl(wl::topk_cluster_kernel<16>, gc, dim3(wl::TOPKC_THREADS), 0, st, p, vec4, cout));
            else
                WL_CUDA_TRY(launch_pdl(wl::topk_cluster_kernel<24>, gc, dim3(wl::TOPKC_THREADS), 0, st, p, vec4, cout));
            WL_CUDA_TRY(cudaGetLastError());
            return WL_OK;
        }
        const dim3 g(p.n_chunks, rows->n_rows);
        WL_CUDA_TRY(launch_pdl(wl::topk_partition_kernel, g, dim3(wl::TOPKM_THREADS), wl::TOPKM_PART_SMEM, st, p));
        WL_CUDA_TRY(launch_pdl(wl::topk_threshold_kernel, dim3(rows->n_rows), dim3(wl::TOPK_THREADS), wl::TOPKM_THR_SMEM, st, p));
        WL_CUDA_TRY(launch_pdl(wl::topk_emit_kernel, g, dim3(wl::TOPKM_THREADS), 0, st, p));
        WL_CUDA_TRY(cudaGetLastError());
        return WL_OK;
    }
    wl::TopkParams p{};
    p.in = index;
    p.in_stride = index_stride;
    p.n_rows = rows->n_rows;
    p.rows_per_seq = rows->rows_per_seq;
    p.len0 = rows->len0;
    p.len_step = rows->len_step;
    p.T = T;
    p.k = k;
    p.cand_idx = cand_idx;
    p.out = sel_out;
    p.out_stride = sel_stride;
    p.n_out = sel_n_out;
    p.seg_len = seg_len;
    p.seg_stride = seg_stride;
    if (ll) {
        p.ll = *ll;
        p.ll_idx_off = ll_idx_off;
    }
    if (lmax <= kTopkRegMax) {
        const int vec4 = aligned16(index) && (index_stride & 3) == 0 && (seg_stride & 3) == 0;
        const dim3 g(rows->n_rows), b(wl::TOPK_THREADS);
        const int per = lmax <= wl::TOPK_THREADS * 4 ? 4 : lmax <= wl::TOPK_THREADS * 8 ? 8
                      : lmax <= wl::TOPK_THREADS * 16 ? 16 : 32;
        auto go = [&](auto kernel) { return launch_pdl(kernel, g, b, 0, st, p, vec4, cout); };
        cudaError_t e;
        if (ll)
            e = per == 4 ? go(wl::topk_reg_kernel<4, true>) : per == 8 ? go(wl::topk_reg_kernel<8, true>)
              : per == 16 ? go(wl::topk_reg_kernel<16, true>) : go(wl::topk_reg_kernel<32, true>);
        else
            e = per == 4 ? go(wl::topk_reg_kernel<4, false>) : per == 8 ? go(wl::topk_reg_kernel<8, false>)
              : per == 16 ? go(wl::topk_reg_kernel<16, false>) : go(wl::topk_reg_kernel<32, false>);
        WL_CUDA_TRY(e);
        return WL_OK;
    }
    const size_t smem = lmax <= wl::TOPK_SMEM_MAX ? (size_t)lmax * 4 : 0;
    WL_CUDA_TRY(launch_pdl(wl::topk_kernel, dim3(rows->n_rows), dim3(wl::TOPK_THREADS), smem, st, p));
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
}

int launch_normalize(const int32_t* in, int64_t in_stride, const int32_t* n_in_dev, int32_t n_in,
                     const wl_rows* rows, int32_t T, int32_t* out, int64_t out_stride, int32_t* n_out,
                     cudaStream_t st) {
    if (!in || !out) return WL_ERR_ARG;
    const size_t smem = (size_t)ceil_div(T, 32) * 4;
    if (smem > 200 * 1024) return WL_ERR_UNSUPPORTED;
    wl::NormParams p{};
    p.in = in;
    p.in_stride = in_stride;
    p.n_in_dev = n_in_dev;
    p.n_in = n_in;
    p.n_rows = rows->n_rows;
    p.rows_per_seq = rows->rows_per_seq;
    p.len0 = rows->len0;
    p.len_step = rows->len_step;
    p.T = T;
    p.out = out;
    p.out_stride = out_stride;
    p.n_out = n_out;
    WL_CUDA_TRY(launch_pdl(wl::sel_normalize_kernel, dim3(rows->n_rows), dim3(wl::TOPK_THREADS), smem, st, p));
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
}

int launch_attn(const wl_attn_cfg* cfg, const wl_latent_cache* c, int32_t T, int64_t len_T,
                const wl_rows* rows, const void* q_abs, const int32_t* sel, int64_t sel_stride,
                const int32_t* sel_n_dev, int32_t sel_n, int64_t win_lo, int64_t win_hi, int32_t split_keys,
                float* o_part, float* lse_part, int32_t max_splits, cudaStream_t st, bool dyn_split = false) {
    if (!c || !c->c_kv || !c->k_rot || !q_abs || !o_part || !lse_part) return WL_ERR_ARG;
    if (!aligned16(c->c_kv) || !aligned16(c->k_rot) || !aligned16(q_abs)) return WL_ERR_ARG;
    if ((c->c_kv_row_stride & 7) || (c->k_rot_row_stride & 7) || (c->c_kv_seq_stride & 7) ||
        (c->k_rot_seq_stride & 7))
        return WL_ERR_ARG;
    if (split_keys < 0 || (split_keys % wl::AT_TILE) || max_splits <= 0) return WL_ERR_ARG;
    if (split_keys == 0 && max_splits != 1 && !dyn_split) return WL_ERR_ARG;
    if (rows->n_rows > 65535 || max_splits > 65535) return WL_ERR_ARG;
    wl::AttnParams p{};
    p.c_kv = static_cast<const __nv_bfloat16*>(c->c_kv);
    p.ckv_row = c->c_kv_row_stride;
    p.ckv_seq = c->c_kv_seq_stride;
    p.k_rot = static_cast<const __nv_bfloat16*>(c->k_rot);
    p.krot_row = c->k_rot_row_stride;
    p.krot_seq = c->k_rot_seq_stride;
    p.T = T;
    p.n_rows = rows->n_rows;
    p.rows_per_seq = rows->rows_per_seq;
    p.len0 = rows->len0;
    p.len_step = rows->len_step;
    p.len_T = (int)len_T;
    p.q_abs = static_cast<const __nv_bfloat16*>(q_abs);
    p.sel = sel;
    p.sel_stride = sel_stride;
    p.sel_n_dev = sel_n_dev;
    p.sel_n = sel_n;
    p.win_lo = win_lo;
    p.win_hi = win_hi;
    p.split_keys = split_keys;
    p.dyn_split = dyn_split ? 1 : 0;
    p.max_splits = max_splits;
    p.o_part = o_part;
    p.lse_part = lse_part;
    p.scale_log2 = cfg->softmax_scale * 1.4426950408889634f;
    // Heads as M = 64, gather / QK / softmax / P.V pipelined over 64-key tiles;
    // grid (splits, rows), each CTA one (o, lse) partial.
    wl::PfParams pp{};
    if (int e = encode_q_map(&pp.tm_q, q_abs, rows->n_rows)) return e;
    // O leaves through TMA stores (plain per-thread stores measured 2-3 us
    // slower per layer-step); plain stores only when the map cannot be made
    pp.o_tma = aligned16(o_part) && encode_o_map(&pp.tm_o, o_part, (int64_t)rows->n_rows * max_splits) == WL_OK;
    WL_CUDA_TRY(launch_pdl(wl::mla_attn64_kernel, dim3(max_splits, rows->n_rows), dim3(wl::PF_THREADS),
                           wl::PfLayout::BYTES, st, p, pp));
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
}

int launch_merge(const float* o_part, const float* lse_part, int32_t n_rows, int32_t n_parts, int64_t row_stride,
                 int64_t part_stride, int64_t lse_row_stride, int64_t lse_part_stride, int32_t n_heads,
                 int32_t dv, float* ctx, float* lse, cudaStream_t st, int64_t ctx_row_stride = 0,
                 int64_t lse_out_row_stride = 0, const wl::P2PRecv* ll = nullptr, int64_t ll_lse_off = 0) {
    if ((!ll && (!o_part || !lse_part)) || !ctx || n_rows <= 0 || n_parts <= 0 || n_parts > 32 || (dv % 128) ||
        n_heads <= 0 || n_rows > 65535)
        return WL_ERR_ARG;
    wl::MergeParams p{o_part, lse_part, n_rows, n_parts, row_stride, part_stride, lse_row_stride,
                      lse_part_stride, n_heads, dv, ctx, lse,
                      ctx_row_stride > 0 ? ctx_row_stride : (int64_t)n_heads * dv,
                      lse_out_row_stride > 0 ? lse_out_row_stride : (int64_t)n_heads};
    if (ll) {
        p.ll = *ll;
        p.ll_lse_off = ll_lse_off;
    }
    if (ll)
        WL_CUDA_TRY(launch_pdl(wl::lse_merge_kernel<true>, dim3(n_heads, dv / 128, n_rows), dim3(32), 0, st, p));
    else if (n_rows < 4)  // few rows: four warps per CTA hide the partials' load latency
        WL_CUDA_TRY(launch_pdl(wl::lse_merge4_kernel, dim3(n_heads, dv / 128, n_rows), dim3(32 * wl::MG_WARPS), 0, st,
                               p));
    else  // enough CTAs to fill the SMs with one warp each
        WL_CUDA_TRY(launch_pdl(wl::lse_merge_kernel<false>, dim3(n_heads, dv / 128, n_rows), dim3(32), 0, st, p));
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
}

// ---- workspace carving ---------------------------------------------------------------
struct DecodeWs {
    float* index;
    int32_t* sel;
    int32_t* cnt;
    float* o_part;
    float* lse_part;
    float* lse_tmp;
    // sharded only
    float* cand_score;
    int32_t* cand_idx;
    float* cand_score_all;
    int32_t* cand_idx_all;
    float* cand_score_rows;
    int32_t* cand_idx_rows;
    float* part_send;
    float* part_recv;
    TopkWs topk;
    size_t bytes;
};

DecodeWs carve_decode(void* base, const wl_attn_cfg* cfg, int32_t T_max, int32_t batch, int32_t nranks) {
    DecodeWs w{};
    size_t off = 0;
    auto take = [&](size_t bytes) -> void* {
        void* p = base ? static_cast<char*>(base) + off : nullptr;
        off += align256(bytes);
        return p;
    };
    const size_t k = (size_t)cfg->index_topk;
    w.index = static_cast<float*>(take((size_t)batch * T_max * 4));
    const size_t sel_cap = (size_t)(nranks > 1 ? (size_t)T_max * nranks : (size_t)T_max);
    w.sel = static_cast<int32_t*>(take((size_t)batch * (sel_cap > k ? sel_cap : k) * 4));
    w.cnt = static_cast<int32_t*>(take((size_t)batch * 4));
    w.o_part = static_cast<float*>(take((size_t)batch * kMaxSplits * wl::AT_H * wl::AT_DV * 4));
    w.lse_part = static_cast<float*>(take((size_t)batch * kMaxSplits * wl::AT_H * 4));
    w.lse_tmp = static_cast<float*>(take((size_t)batch * wl::AT_H * 4));
    {
        void* tb = take(topk_ws_bytes(batch, T_max));
        if (base) w.topk = topk_ws_carve(tb, batch, T_max);
    }
    if (nranks > 1) {
        // one block [scores B x k][indices B x k]: the peer exchange sends it whole
        w.cand_score = static_cast<float*>(take((size_t)batch * k * 8));
        w.cand_idx = reinterpret_cast<int32_t*>(w.cand_score + (size_t)batch * k);
        w.cand_score_all = static_cast<float*>(take((size_t)nranks * batch * k * 4));
        w.cand_idx_all = static_cast<int32_t*>(take((size_t)nranks * batch * k * 4));
        w.cand_score_rows = static_cast<float*>(take((size_t)nranks * batch * k * 4));
        w.cand_idx_rows = static_cast<int32_t*>(take((size_t)nranks * batch * k * 4));
        const size_t part = (size_t)batch * (wl::AT_H * wl::AT_DV + wl::AT_H);
        w.part_send = static_cast<float*>(take(part * 4));
        w.part_recv = static_cast<float*>(take((size_t)nranks * part * 4));
    }
    w.bytes = off + 256;  // + base alignment slack
    return w;
}

void* align_base(void* ws) {
    return reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
}

int check_decode_io(const wl_attn_cfg* cfg, const wl_attn_decode_io* io) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (!io || io->batch <= 0 || io->T <= 0 || !io->q_abs || !io->ctx) return WL_ERR_ARG;
    if (io->T > cfg->T_max) return WL_ERR_T_EXCEEDS_MAX;
    if (io->mode != WL_MODE_OWNER && io->mode != WL_MODE_CONSUMER && io->mode != WL_MODE_DENSE) return WL_ERR_ARG;
    if (io->mode == WL_MODE_OWNER && (!io->q_idx || !io->w_idx || !io->index.keys || !io->index.scale))
        return WL_ERR_ARG;
    if (io->mode == WL_MODE_CONSUMER) {
        if (!io->sel_in) return WL_ERR_NO_INDICES;
        if (!io->sel_n_in && io->sel_n < 0) return WL_ERR_ARG;
        if (io->sel_stride <= 0) return WL_ERR_ARG;
    }
    return WL_OK;
}

// Gather (score, global index) of a rank's local top-k into fixed-size
// candidate rows; slots past the local count get (-inf, INT32_MAX).
__global__ void gather_candidates_kernel(const float* index, long long index_stride, const int* sel,
                                         long long sel_stride, const int* cnt, int k, long long t0,
                                         float* cs, int* ci) {
    const int r = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= k) return;
    const int n = cnt[r];
    float s = -INFINITY;
    int g = 0x7fffffff;
    if (j < n) {
        const int t = sel[(long long)r * sel_stride + j];
        s = index[(long long)r * index_stride + t];
        g = (int)(t0 + t);
    }
    cs[(long long)r * k + j] = s;
    ci[(long long)r * k + j] = g;
}

// The identity selection 0..T-1 of every row (an owner layer with
// index_topk >= T: the reference's top-k returns every key).
__global__ void identity_sel_kernel(int T, int* out, long long stride, int* n_out) {
    wl::pdl_wait();
    wl::pdl_trigger();
    const int r = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x)
        out[(long long)r * stride + i] = i;
    if (blockIdx.x == 0 && threadIdx.x == 0 && n_out) n_out[r] = T;
}

__global__ void row_counts_kernel(int n_rows, int len0, int len_step, int T, int k, int* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    const long long l = (long long)len0 + (long long)r * len_step;
    const int len = (int)(l < T ? l : T);
    out[r] = len < k ? len : k;
}

// [rank][row][k] -> [row][rank*k + j]
__global__ void candidates_to_rows_kernel(const float* s_all, const int* i_all, int nranks, int batch, int k,
                                          float* s_rows, int* i_rows) {
    const long long n = (long long)nranks * batch * k;
    for (long long x = blockIdx.x * (long long)blockDim.x + threadIdx.x; x < n; x += (long long)gridDim.x * blockDim.x) {
        const int j = (int)(x % k);
        const int b = (int)((x / k) % batch);
        const int rk = (int)(x / ((long long)k * batch));
        const long long dst = (long long)b * nranks * k + (long long)rk * k + j;
        s_rows[dst] = s_all[x];
        i_rows[dst] = i_all[x];
    }
}

}  // namespace

// Capacity of the peer exchange (rows per call, selection length) and its
// region layout; larger calls use the NCCL exchange.
constexpr int kP2PMaxRows = 32;
constexpr int kP2PMaxK = 4096;
// Slots hold the wire format: 8 bytes per 4-byte payload word. Region layout:
// [candidate slots: N x kP2PCandSlot][PART slots: N x xslot][GATH slots: N x xslot],
// xslot = the (o, lse) words of kP2PMaxRows rows x 64/N heads (xmerge.cuh).
constexpr long long kP2PCandSlot = (long long)kP2PMaxRows * kP2PMaxK * 2 * 8;  // scores, indices

struct wl_comm {
    ncclComm_t comm;
    int32_t nranks;
    int32_t rank;
    // Peer exchange over NVLink (absent: p2p == false, NCCL carries both exchanges).
    bool p2p;
    uint8_t* region;                           // this rank's exchange region
    uint8_t* peer[wl::P2P_MAX_RANKS];          // every rank's region, mapped here (peer[rank] = region)
    unsigned* ctr;                             // epoch / CTA-done counters
};

namespace {

long long p2p_xslot(int nranks) {
    const long long w = (long long)kP2PMaxRows * (wl::AT_H / nranks) * (wl::AT_DV + 1);
    return (w * 8 + 255) / 256 * 256;
}
long long p2p_off_part(int nranks) { return wl::P2P_OFF_CAND + nranks * kP2PCandSlot; }
long long p2p_off_gath(int nranks) { return p2p_off_part(nranks) + nranks * p2p_xslot(nranks); }
size_t p2p_region_bytes(int nranks) { return (size_t)(p2p_off_gath(nranks) + nranks * p2p_xslot(nranks)); }

bool p2p_allowed() {
    static const bool on = [] {
        const char* e = std::getenv("WL_NO_P2P");
        return !(e && e[0] == '1');
    }();
    return on;
}

void p2p_release(wl_comm* c) {
    for (int p = 0; p < c->nranks && p < wl::P2P_MAX_RANKS; ++p)
        if (c->peer[p] && c->peer[p] != c->region) cudaIpcCloseMemHandle(c->peer[p]);
    if (c->region) cudaFree(c->region);
    if (c->ctr) cudaFree(c->ctr);
    c->region = nullptr;
    c->ctr = nullptr;
    for (auto& q : c->peer) q = nullptr;
    c->p2p = false;
}

// Collective: every rank allocates its region and maps every peer's through
// CUDA IPC handles all-gathered over NCCL. Any failure on any rank leaves the
// peer exchange off everywhere (the outcome is all-reduced).
void p2p_setup(wl_comm* c) {
    const int N = c->nranks;
    if (N < 2 || N > wl::P2P_MAX_RANKS || (wl::AT_H % N) || !p2p_allowed()) return;
    int ok = 1;
    cudaIpcMemHandle_t mine{};
    if (cudaMalloc(&c->region, p2p_region_bytes(N)) != cudaSuccess ||
        cudaMemset(c->region, 0, p2p_region_bytes(N)) != cudaSuccess ||
        cudaMalloc(&c->ctr, 64) != cudaSuccess || cudaMemset(c->ctr, 0, 64) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine, c->region) != cudaSuccess)
        ok = 0;
    cudaGetLastError();
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaStream_t st = nullptr;
    uint8_t* dev = nullptr;
    std::vector<uint8_t> all((size_t)N * 64);
    bool comm_ok = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
                   cudaMalloc(&dev, (size_t)N * 64 + 4 * N) == cudaSuccess &&
                   cudaMemcpy(dev + (size_t)c->rank * 64, &mine, 64, cudaMemcpyHostToDevice) == cudaSuccess;
    comm_ok = comm_ok && ncclAllGather(dev + (size_t)c->rank * 64, dev, 64, ncclUint8, c->comm, st) == ncclSuccess &&
              cudaStreamSynchronize(st) == cudaSuccess &&
              cudaMemcpy(all.data(), dev, (size_t)N * 64, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (comm_ok && ok) {
        for (int p = 0; p < N; ++p) {
            if (p == c->rank) {
                c->peer[p] = c->region;
                continue;
            }
            cudaIpcMemHandle_t h;
            std::memcpy(&h, all.data() + (size_t)p * 64, 64);
            void* ptr = nullptr;
            if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                ok = 0;
                cudaGetLastError();
                break;
            }
            c->peer[p] = static_cast<uint8_t*>(ptr);
        }
    }
    // Agree: the exchange is on only if every rank set it up.
    int* flag = reinterpret_cast<int*>(dev + (size_t)N * 64);
    int agreed = 0;
    if (comm_ok) {
        const int v = (ok && comm_ok) ? 1 : 0;
        comm_ok = cudaMemcpy(flag, &v, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
                  ncclAllReduce(flag, flag, 1, ncclInt32, ncclMin, c->comm, st) == ncclSuccess &&
                  cudaStreamSynchronize(st) == cudaSuccess &&
                  cudaMemcpy(&agreed, flag, 4, cudaMemcpyDeviceToHost) == cudaSuccess;
    }
    if (dev) cudaFree(dev);
    if (st) cudaStreamDestroy(st);
    c->p2p = comm_ok && agreed == 1;
    if (!c->p2p) p2p_release(c);
}

wl::P2PArgs p2p_args(const wl_comm* c) {
    wl::P2PArgs a{};
    for (int p = 0; p < c->nranks; ++p) a.region[p] = c->peer[p];
    a.nranks = c->nranks;
    a.rank = c->rank;
    a.ctr = c->ctr;
    return a;
}

// `bytes` of payload (a multiple of 8) from `src` into slot `rank` of every region.
int launch_put(const wl_comm* c, int type, const void* src, size_t bytes, long long dst_off, long long slot_bytes,
               long long parity_bytes, cudaStream_t st) {
    if (bytes % 8) return WL_ERR_ARG;
    const long long n32 = (long long)(bytes / 4);
    int grid = (int)ceil_div(n32 / 2, 256 * 2);
    grid = grid < 1 ? 1 : (grid > sm_count() ? sm_count() : grid);
    WL_CUDA_TRY(launch_pdl(wl::p2p_put_kernel, dim3(grid), dim3(256), 0, st, p2p_args(c), type,
                           static_cast<const uint32_t*>(src), n32, dst_off, slot_bytes, parity_bytes));
    return WL_OK;
}

wl::P2PRecv p2p_recv(const wl_comm* c, int type, long long off, long long slot_bytes, long long parity_bytes) {
    return wl::P2PRecv{reinterpret_cast<const uint64_t*>(c->region + off), slot_bytes / 8, parity_bytes / 8,
                       c->ctr + type};
}

}  // namespace

extern "C" {

const char* wl_strerror(int s) {
    switch (s) {
        case WL_OK: return "ok";
        case WL_ERR_ARG: return "invalid argument";
        case WL_ERR_T_EXCEEDS_MAX: return "T exceeds the cache capacity T_max";
        case WL_ERR_NO_INDICES: return "consumer layer has no published indexer indices";
        case WL_ERR_CUDA: return "CUDA error";
        case WL_ERR_NCCL: return "NCCL error";
        case WL_ERR_TIMEOUT: return "a bounded device wait timed out";
        case WL_ERR_WORKSPACE: return "workspace missing or too small";
        case WL_ERR_UNSUPPORTED: return "shape not supported by the compiled kernels";
        case WL_ERR_DEVICE: return "device-side bounds check failed";
        default: return "unknown status";
    }
}

int32_t wl_abi_version(void) { return WL_ABI_VERSION; }

int32_t wl_struct_sizes(int64_t* out, int32_t n) {
    const int64_t s[] = {(int64_t)sizeof(wl_attn_cfg),     (int64_t)sizeof(wl_latent_cache),
                         (int64_t)sizeof(wl_index_cache),  (int64_t)sizeof(wl_rows),
                         (int64_t)sizeof(wl_index_share),  (int64_t)sizeof(wl_attn_decode_io),
                         (int64_t)sizeof(wl_attn_prefill_io), (int64_t)sizeof(wl_shard),
                         (int64_t)sizeof(wl_cache_append_io)};
    const int32_t m = (int32_t)(sizeof(s) / sizeof(s[0]));
    for (int32_t i = 0; i < n && i < m && out; ++i) out[i] = s[i];
    return m;
}

void wl_attn_cfg_glm52(wl_attn_cfg* c, int32_t T_max) {
    if (!c) return;
    c->n_heads = 64;
    c->kv_lora = 512;
    c->rope_dim = 64;
    c->idx_heads = 32;
    c->idx_dim = 128;
    c->index_topk = 2048;
    c->softmax_scale = 1.0f / 16.0f;            // (192 + 64)^-0.5
    c->idx_qk_scale = 0.08838834764831845f;     // 128^-0.5
    c->T_max = T_max;
}

// ---- IndexShare -------------------------------------------------------------------
void wl_index_share_reset(wl_index_share* s) {
    if (!s) return;
    const int32_t dense = s->dense;
    std::memset(s, 0, sizeof(*s));
    s->producer = UINT32_MAX;
    s->dense = dense;  // a property of the run, not of the token
}

void wl_index_share_publish(wl_index_share* s, uint32_t layer, const int32_t* idx, const int32_t* n_dev,
                            int64_t stride, int32_t n) {
    if (!s) return;
    s->idx = idx;
    s->n_dev = n_dev;
    s->stride = stride;
    s->n = n;
    s->producer = layer;
}

int wl_index_share_require(const wl_index_share* s, uint32_t layer) {
    if (!s) return WL_ERR_ARG;
    if (s->dense) return WL_OK;
    if (!s->idx) {
        std::fprintf(stderr,
                     "wl_attn: layer %u is \"shared\" but no preceding layer published indexer indices\n",
                     layer);
        return WL_ERR_NO_INDICES;
    }
    return WL_OK;
}

// ---- kernels as entry points ------------------------------------------------------------
int wl_indexer_scores(const wl_attn_cfg* cfg, const wl_index_cache* cache, int32_t T, const wl_rows* rows,
                      const void* q_idx, const float* w_idx, float* index_out, int64_t index_stride,
                      void* stream) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (int e = rows_ok(rows, T)) return e;
    if (T > cfg->T_max) return WL_ERR_T_EXCEEDS_MAX;
    if (int e = ensure_attrs()) return e;
    return launch_indexer(cfg, cache, T, rows, q_idx, w_idx, index_out, index_stride,
                          static_cast<cudaStream_t>(stream));
}

size_t wl_indexer_topk_workspace_bytes(int32_t n_rows, int32_t T) {
    if (n_rows <= 0 || T <= 0) return 0;
    return topk_ws_bytes(n_rows, T);
}

int wl_indexer_topk(const float* index, int64_t index_stride, const wl_rows* rows, int32_t T, int32_t k,
                    const int32_t* cand_idx, int32_t* sel_out, int64_t sel_stride, int32_t* sel_n_out,
                    void* workspace, size_t workspace_bytes, void* stream) {
    if (int e = rows_ok(rows, T)) return e;
    if (index_stride < T) return WL_ERR_ARG;
    if (int e = ensure_attrs()) return e;
    TopkWs ws{};
    const bool use_ws = workspace && workspace_bytes >= topk_ws_bytes(rows->n_rows, T);
    if (use_ws) ws = topk_ws_carve(align_base(workspace), rows->n_rows, T);
    return launch_topk(index, index_stride, rows, T, k, cand_idx, sel_out, sel_stride, sel_n_out,
                       static_cast<cudaStream_t>(stream), use_ws ? &ws : nullptr, false);
}

int wl_sel_normalize(const int32_t* sel_in, int64_t in_stride, const int32_t* n_in_dev, int32_t n_in,
                     const wl_rows* rows, int32_t T, int32_t* sel_out, int64_t out_stride, int32_t* n_out_dev,
                     void* stream) {
    if (int e = rows_ok(rows, T)) return e;
    if (int e = ensure_attrs()) return e;
    return launch_normalize(sel_in, in_stride, n_in_dev, n_in, rows, T, sel_out, out_stride, n_out_dev,
                            static_cast<cudaStream_t>(stream));
}

int wl_mla_sparse_attn(const wl_attn_cfg* cfg, const wl_latent_cache* cache, int32_t T, const wl_rows* rows,
                       const void* q_abs, const int32_t* sel, int64_t sel_stride, const int32_t* sel_n_dev,
                       int32_t sel_n, int64_t win_lo, int64_t win_hi, int32_t split_keys, float* o_part,
                       float* lse_part, int32_t max_splits, void* stream) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (int e = rows_ok(rows, T)) return e;
    if (int e = ensure_attrs()) return e;
    // Keys are positions in [0, win_hi); rows clamp to the window's end.
    return launch_attn(cfg, cache, T, win_hi, rows, q_abs, sel, sel_stride, sel_n_dev, sel_n, win_lo, win_hi,
                       split_keys, o_part, lse_part, max_splits, static_cast<cudaStream_t>(stream));
}

int wl_lse_merge(const float* o_part, const float* lse_part, int32_t n_rows, int32_t n_parts, int64_t row_stride,
                 int64_t part_stride, int64_t lse_row_stride, int64_t lse_part_stride, int32_t n_heads,
                 int32_t kv_lora, float* ctx, float* lse, void* stream) {
    return launch_merge(o_part, lse_part, n_rows, n_parts, row_stride, part_stride, lse_row_stride,
                        lse_part_stride, n_heads, kv_lora, ctx, lse, static_cast<cudaStream_t>(stream));
}

// ---- the indexer's query side ------------------------------------------------------------
int wl_indexer_query(const wl_attn_cfg* cfg, int32_t n, const float* q_resid, int64_t q_resid_row_stride,
                     const void* wq_b, const float* x, int64_t x_row_stride, int32_t hidden,
                     const float* weights_proj, const float* cos, const float* sin, void* q_idx, float* w_idx,
                     void* stream) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (n < 0) return WL_ERR_ARG;
    if (n == 0) return WL_OK;
    if (!q_resid || !wq_b || !x || !weights_proj || !cos || !sin || !q_idx || !w_idx) return WL_ERR_ARG;
    if (!aligned16(q_resid) || (q_resid_row_stride & 3) || q_resid_row_stride < wl::IQ_QL || !aligned16(wq_b) ||
        !aligned16(x) || (x_row_stride & 3) || hidden <= 0 || (hidden % 1024) || x_row_stride < hidden ||
        !aligned16(weights_proj) || (reinterpret_cast<uintptr_t>(q_idx) & 1) ||
        (reinterpret_cast<uintptr_t>(w_idx) & 3) || n > 65535)
        return WL_ERR_ARG;
    if (int e = ensure_attrs()) return e;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    wl::GvParams gp{};
    if (int e = encode_bf16_2d(&gp.tm_w, wq_b, wl::IQ_QL, wl::IQ_H * wl::IQ_D, wl::IQ_QL, 64, wl::GV_M)) return e;
    gp.n = n;
    gp.x = q_resid;
    gp.x_row = q_resid_row_stride;
    gp.out = q_idx;
    gp.out_row = (long long)wl::IQ_H * wl::IQ_D;
    gp.cos = cos;
    gp.sin = sin;
    if (int e = launch_gemv<wl::GV_IDXQ>(gp, dim3(wl::GV_CL, wl::IQ_H * wl::IQ_D / wl::GV_M), st)) return e;
    const float head_scale = (float)(1.0 / std::sqrt((double)wl::IQ_H));
    WL_CUDA_TRY(launch_pdl(wl::idx_head_weights_kernel, dim3(wl::IQ_H, n), dim3(256), 0, st, (int)n, x,
                           (long long)x_row_stride, weights_proj, (int)hidden, head_scale, w_idx, (long long)wl::IQ_H));
    return WL_OK;
}

// ---- the absorption around the attention ---------------------------------------------
int wl_mla_absorb_q(const wl_attn_cfg* cfg, int32_t n, const float* q, int64_t q_row_stride, const void* kv_b,
                    void* q_abs, int64_t q_abs_row_stride, void* stream) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (n < 0) return WL_ERR_ARG;
    if (n == 0) return WL_OK;
    if (!q || !kv_b || !q_abs || (reinterpret_cast<uintptr_t>(kv_b) & 3) || !aligned16(q) || (q_row_stride & 3) ||
        (reinterpret_cast<uintptr_t>(q_abs) & 1) ||
        q_row_stride < wl::PJ_H * wl::PJ_QK || q_abs_row_stride < wl::PJ_H * (wl::PJ_L + wl::PJ_ROPE) ||
        !aligned16(kv_b) || (reinterpret_cast<uintptr_t>(q_abs) & 7) || (q_abs_row_stride & 3))
        return WL_ERR_ARG;
    if (int e = ensure_attrs()) return e;
    wl::GvParams gp{};
    if (int e = encode_bf16_2d(&gp.tm_w, kv_b, wl::PJ_L, (uint64_t)wl::PJ_H * wl::PJ_KVB_ROWS, wl::PJ_L, 64,
                               wl::PJ_NOPE))
        return e;
    gp.n = n;
    gp.x = q;
    gp.x_row = q_row_stride;
    gp.out = q_abs;
    gp.out_row = q_abs_row_stride;
    return launch_gemv<wl::GV_ABSQ>(gp, dim3(wl::PJ_L / wl::GV_M, wl::PJ_H), static_cast<cudaStream_t>(stream));
}

int wl_mla_project_v(const wl_attn_cfg* cfg, int32_t n, const float* ctx, int64_t ctx_row_stride,
                     const void* kv_b, float* out, int64_t out_row_stride, void* stream) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (n < 0) return WL_ERR_ARG;
    if (n == 0) return WL_OK;
    if (!ctx || !kv_b || !out || !aligned16(kv_b) || !aligned16(ctx) || (ctx_row_stride & 3) ||
        !aligned16(out) || (out_row_stride & 3) || ctx_row_stride < wl::PJ_H * wl::PJ_L ||
        out_row_stride < wl::PJ_H * wl::PJ_V)
        return WL_ERR_ARG;
    if (int e = ensure_attrs()) return e;
    wl::GvParams gp{};
    if (int e = encode_bf16_2d(&gp.tm_w, kv_b, wl::PJ_L, (uint64_t)wl::PJ_H * wl::PJ_KVB_ROWS, wl::PJ_L, 64,
                               wl::GV_M))
        return e;
    gp.n = n;
    gp.x = ctx;
    gp.x_row = ctx_row_stride;
    gp.out = out;
    gp.out_row = out_row_stride;
    return launch_gemv<wl::GV_PROJV>(gp, dim3(wl::PJ_V / wl::GV_M, wl::PJ_H), static_cast<cudaStream_t>(stream));
}

// ---- the cache write path -------------------------------------------------------------
int wl_cache_append(const wl_attn_cfg* cfg, const wl_cache_append_io* io, void* stream) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (!io || io->n < 0) return WL_ERR_ARG;
    if (io->n == 0) return WL_OK;
    if (!io->pos || !io->cos || !io->sin || (!io->k_raw && !io->kv_raw)) return WL_ERR_ARG;
    if (io->n_seq < 1 || (!io->seq && io->n_seq != 1)) return WL_ERR_ARG;
    wl::AppendParams p{};
    p.n = io->n;
    p.pos = io->pos;
    p.seq = io->seq;
    p.n_seq = io->n_seq;
    p.T_max = cfg->T_max;
    p.cos = io->cos;
    p.sin = io->sin;
    if (io->k_raw) {
        const wl_index_cache& c = io->index;
        if (!io->k_norm_w || !io->k_norm_b || !c.keys || !c.scale || !aligned16(io->k_raw) || !aligned16(c.keys) ||
            (c.keys_seq_stride & 15) || c.keys_seq_stride < 0 || c.scale_seq_stride < 0)
            return WL_ERR_ARG;
        if (io->seq && (c.keys_seq_stride < (int64_t)cfg->T_max * wl::IDX_D || c.scale_seq_stride < cfg->T_max))
            return WL_ERR_ARG;
        p.k_raw = io->k_raw;
        p.k_w = static_cast<const __nv_bfloat16*>(io->k_norm_w);
        p.k_b = static_cast<const __nv_bfloat16*>(io->k_norm_b);
        p.ln_eps = io->ln_eps;
        p.keys = static_cast<uint8_t*>(const_cast<void*>(c.keys));
        p.keys_seq = c.keys_seq_stride;
        p.scale = const_cast<float*>(c.scale);
        p.scale_seq = c.scale_seq_stride;
    }
    if (io->kv_raw) {
        const wl_latent_cache& c = io->latent;
        if (!io->kv_norm_w || !c.c_kv || !c.k_rot || !aligned16(io->kv_raw) || !aligned16(c.c_kv) ||
            !aligned16(c.k_rot) || (c.c_kv_row_stride & 7) || (c.k_rot_row_stride & 7) ||
            c.c_kv_row_stride < wl::AT_DV || c.k_rot_row_stride < wl::AT_D - wl::AT_DV || (c.c_kv_seq_stride & 7) ||
            (c.k_rot_seq_stride & 7) || c.c_kv_seq_stride < 0 || c.k_rot_seq_stride < 0)
            return WL_ERR_ARG;
        if (io->seq && (c.c_kv_seq_stride < (int64_t)cfg->T_max * c.c_kv_row_stride ||
                        c.k_rot_seq_stride < (int64_t)cfg->T_max * c.k_rot_row_stride))
            return WL_ERR_ARG;
        p.kv_raw = io->kv_raw;
        p.kv_w = static_cast<const __nv_bfloat16*>(io->kv_norm_w);
        p.rms_eps = io->rms_eps;
        p.c_kv = static_cast<__nv_bfloat16*>(const_cast<void*>(c.c_kv));
        p.ckv_row = c.c_kv_row_stride;
        p.ckv_seq = c.c_kv_seq_stride;
        p.k_rot = static_cast<__nv_bfloat16*>(const_cast<void*>(c.k_rot));
        p.krot_row = c.k_rot_row_stride;
        p.krot_seq = c.k_rot_seq_stride;
    }
    const unsigned blocks = (unsigned)ceil_div(io->n, wl::CA_WARPS);
    WL_CUDA_TRY(launch_pdl(wl::cache_append_kernel, dim3(blocks), dim3(32 * wl::CA_WARPS), 0,
                           static_cast<cudaStream_t>(stream), p));
    return WL_OK;
}

// ---- decode --------------------------------------------------------------------------
size_t wl_attn_workspace_bytes(const wl_attn_cfg* cfg, int32_t T_max, int32_t batch) {
    if (!cfg || T_max <= 0 || batch <= 0) return 0;
    return carve_decode(nullptr, cfg, T_max, batch, 1).bytes;
}

// Attention over the selection restricted to this cache's window [t0, t0+T)
// into split-K partials (at most `cap` per row; the workspace holds
// kMaxSplits), returning the split count.
static int decode_attn(const wl_attn_cfg* cfg, const wl_attn_decode_io* io, const DecodeWs& w, int64_t t0,
                       int64_t T_global, const int32_t* sel, const int32_t* cnt, int32_t sel_n, int64_t stride,
                       long long n_max, cudaStream_t st, int cap, int32_t* nsplit_out) {
    const int32_t B = io->batch;
    const wl_rows rows{B, 1, (int32_t)T_global, 0};
    if (n_max <= 0) n_max = 1;
    const int32_t nsplit = splits_for(B, n_max, cap);
    *nsplit_out = nsplit;
    return launch_attn(cfg, &io->latent, io->T, T_global, &rows, io->q_abs, sel, stride, cnt, sel_n, t0,
                       t0 + io->T, 0, w.o_part, w.lse_part, nsplit, st, true);
}

static int decode_local(const wl_attn_cfg* cfg, const wl_attn_decode_io* io, const DecodeWs& w,
                        int64_t t0, int64_t T_global, float* ctx, float* lse, const int32_t* sel,
                        const int32_t* cnt, int32_t sel_n, int64_t stride, long long n_max, cudaStream_t st,
                        int64_t ctx_row_stride = 0, int64_t lse_row_stride = 0, int cap = kMaxSplits) {
    // Attention over the selection restricted to this cache's window [t0, t0+T),
    // then the merge of its split-K partials.
    const int32_t B = io->batch;
    int32_t nsplit = 1;
    if (int e = decode_attn(cfg, io, w, t0, T_global, sel, cnt, sel_n, stride, n_max, st, cap, &nsplit)) return e;
    WL_PHASE(st);
    const int em = launch_merge(w.o_part, w.lse_part, B, nsplit, (int64_t)nsplit * wl::AT_H * wl::AT_DV,
                                (int64_t)wl::AT_H * wl::AT_DV, (int64_t)nsplit * wl::AT_H, wl::AT_H, wl::AT_H,
                                wl::AT_DV, ctx, lse, st, ctx_row_stride, lse_row_stride);
    WL_PHASE(st);
    return em;
}

// Selection for decode: returns the list/count/stride the attention consumes.
static int decode_select(const wl_attn_cfg* cfg, const wl_attn_decode_io* io, const DecodeWs& w,
                         const int32_t** sel, const int32_t** cnt, int64_t* stride, cudaStream_t st) {
    const int32_t B = io->batch, T = io->T;
    const wl_rows rows{B, 1, T, 0};
    if (io->mode == WL_MODE_OWNER && cfg->index_topk >= T && !io->index_out) {
        // Every key is selected whatever the scores: publish the identity list
        // and attend densely (the same list, so the same result bit for bit);
        // no indexer or top-k runs. (A caller that wants the scores sets
        // index_out and gets the full path.)
        int32_t* out = io->sel_out ? io->sel_out : w.sel;
        const int64_t ostride = io->sel_out ? io->sel_stride : T;
        if (io->sel_out && io->sel_stride < T) return WL_ERR_ARG;
        if (io->sel_out || io->sel_n_out)
            WL_CUDA_TRY(launch_pdl(identity_sel_kernel, dim3((unsigned)ceil_div(T, 1024), B), dim3(256), 0, st, (int)T,
                                   out, (long long)ostride, io->sel_n_out));
        *sel = nullptr;
        *cnt = nullptr;
        *stride = 0;
        return WL_OK;
    }
    if (io->mode == WL_MODE_OWNER) {
        float* index = io->index_out ? io->index_out : w.index;
        const int64_t istride = io->index_out ? io->index_stride : T;
        const bool fuse = topk_wants_hist(T, cfg->index_topk);
        if (fuse) WL_CUDA_TRY(hist_zero(w.topk.hist, B, st));
        if (int e = launch_indexer(cfg, &io->index, T, &rows, io->q_idx, io->w_idx, index, istride, st,
                                   fuse ? w.topk.hist : nullptr))
            return e;
        WL_PHASE(st);
        const int32_t kk = cfg->index_topk < T ? cfg->index_topk : T;
        int32_t* out = io->sel_out ? io->sel_out : w.sel;
        const int64_t ostride = io->sel_out ? io->sel_stride : kk;
        if (io->sel_out && io->sel_stride < kk) return WL_ERR_ARG;
        int32_t* n_out = io->sel_n_out ? io->sel_n_out : w.cnt;
        if (int e = launch_topk(index, istride, &rows, T, cfg->index_topk, nullptr, out, ostride, n_out, st, &w.topk,
                                fuse))
            return e;
        WL_PHASE(st);
        *sel = out;
        *cnt = n_out;
        *stride = ostride;
        return WL_OK;
    }
    if (io->mode == WL_MODE_CONSUMER) {
        if (io->sel_flags & WL_SEL_CANONICAL) {
            *sel = io->sel_in;
            *cnt = io->sel_n_in;  // NULL: the attention kernel takes io->sel_n
            *stride = io->sel_stride;
            return WL_OK;
        }
        const int64_t ostride = T;
        if (int e = launch_normalize(io->sel_in, io->sel_stride, io->sel_n_in, io->sel_n, &rows, T, w.sel, ostride,
                                     w.cnt, st))
            return e;
        *sel = w.sel;
        *cnt = w.cnt;
        *stride = ostride;
        return WL_OK;
    }
    *sel = nullptr;
    *cnt = nullptr;
    *stride = 0;
    return WL_OK;
}

int wl_attn_decode(const wl_attn_cfg* cfg, const wl_attn_decode_io* io, void* workspace, size_t workspace_bytes,
                   void* stream) {
    if (int e = check_decode_io(cfg, io)) return e;
    const DecodeWs need = carve_decode(nullptr, cfg, io->T, io->batch, 1);
    if (!workspace || workspace_bytes < need.bytes) return WL_ERR_WORKSPACE;
    if (int e = ensure_attrs()) return e;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const DecodeWs w = carve_decode(align_base(workspace), cfg, io->T, io->batch, 1);
    WL_PHASE(st);  // stamps: start | indexer | top-k (owner) | attention | merge
    const int32_t* sel = nullptr;
    const int32_t* cnt = nullptr;
    int64_t stride = 0;
    if (int e = decode_select(cfg, io, w, &sel, &cnt, &stride, st)) return e;
    long long n_max = io->T;  // dense: every key
    int32_t sel_n = 0;
    if (io->mode == WL_MODE_OWNER) n_max = cfg->index_topk < io->T ? cfg->index_topk : io->T;
    if (io->mode == WL_MODE_CONSUMER) {
        const bool canon = (io->sel_flags & WL_SEL_CANONICAL) != 0;
        n_max = canon ? (io->sel_n_in ? io->sel_stride : io->sel_n) : io->T;
        sel_n = io->sel_n;
    }
    float* lse = io->lse ? io->lse : w.lse_tmp;
    return decode_local(cfg, io, w, 0, io->T, io->ctx, lse, sel, cnt, sel_n, stride, n_max, st);
}

int wl_attn_layer_decode(const wl_attn_cfg* cfg, wl_attn_decode_io* io, int32_t owner, uint32_t layer,
                         wl_index_share* share, void* workspace, size_t workspace_bytes, void* stream) {
    if (!io || !share) return WL_ERR_ARG;
    if (owner) {
        if (!io->sel_out || !io->sel_n_out) return WL_ERR_ARG;  // the published buffer must outlive the call
        io->mode = WL_MODE_OWNER;
        if (int e = wl_attn_decode(cfg, io, workspace, workspace_bytes, stream)) return e;
        // Publish the raw selection (glm_layer_runner.cuh:604).
        wl_index_share_publish(share, layer, io->sel_out, io->sel_n_out, io->sel_stride,
                               cfg->index_topk < io->T ? cfg->index_topk : io->T);
        return WL_OK;
    }
    if (int e = wl_index_share_require(share, layer)) return e;
    if (share->dense) {
        io->mode = WL_MODE_DENSE;
    } else {
        io->mode = WL_MODE_CONSUMER;
        io->sel_in = share->idx;
        io->sel_n_in = share->n_dev;
        io->sel_n = share->n;
        io->sel_stride = share->stride;
        io->sel_flags = WL_SEL_CANONICAL;  // this library only publishes canonical lists
    }
    return wl_attn_decode(cfg, io, workspace, workspace_bytes, stream);
}

// ---- prefill ----------------------------------------------------------------------------
static size_t prefill_ws(const wl_attn_cfg* cfg, int32_t n_q, int32_t T, void* base, float** index,
                         int32_t** sel, int32_t** cnt, float** lse) {
    size_t off = 0;
    auto take = [&](size_t bytes) -> void* {
        void* p = base ? static_cast<char*>(base) + off : nullptr;
        off += align256(bytes);
        return p;
    };
    const size_t k = (size_t)(cfg->index_topk < T ? cfg->index_topk : T);
    *index = static_cast<float*>(take((size_t)n_q * T * 4));
    *sel = static_cast<int32_t*>(take((size_t)n_q * (size_t)T * 4 > (size_t)n_q * k * 4 ? (size_t)n_q * T * 4
                                                                                          : (size_t)n_q * k * 4));
    *cnt = static_cast<int32_t*>(take((size_t)n_q * 4));
    *lse = static_cast<float*>(take((size_t)n_q * wl::AT_H * 4));
    return off + 256;
}

size_t wl_attn_prefill_workspace_bytes(const wl_attn_cfg* cfg, int32_t n_q, int32_t T) {
    if (!cfg || n_q <= 0 || T <= 0) return 0;
    float* a;
    int32_t* b;
    int32_t* c;
    float* d;
    return prefill_ws(cfg, n_q, T, nullptr, &a, &b, &c, &d);
}

int wl_attn_prefill(const wl_attn_cfg* cfg, const wl_attn_prefill_io* io, void* workspace, size_t workspace_bytes,
                    void* stream) {
    if (!cfg_supported(cfg)) return cfg ? WL_ERR_UNSUPPORTED : WL_ERR_ARG;
    if (!io || io->n_q <= 0 || io->pos0 < 0 || !io->q_abs || !io->ctx) return WL_ERR_ARG;
    const int32_t T = io->pos0 + io->n_q;
    if (T > cfg->T_max) return WL_ERR_T_EXCEEDS_MAX;
    if (io->n_q > 65535) return WL_ERR_ARG;
    if (workspace_bytes < wl_attn_prefill_workspace_bytes(cfg, io->n_q, T) || !workspace) return WL_ERR_WORKSPACE;
    if (int e = ensure_attrs()) return e;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* w_index;
    int32_t* w_sel;
    int32_t* w_cnt;
    float* w_lse;
    prefill_ws(cfg, io->n_q, T, align_base(workspace), &w_index, &w_sel, &w_cnt, &w_lse);
    const wl_rows rows{io->n_q, io->n_q, io->pos0 + 1, 1};
    const int32_t* sel = nullptr;
    const int32_t* cnt = nullptr;
    int64_t stride = 0;
    if (io->mode == WL_MODE_OWNER) {
        if (!io->q_idx || !io->w_idx || !io->index.keys || !io->index.scale) return WL_ERR_ARG;
        float* index = io->index_out ? io->index_out : w_index;
        const int64_t istride = io->index_out ? io->index_stride : T;
        if (int e = launch_indexer(cfg, &io->index, T, &rows, io->q_idx, io->w_idx, index, istride, st)) return e;
        const int32_t kk = cfg->index_topk < T ? cfg->index_topk : T;
        int32_t* out = io->sel_out ? io->sel_out : w_sel;
        const int64_t ostride = io->sel_out ? io->sel_stride : kk;
        if (io->sel_out && io->sel_stride < kk) return WL_ERR_ARG;
        int32_t* n_out = io->sel_n_out ? io->sel_n_out : w_cnt;
        if (int e = launch_topk(index, istride, &rows, T, cfg->index_topk, nullptr, out, ostride, n_out, st)) return e;
        sel = out;
        cnt = n_out;
        stride = ostride;
    } else if (io->mode == WL_MODE_CONSUMER) {
        if (!io->sel_in) return WL_ERR_NO_INDICES;
        if (io->sel_flags & WL_SEL_CANONICAL) {
            sel = io->sel_in;
            stride = io->sel_stride;
            if (io->sel_n_in) {
                cnt = io->sel_n_in;
            } else {
                // min(topk, row length) per row, as an owner of this chunk writes.
                row_counts_kernel<<<(unsigned)ceil_div(io->n_q, 256), 256, 0, st>>>(rows.n_rows, rows.len0,
                                                                                    rows.len_step, T,
                                                                                    cfg->index_topk, w_cnt);
                WL_CUDA_TRY(cudaGetLastError());
                cnt = w_cnt;
            }
        } else {
            const int32_t n_in = (int32_t)io->sel_stride;
            if (int e = launch_normalize(io->sel_in, io->sel_stride, io->sel_n_in, n_in, &rows, T, w_sel, T, w_cnt, st))
                return e;
            sel = w_sel;
            cnt = w_cnt;
            stride = T;
        }
    } else if (io->mode != WL_MODE_DENSE) {
        return WL_ERR_ARG;
    }
    float* lse = io->lse ? io->lse : w_lse;
    return launch_attn(cfg, &io->latent, T, T, &rows, io->q_abs, sel, stride, cnt, 0, 0, T, 0, io->ctx, lse, 1, st);
}

int wl_attn_layer_prefill(const wl_attn_cfg* cfg, wl_attn_prefill_io* io, int32_t owner, uint32_t layer,
                          wl_index_share* share, void* workspace, size_t workspace_bytes, void* stream) {
    if (!io || !share) return WL_ERR_ARG;
    if (owner) {
        if (!io->sel_out || !io->sel_n_out) return WL_ERR_ARG;  // the published rows must outlive the call
        io->mode = WL_MODE_OWNER;
        if (int e = wl_attn_prefill(cfg, io, workspace, workspace_bytes, stream)) return e;
        // Publish every row's raw selection, one row per query position (the
        // per-row index buffers of run_prefill_layer_major,
        // glm_layer_runner.cuh:763-770, 954-983).
        const int64_t T = (int64_t)io->pos0 + io->n_q;
        wl_index_share_publish(share, layer, io->sel_out, io->sel_n_out, io->sel_stride,
                               (int32_t)(cfg->index_topk < T ? cfg->index_topk : T));
        return WL_OK;
    }
    if (int e = wl_index_share_require(share, layer)) return e;
    if (share->dense) {
        io->mode = WL_MODE_DENSE;
    } else {
        if (!share->n_dev) return WL_ERR_ARG;  // prefill rows carry their own counts
        io->mode = WL_MODE_CONSUMER;
        io->sel_in = share->idx;
        io->sel_n_in = share->n_dev;
        io->sel_stride = share->stride;
        io->sel_flags = WL_SEL_CANONICAL;
    }
    return wl_attn_prefill(cfg, io, workspace, workspace_bytes, stream);
}

// ---- sharded decode ----------------------------------------------------------------------------
int wl_comm_unique_id(uint8_t id_out[128]) {
    if (!id_out) return WL_ERR_ARG;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return WL_ERR_NCCL;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    std::memcpy(id_out, &id, 128);
    return WL_OK;
}

int wl_comm_create(const uint8_t id[128], int32_t nranks, int32_t rank, wl_comm** out) {
    if (!id || !out || nranks <= 0 || rank < 0 || rank >= nranks) return WL_ERR_ARG;
    ncclUniqueId uid;
    std::memcpy(&uid, id, 128);
    wl_comm* c = new wl_comm{};
    c->nranks = nranks;
    c->rank = rank;
    if (ncclCommInitRank(&c->comm, nranks, uid, rank) != ncclSuccess) {
        delete c;
        return WL_ERR_NCCL;
    }
    p2p_setup(c);
    *out = c;
    return WL_OK;
}

int wl_comm_p2p(const wl_comm* c) { return c && c->p2p ? 1 : 0; }

int wl_comm_destroy(wl_comm* c) {
    if (!c) return WL_ERR_ARG;
    cudaDeviceSynchronize();  // this rank's exchanges are done
    if (c->p2p) {
        // Collective: no rank frees its region while a peer's put may still write it.
        int* one = nullptr;
        cudaStream_t st = nullptr;
        if (cudaMalloc(&one, 4) == cudaSuccess && cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess &&
            ncclAllReduce(one, one, 1, ncclInt32, ncclSum, c->comm, st) == ncclSuccess)
            cudaStreamSynchronize(st);
        if (st) cudaStreamDestroy(st);
        if (one) cudaFree(one);
    }
    p2p_release(c);
    const ncclResult_t r = ncclCommDestroy(c->comm);
    delete c;
    return r == ncclSuccess ? WL_OK : WL_ERR_NCCL;
}

size_t wl_attn_sharded_workspace_bytes(const wl_attn_cfg* cfg, int32_t T_local_max, int32_t batch, int32_t nranks) {
    if (!cfg || T_local_max <= 0 || batch <= 0 || nranks <= 0) return 0;
    return carve_decode(nullptr, cfg, T_local_max, batch, nranks > 1 ? nranks : 2).bytes;
}

int wl_attn_decode_sharded(const wl_attn_cfg* cfg, const wl_attn_decode_io* io, const wl_shard* shard, wl_comm* comm,
                           void* workspace, size_t workspace_bytes, void* stream) {
    if (int e = check_decode_io(cfg, io)) return e;
    if (!shard || !comm || shard->t0 < 0 || shard->T_global < shard->t0 + io->T) return WL_ERR_ARG;
    const int32_t N = comm->nranks;
    const DecodeWs need = carve_decode(nullptr, cfg, io->T, io->batch, N > 1 ? N : 2);
    if (!workspace || workspace_bytes < need.bytes) return WL_ERR_WORKSPACE;
    if (int e = ensure_attrs()) return e;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const DecodeWs w = carve_decode(align_base(workspace), cfg, io->T, io->batch, N > 1 ? N : 2);
    const int32_t B = io->batch, T = io->T, k = cfg->index_topk;
    const int64_t Tg = shard->T_global, t0 = shard->t0;
    const int32_t kg = (int32_t)(k < Tg ? k : Tg);
    const int64_t rowsz = wl::AT_H * wl::AT_DV + wl::AT_H;
    // Peer exchange when the comm has it and this call fits its slots (and the
    // global top-k can read the candidate slots as segmented rows).
    const bool p2p = comm->p2p && B <= kP2PMaxRows && k <= kP2PMaxK && (k % 32) == 0 &&
                     (int64_t)N * k <= kTopkRegMax;
    // Phase stamps (diagnostics): start | indexer | local top-k | candidate
    // exchange | global top-k | attention | (o, lse) reduce-scatter |
    // all-gather (peer exchange); the NCCL exchange stamps start | indexer |
    // local top-k | candidate exchange | global top-k | attention | local merge
    // | all-gather | merge. A consumer layer has no indexer, top-k or
    // candidate stamps.
    WL_PHASE(st);

    const int32_t* gsel = nullptr;
    const int32_t* gcnt = nullptr;
    int64_t gstride = 0;
    if (io->mode == WL_MODE_OWNER) {
        if (!io->sel_out || !io->sel_n_out || io->sel_stride < kg) return WL_ERR_ARG;
        const wl_rows lrows{B, 1, T, 0};
        float* index = w.index;
        const bool fuse = topk_wants_hist(T, k);
        if (fuse) WL_CUDA_TRY(hist_zero(w.topk.hist, B, st));
        if (int e = launch_indexer(cfg, &io->index, T, &lrows, io->q_idx, io->w_idx, index, T, st,
                                   fuse ? w.topk.hist : nullptr))
            return e;
        const int32_t kl = k < T ? k : T;
        WL_PHASE(st);
        // Local top-k; its selection leaves as (score, global index) candidates,
        // k per row (padded), straight from the top-k's emission where it can.
        const bool cand_direct = T <= kTopkClusterMax;
        const wl::CandOut co{w.cand_score, w.cand_idx, k, k, t0};
        if (int e = launch_topk(index, T, &lrows, T, k, nullptr, w.sel, kl, w.cnt, st, &w.topk, fuse,
                                cand_direct ? &co : nullptr))
            return e;
        if (!cand_direct) {
            gather_candidates_kernel<<<dim3((unsigned)ceil_div(k, 256), B), 256, 0, st>>>(
                index, T, w.sel, kl, w.cnt, k, t0, w.cand_score, w.cand_idx);
            WL_CUDA_TRY(cudaGetLastError());
        }
        WL_PHASE(st);
        const wl_rows crows{B, 1, N * k, 0};
        if (p2p) {
            // Candidates to every rank's slot `rank`; the global top-k waits for all
            // N slots and reads them in place as rows of N segments of k.
            if (int e = launch_put(comm, wl::XCH_CAND, w.cand_score, (size_t)B * k * 8, wl::P2P_OFF_CAND, kP2PCandSlot, 0,
                                   st))
                return e;
            WL_PHASE(st);
            const wl::P2PRecv rc = p2p_recv(comm, wl::XCH_CAND, wl::P2P_OFF_CAND, kP2PCandSlot, 0);
            if (int e = launch_topk(nullptr, k, &crows, N * k, kg, nullptr, io->sel_out, io->sel_stride, io->sel_n_out,
                                    st, nullptr, false, nullptr, k, rc.slot_words, &rc, (int64_t)B * k))
                return e;
        } else {
            if (ncclGroupStart() != ncclSuccess) return WL_ERR_NCCL;
            if (ncclAllGather(w.cand_score, w.cand_score_all, (size_t)B * k, ncclFloat32, comm->comm, st) !=
                    ncclSuccess ||
                ncclAllGather(w.cand_idx, w.cand_idx_all, (size_t)B * k, ncclInt32, comm->comm, st) != ncclSuccess) {
                ncclGroupEnd();
                return WL_ERR_NCCL;
            }
            if (ncclGroupEnd() != ncclSuccess) return WL_ERR_NCCL;
            WL_PHASE(st);
            // Exact global top-k over the candidates; candidate order (rank-major,
            // ascending within a rank) is global key order, so position ties
            // resolve to the lowest global index. The all-gathered [rank][row][k]
            // buffers are read in place as rows of N segments of k.
            if ((k % 32) == 0 && (int64_t)N * k <= kTopkRegMax) {
                if (int e = launch_topk(w.cand_score_all, k, &crows, N * k, kg, w.cand_idx_all, io->sel_out,
                                        io->sel_stride, io->sel_n_out, st, nullptr, false, nullptr, k, (int64_t)B * k))
                    return e;
            } else {
                candidates_to_rows_kernel<<<256, 256, 0, st>>>(w.cand_score_all, w.cand_idx_all, N, B, k,
                                                              w.cand_score_rows, w.cand_idx_rows);
                WL_CUDA_TRY(cudaGetLastError());
                if (int e = launch_topk(w.cand_score_rows, (int64_t)N * k, &crows, N * k, kg, w.cand_idx_rows,
                                        io->sel_out, io->sel_stride, io->sel_n_out, st))
                    return e;
            }
        }
        if (io->index_out) {
            // Local scores into the caller's buffer (this rank's window).
            for (int32_t b = 0; b < B; ++b)
                WL_CUDA_TRY(cudaMemcpy2DAsync(io->index_out + (int64_t)b * io->index_stride, (size_t)T * 4,
                                              index + (int64_t)b * T, (size_t)T * 4, (size_t)T * 4, 1,
                                              cudaMemcpyDeviceToDevice, st));
        }
        WL_PHASE(st);
        gsel = io->sel_out;
        gcnt = io->sel_n_out;
        gstride = io->sel_stride;
    } else if (io->mode == WL_MODE_CONSUMER) {
        const wl_rows grows{B, 1, (int32_t)Tg, 0};
        if (io->sel_flags & WL_SEL_CANONICAL) {
            gsel = io->sel_in;
            gcnt = io->sel_n_in;
            gstride = io->sel_stride;
        } else {
            if (Tg > (int64_t)T * N) return WL_ERR_WORKSPACE;  // normalised lists need B x T_global
            if (int e = launch_normalize(io->sel_in, io->sel_stride, io->sel_n_in, io->sel_n, &grows, (int32_t)Tg, w.sel,
                                         (int32_t)Tg, w.cnt, st))
                return e;
            gsel = w.sel;
            gcnt = w.cnt;
            gstride = Tg;
        }
    }
    // Attention over this rank's part of the global list (its window of keys).
    long long n_max = Tg;
    int32_t sel_n = 0;
    if (io->mode == WL_MODE_OWNER) n_max = kg;
    if (io->mode == WL_MODE_CONSUMER) {
        n_max = (gcnt || !(io->sel_flags & WL_SEL_CANONICAL)) ? gstride : io->sel_n;
        sel_n = io->sel_n;
    }
    if (p2p) {
        // Split-K partials, then the (o, lse) reduce-scatter over heads and the
        // all-gather of the merged slices (xmerge.cuh).
        int32_t nsplit = 1;
        if (int e = decode_attn(cfg, io, w, t0, Tg, gsel, gcnt, sel_n, gstride, n_max, st, kMaxSplits, &nsplit))
            return e;
        WL_PHASE(st);
        wl::XMergeParams xp{};
        xp.a = p2p_args(comm);
        xp.B = B;
        xp.hs = wl::AT_H / N;
        xp.nsplit = nsplit;
        xp.o_part = w.o_part;
        xp.lse_part = w.lse_part;
        xp.part_off = p2p_off_part(N);
        xp.part_slot = p2p_xslot(N);
        xp.gath_off = p2p_off_gath(N);
        xp.gath_slot = p2p_xslot(N);
        xp.ctx = io->ctx;
        xp.lse = io->lse;
        WL_CUDA_TRY(launch_pdl(wl::xscatter_kernel, dim3(wl::AT_H / wl::XS_HEADS, wl::AT_DV / 128, B), dim3(32 * wl::XS_HEADS), 0, st, xp));
        WL_PHASE(st);
        WL_CUDA_TRY(launch_pdl(wl::xgather_kernel<true>, dim3(xp.hs, wl::AT_DV / 128, B), dim3(32 * N), 0, st, xp));
        WL_PHASE(st);
        return WL_OK;
    }
    // NCCL: local partial merged over its splits straight into the exchange
    // layout [row][64 * 512 + 64], all-gathered, then merged over the ranks.
    if (int e = decode_local(cfg, io, w, t0, Tg, w.part_send, w.part_send + wl::AT_H * wl::AT_DV, gsel, gcnt, sel_n,
                             gstride, n_max, st, rowsz, rowsz))
        return e;
    const size_t per = (size_t)B * rowsz;
    float* lse = io->lse ? io->lse : w.lse_tmp;
    if (ncclAllGather(w.part_send, w.part_recv, per, ncclFloat32, comm->comm, st) != ncclSuccess) return WL_ERR_NCCL;
    WL_PHASE(st);
    // part_recv: [rank][row][64*512 + 64]
    const int em = launch_merge(w.part_recv, w.part_recv + wl::AT_H * wl::AT_DV, B, N, rowsz, (int64_t)B * rowsz,
                                rowsz, (int64_t)B * rowsz, wl::AT_H, wl::AT_DV, io->ctx, lse, st);
    WL_PHASE(st);
    return em;
}

// ---- decode attention without any allocation ------------------------------------------
// For callers that cannot allocate device memory at all (for example code that
// runs where cudaMalloc is not allowed, or an embedding runtime that owns every
// allocation and hands out only input/output buffers): the split-K partials of
// the decode attention live in this fixed array instead of a caller workspace.
// Every GPU that loads the library holds it until the process exits.
constexpr int kNoAllocMaxRows = 4;
constexpr int kNoAllocMaxSplits = 16;
constexpr size_t kNoAllocPartFloats = (size_t)kNoAllocMaxRows * kNoAllocMaxSplits * wl::AT_H * wl::AT_DV;
constexpr size_t kNoAllocLseFloats = (size_t)kNoAllocMaxRows * kNoAllocMaxSplits * wl::AT_H;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocPartFloats + kNoAllocLseFloats +
                                                         (size_t)kNoAllocMaxRows * wl::AT_H];
static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[kMaxDevices];

int wl_attn_decode_noalloc(const wl_attn_cfg* cfg, const wl_attn_decode_io* io, void* stream) {
    if (int e = check_decode_io(cfg, io)) return e;
    if (io->mode == WL_MODE_OWNER) return WL_ERR_UNSUPPORTED;  // the indexer and top-k need T-sized scratch
    if (io->mode == WL_MODE_CONSUMER && !(io->sel_flags & WL_SEL_CANONICAL)) return WL_ERR_UNSUPPORTED;
    if (io->batch > kNoAllocMaxRows) {
        std::fprintf(stderr, "wl_attn_decode_noalloc: batch %d exceeds the fixed scratch's maximum of %d rows\n",
                     io->batch, kNoAllocMaxRows);
        return WL_ERR_WORKSPACE;
    }
    if (int e = ensure_attrs()) return e;
    int dev = 0;
    WL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return WL_ERR_CUDA;
    float* base = nullptr;
    {
        // First call on this device: resolve the array's device address (the
        // host-side name is only a stand-in). Later calls reuse it.
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void* p = nullptr;
            WL_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            g_noalloc_ptr[dev] = static_cast<float*>(p);
        }
        base = g_noalloc_ptr[dev];
    }
    // Nothing needs clearing: the attention kernel writes the lse of every
    // split slot it may use (-inf for an empty split), and the merge reads the
    // o of non-empty splits only, which the same call has written.
    DecodeWs w{};
    w.o_part = base;
    w.lse_part = base + kNoAllocPartFloats;
    w.lse_tmp = base + kNoAllocPartFloats + kNoAllocLseFloats;
    long long n_max = io->T;
    int32_t sel_n = 0;
    const int32_t* sel = nullptr;
    int64_t stride = 0;
    if (io->mode == WL_MODE_CONSUMER) {
        sel = io->sel_in;
        stride = io->sel_stride;
        n_max = io->sel_n_in ? io->sel_stride : io->sel_n;
        sel_n = io->sel_n;
    }
    float* lse = io->lse ? io->lse : w.lse_tmp;
    return decode_local(cfg, io, w, 0, io->T, io->ctx, lse, sel, io->sel_n_in, sel_n, stride, n_max,
                        static_cast<cudaStream_t>(stream), 0, 0, kNoAllocMaxSplits);
}

// ---- diagnostics ---------------------------------------------------------------------------
int wl_diag_set_wait_limit(int64_t cycles) {
    const long long v = cycles > 0 ? (long long)cycles : wl::WL_WAIT_CYCLES_DEFAULT;
    WL_CUDA_TRY(cudaMemcpyToSymbol(wl::g_wait_cycles, &v, sizeof(v)));
    return WL_OK;
}

int wl_diag_phase_stamps(uint64_t* dev_buf, int32_t cap) {
    if (dev_buf && cap <= 0) return WL_ERR_ARG;
    std::lock_guard<std::mutex> lk(g_ph_mu);
    g_ph_buf = reinterpret_cast<unsigned long long*>(dev_buf);
    g_ph_cap = dev_buf ? cap : 0;
    g_ph_n = 0;
    return WL_OK;
}

int32_t wl_diag_phase_count(void) {
    std::lock_guard<std::mutex> lk(g_ph_mu);
    return g_ph_n;
}

size_t wl_diag_xmerge_bytes(int32_t nranks) {
    if (nranks < 2 || nranks > wl::P2P_MAX_RANKS || (wl::AT_H % nranks)) return 0;
    return (size_t)nranks * (p2p_region_bytes(nranks) + 256);
}

int wl_diag_xmerge(int32_t nranks, int32_t batch, int32_t nsplit, const float* o_part, const float* lse_part,
                   void* regions, size_t regions_bytes, float* ctx, float* lse, void* stream) {
    const size_t need = wl_diag_xmerge_bytes(nranks);
    if (!need || batch <= 0 || batch > kP2PMaxRows || nsplit <= 0 || nsplit > 32 || !o_part || !lse_part ||
        !regions || regions_bytes < need || !ctx || !aligned16(regions))
        return WL_ERR_ARG;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t rb = p2p_region_bytes(nranks);
    uint8_t* base = static_cast<uint8_t*>(regions);
    auto region = [&](int q) { return base + (size_t)q * rb; };
    auto ctr = [&](int q) { return reinterpret_cast<unsigned*>(base + (size_t)nranks * rb + (size_t)q * 64); };
    const int64_t part = (int64_t)batch * nsplit;
    auto params = [&](int r) {
        wl::XMergeParams xp{};
        for (int q = 0; q < nranks; ++q) xp.a.region[q] = region(q);
        xp.a.nranks = nranks;
        xp.a.rank = r;
        xp.a.ctr = ctr(r);
        xp.B = batch;
        xp.hs = wl::AT_H / nranks;
        xp.nsplit = nsplit;
        xp.o_part = o_part + (int64_t)r * part * wl::AT_H * wl::AT_DV;
        xp.lse_part = lse_part + (int64_t)r * part * wl::AT_H;
        xp.part_off = p2p_off_part(nranks);
        xp.part_slot = p2p_xslot(nranks);
        xp.gath_off = p2p_off_gath(nranks);
        xp.gath_slot = p2p_xslot(nranks);
        xp.ctx = ctx + (int64_t)r * batch * wl::AT_H * wl::AT_DV;
        xp.lse = lse ? lse + (int64_t)r * batch * wl::AT_H : nullptr;
        return xp;
    };
    // Every stage of every emulated rank runs after the stage it reads from has
    // completed on every rank, so no wait depends on a kernel still to come.
    for (int r = 0; r < nranks; ++r)
        wl::xscatter_kernel<<<dim3(wl::AT_H / wl::XS_HEADS, wl::AT_DV / 128, batch), 32 * wl::XS_HEADS, 0, st>>>(params(r));
    for (int r = 0; r < nranks; ++r)
        wl::xgather_kernel<false><<<dim3(wl::AT_H / nranks, wl::AT_DV / 128, batch), 32 * nranks, 0, st>>>(params(r));
    for (int r = 0; r < nranks; ++r)
        wl::xunpack_kernel<<<dim3(wl::AT_H, wl::AT_DV / 128, batch), 32, 0, st>>>(params(r));
    WL_CUDA_TRY(cudaGetLastError());
    return WL_OK;
}

int wl_diag_merge_exchange(const void* region, int64_t slot_words, const uint32_t* epoch_ctr, int32_t n_rows,
                           int32_t n_parts, float* ctx, float* lse, void* stream) {
    if (!region || !epoch_ctr || !ctx || slot_words <= 0 || !aligned16(region)) return WL_ERR_ARG;
    const int64_t rowsz = wl::AT_H * wl::AT_DV + wl::AT_H;
    if (slot_words < (int64_t)n_rows * rowsz) return WL_ERR_ARG;
    const wl::P2PRecv rp{static_cast<const uint64_t*>(region), slot_words, 0, epoch_ctr};
    return launch_merge(nullptr, nullptr, n_rows, n_parts, rowsz, slot_words, rowsz, slot_words, wl::AT_H,
                        wl::AT_DV, ctx, lse, static_cast<cudaStream_t>(stream), 0, 0, &rp, wl::AT_H * wl::AT_DV);
}

int wl_device_error(int32_t clear, uint32_t* detail) {
    WL_CUDA_TRY(cudaDeviceSynchronize());
    unsigned w = 0;
    WL_CUDA_TRY(cudaMemcpyFromSymbol(&w, wl::g_err_word, sizeof(w)));
    if (detail) *detail = w;
    if (clear) {
        const unsigned z = 0;
        WL_CUDA_TRY(cudaMemcpyToSymbol(wl::g_err_word, &z, sizeof(z)));
    }
    if (w == 0) return WL_OK;
    const unsigned code = w >> 24;
    return code == wl::ERRC_TIMEOUT ? WL_ERR_TIMEOUT : WL_ERR_DEVICE;
}

}  // extern "C"
