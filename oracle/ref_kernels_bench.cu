// ref_kernels_bench.cu — TEST / BASELINE INFRASTRUCTURE ONLY: times the
// reference's own CUDA kernels for the attention substep on this GPU, as the
// GPU row to compare this library's kernels with. Nothing in windlass_b200
// links or loads it; bench.py runs the built binary (oracle/_ref/) beside its
// CPU baseline and reports the numbers in its extras.
//
// Built by oracle/build_ref.sh from the reference's headers where they lie
// (src/glm_kernels.cuh, src/glm_layer_runner.cuh of ssubbotin/windlass,
// compiled unmodified for sm_100a); this file holds only the timing harness.
//
// The timed block is the one this library's wl_attn_decode replaces
// (src/glm_layer_runner.cuh:582-644), with the reference's own launch shapes:
//   owner:    indexer_scores_relu -> indexer_combine -> indexer_topk (1 CTA)
//             -> index_mask_fill/scatter -> mla_decode_absorbed (64 CTAs)
//   consumer: index_mask_fill/scatter -> mla_decode_absorbed
// in the reference's formats (bf16 index keys, fp32 queries, fp32 latent
// cache), batch 1, on seeded random inputs. The query side (wq_b, rope, head
// weights) and the absorption are outside the block, as in this library.
// Output: one JSON line per configuration.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "glm_layer_runner.cuh"

namespace {

#define CK(x)                                                                                \
    do {                                                                                     \
        cudaError_t e_ = (x);                                                                \
        if (e_ != cudaSuccess) {                                                             \
            std::fprintf(stderr, "%s failed: %s\n", #x, cudaGetErrorString(e_));             \
            std::exit(1);                                                                    \
        }                                                                                    \
    } while (0)

__global__ void fill_normal(float* p, size_t n, unsigned seed, float scale) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        // two hashed uniforms -> one Box-Muller normal
        unsigned a = (unsigned)i * 2654435761u ^ seed, b = (unsigned)(i >> 32) * 40503u ^ (seed * 977u + (unsigned)i);
        a ^= a >> 15; a *= 2246822519u; a ^= a >> 13; a *= 3266489917u; a ^= a >> 16;
        b ^= b >> 15; b *= 2246822519u; b ^= b >> 13; b *= 3266489917u; b ^= b >> 16;
        const float u1 = (a + 1.0f) * (1.0f / 4294967296.0f), u2 = b * (1.0f / 4294967296.0f);
        p[i] = scale * sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
    }
}
__global__ void to_bf16_bits(const float* in, uint16_t* out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const uint32_t u = __float_as_uint(in[i]);
        out[i] = (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
    }
}

struct Case {
    uint32_t T;
    bool owner;
};

float run_case(const Case& c, int iters) {
    const uint32_t H = 32, D = 128, HN = 64, L = 512, R = 64, DH = 256, K = 2048;
    const uint32_t T = c.T;
    float *q, *qabs, *kvc, *krot, *ctx, *kf, *w, *scores, *index, *scores_g = nullptr;
    uint16_t* kb;
    int32_t* sel;
    uint32_t* sel_n;
    uint8_t* mask;
    CK(cudaMalloc(&q, HN * DH * 4));
    CK(cudaMalloc(&qabs, HN * L * 4));
    CK(cudaMalloc(&kvc, (size_t)T * L * 4));
    CK(cudaMalloc(&krot, (size_t)T * R * 4));
    CK(cudaMalloc(&ctx, HN * L * 4));
    CK(cudaMalloc(&kf, (size_t)T * D * 4));
    CK(cudaMalloc(&kb, (size_t)T * D * 2));
    CK(cudaMalloc(&w, H * 4));
    CK(cudaMalloc(&scores, (size_t)H * T * 4));
    CK(cudaMalloc(&index, (size_t)T * 4));
    CK(cudaMalloc(&sel, K * 4));
    CK(cudaMalloc(&sel_n, 4));
    CK(cudaMalloc(&mask, T));
    float* qi;
    CK(cudaMalloc(&qi, H * D * 4));
    fill_normal<<<256, 256>>>(q, HN * DH, 1, 1.f);
    fill_normal<<<256, 256>>>(qabs, HN * L, 2, 1.f);
    fill_normal<<<1024, 256>>>(kvc, (size_t)T * L, 3, 1.f);
    fill_normal<<<1024, 256>>>(krot, (size_t)T * R, 4, 1.f);
    fill_normal<<<1024, 256>>>(kf, (size_t)T * D, 5, 1.f);
    to_bf16_bits<<<1024, 256>>>(kf, kb, (size_t)T * D);
    fill_normal<<<1, 32>>>(w, H, 6, 0.5f);
    fill_normal<<<16, 256>>>(qi, H * D, 7, 1.f);
    CK(cudaGetLastError());
    const size_t smem = (size_t)T * sizeof(float);
    if (smem > glm::mla_smem_capacity()) CK(cudaMalloc(&scores_g, (size_t)HN * T * 4));
    const uint32_t k_sel = K < T ? K : T;
    auto step = [&]() {
        if (c.owner) {
            glm::indexer_scores_relu<<<(H * T + 7) / 8, dim3(32, 8)>>>(qi, kb, scores, H, T, D,
                                                                       1.0f / std::sqrt((float)D));
            glm::indexer_combine<<<(T + 255) / 256, 256>>>(scores, w, index, H, T);
            glm::indexer_topk<<<1, 256>>>(index, T, k_sel, sel, sel_n);
        }
        glm::launch_build_index_mask(sel, k_sel, mask, T);
        glm::mla_decode_absorbed<<<HN, 256, scores_g ? 0 : smem>>>(q, qabs, kvc, krot, ctx, T, DH, 192, R, L,
                                                                   1.0f / std::sqrt((float)DH), mask, scores_g);
    };
    if (!c.owner) {  // a consumer reads a published selection: take the owner's once
        glm::indexer_scores_relu<<<(H * T + 7) / 8, dim3(32, 8)>>>(qi, kb, scores, H, T, D, 1.0f / std::sqrt((float)D));
        glm::indexer_combine<<<(T + 255) / 256, 256>>>(scores, w, index, H, T);
        glm::indexer_topk<<<1, 256>>>(index, T, k_sel, sel, sel_n);
    }
    for (int i = 0; i < 3; ++i) step();
    CK(cudaDeviceSynchronize());
    cudaEvent_t a, b;
    CK(cudaEventCreate(&a));
    CK(cudaEventCreate(&b));
    CK(cudaEventRecord(a));
    for (int i = 0; i < iters; ++i) step();
    CK(cudaEventRecord(b));
    CK(cudaEventSynchronize(b));
    CK(cudaGetLastError());
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, a, b));
    for (void* p : {(void*)q, (void*)qabs, (void*)kvc, (void*)krot, (void*)ctx, (void*)kf, (void*)kb, (void*)w,
                    (void*)scores, (void*)index, (void*)sel, (void*)sel_n, (void*)mask, (void*)qi})
        cudaFree(p);
    if (scores_g) cudaFree(scores_g);
    return ms * 1e3f / iters;
}

}  // namespace

int main(int argc, char** argv) {
    const int iters = argc > 1 ? std::atoi(argv[1]) : 10;
    const Case cases[] = {{1024, true}, {4096, true}, {4096, false}, {32768, true}, {32768, false}, {131072, true}};
    for (const Case& c : cases) {
        const int it = c.T >= 131072 ? (iters > 3 ? 3 : iters) : iters;
        const float us = run_case(c, it);
        std::printf("{\"T\": %u, \"mode\": \"%s\", \"us_per_layer\": %.2f, \"iters\": %d}\n", c.T,
                    c.owner ? "owner" : "consumer", us, it);
        std::fflush(stdout);
    }
    return 0;
}
