/*
 * c_abi_roundtrip.c -- the warp_div C ABI (include/fcai_warp_div.h) from plain
 * C99, with no Python or torch: plan, encode, pack and decode of seeded
 * symbols through device buffers that the caller owns, as a binding of the
 * reference's encode_warp_div / decode_warp_div (coders/cuda/ans_gpu.cpp:25-30)
 * would call it.  The symbols run past both ends of the CDF tables, so escapes
 * are coded too.  Exits 0 and prints "c-abi ok" when both decodes (checked and
 * unchecked) return the symbols; tests/test_c_abi.py builds and runs it.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "fcai_warp_div.h"

#define CUDA_OK(call)                                                                  \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));                \
            return 1;                                                                  \
        }                                                                              \
    } while (0)
#define FCAI_CALL(call)                                                                \
    do {                                                                               \
        int rc_ = (call);                                                              \
        if (rc_ != FCAI_OK) {                                                          \
            fprintf(stderr, "%s: status %d (%s)\n", #call, rc_, fcai_last_error());    \
            return 1;                                                                  \
        }                                                                              \
    } while (0)

enum { B = 3, C = 16, HW = 200, N = C * HW, P = 4, L = 34 };

static uint32_t rng_state = 12345u;
static uint32_t next_u32(void) {
    rng_state = rng_state * 1664525u + 1013904223u;
    return rng_state;
}

int main(void) {
    /* per channel: 33 coded symbols (the last one is the escape symbol), a
     * two-sided geometric pmf of 65536 slots centred per channel */
    static int32_t cdfs[C * L], sizes[C], offsets[C], symbols[B * N], decoded[B * N];
    for (int c = 0; c < C; ++c) {
        int32_t freq[L - 1];
        int32_t total = 0;
        for (int i = 0; i < L - 1; ++i) {
            int d = i - 12 - (c % 5);
            if (d < 0) d = -d;
            freq[i] = 1 + (int32_t)(4000.0 / (1 << (d < 12 ? d : 12)));
            total += freq[i];
        }
        freq[12] += 65536 - total; /* the mode takes the rest */
        cdfs[c * L] = 0;
        for (int i = 0; i < L - 1; ++i) cdfs[c * L + i + 1] = cdfs[c * L + i] + freq[i];
        sizes[c] = L;
        offsets[c] = -12;
    }
    for (int i = 0; i < B * N; ++i) {
        int32_t v = (int32_t)(next_u32() % 9u) - 4; /* mostly near the mode */
        if (next_u32() % 50u == 0u) v = (int32_t)(next_u32() % 101u) - 50; /* escapes both ways */
        symbols[i] = v;
    }

    fcai_warp_div_plan plan;
    FCAI_CALL(fcai_warp_div_plan_create(B, N, C, P, &plan));
    const int32_t K = plan.chunks;

    int32_t *d_sym, *d_cdfs, *d_sizes, *d_offs, *d_out;
    uint32_t *d_rounds;
    void *d_ws, *d_dws;
    const int64_t dws_bytes = 256 + ((8 * (int64_t)B * K + 255) / 256) * 256;
    CUDA_OK(cudaMalloc((void **)&d_sym, sizeof symbols));
    CUDA_OK(cudaMalloc((void **)&d_out, sizeof decoded));
    CUDA_OK(cudaMalloc((void **)&d_cdfs, sizeof cdfs));
    CUDA_OK(cudaMalloc((void **)&d_sizes, sizeof sizes));
    CUDA_OK(cudaMalloc((void **)&d_offs, sizeof offsets));
    CUDA_OK(cudaMalloc((void **)&d_rounds, sizeof(uint32_t) * (size_t)B * (size_t)K));
    CUDA_OK(cudaMalloc(&d_ws, (size_t)plan.encode_workspace_bytes));
    CUDA_OK(cudaMalloc(&d_dws, (size_t)dws_bytes));
    CUDA_OK(cudaMemset(d_ws, 0, (size_t)plan.encode_workspace_bytes));
    CUDA_OK(cudaMemset(d_dws, 0, (size_t)dws_bytes));
    CUDA_OK(cudaMemcpy(d_sym, symbols, sizeof symbols, cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(d_cdfs, cdfs, sizeof cdfs, cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(d_sizes, sizes, sizeof sizes, cudaMemcpyHostToDevice));
    CUDA_OK(cudaMemcpy(d_offs, offsets, sizeof offsets, cudaMemcpyHostToDevice));

    fcai_warp_div_encode_info info;
    memset(&info, 0, sizeof info);
    FCAI_CALL(fcai_warp_div_encode(d_sym, NULL, B, N, d_cdfs, C, L, d_sizes, d_offs, P, d_ws,
                                   plan.encode_workspace_bytes, d_rounds, &info, NULL));
    if (info.packed_bytes <= info.header_bytes || info.packed_bytes > plan.max_packed_bytes ||
        info.chunk_len != plan.chunk_len || info.index_layout_is_channel != 1) {
        fprintf(stderr, "unexpected encode info: %lld bytes\n", (long long)info.packed_bytes);
        return 1;
    }
    uint8_t *d_packed;
    CUDA_OK(cudaMalloc((void **)&d_packed, (size_t)info.packed_bytes));
    FCAI_CALL(fcai_warp_div_encode_pack(d_ws, plan.encode_workspace_bytes, B, N, C, P, d_packed, info.packed_bytes,
                                        NULL));

    for (int32_t check = 1; check >= 0; --check) {
        int32_t layout = -1;
        CUDA_OK(cudaMemset(d_out, 0, sizeof decoded));
        FCAI_CALL(fcai_warp_div_decode(d_packed, info.packed_bytes, d_rounds, K, info.header_bytes, info.chunk_len,
                                       NULL, B, N, d_cdfs, C, L, d_sizes, d_offs, d_out, d_dws, dws_bytes, check,
                                       check ? &layout : NULL, NULL));
        CUDA_OK(cudaMemcpy(decoded, d_out, sizeof decoded, cudaMemcpyDeviceToHost));
        if (memcmp(decoded, symbols, sizeof symbols) != 0 || (check && layout != 1)) {
            fprintf(stderr, "decode (check=%d) does not return the symbols\n", (int)check);
            return 1;
        }
    }
    printf("c-abi ok: %s, %d x %d symbols in %lld payload bytes\n", fcai_version(), (int)B, (int)N,
           (long long)info.packed_bytes);
    cudaFree(d_packed);
    cudaFree(d_dws);
    cudaFree(d_ws);
    cudaFree(d_rounds);
    cudaFree(d_offs);
    cudaFree(d_sizes);
    cudaFree(d_cdfs);
    cudaFree(d_out);
    cudaFree(d_sym);
    return 0;
}
