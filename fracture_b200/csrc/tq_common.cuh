// Shared pieces of the TurboQuant kernels: argument block, pool-slot rule,
// exact float32 helpers and the MSB-first bit-stream codec.
#pragma once

#include "common.cuh"

namespace fb {

// Calls of at most this many head vectors (num_tokens * num_kv_heads) take the small-call exact
// kernels of tq_small.cu (a few vectors per CTA, none of the tensor-core kernels' set-up):
// where they beat the tensor-core kernels on B200 (GPU time of graph-replayed calls, head_dim
// 128: compress 6.1 vs 10.0 us at 32 vectors, 7.3 vs 10.5 at 256, 10.5 vs 11.0 at 1024;
// dequantize 5.8 vs 6.7 us at 32 vectors, even at 256).
constexpr int64_t kTqSmallCompressVectors = 1024;
constexpr int64_t kTqSmallDequantVectors = 192;

struct TqArgs {
    const void* input;         // compress: [T, H, d] fp16/bf16
    int in_dtype;
    const float* rotation;     // [d, d] row-major f32
    const float* centroids;    // [2^bits] f32
    int bits;
    int n_levels;
    int64_t num_tokens;
    int num_heads;
    int head_dim;
    const int32_t* block_table;  // nullptr: slot = position
    const int64_t* slot_map;     // when set: pool row of call token t = slot_map[t] (block_table unused)
    int64_t start_pos;
    int64_t pool_rows;
    void* packed_pool;         // [pool_rows, H * P] u8
    void* norms_pool;          // [pool_rows, H] fp16
    unsigned int* err_count;   // optional
    void* output;              // dequant: [T, H, d]
    int out_dtype;
};

// Pool row of call token t, or -1 (and err_count bumped) when out of range.
__device__ __forceinline__ int64_t tq_slot(const TqArgs& a, int64_t t) {
    const int64_t pos = a.start_pos + t;
    int64_t slot;
    if (a.slot_map) {
        slot = __ldg(a.slot_map + t);
    } else if (a.block_table) {
        const int32_t b = __ldg(a.block_table + (pos >> 4));
        slot = b < 0 ? -1 : (int64_t)b * 16 + (pos & 15);
    } else {
        slot = pos;
    }
    if (slot < 0 || slot >= a.pool_rows) {
        if (a.err_count) atomicAdd(a.err_count, 1u);
        return -1;
    }
    return slot;
}

__device__ __forceinline__ float load_in_f32(const void* p, int dt, int64_t i) {
    if (dt == FB_BF16) return __bfloat162float(((const __nv_bfloat16*)p)[i]);
    if (dt == FB_FP32) return ((const float*)p)[i];
    return __half2float(((const __half*)p)[i]);
}

// float32 L2 norm: sequential sum of separately rounded squares, IEEE sqrt.
__device__ __forceinline__ float exact_norm(const float* x, int d) {
    float s = 0.0f;
    for (int j = 0; j < d; ++j) s = __fadd_rn(s, __fmul_rn(x[j], x[j]));
    return __fsqrt_rn(s);
}

// First index minimising |y - c_k| (strict <), as the reference kernel scans.
__device__ __forceinline__ int nearest_centroid(float y, const float* c, int n) {
    float best = fabsf(__fsub_rn(y, c[0]));
    int bi = 0;
    for (int k = 1; k < n; ++k) {
        const float dist = fabsf(__fsub_rn(y, c[k]));
        if (dist < best) {
            best = dist;
            bi = k;
        }
    }
    return bi;
}

// Byte `byte` of the MSB-first bit stream of codes idx[0..d).
__device__ __forceinline__ uint8_t pack_byte(const uint8_t* idx, int d, int bits, int byte) {
    unsigned v = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const int p = byte * 8 + b;
        const int i = p / bits;
        unsigned bit = 0;
        if (i < d) bit = (idx[i] >> (bits - 1 - (p - i * bits))) & 1u;
        v = (v << 1) | bit;
    }
    return (uint8_t)v;
}

__device__ __forceinline__ int unpack_code(const uint8_t* row, int i, int bits) {
    const int p = i * bits;
    const int byte = p >> 3, off = p & 7;
    unsigned w = (unsigned)row[byte] << 8;
    if (off + bits > 8) w |= row[byte + 1];
    return (int)((w >> (16 - off - bits)) & ((1u << bits) - 1u));
}

int tq_compress_exact(const TqArgs& a, cudaStream_t s);
int tq_dequant_exact(const TqArgs& a, cudaStream_t s);
bool tq_small_compress_call(const TqArgs& a);
bool tq_small_dequant_call(const TqArgs& a);
int tq_compress_small(const TqArgs& a, cudaStream_t s);
int tq_compress_small_pair(const TqArgs& k, const TqArgs& v, cudaStream_t s);
int tq_dequant_small(const TqArgs& a, cudaStream_t s);

}  // namespace fb
