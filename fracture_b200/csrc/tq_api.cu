// C entry points of the TurboQuant kernels: argument checks and dispatch.
//
// Reference ABI: launch_turboquant_compress / launch_turboquant_decompress
// (backends/fracture-cuda/src/ffi.rs:220-247) write/read the compact
// [T, Hkv * P] layout; they are the paged entry points with no block table.

#include <atomic>

#include "common.cuh"
#include "tq_common.cuh"

namespace fb {
int tq_compress_umma(const TqArgs& a, cudaStream_t s, bool* handled);
int tq_compress_umma_pair(const TqArgs& k, const TqArgs& v, cudaStream_t s, bool* handled);
int tq_dequant_umma(const TqArgs& a, cudaStream_t s, bool* handled);
int tq_dequant_umma_pair(const TqArgs& k, const TqArgs& v, cudaStream_t s, bool* handled);
}

using namespace fb;

// Calls served per path since the library was loaded: compress small / tensor-core / exact, then
// dequantize small / tensor-core / exact, then K+V compress and K+V dequantize pairs served by one
// tensor-core launch, then paged attention calls served by the CUDA-core, the per-head
// tensor-core and the streamed tensor-core kernel (fb_tq_path_counts).
constexpr int kTqPaths = 12;
static std::atomic<unsigned long long> g_tq_path_calls[kTqPaths];

static int count_path(int which, int rc) {
    if (rc == 0) g_tq_path_calls[which].fetch_add(1, std::memory_order_relaxed);
    return rc;
}

namespace fb {
int tq_count_path(int which, int rc) { return count_path(which, rc); }
}

static bool tq_bits_ok(int bits) { return bits == 2 || bits == 3 || bits == 4 || bits == 8; }

static int tq_check_common(int bits, int64_t num_tokens, int num_kv_heads, int head_dim, int64_t pool_rows) {
    if (!tq_bits_ok(bits) || num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || head_dim > 192 || pool_rows < 0)
        return (int)cudaErrorInvalidValue;
    return 0;
}

// Checks one compress call and fills its argument block (a.num_tokens == 0: nothing to do).
static int tq_compress_args(const void* input, int dtype, const float* rotation, const float* centroids, int bits,
                            int64_t num_tokens, int num_kv_heads, int head_dim, const int32_t* block_table,
                            const int64_t* slot_map, int64_t start_pos, int64_t num_pool_rows, void* packed_pool,
                            void* norms_pool, unsigned int* err_count, TqArgs* out) {
    *out = TqArgs{};
    int rc = tq_check_common(bits, num_tokens, num_kv_heads, head_dim, num_pool_rows);
    if (rc) return rc;
    if (dtype != FB_FP16 && dtype != FB_BF16 && dtype != FB_FP32) return (int)cudaErrorInvalidValue;
    if (start_pos < 0) return (int)cudaErrorInvalidValue;
    if (num_tokens == 0) return 0;
    if (!input || !rotation || !centroids || !packed_pool || !norms_pool) return (int)cudaErrorInvalidValue;
    TqArgs& a = *out;
    a.input = input;
    a.in_dtype = dtype;
    a.rotation = rotation;
    a.centroids = centroids;
    a.bits = bits;
    a.n_levels = 1 << bits;
    a.num_tokens = num_tokens;
    a.num_heads = num_kv_heads;
    a.head_dim = head_dim;
    a.block_table = block_table;
    a.slot_map = slot_map;
    a.start_pos = start_pos;
    a.pool_rows = num_pool_rows;
    a.packed_pool = packed_pool;
    a.norms_pool = norms_pool;
    a.err_count = err_count;
    return 0;
}

// Small calls take the few-vectors-per-CTA kernels, the rest the tensor-core kernel where it
// applies, else the exact CUDA-core kernel.
static int tq_compress_dispatch(const TqArgs& a, void* stream) {
    if (tq_small_compress_call(a)) return count_path(0, tq_compress_small(a, (cudaStream_t)stream));
    bool handled = false;
    const int rc = tq_compress_umma(a, (cudaStream_t)stream, &handled);
    if (handled) return count_path(1, rc);
    return count_path(2, tq_compress_exact(a, (cudaStream_t)stream));
}

static int tq_compress_any(const void* input, int dtype, const float* rotation, const float* centroids, int bits,
                           int64_t num_tokens, int num_kv_heads, int head_dim, const int32_t* block_table,
                           const int64_t* slot_map, int64_t start_pos, int64_t num_pool_rows, void* packed_pool,
                           void* norms_pool, unsigned int* err_count, void* stream) {
    TqArgs a;
    const int rc = tq_compress_args(input, dtype, rotation, centroids, bits, num_tokens, num_kv_heads, head_dim,
                                    block_table, slot_map, start_pos, num_pool_rows, packed_pool, norms_pool,
                                    err_count, &a);
    if (rc || a.num_tokens == 0) return rc;
    return tq_compress_dispatch(a, stream);
}

// K and V of one append (same tokens, heads and pool rows): small calls take one small-call launch
// for both, larger ones one tensor-core launch where the widths allow it, else two calls.
static int tq_compress_kv_dispatch(const TqArgs& k, const TqArgs& v, void* stream) {
    if (tq_small_compress_call(k)) return count_path(11, tq_compress_small_pair(k, v, (cudaStream_t)stream));
    bool handled = false;
    const int rc = tq_compress_umma_pair(k, v, (cudaStream_t)stream, &handled);
    if (handled) return count_path(6, rc);
    const int rk = tq_compress_dispatch(k, stream);
    if (rk) return rk;
    return tq_compress_dispatch(v, stream);
}

extern "C" int fb_launch_tq_compress_paged(const void* input, int dtype, const float* rotation, const float* centroids,
                                           int bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                           const int32_t* block_table, int64_t start_pos, int64_t num_pool_rows,
                                           void* packed_pool, void* norms_pool, unsigned int* err_count, void* stream) {
    return tq_compress_any(input, dtype, rotation, centroids, bits, num_tokens, num_kv_heads, head_dim, block_table,
                           nullptr, start_pos, num_pool_rows, packed_pool, norms_pool, err_count, stream);
}

// K and V of one append: one tensor-core launch for both where they qualify, else two calls.
extern "C" int fb_launch_tq_compress_kv_paged(const void* k_input, const void* v_input, int dtype,
                                              const float* k_rotation, const float* v_rotation,
                                              const float* k_centroids, const float* v_centroids, int key_bits,
                                              int value_bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                              const int32_t* block_table, int64_t start_pos, int64_t num_pool_rows,
                                              void* k_packed_pool, void* k_norms_pool, void* v_packed_pool,
                                              void* v_norms_pool, unsigned int* err_count, void* stream) {
    TqArgs k, v;
    int rc = tq_compress_args(k_input, dtype, k_rotation, k_centroids, key_bits, num_tokens, num_kv_heads, head_dim,
                              block_table, nullptr, start_pos, num_pool_rows, k_packed_pool, k_norms_pool, err_count,
                              &k);
    if (rc) return rc;
    rc = tq_compress_args(v_input, dtype, v_rotation, v_centroids, value_bits, num_tokens, num_kv_heads, head_dim,
                          block_table, nullptr, start_pos, num_pool_rows, v_packed_pool, v_norms_pool, err_count, &v);
    if (rc || num_tokens == 0) return rc;
    return tq_compress_kv_dispatch(k, v, stream);
}

// K and V of a batched append through one slot map (one launch for both where they qualify).
extern "C" int fb_launch_tq_compress_kv_slots(const void* k_input, const void* v_input, int dtype,
                                              const float* k_rotation, const float* v_rotation,
                                              const float* k_centroids, const float* v_centroids, int key_bits,
                                              int value_bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                              const int64_t* slot_map, int64_t num_pool_rows, void* k_packed_pool,
                                              void* k_norms_pool, void* v_packed_pool, void* v_norms_pool,
                                              unsigned int* err_count, void* stream) {
    if (!slot_map && num_tokens > 0) return (int)cudaErrorInvalidValue;
    TqArgs k, v;
    int rc = tq_compress_args(k_input, dtype, k_rotation, k_centroids, key_bits, num_tokens, num_kv_heads, head_dim,
                              nullptr, slot_map, 0, num_pool_rows, k_packed_pool, k_norms_pool, err_count, &k);
    if (rc) return rc;
    rc = tq_compress_args(v_input, dtype, v_rotation, v_centroids, value_bits, num_tokens, num_kv_heads, head_dim,
                          nullptr, slot_map, 0, num_pool_rows, v_packed_pool, v_norms_pool, err_count, &v);
    if (rc || num_tokens == 0) return rc;
    return tq_compress_kv_dispatch(k, v, stream);
}

// Batched append: token t of the call goes to pool row slot_map[t] (negative or out of range:
// skipped and counted in err_count); one launch for the new tokens of many sequences.
extern "C" int fb_launch_tq_compress_slots(const void* input, int dtype, const float* rotation, const float* centroids,
                                           int bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                           const int64_t* slot_map, int64_t num_pool_rows, void* packed_pool,
                                           void* norms_pool, unsigned int* err_count, void* stream) {
    if (!slot_map && num_tokens > 0) return (int)cudaErrorInvalidValue;
    return tq_compress_any(input, dtype, rotation, centroids, bits, num_tokens, num_kv_heads, head_dim, nullptr,
                           slot_map, 0, num_pool_rows, packed_pool, norms_pool, err_count, stream);
}

// Checks one dequantize call and fills its argument block (a.num_tokens == 0: nothing to do).
static int tq_dequant_args(const void* packed_pool, const void* norms_pool, const float* rotation,
                           const float* centroids, int bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                           const int32_t* block_table, const int64_t* slot_map, int64_t start_pos,
                           int64_t num_pool_rows, void* output, int dtype, TqArgs* out) {
    *out = TqArgs{};
    int rc = tq_check_common(bits, num_tokens, num_kv_heads, head_dim, num_pool_rows);
    if (rc) return rc;
    if (dtype != FB_FP16 && dtype != FB_BF16 && dtype != FB_FP32) return (int)cudaErrorInvalidValue;
    if (start_pos < 0) return (int)cudaErrorInvalidValue;
    if (num_tokens == 0) return 0;
    if (!packed_pool || !norms_pool || !rotation || !centroids || !output) return (int)cudaErrorInvalidValue;
    TqArgs& a = *out;
    a.rotation = rotation;
    a.centroids = centroids;
    a.bits = bits;
    a.n_levels = 1 << bits;
    a.num_tokens = num_tokens;
    a.num_heads = num_kv_heads;
    a.head_dim = head_dim;
    a.block_table = block_table;
    a.slot_map = slot_map;
    a.start_pos = start_pos;
    a.pool_rows = num_pool_rows;
    a.packed_pool = const_cast<void*>(packed_pool);
    a.norms_pool = const_cast<void*>(norms_pool);
    a.output = output;
    a.out_dtype = dtype;
    return 0;
}

static int tq_dequant_dispatch(const TqArgs& a, void* stream) {
    if (tq_small_dequant_call(a)) return count_path(3, tq_dequant_small(a, (cudaStream_t)stream));
    bool handled = false;
    const int rc = tq_dequant_umma(a, (cudaStream_t)stream, &handled);
    if (handled) return count_path(4, rc);
    return count_path(5, tq_dequant_exact(a, (cudaStream_t)stream));
}

static int tq_dequant_any(const void* packed_pool, const void* norms_pool, const float* rotation,
                          const float* centroids, int bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                          const int32_t* block_table, const int64_t* slot_map, int64_t start_pos,
                          int64_t num_pool_rows, void* output, int dtype, void* stream) {
    TqArgs a;
    const int rc = tq_dequant_args(packed_pool, norms_pool, rotation, centroids, bits, num_tokens, num_kv_heads,
                                   head_dim, block_table, slot_map, start_pos, num_pool_rows, output, dtype, &a);
    if (rc || a.num_tokens == 0) return rc;
    return tq_dequant_dispatch(a, stream);
}

// K and V of one cache read: one tensor-core launch for both where they qualify, else two calls.
extern "C" int fb_launch_tq_dequant_kv_paged(const void* k_packed_pool, const void* k_norms_pool,
                                             const void* v_packed_pool, const void* v_norms_pool,
                                             const float* k_rotation, const float* v_rotation,
                                             const float* k_centroids, const float* v_centroids, int key_bits,
                                             int value_bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                             const int32_t* block_table, int64_t start_pos, int64_t num_pool_rows,
                                             void* k_output, void* v_output, int dtype, void* stream) {
    TqArgs k, v;
    int rc = tq_dequant_args(k_packed_pool, k_norms_pool, k_rotation, k_centroids, key_bits, num_tokens, num_kv_heads,
                             head_dim, block_table, nullptr, start_pos, num_pool_rows, k_output, dtype, &k);
    if (rc) return rc;
    rc = tq_dequant_args(v_packed_pool, v_norms_pool, v_rotation, v_centroids, value_bits, num_tokens, num_kv_heads,
                         head_dim, block_table, nullptr, start_pos, num_pool_rows, v_output, dtype, &v);
    if (rc || num_tokens == 0) return rc;
    if (!tq_small_dequant_call(k)) {
        bool handled = false;
        rc = tq_dequant_umma_pair(k, v, (cudaStream_t)stream, &handled);
        if (handled) return count_path(7, rc);
    }
    rc = tq_dequant_dispatch(k, stream);
    if (rc) return rc;
    return tq_dequant_dispatch(v, stream);
}

extern "C" int fb_launch_tq_dequant_paged(const void* packed_pool, const void* norms_pool, const float* rotation,
                                          const float* centroids, int bits, int64_t num_tokens, int num_kv_heads,
                                          int head_dim, const int32_t* block_table, int64_t start_pos,
                                          int64_t num_pool_rows, void* output, int dtype, void* stream) {
    return tq_dequant_any(packed_pool, norms_pool, rotation, centroids, bits, num_tokens, num_kv_heads, head_dim,
                          block_table, nullptr, start_pos, num_pool_rows, output, dtype, stream);
}

// Gather by slot map: output token t from pool row slot_map[t] (no row: zeros).
extern "C" int fb_launch_tq_dequant_slots(const void* packed_pool, const void* norms_pool, const float* rotation,
                                          const float* centroids, int bits, int64_t num_tokens, int num_kv_heads,
                                          int head_dim, const int64_t* slot_map, int64_t num_pool_rows, void* output,
                                          int dtype, void* stream) {
    if (!slot_map && num_tokens > 0) return (int)cudaErrorInvalidValue;
    return tq_dequant_any(packed_pool, norms_pool, rotation, centroids, bits, num_tokens, num_kv_heads, head_dim,
                          nullptr, slot_map, 0, num_pool_rows, output, dtype, stream);
}

extern "C" int launch_turboquant_compress(const void* input, const float* rotation, const float* centroids,
                                          void* packed_out, void* norms_out, int num_tokens, int num_kv_heads,
                                          int head_dim, int n_levels, int bits, int packed_dim_per_head,
                                          void* stream) {
    if (!tq_bits_ok(bits) || n_levels != (1 << bits) || head_dim <= 0 ||
        packed_dim_per_head != (head_dim * bits + 7) / 8)
        return (int)cudaErrorInvalidValue;
    return fb_launch_tq_compress_paged(input, FB_FP16, rotation, centroids, bits, num_tokens, num_kv_heads, head_dim,
                                       nullptr, 0, num_tokens, packed_out, norms_out, nullptr, stream);
}

extern "C" int launch_turboquant_decompress(const void* packed_in, const void* norms_in, const float* rotation,
                                            const float* centroids, void* output, int num_tokens, int num_kv_heads,
                                            int head_dim, int bits, int packed_dim_per_head, void* stream) {
    if (!tq_bits_ok(bits) || head_dim <= 0 || packed_dim_per_head != (head_dim * bits + 7) / 8)
        return (int)cudaErrorInvalidValue;
    return fb_launch_tq_dequant_paged(packed_in, norms_in, rotation, centroids, bits, num_tokens, num_kv_heads,
                                      head_dim, nullptr, 0, num_tokens, output, FB_FP16, stream);
}

extern "C" int fb_tq_path_counts(unsigned long long* counts, int n) {
    if (!counts || n < 0) return (int)cudaErrorInvalidValue;
    for (int i = 0; i < n && i < kTqPaths; ++i) counts[i] = g_tq_path_calls[i].load(std::memory_order_relaxed);
    return 0;
}
