/*
 * fracture_b200 — C ABI of the B200 (sm_100a) implementation of Fracture's
 * per-layer elementwise hot path and TurboQuant KV compression.
 *
 * Three layers of entry points, all plain C (pointers, sizes, ints):
 *
 *  1. The reference kernel ABI. Same names, argument lists and meaning as the
 *     `extern "C"` kernels Fracture's CUDA backend links today
 *     (backends/fracture-cuda/src/ffi.rs:141-249, implemented by
 *     backends/fracture-cuda/kernels/*.cu). FP16 tensors, cudaError_t return,
 *     enqueued on `stream`. Linking this library instead of
 *     libfracture_kernels.a changes nothing above the FFI.
 *
 *  2. New kernel entry points: dtype-generic (FP16 / BF16 / FP32) versions,
 *     the fused residual-add + RMSNorm, one-launch Q+K RoPE, TurboQuant
 *     compress / dequantize straight into a paged pool, and paged attention
 *     over the TurboQuant and the FP16/BF16 caches. Host-table builders
 *     (RoPE frequencies incl. llama3 scaling, Lloyd-Max codebook, Haar
 *     rotation) restate crates/fracture-core on the host.
 *
 *  3. A backend object that mirrors `trait Backend`
 *     (crates/fracture-core/src/backend.rs:8-223) over opaque tensor handles,
 *     so the Rust `CudaBackend` can be replaced by a thin shim, plus the
 *     quantized paged KV cache of crates/fracture-engine/src/
 *     quantized_paged_kv_cache.rs with its append_kv fused into one launch,
 *     and the FP16/BF16 paged KV cache of paged_kv_cache.rs.
 *
 * Stream order: every call is ordered after the work already on its stream.
 * Decode-sized elementwise, RoPE, small TurboQuant and paged-attention launches
 * are programmatic dependent launches: they may be scheduled while the previous
 * kernel on the stream drains, and wait for it to complete (its writes
 * visible) before they touch memory, so the ordering is the same.
 *
 * Return values: layer 1 and 2 return a cudaError_t value (0 = success;
 * cudaErrorInvalidValue = 1 for arguments rejected by the host-side checks,
 * before anything is enqueued). Layer 3 returns an fb_status and records a
 * message retrievable with fb_last_error().
 */
#ifndef FRACTURE_B200_H
#define FRACTURE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage dtypes, in the reference's DType order (crates/fracture-core/src/dtype.rs:5-11). */
enum fb_dtype { FB_FP16 = 0, FB_FP32 = 1, FB_BF16 = 2, FB_INT8 = 3, FB_INT4 = 4 };

/* ======================================================================== */
/* 1. Reference kernel ABI (backends/fracture-cuda/src/ffi.rs:141-249)       */
/* ======================================================================== */

/* ffi.rs:142-150; kernels/rmsnorm.cu:69-85. output = x * rsqrt(mean(x^2)+eps) * w, FP16 [rows, cols]. */
int launch_rmsnorm(void* output, const void* input, const void* weight, float eps, int rows, int cols,
                   void* stream);

/* ffi.rs:152-162; kernels/rope.cu:51-82. In-place split-half RoPE on Q [T,Hq,d] and K [T,Hkv,d] FP16.
 * positions: device u32 [T]; freq_table: device f32 [d/2]. One launch covers Q and K. */
int launch_rope(void* q, void* k, const uint32_t* positions, const float* freq_table, int num_tokens,
                int num_q_heads, int num_kv_heads, int head_dim, void* stream);

/* ffi.rs:164-170; kernels/silu_mul.cu:25-38. output = silu(gate) * up, FP16 [n]. */
int launch_silu_mul(void* output, const void* gate, const void* up, int n, void* stream);

/* ffi.rs:200-208; kernels/embedding.cu:30-47. output[t] = table[ids[t]] (zero row when id >= vocab). */
int launch_embedding(void* output, const void* table, const uint32_t* token_ids, int num_tokens,
                     int hidden_dim, int vocab_size, void* stream);

/* ffi.rs:210-216; kernels/add.cu:16-29. output = a + b, FP16 [n] (output may alias a or b). */
int launch_add(void* output, const void* a, const void* b, int n, void* stream);

/* ffi.rs:220-233; kernels/turboquant_compress.cu:189-222. input FP16 [T,Hkv,d]; rotation f32 [d,d];
 * centroids f32 [n_levels]; packed_out u8 [T, Hkv*packed_dim_per_head]; norms_out FP16 [T,Hkv].
 * bits: 2, 3, 4 or 8 (3 is an extension: MSB-first bit stream). */
int launch_turboquant_compress(const void* input, const float* rotation, const float* centroids,
                               void* packed_out, void* norms_out, int num_tokens, int num_kv_heads,
                               int head_dim, int n_levels, int bits, int packed_dim_per_head,
                               void* stream);

/* ffi.rs:235-247; kernels/turboquant_decompress.cu:96-127. Inverse of the above into FP16 [T,Hkv,d]. */
int launch_turboquant_decompress(const void* packed_in, const void* norms_in, const float* rotation,
                                 const float* centroids, void* output, int num_tokens, int num_kv_heads,
                                 int head_dim, int bits, int packed_dim_per_head, void* stream);
/* ffi.rs:186-200 (attention_paged.cu:161-185): GQA attention of num_tokens FP16 query tokens of one
 * sequence over its FP16 paged KV cache; block_table (device int32, num_blocks_in_seq entries)
 * maps logical block pos/16 to a physical block whose K and V rows sit at k_block_ptrs[b],
 * v_block_ptrs[b] (device arrays of device pointers, [16, Hkv, d] each). Token t attends positions
 * [0, min(start_pos + t + 1, kv_len)). head_dim 128, Hq/Hkv in {1, 2, 4, 8}; float32 math. Uses a
 * device workspace owned by this library, one per device and stream, grown to the largest call on
 * that stream and kept until exit (calls on different streams may run at the same time). Growing
 * it calls cudaFree/cudaMalloc, which a stream being captured into a CUDA graph refuses: make a
 * call of the largest size on the stream before capturing. The workspace is keyed by the stream
 * handle, so do not call on a handle that was destroyed and reused while work queued on the old
 * stream may still be running. */
int launch_paged_attention(void* output, const void* q, const int* block_table, const void** k_block_ptrs,
                           const void** v_block_ptrs, int num_tokens, int num_q_heads, int num_kv_heads,
                           int head_dim, int kv_len, int start_pos, int num_blocks_in_seq, void* stream);

/* ffi.rs:251-274 (attention_paged_tq.cu:261-309): attention of num_tokens FP16 query tokens of one
 * sequence over its TurboQuant-compressed paged cache; block_table (device int32) maps logical
 * block pos/16 to a physical block whose packed K/V rows and norms sit at k_packed_ptrs[b],
 * k_norms_ptrs[b], ... (device arrays of device pointers, [16, Hkv*P] and [16, Hkv]). Token t
 * attends positions [0, min(start_pos + t + 1, kv_len)). head_dim 128, Hq/Hkv in {1, 2, 4, 8},
 * 2/3/4/8-bit codes; k_rotation 16-byte aligned. The reference's math with FP32 accumulation:
 * 2- and 4-bit codes on the tensor cores (centroid values, rotated queries and softmax weights as
 * fp16 operands), 3- and 8-bit codes on CUDA cores in float32 with the 3-bit centroid values read
 * as fp16; all within the 2e-3 FP bar of the float32 statement. Uses a device workspace owned by
 * this library, one per device and stream, grown to the largest call on that stream and kept until
 * exit (calls on different streams may run at the same time), with the same two caveats as
 * launch_paged_attention: a warm-up call of the largest size before graph capture, and no call on
 * a recycled stream handle while the old stream's work may still be running. */
int launch_attention_paged_tq(void* output, const void* q, const int* block_table, const void** k_packed_ptrs,
                              const void** k_norms_ptrs, const void** v_packed_ptrs, const void** v_norms_ptrs,
                              const float* k_rotation, const float* v_rotation, const float* k_centroids,
                              const float* v_centroids, int num_tokens, int num_q_heads, int num_kv_heads,
                              int head_dim, int kv_len, int start_pos, int key_bits, int value_bits,
                              int k_packed_dim_per_head, int v_packed_dim_per_head, void* stream);

/* launch_attention_paged_tq for callers that cannot allocate device memory (no counterpart in the
 * reference). An engine that sized its KV pool to take all free memory at start-up cannot have a
 * cudaMalloc succeed mid-step, and a decode loop must not stall on the device-wide synchronisation
 * of the cudaFree that growing launch_attention_paged_tq's workspace implies. This entry point
 * allocates nothing: the rotated queries and split-K partials live in one fixed array of
 * FB_TQA_NOALLOC_SCRATCH_BYTES (4 MiB) of device memory inside the library image, which every GPU
 * that loads the library holds until the process exits. Same arguments, kernels and results as
 * launch_attention_paged_tq (bit for bit). A call needs
 *   num_tokens * num_q_heads * (512 + 520 * ceil(kv_len / 256)) bytes
 * of it (one decode token with 32 Q heads: contexts up to 64,256 positions); a larger call returns
 * cudaErrorInvalidValue, with the reason in fb_last_error(), before anything is enqueued. The
 * first call on a device looks the array's device address up (cudaGetSymbolAddress), so make it
 * before any stream capture. Every call shares the array and it keeps the last call's contents
 * (nothing needs clearing: each call writes what it reads), so calls that can overlap on the GPU
 * (on two streams, or from two threads without ordering) race; order them on one stream. */
#define FB_TQA_NOALLOC_SCRATCH_BYTES ((size_t)4 << 20)
int launch_attention_paged_tq_noalloc(void* output, const void* q, const int* block_table,
                                      const void** k_packed_ptrs, const void** k_norms_ptrs,
                                      const void** v_packed_ptrs, const void** v_norms_ptrs,
                                      const float* k_rotation, const float* v_rotation, const float* k_centroids,
                                      const float* v_centroids, int num_tokens, int num_q_heads, int num_kv_heads,
                                      int head_dim, int kv_len, int start_pos, int key_bits, int value_bits,
                                      int k_packed_dim_per_head, int v_packed_dim_per_head, void* stream);

/* ======================================================================== */
/* 2. New kernel entry points                                               */
/* ======================================================================== */

/* Embedding gather for any storage dtype (replaces embedding.cu:7-28). */
int fb_launch_embedding(void* output, const void* table, const uint32_t* token_ids, int64_t num_tokens,
                        int64_t hidden_dim, int64_t vocab_size, int dtype, void* stream);

/* out = a + b with one rounding to dtype (replaces add.cu:5-14). */
int fb_launch_add(void* output, const void* a, const void* b, int64_t n, int dtype, void* stream);

/* RMSNorm for any storage dtype (replaces rmsnorm.cu:10-67). */
int fb_launch_rmsnorm(void* output, const void* input, const void* weight, float eps, int64_t rows,
                      int64_t cols, int dtype, void* stream);

/* Fused residual add + RMSNorm: h <- round(h + residual); normed <- round(h * rsqrt(mean(h^2)+eps) * w).
 * Replaces the engine's back-to-back add(h, r, h); rmsnorm(h, w, eps, normed)
 * (crates/fracture-engine/src/batched.rs:393-396, engine.rs:364-371). No reference counterpart. */
int fb_launch_add_rmsnorm(void* h_inout, const void* residual, const void* weight, void* normed_out,
                          float eps, int64_t rows, int64_t cols, int dtype, void* stream);

/* In-place RoPE on Q and K in one launch, any storage dtype (replaces rope.cu:20-82). */
int fb_launch_rope(void* q, void* k, const uint32_t* positions, const float* freq_table, int64_t num_tokens,
                   int num_q_heads, int num_kv_heads, int head_dim, int dtype, void* stream);

/* silu(gate) * up for any storage dtype (replaces silu_mul.cu:8-23). */
int fb_launch_silu_mul(void* output, const void* gate, const void* up, int64_t n, int dtype, void* stream);

/* TurboQuant compress written straight into a paged pool.
 * input: [num_tokens, Hkv, d] (FP16 or BF16, `dtype`); rotation f32 [d,d] row-major; centroids f32 [2^bits].
 * Token t (position start_pos + t of the sequence) lands in pool row
 *   slot = block_table[(start_pos+t)/16]*16 + (start_pos+t)%16
 * i.e. packed_pool[slot, h*P .. h*P+P) and norms_pool[slot, h] (FP16), P = ceil(d*bits/8), which is
 * the per-block layout of the reference's block tensors (quantized_paged_kv_cache.rs:82-133) placed
 * back to back. block_table == NULL means slot = t (the reference's compress-to-scratch layout).
 * num_pool_rows bounds every slot (rejected on device: the token is skipped and *err_count bumped
 * when err_count != NULL). Replaces turboquant_compress + 4x copy_rows per block segment
 * (quantized_paged_kv_cache.rs:417-497). Index results equal the exact float32 statement
 * (sequential sums, true division) bit for bit. */
int fb_launch_tq_compress_paged(const void* input, int dtype, const float* rotation, const float* centroids,
                                int bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                const int32_t* block_table, int64_t start_pos, int64_t num_pool_rows,
                                void* packed_pool, void* norms_pool, unsigned int* err_count, void* stream);

/* K and V of one append in one call (no reference counterpart; replaces the two compress calls of
 * quantized_paged_kv_cache.rs:417-438): fb_launch_tq_compress_paged for the keys (k_*, key_bits)
 * and for the values (v_*, value_bits), same tokens, block table and pool rows. Where both take
 * the tensor-core kernel (head_dim 128, FP16 or BF16, 2/3/4-bit codes of equal width, or 4-bit
 * keys with 2-bit values) they run as one launch whose grid is split between K and V; calls small
 * enough for the small-call kernel (decode steps: at most 1024 head vectors each) also run as one
 * launch of that kernel for both; otherwise as two calls. Results equal the two separate calls bit
 * for bit. */
int fb_launch_tq_compress_kv_paged(const void* k_input, const void* v_input, int dtype, const float* k_rotation,
                                   const float* v_rotation, const float* k_centroids, const float* v_centroids,
                                   int key_bits, int value_bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                   const int32_t* block_table, int64_t start_pos, int64_t num_pool_rows,
                                   void* k_packed_pool, void* k_norms_pool, void* v_packed_pool, void* v_norms_pool,
                                   unsigned int* err_count, void* stream);

/* Which TurboQuant kernels served the compress / dequantize calls made so far in this process (no
 * reference counterpart; for tests and diagnostics): counts[0..2] = compress calls that took the
 * small-call kernel (tq_small.cu), the tensor-core kernel (tq_umma.cu) and the exact CUDA-core
 * kernel (tq_exact.cu); counts[3..5] the same for dequantize; counts[6] = K+V pairs of
 * fb_launch_tq_compress_kv_paged served by one tensor-core launch; counts[7] the same for
 * fb_launch_tq_dequant_kv_paged; counts[8..10] = paged-attention calls (every TurboQuant attention
 * entry point) whose main kernel was the CUDA-core one, the per-head tensor-core one and the
 * streamed tensor-core one; counts[11] = K+V pairs of fb_launch_tq_compress_kv_paged or
 * fb_launch_tq_compress_kv_slots served by one small-call launch. Writes min(n, 12) counters. */
int fb_tq_path_counts(unsigned long long* counts, int n);

/* Batched append (no reference counterpart; the reference appends one sequence at a time,
 * quantized_paged_kv_cache.rs:404-500, called per sequence from batched.rs:324-350): as
 * fb_launch_tq_compress_paged, but call token t goes to pool row slot_map[t] (int64; negative or
 * >= num_pool_rows: skipped and counted in err_count once per head vector), so one launch writes the
 * new tokens of many sequences. */
int fb_launch_tq_compress_slots(const void* input, int dtype, const float* rotation, const float* centroids,
                                int bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                const int64_t* slot_map, int64_t num_pool_rows, void* packed_pool,
                                void* norms_pool, unsigned int* err_count, void* stream);

/* K and V of one batched append in one call (no reference counterpart; the reference compresses K
 * and V separately, quantized_paged_kv_cache.rs:417-438): fb_launch_tq_compress_slots for the keys
 * (k_*, key_bits) and for the values (v_*, value_bits) through the same slot map, with the launch
 * sharing of fb_launch_tq_compress_kv_paged (one small-call launch for both at decode sizes, one
 * tensor-core launch where both qualify). Results equal the two separate calls bit for bit. */
int fb_launch_tq_compress_kv_slots(const void* k_input, const void* v_input, int dtype, const float* k_rotation,
                                   const float* v_rotation, const float* k_centroids, const float* v_centroids,
                                   int key_bits, int value_bits, int64_t num_tokens, int num_kv_heads, int head_dim,
                                   const int64_t* slot_map, int64_t num_pool_rows, void* k_packed_pool,
                                   void* k_norms_pool, void* v_packed_pool, void* v_norms_pool,
                                   unsigned int* err_count, void* stream);

/* TurboQuant dequantize from a paged pool into [num_tokens, Hkv, d] (`dtype` FP16/BF16/FP32):
 * x = (Pi^T @ centroids[idx]) * norm (replaces turboquant_decompress.cu:21-94). Same slot rule; a
 * token without a valid slot dequantizes to zeros. head_dim 128 with 2/3/4-bit codes and FP16/BF16
 * output runs on the tensor cores (one fp16 pass: within about 1e-4 of the output's magnitude of
 * the float32 statement); every other case evaluates the float32 statement exactly. */
int fb_launch_tq_dequant_paged(const void* packed_pool, const void* norms_pool, const float* rotation,
                               const float* centroids, int bits, int64_t num_tokens, int num_kv_heads,
                               int head_dim, const int32_t* block_table, int64_t start_pos,
                               int64_t num_pool_rows, void* output, int dtype, void* stream);

/* K and V of one cache read in one call (no reference counterpart): fb_launch_tq_dequant_paged for
 * the keys (k_*, key_bits) and the values (v_*, value_bits), same tokens, block table and pool
 * rows, outputs of one `dtype`. Where both take the tensor-core kernel with whole-token tiles
 * (head_dim 128, FP16/BF16 output, 2/3/4-bit codes of equal width or 4-bit keys with 2-bit
 * values, KV head count a multiple of 8 dividing 128, 16-byte aligned pools) they run as one
 * launch whose grid is split between K and V; otherwise as two calls. Results equal the two
 * separate calls bit for bit. */
int fb_launch_tq_dequant_kv_paged(const void* k_packed_pool, const void* k_norms_pool, const void* v_packed_pool,
                                  const void* v_norms_pool, const float* k_rotation, const float* v_rotation,
                                  const float* k_centroids, const float* v_centroids, int key_bits, int value_bits,
                                  int64_t num_tokens, int num_kv_heads, int head_dim, const int32_t* block_table,
                                  int64_t start_pos, int64_t num_pool_rows, void* k_output, void* v_output, int dtype,
                                  void* stream);

/* Gather counterpart of fb_launch_tq_compress_slots (no reference counterpart): output token t is
 * dequantized from pool row slot_map[t] (no row: zeros). Same kernels and tolerance as
 * fb_launch_tq_dequant_paged. */
int fb_launch_tq_dequant_slots(const void* packed_pool, const void* norms_pool, const float* rotation,
                               const float* centroids, int bits, int64_t num_tokens, int num_kv_heads,
                               int head_dim, const int64_t* slot_map, int64_t num_pool_rows, void* output,
                               int dtype, void* stream);

/* TurboQuant paged attention over this library's pools, batched over sequences (no reference
 * counterpart for the batching; the math is attention_paged_tq.cu:56-259, called per sequence
 * from batched.rs:156-193). Queries [num_seqs * q_per_seq, Hq, 128] FP16/BF16 (`dtype`, also the
 * output's), sequence-major; sequence s reads its blocks from block_tables[s * max_blocks_per_seq
 * ...] (device int32; a negative entry leaves its 16 positions out) in the K/V pools laid out as
 * fb_launch_tq_compress_paged writes them; query t of sequence s attends positions
 * [0, min(start_pos[s] + t + 1, kv_lens[s])) (device int32 arrays; max_kv_len bounds kv_lens).
 * Hq/Hkv in {1, 2, 4, 8}; key_bits/value_bits 2, 3, 4 or 8. `workspace` (16-byte aligned, at
 * least num_seqs * q_per_seq * num_q_heads * (512 + 520 * ceil(max_kv_len / 256)) bytes) holds the
 * rotated queries and the split-K partial results, one per chunk of at least 256 positions.
 * fb_tq_attention_workspace_bytes returns that, or more for calls with few query rows: room for
 * up to one partial per 32 positions (at most 160 per head over the rows), with which the
 * streamed kernel splits a short or sparsely batched context into more chunks to give every SM
 * work. A workspace between the two sizes uses the slots it holds.
 * k_rotation 16-byte aligned. Numerics as for launch_attention_paged_tq. */
size_t fb_tq_attention_workspace_bytes(int num_seqs, int q_per_seq, int num_q_heads, int max_kv_len);
int fb_launch_tq_attention_paged(const void* q, int dtype, int num_seqs, int q_per_seq, int num_q_heads,
                                 int num_kv_heads, int head_dim, const void* k_packed_pool, const void* k_norms_pool,
                                 const void* v_packed_pool, const void* v_norms_pool, int64_t num_pool_rows,
                                 const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens,
                                 const int32_t* start_pos, int max_kv_len, const float* k_rotation,
                                 const float* v_rotation, const float* k_centroids, const float* v_centroids,
                                 int key_bits, int value_bits, void* workspace, size_t workspace_bytes, void* output,
                                 void* stream);

/* Paged attention over an FP16/BF16 KV cache, batched over sequences (no reference counterpart for
 * the batching; the math is attention_paged.cu:25-159, called per sequence). Pools
 * [num_pool_rows, Hkv, 128] of `dtype` (the reference's per-block tensors [16, Hkv, d] back to back,
 * pool row = block * 16 + offset); queries and output [num_seqs * q_per_seq, Hq, 128] of `dtype`;
 * block tables, kv_lens, start_pos and the workspace as for fb_launch_tq_attention_paged
 * (fb_attention_workspace_bytes). Queries on a 16-byte boundary take the tensor-core kernel
 * (FP32 accumulation; the softmax weights as the cache's 16-bit type, BF16 ones split into a high
 * and a low part), others the CUDA-core kernel (float32); both within the 2e-3 FP bar. */
size_t fb_attention_workspace_bytes(int num_seqs, int q_per_seq, int num_q_heads, int max_kv_len);
int fb_launch_attention_paged(const void* q, int dtype, int num_seqs, int q_per_seq, int num_q_heads, int num_kv_heads,
                              int head_dim, const void* k_pool, const void* v_pool, int64_t num_pool_rows,
                              const int32_t* block_tables, int max_blocks_per_seq, const int32_t* kv_lens,
                              const int32_t* start_pos, int max_kv_len, void* workspace, size_t workspace_bytes,
                              void* output, void* stream);
/* PagedKvCacheManager::append_kv's row writes (paged_kv_cache.rs:290-315) in one launch: keys and
 * values [num_tokens, Hkv, d] of `dtype` (FP16/BF16/FP32, the pools'), token t written at pool row
 * block_table[(start_pos + t) / 16] * 16 + (start_pos + t) % 16 of k_pool / v_pool
 * ([num_pool_rows, Hkv, d]); a negative block entry or a row past the pool is skipped and counted
 * in err_count (device uint32, optional) once per token. Hkv * d * element size must be a multiple
 * of 16 bytes. */
int fb_launch_kv_append_paged(const void* keys, const void* values, int dtype, int64_t num_tokens, int num_kv_heads,
                              int head_dim, const int32_t* block_table, int64_t start_pos, int64_t num_pool_rows,
                              void* k_pool, void* v_pool, unsigned int* err_count, void* stream);

/* Number of bounded waits that timed out inside the TurboQuant kernels that stage data
 * asynchronously (tensor-core compress and dequantize; paged attention's rotate, streamed and
 * combine kernels) since the library was loaded (0 in normal operation; a timeout abandons the
 * launch's remaining work). */
unsigned int fb_tq_timeouts(void);

/* Host tables. */
/* CudaBackend::precompute_rope_freqs (backends/fracture-cuda/src/lib.rs:133-138): out[d/2] f32. */
int fb_rope_freqs(int head_dim, double theta, float* out);
/* Same, then the Llama 3.1 frequency scaling rule (no reference counterpart; the reference ignores
 * rope scaling). */
int fb_rope_freqs_llama3(int head_dim, double theta, double factor, double low_freq_factor,
                         double high_freq_factor, double original_max_position, float* out);
/* LloydMaxCodebook::compute (crates/fracture-core/src/turboquant.rs:186-250): centroids[2^bits],
 * boundaries[2^bits - 1] (either may be NULL). */
int fb_tq_codebook(int dim, int bits, float* centroids, float* boundaries);
/* generate_rotation_matrix (turboquant.rs:306-338): out[d*d] row-major f32. */
int fb_tq_rotation_matrix(int d, uint64_t seed, float* out);

/* RoPE frequencies from a GGUF model file (no reference counterpart: the reference reads only
 * `{arch}.rope.freq_base`, crates/fracture-gguf/src/parser.rs:482, and calls
 * precompute_rope_freqs(head_dim, theta) at bins/fracture-server-cuda/src/main.rs:104, so Llama
 * 3.1 runs with unscaled frequencies). fb_gguf_rope_params reads the file's rope metadata:
 * theta (`{arch}.rope.freq_base`, default 500000 as in the reference), `rope.dimension_count`,
 * `rope.scaling.{type,factor,original_context_length,low_freq_factor,high_freq_factor}`
 * (defaults 1, 8192, 1, 4) and whether a `rope_freqs.weight` F32 tensor of per-pair divisors is
 * present (what llama.cpp's converter writes for Llama 3.1). fb_rope_freqs_from_gguf builds the
 * head_dim/2 table the RoPE kernels take: base / divisors when the tensor is there, else the llama3
 * rule (fb_rope_freqs_llama3) for scaling type "llama3", base / factor for "linear", else the
 * reference's table (fb_rope_freqs). Host only; returns 0, or non-zero with the reason in
 * fb_gguf_last_error(). */
enum fb_rope_scaling { FB_ROPE_SCALING_NONE = 0, FB_ROPE_SCALING_LINEAR = 1, FB_ROPE_SCALING_LLAMA3 = 2,
                       FB_ROPE_SCALING_FACTORS = 3 };
typedef struct fb_rope_params {
    double theta, factor, original_context, low_freq_factor, high_freq_factor;
    int32_t scaling;           /* enum fb_rope_scaling */
    int32_t head_dim;          /* rope.dimension_count, 0 when absent */
    int32_t num_freq_factors;  /* entries of rope_freqs.weight, 0 when absent */
    int32_t pad0;
} fb_rope_params;
int fb_gguf_rope_params(const char* path, fb_rope_params* out);
int fb_rope_freqs_from_gguf(const char* path, int head_dim, float* out);
const char* fb_gguf_last_error(void);

/* ======================================================================== */
/* 3. Backend object (mirror of trait Backend)                              */
/* ======================================================================== */

/* Status codes, one per FractureError variant the backend can raise (crates/fracture-core/src/error.rs:7-50). */
enum fb_status {
    FB_OK = 0,
    FB_ERR_BACKEND = 1,          /* FractureError::Backend("CUDA error (N): msg" ...) */
    FB_ERR_OUT_OF_MEMORY = 2,    /* FractureError::OutOfMemory */
    FB_ERR_INVALID_SHAPE = 3,    /* FractureError::InvalidShape */
    FB_ERR_TENSOR_NOT_FOUND = 4, /* FractureError::TensorNotFound("tensor id N") */
    FB_ERR_UNSUPPORTED_DTYPE = 5,/* FractureError::UnsupportedDType */
    FB_ERR_KV_CACHE = 6,         /* FractureError::KvCache */
    FB_ERR_MODEL_CONFIG = 7      /* FractureError::ModelConfig */
};

/* DeviceTensor {id, shape, dtype} (crates/fracture-core/src/tensor.rs:14-18). Views share the id. */
typedef struct fb_tensor {
    uint64_t id;
    int32_t dtype;
    int32_t ndim;
    int64_t shape[4];
} fb_tensor;

typedef struct fb_backend fb_backend;

/* Message of the last failing fb_* call on the calling thread ("" if none). */
const char* fb_last_error(void);

/* CudaBackend::new (src/lib.rs:76-114): device, own stream. */
int fb_backend_create(int device, fb_backend** out);
int fb_backend_destroy(fb_backend* b);
int fb_backend_stream(fb_backend* b, void** stream_out);
int fb_backend_device_name(fb_backend* b, char* buf, size_t cap);
int fb_backend_total_memory(fb_backend* b, size_t* out);
int fb_backend_available_memory(fb_backend* b, size_t* out);

/* Memory (backend.rs:11-20). */
int fb_alloc(fb_backend* b, const int64_t* shape, int ndim, int dtype, fb_tensor* out);
int fb_free(fb_backend* b, const fb_tensor* t);
int fb_copy_to_device(fb_backend* b, const fb_tensor* dst, const void* src, size_t src_len);
int fb_copy_to_host(fb_backend* b, const fb_tensor* src, void* dst, size_t dst_len);
/* Register memory owned by the caller (not freed by the backend). */
int fb_register_external(fb_backend* b, void* dev_ptr, const int64_t* shape, int ndim, int dtype, fb_tensor* out);
int fb_get_ptr(fb_backend* b, const fb_tensor* t, void** out);

/* Compute (backend.rs:30-117, 166-178). */
int fb_rmsnorm(fb_backend* b, const fb_tensor* input, const fb_tensor* weight, double eps, const fb_tensor* out);
int fb_rope(fb_backend* b, const fb_tensor* q, const fb_tensor* k, const uint32_t* positions, size_t num_positions,
            double theta, size_t head_dim);
int fb_silu_mul(fb_backend* b, const fb_tensor* gate, const fb_tensor* up, const fb_tensor* out);
int fb_embedding(fb_backend* b, const uint32_t* token_ids, size_t num_tokens, const fb_tensor* table,
                 const fb_tensor* out);
/* add(a, b, out). When out aliases a and the next op is rmsnorm(a, ...), the two run as one fused
 * launch (deferred add; any other use of a or b first runs the pending add). */
int fb_add(fb_backend* b, const fb_tensor* a, const fb_tensor* bb, const fb_tensor* out);
int fb_copy_rows(fb_backend* b, const fb_tensor* src, const fb_tensor* dst, size_t src_offset, size_t dst_offset,
                 size_t count);
int fb_turboquant_compress(fb_backend* b, const fb_tensor* input, const fb_tensor* rotation,
                           const fb_tensor* centroids, uint8_t bits, const fb_tensor* packed_out,
                           const fb_tensor* norms_out);
int fb_synchronize(fb_backend* b);
/* precompute_rope_freqs (src/lib.rs:133) and its llama3 variant. */
int fb_precompute_rope_freqs(fb_backend* b, size_t head_dim, double theta);
int fb_precompute_rope_freqs_llama3(fb_backend* b, size_t head_dim, double theta, double factor,
                                    double low_freq_factor, double high_freq_factor, double original_max_position);
/* precompute_rope_freqs from a GGUF model file: the table of fb_rope_freqs_from_gguf uploaded as
 * the backend's RoPE table (the call-site change for bins/fracture-server-cuda/src/main.rs:104). */
int fb_precompute_rope_freqs_gguf(fb_backend* b, size_t head_dim, const char* gguf_path);

/* Timers (backend.rs:132-143; src/timers.rs). */
int fb_create_timer(fb_backend* b, uint64_t* timer);
int fb_start_timer(fb_backend* b, uint64_t timer);
int fb_stop_timer(fb_backend* b, uint64_t timer, float* ms);
int fb_destroy_timer(fb_backend* b, uint64_t timer);

/* Quantized paged KV cache (crates/fracture-engine/src/quantized_paged_kv_cache.rs). */
typedef struct fb_tq_config {
    uint8_t key_bits, value_bits, protected_bits, pad0;
    uint32_t protected_layers;
    uint32_t residual_tokens;
    uint64_t seed;
} fb_tq_config;

typedef struct fb_tq_cache fb_tq_cache;

int fb_tq_cache_create(fb_backend* b, size_t num_blocks, size_t num_layers, size_t num_kv_heads, size_t head_dim,
                       const fb_tq_config* cfg, fb_tq_cache** out);
int fb_tq_cache_destroy(fb_tq_cache* c);
int fb_tq_cache_alloc(fb_tq_cache* c, uint64_t* handle);
int fb_tq_cache_free(fb_tq_cache* c, uint64_t handle);
/* keys / values: [N, Hkv, d] FP16 or BF16 tensors of the backend. One launch per K and per V. */
int fb_tq_cache_append_kv(fb_tq_cache* c, uint64_t handle, size_t layer, const fb_tensor* keys,
                          const fb_tensor* values);
int fb_tq_cache_block_table(fb_tq_cache* c, uint64_t handle, int32_t* out, size_t cap, size_t* len);
int fb_tq_cache_seq_len(fb_tq_cache* c, uint64_t handle, size_t* out);
int fb_tq_cache_num_free_blocks(fb_tq_cache* c, size_t* out);
/* Device pointers of one layer's pool (kv: 0 = K, 1 = V) and of its tables, for attention kernels. */
int fb_tq_cache_pool(fb_tq_cache* c, size_t layer, int kv, void** packed, void** norms, void** rotation,
                     void** centroids, int* bits);
/* Dequantize a sequence's first `count` tokens of one layer into `out` ([count, Hkv, d]). */
int fb_tq_cache_dequant(fb_tq_cache* c, uint64_t handle, size_t layer, int kv, size_t count, const fb_tensor* out);
/* QuantizedKvCacheManager's attention (batched.rs:143-193 -> Backend::attention_paged_tq,
 * backend.rs:180-222): q [N, Hq, d] FP16/BF16 (Hq a multiple of Hkv, Hq/Hkv in {1, 2, 4, 8}, d 128),
 * tokens of the sequence at positions start_pos.., attending the sequence's first kv_len cached
 * positions of `layer` (token t: positions [0, min(start_pos + t + 1, kv_len))); out like q. The
 * workspace is the cache's, grown to the largest call. */
int fb_tq_cache_attention(fb_tq_cache* c, uint64_t handle, size_t layer, const fb_tensor* q, size_t kv_len,
                          size_t start_pos, const fb_tensor* out);

/* PagedKvCacheManager (crates/fracture-engine/src/paged_kv_cache.rs:207-370) for the uncompressed
 * cache: per-layer K and V pools [num_blocks * 16, Hkv, d] of `dtype` (FP16/BF16), blocks of 16
 * tokens from a free list. alloc takes one initial block (:231-249); append_kv takes blocks on
 * layer 0 and writes every layer's rows with one launch for K and V (:253-315); out of blocks is
 * FB_ERR_OUT_OF_MEMORY as in the reference's BlockPool. attention: q and out [N, Hq, d] of the
 * cache's dtype, tokens at positions start_pos.. attending the first kv_len cached positions
 * (Backend::attention_paged, backend.rs:66-88). */
typedef struct fb_kv_cache fb_kv_cache;
int fb_kv_cache_create(fb_backend* b, size_t num_blocks, size_t num_layers, size_t num_kv_heads, size_t head_dim,
                       int dtype, fb_kv_cache** out);
int fb_kv_cache_destroy(fb_kv_cache* c);
int fb_kv_cache_alloc(fb_kv_cache* c, uint64_t* handle);
int fb_kv_cache_free(fb_kv_cache* c, uint64_t handle);
int fb_kv_cache_append_kv(fb_kv_cache* c, uint64_t handle, size_t layer, const fb_tensor* keys,
                          const fb_tensor* values);
int fb_kv_cache_block_table(fb_kv_cache* c, uint64_t handle, int32_t* out, size_t cap, size_t* len);
int fb_kv_cache_seq_len(fb_kv_cache* c, uint64_t handle, size_t* len, size_t* last_block_tokens);
int fb_kv_cache_num_free_blocks(fb_kv_cache* c, size_t* out);
int fb_kv_cache_pool(fb_kv_cache* c, size_t layer, void** k_pool, void** v_pool);
int fb_kv_cache_attention(fb_kv_cache* c, uint64_t handle, size_t layer, const fb_tensor* q, size_t kv_len,
                          size_t start_pos, const fb_tensor* out);

#ifdef __cplusplus
}
#endif

#endif /* FRACTURE_B200_H */
