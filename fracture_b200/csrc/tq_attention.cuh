// Definitions shared by the TurboQuant paged-attention kernels (tq_attention.cu: the rotation,
// the CUDA-core and first tensor-core kernels and the combine; tq_attention_stream.cu: the
// streamed tensor-core kernel): the call's arguments, the two ways of finding a block's rows,
// and the mma.sync helpers.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "common.cuh"
#include "tq_sm100.cuh"

namespace fb {
namespace tqa {

constexpr int D = 128;
constexpr int CH = 256;       // positions per chunk: one per thread of tqa_chunk
constexpr int THREADS = 256;
constexpr int NWARPS = THREADS / 32;
constexpr int MAXG = 8;
constexpr int PART = D + 2;   // floats per chunk partial: max, sum, acc[D]

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

struct AttnArgs {
    const void* q;
    int dtype;  // of q and out: FB_FP16 or FB_BF16
    int num_seqs, q_per_seq, hq, hkv;
    const int32_t* block_tables;  // [num_seqs, max_blocks]
    int max_blocks;
    const int32_t* kv_lens;    // [num_seqs] (null: kv_len for every sequence)
    const int32_t* start_pos;  // [num_seqs] (null: start for every sequence)
    int kv_len, start;
    const float* pik;
    const float* piv;
    const float* ck;
    const float* cv;
    float* qrot;   // [rows, hq, D] f32, or f16 when qrot_f16 is set
    int qrot_f16;  // the rotate kernel writes q_rot as fp16 (the streamed kernel's input)
    float* part;   // [rows, hq, nch, PART]
    int nch;       // partial slots per (row, head): the layout's stride (CH-position chunks until a kernel sets its own)
    int slots;     // partial slots per (row, head) the workspace holds (>= nch; the streamed kernel may use more chunks)
    int spc;       // partial slots per chunk (the streamed kernel writes one per block slot)
    int ch;        // positions per chunk
    int rnd;  // tensor-core kernel: rounds of four 16-position tiles per warp and item
    sm100::DivU32 dnch, dhkv, dqps;  // nch, hkv, q_per_seq as multiply-high divisors (tensor-core kernel)
    void* out;
};

// K/V rows in this library's contiguous pools: pool row = block * 16 + offset, head g at
// g * P within it.
struct PoolAddr {
    const uint8_t* kp;
    const __half* kn;
    const uint8_t* vp;
    const __half* vn;
    int64_t pool_rows;
    __device__ bool locate(int32_t blk, int off, int g, int hkv, int pk, int pv, const uint8_t*& krow,
                           const uint8_t*& vrow, float& knorm, float& vnorm) const {
        const int64_t row = (int64_t)blk * 16 + off;
        if (row >= pool_rows) return false;
        const int64_t hr = row * hkv + g;
        krow = kp + hr * pk;
        vrow = vp + hr * pv;
        knorm = __half2float(kn[hr]);
        vnorm = __half2float(vn[hr]);
        return true;
    }
    // Rows of block blk that lie inside the pool (16 unless the pool ends inside the block).
    __device__ int block_rows(int32_t blk) const {
        return (int)max((int64_t)0, min((int64_t)16, pool_rows - (int64_t)blk * 16));
    }
    // KV head g of row `off` of block blk: K codes at kb + off * hkv * pk, its norm at
    // knb[off * hkv]; the same for V.
    __device__ void block_base(int32_t blk, int g, int hkv, int pk, int pv, const uint8_t*& kb, const uint8_t*& vb,
                               const __half*& knb, const __half*& vnb) const {
        const int64_t hr = (int64_t)blk * 16 * hkv + g;
        kb = kp + hr * pk;
        vb = vp + hr * pv;
        knb = kn + hr;
        vnb = vn + hr;
    }
};

// The reference's per-block tensors (attention_paged_tq.cu:123-129): block b's packed K rows
// at kp[b] ([16, hkv * P]), its norms at kn[b] ([16, hkv]); the same for V.
struct BlockPtrAddr {
    const uint8_t* const* kp;
    const __half* const* kn;
    const uint8_t* const* vp;
    const __half* const* vn;
    __device__ bool locate(int32_t blk, int off, int g, int hkv, int pk, int pv, const uint8_t*& krow,
                           const uint8_t*& vrow, float& knorm, float& vnorm) const {
        const int hr = off * hkv + g;
        krow = kp[blk] + hr * pk;
        vrow = vp[blk] + hr * pv;
        knorm = __half2float(kn[blk][hr]);
        vnorm = __half2float(vn[blk][hr]);
        return true;
    }
    __device__ int block_rows(int32_t) const { return 16; }
    __device__ void block_base(int32_t blk, int g, int hkv, int pk, int pv, const uint8_t*& kb, const uint8_t*& vb,
                               const __half*& knb, const __half*& vnb) const {
        kb = kp[blk] + g * pk;
        vb = vp[blk] + g * pv;
        knb = kn[blk] + g;
        vnb = vn[blk] + g;
    }
};

__device__ __forceinline__ int causal_len(const AttnArgs& a, int s, int t) {
    const int kv = a.kv_lens ? a.kv_lens[s] : a.kv_len;
    const int st = a.start_pos ? a.start_pos[s] : a.start;
    return max(0, min(st + t + 1, kv));
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ uint32_t pack_half2(float x, float y) {
    const __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Table address of the code byte b of word w: (byte << 8) | off, off = lane offset (< 256).
__device__ __forceinline__ uint32_t taddr(uint32_t w, uint32_t off, int b) {
    return __byte_perm(w, off, 0x5504u | ((uint32_t)b << 4));
}

}  // namespace tqa
}  // namespace fb
