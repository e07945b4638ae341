// Attention of query tokens over the TurboQuant-compressed paged KV cache, sm_100a.
//
// Replaces backends/fracture-cuda/kernels/attention_paged_tq.cu:56-309 (one CTA per query
// token and Q head, the whole causal range in one CTA, every Q head of a GQA group re-reading
// its KV head's codes). The math is the reference's (attention_paged_tq.cu:12-17): scores in
// K's rotated space, (Pi_k q) . c_k[idx] * k_norm / sqrt(d); softmax over the causal range;
// values accumulated in V's rotated space, sum p * c_v[idx] * v_norm, and rotated back once,
// Pi_v^T acc. Here, with the centroid values read as fp16 (2^-11 relative) and everything else
// in float32:
//
//   tqa_rotate_q    q_rot = Pi_k q for every query token and Q head (a CTA per up to four
//                   query tokens and KV group, Pi_k staged by TMA), into the workspace
//   tqa_chunk       one CTA per (256-position chunk, KV head, query token): thread p scores
//                   position p for all Q heads of the group from the position's packed K
//                   row (pair-of-codes lookup tables, lane-private), the CTA takes the
//                   chunk's softmax maximum and sum, and then warp w accumulates its 32
//                   positions' values (lane l: coordinates 4l..4l+3, every head of the
//                   group) from the V rows staged in shared memory; the chunk's (max, sum,
//                   acc) go to the workspace (split-K over the causal range)
//   tqa_combine     rescales and sums the chunks of each query token and head, divides by
//                   the softmax sum and rotates back with Pi_v^T (a CTA per up to four query
//                   tokens and KV group, Pi_v staged by one bulk copy; thread (h, i): output i
//                   of head h)
//
// With 2- or 4-bit keys and values, tqa_mma (tensor cores, below) replaces tqa_chunk: same
// split-K partials, chunks of 512 to 2048 positions. 3- and 8-bit codes take tqa_chunk.
//
// Each KV head's codes are read once per query token for its whole group of Q heads. A
// position whose block-table entry is negative, or whose pool row is out of range, is left
// out; a query token with no position gives zeros.

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tq_sm100.cuh"
#include "tq_common.cuh"
#include "tq_attention.cuh"

namespace fb {

// Bounded waits of the rotate and combine kernels' staging copies that ran out (fb_tq_timeouts).
__device__ unsigned int g_tqa_timeouts = 0;

// tq_api.cu: counts a served call of path `which` when rc is 0 (fb_tq_path_counts); returns rc.
int tq_count_path(int which, int rc);

namespace tqa {

__device__ __forceinline__ float load_q(const AttnArgs& a, int64_t i) {
    return a.dtype == FB_BF16 ? __bfloat162float(((const __nv_bfloat16*)a.q)[i]) : __half2float(((const __half*)a.q)[i]);
}

constexpr int RQ = 4;  // query rows per rotate / combine CTA

// Bounded wait for a one-shot staging barrier (phase 0); a wait that runs out is counted.
__device__ __forceinline__ bool stage_wait(uint64_t* bar) {
    const long long t0 = clock64();
    while (!sm100::mbar_try_wait(bar, 0))
        if (clock64() - t0 > 4000000000LL) {
            atomicAdd(&g_tqa_timeouts, 1u);
            return false;
        }
    return true;
}

// 2^x (ex2.approx, 2 ulp; 2^-inf = 0)
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct RotateParams {
    CUtensorMap pimap;  // Pi_k: f32 [128][128], box 32 columns x 128 rows, 128-byte swizzle
    AttnArgs a;
    int rows;
};

// Query rows per rotate / combine CTA: RQ when that still gives a CTA to every SM, else fewer.
inline int rows_per_cta(int rows, int hkv) {
    int rq = RQ;
    while (rq > 1 && (int64_t)((rows + rq - 1) / rq) * hkv < num_sms()) rq /= 2;
    return rq;
}

// q_rot[row][h][i] = sum_j Pi_k[i][j] q[row][h][j] for NR query rows and the G heads of KV group
// blockIdx.y. Pi_k arrives by four TMA boxes of 32 columns with the 128-byte swizzle, so thread i
// reads its row 16 bytes at a time without bank conflicts while every thread reads the same query
// words (broadcast); thread i computes coordinate i of all NR * G vectors.
template <int G, int NR>
__global__ void __launch_bounds__(D) tqa_rotate_q(const __grid_constant__ RotateParams R) {
    pdl_trigger();  // the attention kernel's CTAs may start their table set-up meanwhile
    extern __shared__ uint8_t rsm_raw[];
    uint8_t* rsm = rsm_raw + ((1024u - (smem_addr(rsm_raw) & 1023u)) & 1023u);
    float* pis = (float*)rsm;               // 4 x [128 rows][32 columns], swizzled
    float* qs = (float*)(rsm + D * D * 4);  // [NR * G][D]
    uint64_t* bar = (uint64_t*)(qs + NR * G * D);
    const AttnArgs& a = R.a;
    const int r0 = blockIdx.x * NR, g = blockIdx.y, i = threadIdx.x;
    const int nr = min(NR, R.rows - r0);
    if (i == 0) {
        sm100::mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_begin();
    if (i == 0) {
        sm100::mbar_expect_tx(bar, D * D * 4);
        for (int c = 0; c < 4; ++c) sm100::tma_load_2d(pis + c * 32 * D, &R.pimap, bar, 32 * c, 0);
    }
    {
        float qv[NR * G];  // every query load in flight before the first store
#pragma unroll
        for (int k = 0; k < NR * G; ++k) {
            const int e = i + k * D, rr = e / (G * D);
            qv[k] = rr < nr ? load_q(a, ((int64_t)(r0 + rr) * a.hq + g * G) * D + (e - rr * G * D)) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < NR * G; ++k) qs[i + k * D] = qv[k];
    }
    __syncthreads();
    if (!stage_wait(bar)) return;
    float acc[NR * G];
#pragma unroll
    for (int v = 0; v < NR * G; ++v) acc[v] = 0.0f;
#pragma unroll 2
    for (int m = 0; m < D / 4; ++m) {  // columns 4m .. 4m + 3
        const float4 p = *(const float4*)(pis + (m >> 3) * 32 * D + i * 32 + (((m & 7) ^ (i & 7)) << 2));
#pragma unroll
        for (int v = 0; v < NR * G; ++v) {
            const float4 x = *(const float4*)(qs + v * D + 4 * m);
            acc[v] = fmaf(p.x, x.x, acc[v]);
            acc[v] = fmaf(p.y, x.y, acc[v]);
            acc[v] = fmaf(p.z, x.z, acc[v]);
            acc[v] = fmaf(p.w, x.w, acc[v]);
        }
    }
#pragma unroll
    for (int v = 0; v < NR * G; ++v) {
        const int rr = v / G;
        if (rr < nr) {
            const int64_t o = ((int64_t)(r0 + rr) * a.hq + g * G + (v - rr * G)) * D + i;
            if (a.qrot_f16) ((__half*)a.qrot)[o] = __float2half_rn(acc[v]);
            else a.qrot[o] = acc[v];
        }
    }
}

// For calls with few rows: CTA (row, group g, slice z) computes coordinates 32z .. 32z + 31 of the
// G heads of KV group g, so that the launch spreads over four times as many SMs and each CTA
// reads a quarter of Pi_k. Thread (h, i) = (tid / 32, tid % 32) computes coordinate 32z + i of
// head h; its Pi_k row sits in shared memory at a stride of D + 4 floats (the 16-byte reads of
// a quarter-warp fall in different banks), the head's query is read by the whole warp at once.
__global__ void __launch_bounds__(8 * 32) tqa_rotate_q_slice(AttnArgs a) {
    pdl_trigger();  // the attention kernel's CTAs may start their table set-up meanwhile
    __shared__ __align__(16) float pis[32][D + 4];
    __shared__ __align__(16) float qs[MAXG][D];
    const int row = blockIdx.x, g = blockIdx.y, z = blockIdx.z;
    const int G = a.hq / a.hkv, tid = threadIdx.x, h = tid >> 5, i = tid & 31;
    pdl_begin();
    // the slice of Pi_k: 32 rows of 512 bytes, 16 bytes per thread and step
    for (int e = tid; e < 32 * D / 4; e += blockDim.x) {
        const int r = e / (D / 4), c = e - r * (D / 4);
        const uint32_t dst = smem_addr(&pis[r][4 * c]);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(a.pik + (int64_t)(32 * z + r) * D + 4 * c)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    for (int e = tid; e < G * D; e += blockDim.x)
        qs[e / D][e % D] = load_q(a, ((int64_t)row * a.hq + g * G) * D + e);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    float acc = 0.0f;
#pragma unroll 8
    for (int m = 0; m < D / 4; ++m) {
        const float4 p = *(const float4*)&pis[i][4 * m];
        const float4 x = *(const float4*)&qs[h][4 * m];
        acc = fmaf(p.x, x.x, acc);
        acc = fmaf(p.y, x.y, acc);
        acc = fmaf(p.z, x.z, acc);
        acc = fmaf(p.w, x.w, acc);
    }
    const int64_t o = ((int64_t)row * a.hq + g * G + h) * D + 32 * z + i;
    if (a.qrot_f16) ((__half*)a.qrot)[o] = __float2half_rn(acc);
    else a.qrot[o] = acc;
}

// One launch of tqa_rotate_q for the call's rows (Pi_k 16-byte aligned, as every entry point checks).
inline int launch_rotate(const AttnArgs& a, int rows, cudaStream_t s) {
    if ((int64_t)rows * a.hkv * 4 <= 2LL * num_sms()) {  // few rows: four slices per (row, group)
        launch_pdl_smem(tqa_rotate_q_slice, dim3(rows, a.hkv, 4), dim3(32 * (a.hq / a.hkv)), 0, s, a);
        return (int)cudaGetLastError();
    }
    auto encode = sm100::tensor_map_encoder();
    if (!encode) return (int)cudaErrorNotSupported;
    RotateParams R;
    memset(&R, 0, sizeof R);
    const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)D};
    const cuuint64_t strides[1] = {(cuuint64_t)D * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)D};
    const cuuint32_t estr[2] = {1, 1};
    if (encode(&R.pimap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.pik), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return (int)cudaErrorInvalidValue;
    R.a = a;
    R.rows = rows;
    const int G = a.hq / a.hkv, rq = rows_per_cta(rows, a.hkv);
    const size_t smem = 1024 + (size_t)D * D * 4 + (size_t)rq * G * D * 4 + 16;
    using Kern = void (*)(RotateParams);
    static const Kern kerns[4][3] = {{tqa_rotate_q<1, 1>, tqa_rotate_q<1, 2>, tqa_rotate_q<1, 4>},
                                     {tqa_rotate_q<2, 1>, tqa_rotate_q<2, 2>, tqa_rotate_q<2, 4>},
                                     {tqa_rotate_q<4, 1>, tqa_rotate_q<4, 2>, tqa_rotate_q<4, 4>},
                                     {tqa_rotate_q<8, 1>, tqa_rotate_q<8, 2>, tqa_rotate_q<8, 4>}};
    const Kern kern = kerns[G == 1 ? 0 : G == 2 ? 1 : G == 4 ? 2 : 3][rq == 1 ? 0 : rq == 2 ? 1 : 2];
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    launch_pdl_smem(kern, dim3((rows + rq - 1) / rq, a.hkv), dim3(D), smem, s, R);
    return (int)cudaGetLastError();
}

// Decoding tables, 32 lane-private copies side by side (a warp's lookups hit 32 banks). Pair
// tables (2-, 3- and 4-bit codes): the 2*BITS bits of two adjacent codes -> half2 (first code,
// second code; the centroids rounded to fp16, 2^-11 relative, one shared-memory wavefront per
// lookup). 8-bit codes: code -> float.
template <int BITS>
struct Lut {
    static constexpr bool pair = BITS <= 4;
    static constexpr int entries = pair ? (1 << (2 * BITS)) : 256;
    static constexpr int copies = 32;
    static constexpr int entry_bytes = 4;
    static constexpr int bytes = entries * copies * entry_bytes;
};

// One thread per entry writes its 128 bytes of copies as eight 16-byte stores, starting at a
// thread-dependent chunk so a quarter-warp's stores fall in eight different bank groups.
template <int BITS>
__device__ __forceinline__ void build_lut(uint8_t* lut, const float* cen) {
    using L = Lut<BITS>;
    static_assert(L::copies * L::entry_bytes == 128, "one 128-byte row of copies per entry");
    for (int ent = threadIdx.x; ent < L::entries; ent += blockDim.x) {
        float4 v;
        if constexpr (L::pair) {
            const __half2 h = __floats2half2_rn(__ldg(cen + (ent >> BITS)), __ldg(cen + (ent & ((1 << BITS) - 1))));
            const float f = *reinterpret_cast<const float*>(&h);
            v = make_float4(f, f, f, f);
        } else {
            const float a = __ldg(cen + ent);
            v = make_float4(a, a, a, a);
        }
        float4* row = (float4*)(lut + ent * 128);
#pragma unroll
        for (int k = 0; k < 8; ++k) row[(k + threadIdx.x) & 7] = v;
    }
}

template <int BITS>
__device__ __forceinline__ float2 lut_pair(uint32_t lane_base, uint32_t idx) {
    uint32_t w;
    asm("ld.shared.b32 %0, [%1];" : "=r"(w) : "r"(lane_base + idx * 128u));
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
__device__ __forceinline__ float lut_one(uint32_t lane_base, uint32_t idx) {
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(lane_base + idx * (32u * 4u)));
    return v;
}

// Code pair m (coordinates 2m, 2m+1) of a row held as 32-bit little-endian words of its
// MSB-first bit stream, as a table index (2-, 3-, 4-bit codes).
template <int BITS>
__device__ __forceinline__ uint32_t pair_index(const uint32_t* w, int m) {
    if constexpr (BITS == 4) {
        return (w[m >> 2] >> (8 * (m & 3))) & 0xffu;  // byte m
    } else if constexpr (BITS == 2) {
        const uint32_t byte = (w[m >> 3] >> (8 * ((m >> 1) & 3))) & 0xffu;  // byte m/2, high nibble first
        return (m & 1) ? (byte & 15u) : (byte >> 4);
    } else {
        // 3-bit: 8 codes per 3 bytes; pair m is bits 18 - 6 (m & 3) of the big-endian 24-bit
        // value of bytes 3c, 3c+1, 3c+2, c = m / 4
        const int c = m >> 2, b0 = 3 * c;
        const uint32_t x0 = (w[b0 >> 2] >> (8 * (b0 & 3))) & 0xffu;
        const uint32_t x1 = (w[(b0 + 1) >> 2] >> (8 * ((b0 + 1) & 3))) & 0xffu;
        const uint32_t x2 = (w[(b0 + 2) >> 2] >> (8 * ((b0 + 2) & 3))) & 0xffu;
        const uint32_t v24 = (x0 << 16) | (x1 << 8) | x2;
        return (v24 >> (18 - 6 * (m & 3))) & 63u;
    }
}

template <int KB, int VB, int G>
struct ChunkSmem {
    static constexpr int PV = D * VB / 8;
    static constexpr int qr_off = 0;                                   // [G][D] f32
    static constexpr int lutk_off = qr_off + G * D * 4;  // K table, then the warps' sums [NWARPS][G][D]
    static constexpr int lutk_bytes = Lut<KB>::bytes > NWARPS * G * D * 4 ? Lut<KB>::bytes : NWARPS * G * D * 4;
    static constexpr int lutv_off = lutk_off + lutk_bytes;
    static constexpr int vs_bytes = CH * PV;
    static constexpr int vs_off = lutv_off + Lut<VB>::bytes;           // V rows of the chunk
    static constexpr int w_off = vs_off + vs_bytes;                    // [CH][G] f32 weights
    static constexpr int red_off = w_off + G * CH * 4;                 // [NWARPS][G] f32
    static constexpr int bytes = red_off + NWARPS * G * 4 + 16;
};

template <int KB, int VB, int G, typename Addr>
__global__ void __launch_bounds__(THREADS) tqa_chunk(AttnArgs a, Addr ad) {
    using S = ChunkSmem<KB, VB, G>;
    constexpr int PK = D * KB / 8, PV = D * VB / 8;
    extern __shared__ __align__(16) uint8_t sm[];
    float* qr = (float*)(sm + S::qr_off);
    uint8_t* lutk = sm + S::lutk_off;
    uint8_t* lutv = sm + S::lutv_off;
    uint8_t* vs = sm + S::vs_off;
    float* ws = (float*)(sm + S::w_off);
    static_assert(G % 4 == 0, "weights are read four heads at a time");
    float* red = (float*)(sm + S::red_off);

    const int row = blockIdx.z, g = blockIdx.y, c = blockIdx.x;
    const int s = row / a.q_per_seq, t = row - s * a.q_per_seq;
    const int L = causal_len(a, s, t);
    const int p0 = c * CH;
    if (p0 >= L) return;  // the whole CTA: chunk past the causal range
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int GA = a.hq / a.hkv;  // heads of the group (<= G; the others are computed on zeros)
    build_lut<KB>(lutk, a.ck);
    build_lut<VB>(lutv, a.cv);
    for (int e = tid; e < G * D; e += THREADS) qr[e] = e < GA * D ? a.qrot[((int64_t)row * a.hq + g * GA) * D + e] : 0.0f;
    __syncthreads();

    // ── scores: thread tid takes position p0 + tid ──
    const int p = p0 + tid;
    bool valid = p < L && (p >> 4) < a.max_blocks;
    const uint8_t* krow = nullptr;
    const uint8_t* vrow = nullptr;
    float knorm = 0.0f, vnorm = 0.0f;
    if (valid) {
        const int32_t blk = a.block_tables[(int64_t)s * a.max_blocks + (p >> 4)];
        valid = blk >= 0 && ad.locate(blk, p & 15, g, a.hkv, PK, PV, krow, vrow, knorm, vnorm);
    }
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = 0.0f;
    if (valid) {
        uint32_t kw[PK / 4];
#pragma unroll
        for (int k = 0; k < PK / 16; ++k) {
            const uint4 u = __ldg((const uint4*)krow + k);
            kw[4 * k] = u.x;
            kw[4 * k + 1] = u.y;
            kw[4 * k + 2] = u.z;
            kw[4 * k + 3] = u.w;
        }
#pragma unroll
        for (int k = 0; k < PV / 16; ++k) ((uint4*)(vs + tid * PV))[k] = __ldg((const uint4*)vrow + k);
        if constexpr (Lut<KB>::pair) {
            // two running sums per head (even and odd coordinates) in one packed register pair:
            // one two-wide FMA per code pair and head; q_rot four coordinates per load
            const uint32_t lb = smem_addr(lutk) + lane * 4u;
            float2 s2[G];
#pragma unroll
            for (int h = 0; h < G; ++h) s2[h] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int m = 0; m < D / 2; m += 2) {  // unrolled: the code words stay in registers
                const float2 c0 = lut_pair<KB>(lb, pair_index<KB>(kw, m));
                const float2 c1 = lut_pair<KB>(lb, pair_index<KB>(kw, m + 1));
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float4 qq = *(const float4*)&qr[h * D + 2 * m];
                    s2[h] = __ffma2_rn(make_float2(qq.x, qq.y), c0, s2[h]);
                    s2[h] = __ffma2_rn(make_float2(qq.z, qq.w), c1, s2[h]);
                }
            }
#pragma unroll
            for (int h = 0; h < G; ++h) sc[h] = s2[h].x + s2[h].y;
        } else {
            const uint32_t lb = smem_addr(lutk) + lane * 4u;
            float2 s2[G];
#pragma unroll
            for (int h = 0; h < G; ++h) s2[h] = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < D; j += 2) {
                const float2 cc = make_float2(lut_one(lb, (kw[j >> 2] >> (8 * (j & 3))) & 0xffu),
                                              lut_one(lb, (kw[j >> 2] >> (8 * ((j + 1) & 3))) & 0xffu));
#pragma unroll
                for (int h = 0; h < G; ++h) s2[h] = __ffma2_rn(*(const float2*)&qr[h * D + j], cc, s2[h]);
            }
#pragma unroll
            for (int h = 0; h < G; ++h) sc[h] = s2[h].x + s2[h].y;
        }
        const float f = knorm * rsqrtf((float)D);
#pragma unroll
        for (int h = 0; h < G; ++h) sc[h] *= f;
    }

    // ── softmax over the chunk: maximum, then weights exp(s - max) * v_norm and their sum ──
    float mx[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        float v = valid ? sc[h] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[warp * G + h] = v;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; ++h) {
        float v = red[h];
        for (int w = 1; w < NWARPS; ++w) v = fmaxf(v, red[w * G + h]);
        mx[h] = v;  // finite: the chunk holds at least position p0 < L, unless every block is missing
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const float e = valid ? expf(sc[h] - mx[h]) : 0.0f;
        ws[tid * G + h] = e * vnorm;
        float v = e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp * G + h] = v;
    }
    __syncthreads();

    // ── values: warp w takes its 32 positions, lane l coordinates 4l..4l+3 of every head ──
    float2 acc[G][2];  // coordinates (4l, 4l+1) and (4l+2, 4l+3) of each head
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h][0] = acc[h][1] = make_float2(0.0f, 0.0f);
    {
        const uint32_t lb = smem_addr(lutv) + lane * 4u;
        const int jn = min(32, L - (p0 + warp * 32));
        for (int j = 0; j < jn; ++j) {
            const int pl = warp * 32 + j;
            const uint8_t* r = vs + pl * PV;
            float2 a0, a1;  // values of coordinates (4l, 4l+1) and (4l+2, 4l+3)
            if constexpr (VB == 4) {
                const uint32_t b2 = *(const uint16_t*)(r + 2 * lane);  // bytes 2l, 2l+1
                a0 = lut_pair<4>(lb, b2 & 0xffu);
                a1 = lut_pair<4>(lb, b2 >> 8);
            } else if constexpr (VB == 2) {
                const uint32_t byte = r[lane];
                a0 = lut_pair<2>(lb, byte >> 4);
                a1 = lut_pair<2>(lb, byte & 15u);
            } else if constexpr (VB == 3) {
                const int bit = 12 * lane, b = bit >> 3;
                const uint32_t v16 = ((uint32_t)r[b] << 8) | r[b + 1];
                const uint32_t v12 = (bit & 7) ? (v16 & 0xfffu) : (v16 >> 4);
                a0 = lut_pair<3>(lb, v12 >> 6);
                a1 = lut_pair<3>(lb, v12 & 63u);
            } else {
                const uint32_t w4 = *(const uint32_t*)(r + 4 * lane);
                a0 = make_float2(lut_one(lb, w4 & 0xffu), lut_one(lb, (w4 >> 8) & 0xffu));
                a1 = make_float2(lut_one(lb, (w4 >> 16) & 0xffu), lut_one(lb, w4 >> 24));
            }
            const float* wp = ws + pl * G;  // this position's weights, G consecutive floats
#pragma unroll
            for (int h4 = 0; h4 < G; h4 += 4) {
                const float4 w4 = *(const float4*)(wp + h4);
                const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 w2 = make_float2(wv[k], wv[k]);
                    acc[h4 + k][0] = __ffma2_rn(w2, a0, acc[h4 + k][0]);
                    acc[h4 + k][1] = __ffma2_rn(w2, a1, acc[h4 + k][1]);
                }
            }
        }
    }
    // the warps' sums, added in warp order (the K table is no longer read: several barriers
    // separate its last use from here)
    float* accs = (float*)lutk;
#pragma unroll
    for (int h = 0; h < G; ++h)
        *(float4*)&accs[(warp * G + h) * D + 4 * lane] = make_float4(acc[h][0].x, acc[h][0].y, acc[h][1].x, acc[h][1].y);
    __syncthreads();
    float* part = a.part + (((int64_t)row * a.hq + g * GA) * a.nch + c) * PART;
    for (int e = tid; e < GA * D; e += THREADS) {
        const int h = e / D, i = e - h * D;
        float v = 0.0f;
        for (int w = 0; w < NWARPS; ++w) v += accs[(w * G + h) * D + i];
        part[(int64_t)h * a.nch * PART + 2 + i] = v;
    }
    if (tid < GA) {
        float l = 0.0f;
        for (int w = 0; w < NWARPS; ++w) l += red[w * G + tid];
        float* ph = part + (int64_t)tid * a.nch * PART;
        ph[0] = mx[tid];
        ph[1] = l;
    }
}

// out[row][h][i] = sum_j Pi_v[j][i] * (sum_c acc_c[j] e^(m_c - M)) / (sum_c l_c e^(m_c - M)) for NR
// query rows of KV group blockIdx.y: the chunks' partials are summed while one bulk copy brings
// Pi_v into shared memory; the rotation back reads column i of Pi_v (consecutive words across
// threads) once for the CTA's rows.
template <int NR>
__global__ void __launch_bounds__(4 * D) tqa_combine(AttnArgs a, int rows) {
    extern __shared__ __align__(16) float csm[];
    float* pvs = csm;           // [D][D]
    float* accs = csm + D * D;  // [NR][G][D]
    const int G = a.hq / a.hkv, GT = min(G, 4);  // heads per KV group; head lanes of the CTA
    uint64_t* bar = (uint64_t*)(accs + RQ * G * D);
    const int r0 = blockIdx.x * NR, g = blockIdx.y, tid = threadIdx.x;
    const int hh = tid / D, i = tid - hh * D;
    const int nr = min(NR, rows - r0);
    const bool bulk = ((uintptr_t)a.piv & 15) == 0;
    if (tid == 0) {
        sm100::mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Pi_v is read before the wait for the chunk kernel: run() launches this kernel right after
    // one of this file's chunk kernels (tqa_stream, tqa_mma, tqa_chunk), none of which writes the
    // rotation, so the copy overlaps that kernel's tail. A chain that puts another kernel in
    // between must move the copy after pdl_begin().
    if (bulk && tid == 0) {
        sm100::mbar_expect_tx(bar, D * D * 4);
        sm100::bulk_load(pvs, a.piv, D * D * 4, bar);
    }
    pdl_begin();
    if (!bulk)
        for (int e = tid; e < D * D; e += GT * D) pvs[e] = __ldg(a.piv + e);
    // weights e^(m_c - M) as exp2 of log2(e)-scaled differences (ex2.approx, 2 ulp); a chunk
    // with no position has m = -inf and weight 0
    auto weight = [](float m, float Ml) {
        float f;
        asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(f) : "f"(fmaf(m, 1.4426950408889634f, -Ml)));
        return f;
    };
    // Thread (hh, i) sums output i of heads hh, hh + 4 of each row. With at most CMAX chunks, a
    // row's maxima, sums and accumulator values are requested at once (one round trip to L2);
    // else two passes (the maxima, then the weighted sums), eight chunks' loads at a time.
    constexpr int CMAX = 16;
    for (int rr = 0; rr < nr; ++rr) {
        const int row = r0 + rr;
        const int s = row / a.q_per_seq, t = row - s * a.q_per_seq;
        const int L = causal_len(a, s, t);
        const int nc = min((L + a.ch - 1) / a.ch * a.spc, a.nch);  // kv_lens past max_kv_len: the chunks computed
        for (int h = hh; h < G; h += 4) {
            const float* ph = a.part + ((int64_t)row * a.hq + g * G + h) * a.nch * PART;
            float l = 0.0f, v = 0.0f;
            if (nc <= CMAX) {
                float mm[CMAX], ll[CMAX], vv[CMAX];
#pragma unroll
                for (int c = 0; c < CMAX; ++c) {
                    const bool in = c < nc;
                    mm[c] = in ? ph[c * PART] : -INFINITY;
                    ll[c] = in ? ph[c * PART + 1] : 0.0f;
                    vv[c] = in ? ph[c * PART + 2 + i] : 0.0f;
                }
                float M = -INFINITY;
#pragma unroll
                for (int c = 0; c < CMAX; ++c) M = fmaxf(M, mm[c]);
                if (M > -INFINITY) {
                    const float Ml = M * 1.4426950408889634f;
#pragma unroll
                    for (int c = 0; c < CMAX; ++c) {
                        const float f = weight(mm[c], Ml);
                        l = fmaf(ll[c], f, l);
                        v = fmaf(vv[c], f, v);
                    }
                }
            } else {
                float M = -INFINITY;
                for (int c0 = 0; c0 < nc; c0 += 8) {
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (c0 + k < nc) M = fmaxf(M, ph[(c0 + k) * PART]);
                }
                if (M > -INFINITY) {
                    const float Ml = M * 1.4426950408889634f;
                    for (int c0 = 0; c0 < nc; c0 += 8) {
                        float m8[8], l8[8], v8[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const int c = c0 + k;
                            m8[k] = c < nc ? ph[c * PART] : -INFINITY;
                            l8[k] = c < nc ? ph[c * PART + 1] : 0.0f;
                            v8[k] = c < nc ? ph[c * PART + 2 + i] : 0.0f;
                        }
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const float f = weight(m8[k], Ml);
                            l = fmaf(l8[k], f, l);
                            v = fmaf(v8[k], f, v);
                        }
                    }
                }
            }
            accs[(rr * G + h) * D + i] = l > 0.0f ? v / l : 0.0f;
        }
    }
    __syncthreads();
    if (bulk && !stage_wait(bar)) return;
    for (int h = hh; h < G; h += 4) {
        float o[NR];
#pragma unroll
        for (int rr = 0; rr < NR; ++rr) o[rr] = 0.0f;
#pragma unroll 4
        for (int j = 0; j < D; ++j) {
            const float p = pvs[j * D + i];
#pragma unroll
            for (int rr = 0; rr < NR; ++rr) o[rr] = fmaf(p, accs[(rr * G + h) * D + j], o[rr]);
        }
#pragma unroll
        for (int rr = 0; rr < NR; ++rr) {
            if (rr >= nr) break;
            const int64_t e = ((int64_t)(r0 + rr) * a.hq + g * G + h) * D + i;
            if (a.dtype == FB_BF16) ((__nv_bfloat16*)a.out)[e] = __float2bfloat16_rn(o[rr]);
            else ((__half*)a.out)[e] = __float2half_rn(o[rr]);
        }
    }
}

// The combine for calls with few rows: one CTA per (query row, HPC Q heads), so that a call of
// one or a few rows still spreads over many SMs, and the partials of a head split over the CL
// (4 or 8) 128-thread chunk lanes (lane k takes chunks k, k + CL, ...), each keeping a running maximum, sum
// and accumulator (eight or sixteen chunks' loads in flight at a time), merged through shared memory. Then
// as tqa_combine: divide by the sum, rotate back by Pi_v (the CL lanes each take 128 / CL of the 128
// terms), convert.
template <int CL>
__global__ void __launch_bounds__(CL * D) tqa_combine_deep(AttnArgs a, int hpc) {
    extern __shared__ __align__(16) float csm[];
    float* pvs = csm;                  // [D][D]
    float* mv = csm + D * D;           // [CL][D] lane accumulators, then [CL][D] rotation partials
    float* ms = mv + CL * D;           // [CL] lane maxima (log2 units)
    float* ls = ms + CL;               // [CL] lane sums
    float* acc = ls + CL;              // [D] the head's normalised accumulator
    uint64_t* bar = (uint64_t*)(acc + D);
    const int row = blockIdx.x, tid = threadIdx.x;
    const int cl = tid / D, i = tid - cl * D;
    const bool bulk = ((uintptr_t)a.piv & 15) == 0;
    if (tid == 0) {
        sm100::mbar_init(bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Pi_v before the wait, as in tqa_combine (same launch order, same invariant)
    if (bulk && tid == 0) {
        sm100::mbar_expect_tx(bar, D * D * 4);
        sm100::bulk_load(pvs, a.piv, D * D * 4, bar);
    }
    pdl_begin();
    if (!bulk)
        for (int e = tid; e < D * D; e += CL * D) pvs[e] = __ldg(a.piv + e);
    const int s = row / a.q_per_seq, t = row - s * a.q_per_seq;
    const int L = causal_len(a, s, t);
    const int nc = min((L + a.ch - 1) / a.ch * a.spc, a.nch);
    bool have_pv = !bulk;
    // a lane's chunks, DB at a time with their loads in flight together: 16 when a lane has more
    // than 8 (fewer round trips), else 8 (no loads masked off)
    auto merge = [&](auto dbc, const float* ph, float& m, float& l, float& v) {
        constexpr int DB = decltype(dbc)::value;
        for (int k0 = 0; cl + CL * k0 < nc; k0 += DB) {
            float m8[DB], l8[DB], v8[DB];
#pragma unroll
            for (int k = 0; k < DB; ++k) {
                const int c = cl + CL * (k0 + k);
                const bool in = c < nc;
                m8[k] = in ? ph[c * PART] * 1.4426950408889634f : -INFINITY;
                l8[k] = in ? ph[c * PART + 1] : 0.0f;
                v8[k] = in ? ph[c * PART + 2 + i] : 0.0f;
            }
            float bm = m8[0];
#pragma unroll
            for (int k = 1; k < DB; ++k) bm = fmaxf(bm, m8[k]);
            if (bm > m) {  // m = -inf before: l and v are 0 and stay 0
                const float f = ex2f(m - bm);
                l *= f;
                v *= f;
                m = bm;
            }
            if (m > -INFINITY) {
#pragma unroll
                for (int k = 0; k < DB; ++k) {
                    const float f = ex2f(m8[k] - m);
                    l = fmaf(l8[k], f, l);
                    v = fmaf(v8[k], f, v);
                }
            }
        }
    };
    for (int hk = 0; hk < hpc; ++hk) {
        const int h = blockIdx.y * hpc + hk;
        const float* ph = a.part + ((int64_t)row * a.hq + h) * a.nch * PART;
        float m = -INFINITY, l = 0.0f, v = 0.0f;
        if (nc > 8 * CL) merge(std::integral_constant<int, 16>{}, ph, m, l, v);
        else merge(std::integral_constant<int, 8>{}, ph, m, l, v);
        mv[cl * D + i] = v;
        if (i == 0) {
            ms[cl] = m;
            ls[cl] = l;
        }
        __syncthreads();
        if (cl == 0) {
            float M = ms[0];
#pragma unroll
            for (int k = 1; k < CL; ++k) M = fmaxf(M, ms[k]);
            float lt = 0.0f, vt = 0.0f;
            if (M > -INFINITY) {
#pragma unroll
                for (int k = 0; k < CL; ++k) {
                    const float f = ex2f(ms[k] - M);
                    lt = fmaf(ls[k], f, lt);
                    vt = fmaf(mv[k * D + i], f, vt);
                }
            }
            acc[i] = lt > 0.0f ? vt / lt : 0.0f;
        }
        __syncthreads();
        if (!have_pv) {
            if (!stage_wait(bar)) return;
            have_pv = true;
        }
        float o = 0.0f;
        constexpr int JL = D / CL;  // terms of the rotation per lane
#pragma unroll 8
        for (int j = JL * cl; j < JL * cl + JL; ++j) o = fmaf(pvs[j * D + i], acc[j], o);
        mv[cl * D + i] = o;
        __syncthreads();
        if (cl == 0) {
            o = mv[i];
#pragma unroll
            for (int k = 1; k < CL; ++k) o += mv[k * D + i];
            const int64_t e = ((int64_t)row * a.hq + h) * D + i;
            if (a.dtype == FB_BF16) ((__nv_bfloat16*)a.out)[e] = __float2bfloat16_rn(o);
            else ((__half*)a.out)[e] = __float2half_rn(o);
        }
        __syncthreads();  // mv, ms, ls and acc are reused by the next head
    }
}

// One launch of the combine for the call's rows: tqa_combine_deep when one CTA per (row group,
// KV head) would leave SMs idle and a row has more partials than tqa_combine requests at once
// (its threads would wait on one round trip to memory after another), else tqa_combine.
inline int launch_combine(const AttnArgs& a, int rows, cudaStream_t s) {
    const int G = a.hq / a.hkv;
    if ((int64_t)rows * a.hkv < num_sms() && a.nch > 16) {
        int hpc = 1;  // heads per CTA: at most two CTAs per SM
        while ((int64_t)rows * a.hq / hpc > 2LL * num_sms() && hpc < G) hpc *= 2;
        // eight chunk lanes when the CTAs fill at most half the SMs and a row has 64 chunks or
        // more (one round of loads per lane), else four
        const bool wide = (int64_t)rows * a.hq / hpc * 2 <= num_sms() && a.nch >= 64;
        const int cl = wide ? 8 : 4;
        auto kern = wide ? tqa_combine_deep<8> : tqa_combine_deep<4>;
        const size_t smem = (size_t)D * D * 4 + (size_t)(cl * D + 2 * cl + D) * 4 + 16;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        launch_pdl_smem(kern, dim3(rows, a.hq / hpc), dim3(cl * D), smem, s, a, hpc);
        return (int)cudaGetLastError();
    }
    const size_t smem = (size_t)D * D * 4 + (size_t)RQ * G * D * 4 + 16;
    const int rq = rows_per_cta(rows, a.hkv);
    void (*kern)(AttnArgs, int) = rq == 1 ? tqa_combine<1> : rq == 2 ? tqa_combine<2> : tqa_combine<4>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    launch_pdl_smem(kern, dim3((rows + rq - 1) / rq, a.hkv), dim3(std::min(G, 4) * D), smem, s, a, rows);
    return (int)cudaGetLastError();
}

// ── tensor-core path: 2- and 4-bit keys and values ──
//
// One work item = (chunk of 512 x rnd positions, KV head, query token), rnd = 1, 2 or 4 chosen per
// call (tc_chunks); a persistent CTA takes items in turn and builds its decoding tables once.
// Warp w takes positions 64 rnd w .. 64 rnd (w + 1) - 1 of the chunk in rnd rounds of four
// 16-position tiles (a round's codes all requested before any is
// used), keeps a running softmax (maximum, sum, accumulator) per head across the rounds, and
// does both contractions with mma.sync m16n8k16 (FP16 operands, FP32 accumulators), the
// operands decoded in registers:
//
//   scores   S[16 positions x 8 heads] = K_tile[16 x 128] . Q^T: lane (r, t) = (lane / 4,
//            lane % 4) reads bytes of rows r and r + 8 holding code pairs 16t..16t+15 and
//            turns each pair into an A register with one table lookup (pair -> half2); the
//            MMA's k index 2t+e of step kk stands for coordinate 32t + 4kk + e (+2 for the
//            upper half), and the B registers hold q_rot of head r at the same coordinates.
//   values   acc^T[128 dims x 8 heads] += V_tile^T[128 x 16 positions] . P[16 x 8]: lane
//            (r, t) owns dims 16r..16r+15 (MMA m-tile mt: rows r and r + 8 are dims 16r + 2mt
//            and 16r + 2mt + 1) and positions 2t, 2t+1, 2t+8, 2t+9; an A register holds one
//            dim at two adjacent positions, so the V table is indexed by the codes of the two
//            positions (cross-position pairs). The weights P go through shared memory and come
//            back transposed (ldmatrix .trans) as B registers.
//
// Table lookups: entry e at byte 256e, 32 lane-private copies of the K pair value at
// 256e + 4 lane and of the V pair value at 256e + 128 + 4 lane, so the address is one byte
// permute of the code byte and the lane offset, and a warp's lookups hit 32 banks. At the end
// of an item the warps' results are rescaled to the item's maximum and added in warp order.

namespace tc {
constexpr int TILE = 16, TPW = 4, MAX_RND = 4;  // an item: NWARPS * rnd * TPW * TILE positions, rnd <= MAX_RND

template <int KB, int VB>
struct Smem {
    static constexpr int ke = 1 << (2 * KB), ve = 1 << (2 * VB);
    static constexpr int entries = ke > ve ? ke : ve;
    static constexpr int acc_off = entries * 256;                       // [NWARPS][8][D] f32
    static constexpr int p_off = acc_off + NWARPS * 8 * D * 4;          // [NWARPS][TPW][16][8] f16
    static constexpr int mx_off = p_off + NWARPS * TPW * TILE * 8 * 2;  // [NWARPS][8] f32
    static constexpr int l_off = mx_off + NWARPS * 8 * 4;               // [NWARPS][8] f32
    static constexpr int q_off = l_off + NWARPS * 8 * 4;              // [8 steps][32 lanes] uint2
    static constexpr int bytes = q_off + 8 * 32 * 8;
};

}  // namespace tc

template <int KB, int VB, typename Addr>
__global__ void __launch_bounds__(THREADS, 2) tqa_mma(AttnArgs a, Addr ad, int items) {
    using namespace tc;
    using S = Smem<KB, VB>;
    constexpr int PK = D * KB / 8, PV = D * VB / 8;
    constexpr int KW = PK / 16;  // 32-bit words of a K row per lane (rows are split in four)
    constexpr int VW = PV / 32;  // 32-bit words of a V row per lane (rows are split in eight)
    extern __shared__ __align__(16) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, r = lane >> 2, t = lane & 3;

    for (int j = tid; j < S::ke + S::ve; j += THREADS) {
        const bool key = j < S::ke;
        const int e = key ? j : j - S::ke, bits = key ? KB : VB;
        const float* cen = key ? a.ck : a.cv;
        const uint32_t w = pack_half2(__ldg(cen + (e >> bits)), __ldg(cen + (e & ((1 << bits) - 1))));
        uint4* row = (uint4*)(sm + e * 256 + (key ? 0 : 128));
#pragma unroll
        for (int k = 0; k < 8; ++k) row[(k + j) & 7] = make_uint4(w, w, w, w);
    }
    // The tables above read only the codebooks, before the wait: this is safe because run() always
    // launches tqa_rotate_q (which waits for the work before it) right before this kernel, and
    // nothing writes the codebooks in between. A chain that drops or reorders rotate_q must move
    // the table build after pdl_begin().
    pdl_begin();  // what follows reads the rotate kernel's output
    __syncthreads();
    auto lut = [&](uint32_t addr) { return *reinterpret_cast<const uint32_t*>(sm + addr); };

    const int GA = a.hq / a.hkv;
    float* accs = (float*)(sm + S::acc_off);
    __half* pb = (__half*)(sm + S::p_off) + warp * TPW * TILE * 8;
    float* rmx = (float*)(sm + S::mx_off);
    float* rl = (float*)(sm + S::l_off);
    uint2* qf = (uint2*)(sm + S::q_off);
    const uint32_t kof = 4u * lane, vof = 128u + 4u * lane;
    const float rs = rsqrtf((float)D);
    const int64_t kst = (int64_t)a.hkv * PK, vst = (int64_t)a.hkv * PV;

    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const uint32_t rest = sm100::divu32((uint32_t)item, a.dnch), rw_ = sm100::divu32(rest, a.dhkv);
        const int c = item - (int)rest * a.nch, g = (int)rest - (int)rw_ * a.hkv, row = (int)rw_;
        const int s = (int)sm100::divu32(rw_, a.dqps), tq = row - s * a.q_per_seq;
        const int L = causal_len(a, s, tq);
        const int p0 = c * a.ch;
        if (p0 >= L) continue;  // the whole CTA

        // B registers of the score MMA, step kk, lane (r, t): q_rot of head r (zeros past the
        // group) at coordinates 32t + 4kk .. 32t + 4kk + 3 as two half2, staged in shared memory
        // in that order (one conflict-free 8-byte load per lane and step; the barrier below the
        // code loads publishes them); thread (kk, lane) = (warp, lane)
        {
            const float4 f = r < GA ? __ldg((const float4*)(a.qrot + ((int64_t)row * a.hq + g * GA + r) * D + 32 * t +
                                                            4 * warp))
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            qf[warp * 32 + lane] = make_uint2(pack_half2(f.x, f.y), pack_half2(f.z, f.w));
        }

        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // heads 2t, 2t + 1: running softmax
        float acc[8][4];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;
#pragma unroll 1
        for (int rd = 0; rd < a.rnd; ++rd) {
        // codes and norms of the round's four tiles of the warp, all requested before any is used
        const int pw = p0 + (warp * a.rnd + rd) * TPW * TILE;
        uint32_t kw[TPW][2][KW], vw[TPW][4][VW];
        float kn[TPW][2], vn[TPW][2];
        int nv[TPW];
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
            const int ps = pw + i * TILE;
            const uint8_t *kb = nullptr, *vb = nullptr;
            const __half *knb = nullptr, *vnb = nullptr;
            int n = 0;
            if (ps < L && (ps >> 4) < a.max_blocks) {
                const int32_t blk = a.block_tables[(int64_t)s * a.max_blocks + (ps >> 4)];
                if (blk >= 0) n = min(min(TILE, L - ps), ad.block_rows(blk));
                if (n > 0) ad.block_base(blk, g, a.hkv, PK, PV, kb, vb, knb, vnb);
            }
            nv[i] = n;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int off = r + 8 * h;
                const bool ok = off < n;
                if constexpr (KW == 4) {
                    const uint4 u = ok ? __ldg((const uint4*)(kb + off * kst + 16 * t)) : make_uint4(0, 0, 0, 0);
                    kw[i][h][0] = u.x;
                    kw[i][h][1] = u.y;
                    kw[i][h][2] = u.z;
                    kw[i][h][3] = u.w;
                } else {
                    const uint2 u = ok ? __ldg((const uint2*)(kb + off * kst + 8 * t)) : make_uint2(0, 0);
                    kw[i][h][0] = u.x;
                    kw[i][h][1] = u.y;
                }
                kn[i][h] = ok ? __half2float(knb[off * a.hkv]) : 0.0f;
                vn[i][h] = ok ? __half2float(vnb[off * a.hkv]) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int off = 2 * t + (u & 1) + 8 * (u >> 1);
                const bool ok = off < n;
                if constexpr (VW == 1) {
                    vw[i][u][0] = ok ? __ldg((const uint32_t*)(vb + off * vst + 4 * r)) : 0u;
                } else {
                    const uint2 x = ok ? __ldg((const uint2*)(vb + off * vst + 8 * r)) : make_uint2(0, 0);
                    vw[i][u][0] = x.x;
                    vw[i][u][1] = x.y;
                }
            }
        }

        if (rd == 0) __syncthreads();  // the staged query fragments

        // ── scores ──
        float sc[TPW][4];
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
            float c4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (nv[i] > 0) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    uint32_t a0, a1, a2, a3;
                    if constexpr (KB == 4) {  // pair 2kk: byte 2kk of the lane's 16; pair 2kk + 1: the next
                        const uint32_t w0 = kw[i][0][kk >> 1], w1 = kw[i][1][kk >> 1];
                        const int b = 2 * (kk & 1);
                        a0 = lut(taddr(w0, kof, b));
                        a1 = lut(taddr(w1, kof, b));
                        a2 = lut(taddr(w0, kof, b + 1));
                        a3 = lut(taddr(w1, kof, b + 1));
                    } else {  // pair 2kk: high nibble of byte kk of the lane's 8; pair 2kk + 1: low nibble
                        const uint32_t w0 = kw[i][0][kk >> 2], w1 = kw[i][1][kk >> 2];
                        const int b = kk & 3;
                        a0 = lut(taddr((w0 >> 4) & 0x0f0f0f0fu, kof, b));
                        a1 = lut(taddr((w1 >> 4) & 0x0f0f0f0fu, kof, b));
                        a2 = lut(taddr(w0 & 0x0f0f0f0fu, kof, b));
                        a3 = lut(taddr(w1 & 0x0f0f0f0fu, kof, b));
                    }
                    const uint2 qb = qf[kk * 32 + lane];
                    mma16816(c4, a0, a1, a2, a3, qb.x, qb.y);
                }
            }
            const float f0 = kn[i][0] * rs, f1 = kn[i][1] * rs;
            sc[i][0] = r < nv[i] ? c4[0] * f0 : -INFINITY;
            sc[i][1] = r < nv[i] ? c4[1] * f0 : -INFINITY;
            sc[i][2] = r + 8 < nv[i] ? c4[2] * f1 : -INFINITY;
            sc[i][3] = r + 8 < nv[i] ? c4[3] * f1 : -INFINITY;
        }

        // ── running softmax of the warp: the round's maximum per head, the sums so far rescaled
        // when it grows, weights exp(s - max) * v_norm ──
        float t0 = -INFINITY, t1 = -INFINITY;
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
            t0 = fmaxf(t0, fmaxf(sc[i][0], sc[i][2]));
            t1 = fmaxf(t1, fmaxf(sc[i][1], sc[i][3]));
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
            t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
        }
        if (t0 > m0 || t1 > m1) {
            const float g0 = t0 > m0 ? __expf(m0 - t0) : 1.0f, g1 = t1 > m1 ? __expf(m1 - t1) : 1.0f;
            m0 = fmaxf(m0, t0);
            m1 = fmaxf(m1, t1);
            l0 *= g0;
            l1 *= g1;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                acc[mt][0] *= g0;
                acc[mt][2] *= g0;
                acc[mt][1] *= g1;
                acc[mt][3] *= g1;
            }
        }
        const bool any = m0 > -INFINITY;  // some position of the warp's rounds so far is in the cache
        __syncwarp();  // the previous round's weights have been read
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
            const float e0 = any ? __expf(sc[i][0] - m0) : 0.0f, e1 = any ? __expf(sc[i][1] - m1) : 0.0f;
            const float e2 = any ? __expf(sc[i][2] - m0) : 0.0f, e3 = any ? __expf(sc[i][3] - m1) : 0.0f;
            l0 += e0 + e2;
            l1 += e1 + e3;
            uint32_t* pr = (uint32_t*)(pb + (i * TILE + r) * 8 + 2 * t);
            pr[0] = pack_half2(e0 * vn[i][0], e1 * vn[i][0]);
            pr[8 * 4] = pack_half2(e2 * vn[i][1], e3 * vn[i][1]);  // row r + 8
        }
        __syncwarp();

        // ── values ──
#pragma unroll
        for (int i = 0; i < TPW; ++i) {
            if (nv[i] == 0) continue;
            uint32_t b0, b1;
            ldsm_x2_trans(b0, b1, (uint32_t)__cvta_generic_to_shared(pb + (i * TILE + (lane & 15)) * 8));
            if constexpr (VB == 2) {
                // X[j] byte q: (code of dim 4q + j at position 2t) << 2 | (same dim at 2t + 1);
                // Y[j]: positions 2t + 8, 2t + 9
                uint32_t X[4], Y[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int sh = 6 - 2 * j;
                    X[j] = ((vw[i][0][0] >> sh << 2) & 0x0c0c0c0cu) | ((vw[i][1][0] >> sh) & 0x03030303u);
                    Y[j] = ((vw[i][2][0] >> sh << 2) & 0x0c0c0c0cu) | ((vw[i][3][0] >> sh) & 0x03030303u);
                }
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    const int b = mt >> 1, j0 = 2 * (mt & 1);
                    mma16816(acc[mt], lut(taddr(X[j0], vof, b)), lut(taddr(X[j0 + 1], vof, b)),
                             lut(taddr(Y[j0], vof, b)), lut(taddr(Y[j0 + 1], vof, b)), b0, b1);
                }
            } else {
                // H[u] byte q: (high nibble of byte 4u + q at position 2t) << 4 | (same at 2t + 1),
                // the dim 2(4u + q); L[u]: low nibbles, dim 2(4u + q) + 1; H2/L2: positions 2t + 8, 2t + 9
                uint32_t H[2], Lo[2], H2[2], L2[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    H[u] = (vw[i][0][u] & 0xf0f0f0f0u) | ((vw[i][1][u] >> 4) & 0x0f0f0f0fu);
                    Lo[u] = ((vw[i][0][u] << 4) & 0xf0f0f0f0u) | (vw[i][1][u] & 0x0f0f0f0fu);
                    H2[u] = (vw[i][2][u] & 0xf0f0f0f0u) | ((vw[i][3][u] >> 4) & 0x0f0f0f0fu);
                    L2[u] = ((vw[i][2][u] << 4) & 0xf0f0f0f0u) | (vw[i][3][u] & 0x0f0f0f0fu);
                }
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    const int u = mt >> 2, b = mt & 3;
                    mma16816(acc[mt], lut(taddr(H[u], vof, b)), lut(taddr(Lo[u], vof, b)), lut(taddr(H2[u], vof, b)),
                             lut(taddr(L2[u], vof, b)), b0, b1);
                }
            }
        }

        }  // rounds

        // ── the warps' results, rescaled to the item's maximum and added in warp order ──
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, o);
            l1 += __shfl_xor_sync(0xffffffffu, l1, o);
        }
        if (r == 0) {
            rmx[warp * 8 + 2 * t] = m0;
            rmx[warp * 8 + 2 * t + 1] = m1;
            rl[warp * 8 + 2 * t] = l0;
            rl[warp * 8 + 2 * t + 1] = l1;
        }
        {
            float* a0 = accs + (warp * 8 + 2 * t) * D + 16 * r;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                *(float2*)(a0 + 2 * mt) = make_float2(acc[mt][0], acc[mt][2]);
                *(float2*)(a0 + D + 2 * mt) = make_float2(acc[mt][1], acc[mt][3]);
            }
        }
        __syncthreads();
        float* part = a.part + (((int64_t)row * a.hq + g * GA) * a.nch + c) * PART;
        for (int e = tid; e < GA * D; e += THREADS) {
            const int h = e / D, i = e - h * D;
            float M = rmx[h];
#pragma unroll
            for (int w = 1; w < NWARPS; ++w) M = fmaxf(M, rmx[w * 8 + h]);
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < NWARPS; ++w) {
                const float mw = rmx[w * 8 + h];
                if (mw > -INFINITY) v = fmaf(accs[(w * 8 + h) * D + i], __expf(mw - M), v);
            }
            part[(int64_t)h * a.nch * PART + 2 + i] = v;
            if (i == 0) {
                float l = 0.0f;
#pragma unroll
                for (int w = 0; w < NWARPS; ++w) {
                    const float mw = rmx[w * 8 + h];
                    if (mw > -INFINITY) l = fmaf(rl[w * 8 + h], __expf(mw - M), l);
                }
                part[(int64_t)h * a.nch * PART] = M;
                part[(int64_t)h * a.nch * PART + 1] = l;
            }
        }
        __syncthreads();  // the next item rewrites the maxima and sums
    }
}

size_t workspace_bytes(int64_t rows, int hq, int64_t nch) {
    return (size_t)rows * hq * D * 4 + (size_t)rows * hq * nch * PART * 4;
}

// Partial slots per (row, head) a workspace is sized for: one per CH positions (the least any
// call needs), and for calls with few query rows up to one per 32 positions, at most 160 over
// the rows: the streamed kernel then splits a context into more, shorter chunks to give every
// SM an item.
int64_t partial_slots(int64_t rows, int max_kv_len) {
    const int64_t nch = (max_kv_len + CH - 1) / CH;
    if (rows <= 0) return nch;
    return std::max<int64_t>(nch, std::min<int64_t>((max_kv_len + 31) / 32, 160 / rows));
}

// The slots a call uses: what a workspace of `bytes` holds past the rotated queries, capped at
// partial_slots() so that the choice of chunks (and so the result) does not depend on how much
// larger than that the caller made the workspace; at least nch (the entry points check that).
int call_slots(size_t bytes, int64_t rows, int hq, int max_kv_len) {
    const int64_t nch = (max_kv_len + CH - 1) / CH;
    const size_t q = (size_t)rows * hq * D * 4, per = (size_t)rows * hq * PART * 4;
    const int64_t held = bytes > q && per > 0 ? (int64_t)((bytes - q) / per) : 0;
    return (int)std::max<int64_t>(nch, std::min<int64_t>(held, partial_slots(rows, max_kv_len)));
}

template <int KB, int VB, int G, typename Addr>
int launch_chunk(const AttnArgs& a, const Addr& ad, cudaStream_t s) {
    constexpr int smem = ChunkSmem<KB, VB, G>::bytes;
    auto kern = tqa_chunk<KB, VB, G, Addr>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    const int rows = a.num_seqs * a.q_per_seq;
    kern<<<dim3(a.nch, a.hkv, rows), THREADS, smem, s>>>(a, ad);
    return (int)cudaGetLastError();
}

template <int KB, int VB, typename Addr>
int dispatch_g(const AttnArgs& a, const Addr& ad, cudaStream_t s) {
    // groups of 1, 2 or 4 Q heads share the 4-head kernel
    return a.hq / a.hkv <= 4 ? launch_chunk<KB, VB, 4>(a, ad, s) : launch_chunk<KB, VB, 8>(a, ad, s);
}

template <int KB, typename Addr>
int dispatch_vb(const AttnArgs& a, int vb, const Addr& ad, cudaStream_t s) {
    switch (vb) {
        case 2: return dispatch_g<KB, 2>(a, ad, s);
        case 3: return dispatch_g<KB, 3>(a, ad, s);
        case 4: return dispatch_g<KB, 4>(a, ad, s);
        default: return dispatch_g<KB, 8>(a, ad, s);
    }
}

// One CTA per SM slot, each walking the items (chunk, KV head, query token) in turn.
template <int KB, int VB, typename Addr>
int launch_tc(const AttnArgs& a, const Addr& ad, cudaStream_t s) {
    constexpr int smem = tc::Smem<KB, VB>::bytes;
    auto kern = tqa_mma<KB, VB, Addr>;
    static std::atomic<int> slots[64];  // CTAs per device, found on the first launch on that device
    // (two threads making their first launch at once both compute the same value)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    if (slots[dev].load(std::memory_order_relaxed) == 0) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return (int)e;
        int per_sm = 0, sms = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, THREADS, smem);
        if (e != cudaSuccess) return (int)e;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return (int)e;
        if (per_sm < 1) return (int)cudaErrorInvalidConfiguration;
        slots[dev].store(per_sm * sms, std::memory_order_relaxed);
    }
    const int64_t items = (int64_t)a.nch * a.hkv * a.num_seqs * a.q_per_seq;
    if (items > INT32_MAX) return (int)cudaErrorInvalidValue;
    const int grid = (int)std::min<int64_t>(items, slots[dev].load(std::memory_order_relaxed));
    AttnArgs b = a;
    b.dnch = sm100::make_divu32((uint32_t)a.nch);
    b.dhkv = sm100::make_divu32((uint32_t)a.hkv);
    b.dqps = sm100::make_divu32((uint32_t)a.q_per_seq);
    launch_pdl_smem(kern, dim3(grid), dim3(THREADS), (size_t)smem, s, b, ad, (int)items);
    return (int)cudaGetLastError();
}

template <int KB, typename Addr>
int dispatch_tc(const AttnArgs& a, int vb, const Addr& ad, cudaStream_t s) {
    return vb == 2 ? launch_tc<KB, 2>(a, ad, s) : launch_tc<KB, 4>(a, ad, s);
}

bool tc_ok(int kb, int vb) { return (kb == 2 || kb == 4) && (vb == 2 || vb == 4); }

// Items of the tensor-core kernel as long as they still fill three quarters of one wave of CTA
// slots (two CTAs per SM): long items pay the per-item cost (query staging, the warps'
// reduction, one partial) over more positions, short ones keep small batches spread over the
// SMs. (Measured at 8192-token contexts: 8 sequences, 256 items of 2048 positions, ran in 56 us
// against 72 us for 1024 items of 512; 1 sequence, 128 items of 512, in 37 us against 48 us for
// 32 items of 2048.)
inline void tc_chunks(AttnArgs& a, int64_t positions, int64_t rows) {
    int rnd = tc::MAX_RND;
    const int64_t per_round = (int64_t)NWARPS * tc::TPW * tc::TILE;
    while (rnd > 1 && (positions + per_round * rnd - 1) / (per_round * rnd) * a.hkv * rows * 4 < 3LL * 2 * num_sms())
        rnd /= 2;
    a.rnd = rnd;
    a.ch = (int)(per_round * rnd);
    a.nch = (int)((positions + a.ch - 1) / a.ch);
}

// tq_attention_stream.cu: the streamed tensor-core kernel (pools or per-block buffers).
bool stream_ok(const AttnArgs& a, int kb, int vb, const PoolAddr& ad);
bool stream_ok(const AttnArgs& a, int kb, int vb, const BlockPtrAddr& ad);
int stream_launch(AttnArgs& a, int kb, int vb, const PoolAddr& ad, cudaStream_t s);
int stream_launch(AttnArgs& a, int kb, int vb, const BlockPtrAddr& ad, cudaStream_t s);

template <typename Addr>
int run(AttnArgs a, int kb, int vb, const Addr& ad, cudaStream_t s) {
    const int rows = a.num_seqs * a.q_per_seq;
    if (rows == 0) return 0;
    a.spc = 1;
    const bool streamed = a.nch > 0 && stream_ok(a, kb, vb, ad);
    a.qrot_f16 = streamed ? 1 : 0;
    int rc = launch_rotate(a, rows, s);
    if (rc) return rc;
    // a.nch counts CH-position chunks (the workspace is sized for them); the tensor-core
    // paths take larger chunks, so they use fewer of the same partial slots
    a.ch = CH;
    if (streamed) {
        rc = tq_count_path(10, stream_launch(a, kb, vb, ad, s));  // sets a.ch, a.spc, a.nch
        if (rc) return rc;
        return launch_combine(a, rows, s);
    }
    if (tc_ok(kb, vb)) {
        tc_chunks(a, (int64_t)a.nch * CH, rows);
        if (a.nch > 0) {
            rc = tq_count_path(9, kb == 2 ? dispatch_tc<2>(a, vb, ad, s) : dispatch_tc<4>(a, vb, ad, s));
            if (rc) return rc;
        }
    } else if (a.nch > 0) {
        switch (kb) {
            case 2: rc = dispatch_vb<2>(a, vb, ad, s); break;
            case 3: rc = dispatch_vb<3>(a, vb, ad, s); break;
            case 4: rc = dispatch_vb<4>(a, vb, ad, s); break;
            default: rc = dispatch_vb<8>(a, vb, ad, s); break;
        }
        if (tq_count_path(8, rc)) return rc;
    }
    return launch_combine(a, rows, s);
}

bool bits_ok(int b) { return b == 2 || b == 3 || b == 4 || b == 8; }

bool shape_ok(int hq, int hkv, int head_dim) {
    if (head_dim != D || hkv <= 0 || hq <= 0 || hq % hkv) return false;
    const int G = hq / hkv;
    return G == 1 || G == 2 || G == 4 || G == 8;
}

}  // namespace tqa

void set_last_error(const char* msg);

// The least workspace a call takes, and the size that lets it use every partial slot it may.
size_t tq_attention_ws_bytes(int64_t rows, int hq, int max_kv_len) {
    return tqa::workspace_bytes(rows, hq, (max_kv_len + tqa::CH - 1) / tqa::CH);
}
size_t tq_attention_ws_bytes_full(int64_t rows, int hq, int max_kv_len) {
    return tqa::workspace_bytes(rows, hq, tqa::partial_slots(rows, max_kv_len));
}

// One sequence over the contiguous pools, with host scalars for its length and start (the
// backend object's cache manager).
int tq_attention_one_seq(const void* q, int dtype, int num_tokens, int hq, int hkv, int head_dim, const void* kp,
                         const void* kn, const void* vp, const void* vn, int64_t pool_rows, const int32_t* block_table,
                         int num_blocks, int kv_len, int start_pos, const float* pik, const float* piv,
                         const float* ck, const float* cv, int kb, int vb, void* workspace, size_t ws_bytes,
                         void* out, cudaStream_t s) {
    if ((dtype != FB_FP16 && dtype != FB_BF16) || !tqa::shape_ok(hq, hkv, head_dim) || !tqa::bits_ok(kb) ||
        !tqa::bits_ok(vb) || num_tokens < 0 || num_tokens > 65535 || kv_len < 0 || start_pos < 0)
        return (int)cudaErrorInvalidValue;
    if (num_tokens == 0) return 0;
    if (ws_bytes < tq_attention_ws_bytes(num_tokens, hq, kv_len) || !aligned16(workspace) || !aligned16(kp) ||
        !aligned16(vp) || !aligned16(pik))
        return (int)cudaErrorInvalidValue;
    tqa::AttnArgs a{};
    a.q = q;
    a.dtype = dtype;
    a.num_seqs = 1;
    a.q_per_seq = num_tokens;
    a.hq = hq;
    a.hkv = hkv;
    a.block_tables = block_table;
    a.max_blocks = num_blocks;
    a.kv_len = kv_len;
    a.start = start_pos;
    a.pik = pik;
    a.piv = piv;
    a.ck = ck;
    a.cv = cv;
    a.qrot = (float*)workspace;
    a.part = a.qrot + (int64_t)num_tokens * hq * tqa::D;
    a.nch = (kv_len + tqa::CH - 1) / tqa::CH;
    a.slots = tqa::call_slots(ws_bytes, num_tokens, hq, kv_len);
    a.out = out;
    tqa::PoolAddr ad{(const uint8_t*)kp, (const __half*)kn, (const uint8_t*)vp, (const __half*)vn, pool_rows};
    return tqa::run(a, kb, vb, ad, s);
}

}  // namespace fb

using namespace fb;

extern "C" size_t fb_tq_attention_workspace_bytes(int num_seqs, int q_per_seq, int num_q_heads, int max_kv_len) {
    if (num_seqs < 0 || q_per_seq < 0 || num_q_heads <= 0 || max_kv_len < 0) return 0;
    return tq_attention_ws_bytes_full((int64_t)num_seqs * q_per_seq, num_q_heads, max_kv_len);
}

extern "C" int fb_launch_tq_attention_paged(const void* q, int dtype, int num_seqs, int q_per_seq, int num_q_heads,
                                            int num_kv_heads, int head_dim, const void* k_packed_pool,
                                            const void* k_norms_pool, const void* v_packed_pool,
                                            const void* v_norms_pool, int64_t num_pool_rows,
                                            const int32_t* block_tables, int max_blocks_per_seq,
                                            const int32_t* kv_lens, const int32_t* start_pos, int max_kv_len,
                                            const float* k_rotation, const float* v_rotation,
                                            const float* k_centroids, const float* v_centroids, int key_bits,
                                            int value_bits, void* workspace, size_t workspace_bytes, void* output,
                                            void* stream) {
    if (dtype != FB_FP16 && dtype != FB_BF16) return (int)cudaErrorInvalidValue;
    if (!tqa::shape_ok(num_q_heads, num_kv_heads, head_dim) || !tqa::bits_ok(key_bits) || !tqa::bits_ok(value_bits))
        return (int)cudaErrorInvalidValue;
    if (num_seqs < 0 || q_per_seq < 0 || max_blocks_per_seq < 0 || max_kv_len < 0 || num_pool_rows < 0)
        return (int)cudaErrorInvalidValue;
    if ((int64_t)num_seqs * q_per_seq == 0) return 0;
    if (!q || !output || !k_rotation || !v_rotation || !k_centroids || !v_centroids || !kv_lens || !start_pos)
        return (int)cudaErrorInvalidValue;
    if (max_kv_len > 0 && (!block_tables || !k_packed_pool || !k_norms_pool || !v_packed_pool || !v_norms_pool))
        return (int)cudaErrorInvalidValue;
    if (!aligned16(k_packed_pool) || !aligned16(v_packed_pool) || !aligned16(k_rotation) || !aligned16(workspace))
        return (int)cudaErrorInvalidValue;
    const int nch = (max_kv_len + tqa::CH - 1) / tqa::CH;
    const int64_t rows = (int64_t)num_seqs * q_per_seq;
    if (rows > 65535 || nch > (1 << 30) || !workspace ||
        workspace_bytes < tqa::workspace_bytes(rows, num_q_heads, nch)) {
        set_last_error("fb_launch_tq_attention_paged: workspace missing or smaller than rows x heads x "
                       "(512 + 520 x ceil(max_kv_len / 256)) bytes, or more than 65535 query rows");
        return (int)cudaErrorInvalidValue;
    }
    tqa::AttnArgs a{};
    a.q = q;
    a.dtype = dtype;
    a.num_seqs = num_seqs;
    a.q_per_seq = q_per_seq;
    a.hq = num_q_heads;
    a.hkv = num_kv_heads;
    a.block_tables = block_tables;
    a.max_blocks = max_blocks_per_seq;
    a.kv_lens = kv_lens;
    a.start_pos = start_pos;
    a.pik = k_rotation;
    a.piv = v_rotation;
    a.ck = k_centroids;
    a.cv = v_centroids;
    a.qrot = (float*)workspace;
    a.part = a.qrot + rows * num_q_heads * tqa::D;
    a.nch = nch;
    a.slots = tqa::call_slots(workspace_bytes, rows, num_q_heads, max_kv_len);
    a.out = output;
    tqa::PoolAddr ad{(const uint8_t*)k_packed_pool, (const __half*)k_norms_pool, (const uint8_t*)v_packed_pool,
                     (const __half*)v_norms_pool, num_pool_rows};
    return tqa::run(a, key_bits, value_bits, ad, (cudaStream_t)stream);
}

// The reference ABI (ffi.rs:251-274, attention_paged_tq.cu:261-309): one sequence, FP16, a
// device block table and per-block pointer arrays. ref_abi_check validates a call and sizes its
// workspace; ref_abi_run enqueues it on a given workspace.
namespace {

int ref_abi_check(const void* output, const void* q, const int* block_table, const void** k_packed_ptrs,
                  const void** k_norms_ptrs, const void** v_packed_ptrs, const void** v_norms_ptrs,
                  const float* k_rotation, const float* v_rotation, const float* k_centroids,
                  const float* v_centroids, int num_tokens, int num_q_heads, int num_kv_heads, int head_dim,
                  int kv_len, int start_pos, int key_bits, int value_bits, int k_packed_dim_per_head,
                  int v_packed_dim_per_head, size_t* need, size_t* want) {
    *need = *want = 0;
    if (!tqa::shape_ok(num_q_heads, num_kv_heads, head_dim) || !tqa::bits_ok(key_bits) || !tqa::bits_ok(value_bits))
        return (int)cudaErrorInvalidValue;
    if (k_packed_dim_per_head != (head_dim * key_bits + 7) / 8 ||
        v_packed_dim_per_head != (head_dim * value_bits + 7) / 8)
        return (int)cudaErrorInvalidValue;
    if (num_tokens < 0 || kv_len < 0 || start_pos < 0 || num_tokens > 65535) return (int)cudaErrorInvalidValue;
    if (num_tokens == 0) return 0;
    if (!output || !q || !k_rotation || !v_rotation || !k_centroids || !v_centroids) return (int)cudaErrorInvalidValue;
    if (!aligned16(k_rotation)) return (int)cudaErrorInvalidValue;  // read 16 bytes at a time
    if (kv_len > 0 && (!block_table || !k_packed_ptrs || !k_norms_ptrs || !v_packed_ptrs || !v_norms_ptrs))
        return (int)cudaErrorInvalidValue;
    const int nch = (kv_len + tqa::CH - 1) / tqa::CH;
    *need = tqa::workspace_bytes(num_tokens, num_q_heads, nch);
    // the workspace for all the call's partial slots, but no larger than the no-allocation
    // variant's scratch (unless the call needs more): both entry points then split a context into
    // the same chunks and agree bit for bit
    *want = std::max(*need, std::min(tq_attention_ws_bytes_full(num_tokens, num_q_heads, kv_len),
                                     (size_t)FB_TQA_NOALLOC_SCRATCH_BYTES));
    return 0;
}

int ref_abi_run(void* ws, size_t ws_bytes, void* output, const void* q, const int* block_table, const void** k_packed_ptrs,
                const void** k_norms_ptrs, const void** v_packed_ptrs, const void** v_norms_ptrs,
                const float* k_rotation, const float* v_rotation, const float* k_centroids, const float* v_centroids,
                int num_tokens, int num_q_heads, int num_kv_heads, int kv_len, int start_pos, int key_bits,
                int value_bits, void* stream) {
    tqa::AttnArgs a{};
    a.q = q;
    a.dtype = FB_FP16;
    a.num_seqs = 1;
    a.q_per_seq = num_tokens;
    a.hq = num_q_heads;
    a.hkv = num_kv_heads;
    a.block_tables = block_table;
    a.max_blocks = (kv_len + 15) / 16;
    a.kv_len = kv_len;
    a.start = start_pos;
    a.pik = k_rotation;
    a.piv = v_rotation;
    a.ck = k_centroids;
    a.cv = v_centroids;
    a.qrot = (float*)ws;
    a.part = a.qrot + (int64_t)num_tokens * num_q_heads * tqa::D;
    a.nch = (kv_len + tqa::CH - 1) / tqa::CH;
    a.slots = tqa::call_slots(ws_bytes, num_tokens, num_q_heads, kv_len);
    a.out = output;
    tqa::BlockPtrAddr ad{(const uint8_t* const*)k_packed_ptrs, (const __half* const*)k_norms_ptrs,
                         (const uint8_t* const*)v_packed_ptrs, (const __half* const*)v_norms_ptrs};
    return tqa::run(a, key_bits, value_bits, ad, (cudaStream_t)stream);
}

}  // namespace

// The workspace is this library's, one per device and stream, grown to the largest call on that
// stream and kept.
extern "C" int launch_attention_paged_tq(void* output, const void* q, const int* block_table, const void** k_packed_ptrs,
                                         const void** k_norms_ptrs, const void** v_packed_ptrs,
                                         const void** v_norms_ptrs, const float* k_rotation, const float* v_rotation,
                                         const float* k_centroids, const float* v_centroids, int num_tokens,
                                         int num_q_heads, int num_kv_heads, int head_dim, int kv_len, int start_pos,
                                         int key_bits, int value_bits, int k_packed_dim_per_head,
                                         int v_packed_dim_per_head, void* stream) {
    size_t need = 0, want = 0;
    const int rc = ref_abi_check(output, q, block_table, k_packed_ptrs, k_norms_ptrs, v_packed_ptrs, v_norms_ptrs,
                                 k_rotation, v_rotation, k_centroids, v_centroids, num_tokens, num_q_heads,
                                 num_kv_heads, head_dim, kv_len, start_pos, key_bits, value_bits,
                                 k_packed_dim_per_head, v_packed_dim_per_head, &need, &want);
    if (rc || num_tokens == 0) return rc;
    return with_stream_workspace(stream, want, [&](void* ws) {
        return ref_abi_run(ws, want, output, q, block_table, k_packed_ptrs, k_norms_ptrs, v_packed_ptrs, v_norms_ptrs,
                           k_rotation, v_rotation, k_centroids, v_centroids, num_tokens, num_q_heads, num_kv_heads,
                           kv_len, start_pos, key_bits, value_bits, stream);
    });
}

// ── launch_attention_paged_tq without any allocation ─────────────────────────
//
// Some callers cannot allocate device memory when they call attention: an engine whose KV pool
// was sized to take all free memory at start-up (a cudaMalloc mid-step would fail), and a decode
// loop that must not stall on the device-wide synchronisation cudaFree implies when the library
// workspace of launch_attention_paged_tq grows. This variant keeps the rotated queries and the
// split-K partials in a fixed array of device memory that is part of the library image instead.
//
// The array is a file-scope __device__ variable: every GPU on which the library's module is
// loaded holds its kTqaNoAllocScratchBytes until the process exits. In host code its name is a
// host-side stand-in, not a device address, so the address handed to the kernels comes from
// cudaGetSymbolAddress, looked up once per device (with that device current) on the first call
// made on it. All calls share the array and it keeps the last call's contents: nothing in it has
// to start at zero (the kernels write every rotated query and every partial the combine step
// reads before reading it), but two calls that can overlap on the GPU (on different streams, or
// on different host threads without ordering) race on it.

constexpr size_t kTqaNoAllocScratchBytes = FB_TQA_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_tqa_noalloc_scratch[kTqaNoAllocScratchBytes];

namespace {

std::mutex g_tqa_noalloc_mu;
void* g_tqa_noalloc_addr[64];  // device address of g_tqa_noalloc_scratch, per device ordinal

int tqa_noalloc_scratch(void** addr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_tqa_noalloc_mu);
    if (!g_tqa_noalloc_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_tqa_noalloc_scratch);
        if (e != cudaSuccess) return (int)e;
        g_tqa_noalloc_addr[dev] = p;
    }
    *addr = g_tqa_noalloc_addr[dev];
    return 0;
}

}  // namespace

extern "C" int launch_attention_paged_tq_noalloc(void* output, const void* q, const int* block_table,
                                                 const void** k_packed_ptrs, const void** k_norms_ptrs,
                                                 const void** v_packed_ptrs, const void** v_norms_ptrs,
                                                 const float* k_rotation, const float* v_rotation,
                                                 const float* k_centroids, const float* v_centroids, int num_tokens,
                                                 int num_q_heads, int num_kv_heads, int head_dim, int kv_len,
                                                 int start_pos, int key_bits, int value_bits,
                                                 int k_packed_dim_per_head, int v_packed_dim_per_head, void* stream) {
    size_t need = 0, want = 0;
    int rc = ref_abi_check(output, q, block_table, k_packed_ptrs, k_norms_ptrs, v_packed_ptrs, v_norms_ptrs,
                           k_rotation, v_rotation, k_centroids, v_centroids, num_tokens, num_q_heads, num_kv_heads,
                           head_dim, kv_len, start_pos, key_bits, value_bits, k_packed_dim_per_head,
                           v_packed_dim_per_head, &need, &want);
    if (rc || num_tokens == 0) return rc;
    if (need > kTqaNoAllocScratchBytes) {
        char msg[256];
        snprintf(msg, sizeof msg,
                 "launch_attention_paged_tq_noalloc: %d query tokens x %d heads over %d positions need %zu bytes "
                 "of scratch, more than its fixed %zu",
                 num_tokens, num_q_heads, kv_len, need, kTqaNoAllocScratchBytes);
        set_last_error(msg);
        return (int)cudaErrorInvalidValue;
    }
    void* ws = nullptr;
    rc = tqa_noalloc_scratch(&ws);
    if (rc) return rc;
    return ref_abi_run(ws, kTqaNoAllocScratchBytes, output, q, block_table, k_packed_ptrs, k_norms_ptrs, v_packed_ptrs, v_norms_ptrs,
                       k_rotation, v_rotation, k_centroids, v_centroids, num_tokens, num_q_heads, num_kv_heads, kv_len,
                       start_pos, key_bits, value_bits, stream);
}

namespace fb {
unsigned int tqa_timeouts() {
    unsigned int v = 0;
    cudaMemcpyFromSymbol(&v, g_tqa_timeouts, sizeof(v));
    return v;
}
}  // namespace fb
