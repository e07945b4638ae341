// TurboQuant compress on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Replaces backends/fracture-cuda/kernels/turboquant_compress.cu:27-222 for
// head_dim 128 and 2/3/4-bit codes. One persistent CTA per SM streams tiles of
// 128 head vectors. A launch serves one compress call, or two (the K and V of an
// append): the grid is split between the calls in proportion to their tiles, and
// each CTA works for one of them only, so a step pays one pipeline fill and one
// tail for both.
//
//   warp 0      TMA producer: [128 vectors x 128] fp16/bf16 tile -> smem (SW128)
//   warp 1      MMA issuer:   acc[v][i] = sum_j x[v][j] * Pi[i][j] on tcgen05,
//               Pi split into 2 fp16 (or 3 bf16) parts so the product is
//               float32-accurate while x stays exact; accumulator in TMEM
//   warps 2-17  epilogue, four warpgroups on their own TMEM accumulators: one
//               thread per vector reads its row of acc from TMEM, derives the
//               norm (|Pi x| = |x|), maps each coordinate to its code through
//               a decision table in shared memory, packs the MSB-first bit
//               stream and writes it straight into its paged-pool row.
//
// Bit-exactness. The reference result is the exact float32 statement
// (sequential sums, true division, first-minimum nearest centroid). The fast
// path agrees with it except for coordinates that land within kRiskBand of a
// decision boundary, and for norms whose fp16 rounding is within kNormBand of a
// tie; those are recomputed here with the exact float32 sequence (tq_common.cuh)
// from the input row, so every stored code and norm equals the exact statement.
//
// Every barrier wait is bounded; on timeout the kernel counts the event in
// g_tq_umma_timeouts (and err_count when given), abandons its loop and still
// frees its TMEM before returning.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "tq_common.cuh"
#include "tq_sm100.cuh"

namespace fb {

__device__ unsigned int g_tq_umma_timeouts = 0;

namespace umma {

using namespace sm100;

constexpr int MAX_STAGES = 4;       // A-tile pipeline depth: 4 with FP16 input, 3 with BF16 (its
                                    // third operand part takes the fourth stage's shared memory)
__host__ __device__ constexpr int stages_for(int nparts) { return nparts == 2 ? 4 : 3; }
constexpr int NB = 128;             // decision-table bins; bin b covers y in [(b - kBin0 -+ 1/2) w]
constexpr int kBin0 = 64;           // the bin centred on y = 0
constexpr float kInvW = 63.5f / 1.02f;  // 1 / bin width: bins span [-1.036, 1.02), and |y| <= 1
constexpr int LUT_COPIES = 32;      // copies per bin, one per lane: a warp's lookups hit 32 banks
constexpr float kRiskBand = 1e-6f;   // |y - boundary| below this: settle with the exact sequence
constexpr float kNormBand = 1e-6f;  // relative band around fp16 rounding ties of the norm
constexpr float kWindowPad = 1e-4f; // a bin owns the boundaries within this distance of its edges
constexpr int EPI_WGS = 4;                 // epilogue warpgroups, one TMEM accumulator each
constexpr int THREADS = 64 + EPI_WGS * 128;  // warp 0 TMA, warp 1 MMA, then the epilogue
constexpr int MAX_REGS = 96;               // 18 warps: up to 5 per scheduler, 16K registers each
constexpr int SQ = 512;                    // settle queue entries per CTA (shared memory)
static_assert(THREADS > NB, "one thread per table bin plus one for the checks");
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// Rows whose fast-path result is not certain (a coordinate within kRiskBand of a
// decision boundary, or a norm within kNormBand of an fp16 rounding tie) are
// queued in shared memory, one entry per uncertain coordinate (or one norm-only
// entry), and settled with the exact float32 sequence by the whole CTA, one entry
// per thread, once its last tile is coded. Rows that need every coordinate settled
// (non-finite input, or no decision table), and rows that find the queue full, are
// settled whole by their epilogue thread at once.
struct FixEntry {
    uint32_t vi;    // vector index (token * heads + head) of the call
    uint32_t info;  // bits 0-6: coordinate; kHasCoord, kFixNorm, kFixAll, kSkip
    int64_t prow;   // pool row (slot * heads + head)
};
constexpr uint32_t kHasCoord = 1u << 8, kFixNorm = 1u << 9, kFixAll = 1u << 10, kSkip = 1u << 11;

struct Misc {
    uint64_t full[MAX_STAGES];
    uint64_t empty[MAX_STAGES];
    uint64_t tfull[EPI_WGS];
    uint64_t tempty[EPI_WGS];
    uint32_t tmem_base;
    int use_exact;  // table could not be built: every row takes the exact path
    float cen[256];
    float bin_mid[NB];      // per-bin table entry before it is copied LUT_COPIES times
    uint32_t bin_base[NB];
    uint32_t sq_tail;  // settle queue: positions reserved (entries at or past SQ are not stored)
    FixEntry sq[SQ];
};

// Byte offsets from the 1024-aligned base of dynamic shared memory.
struct Smem {
    static constexpr int a_off(int nparts) { return nparts * TILE_BYTES; }
    static constexpr int lut_off(int nparts) { return a_off(nparts) + stages_for(nparts) * TILE_BYTES; }
    static constexpr int misc_off(int nparts) { return lut_off(nparts) + NB * LUT_COPIES * 4; }
    static constexpr int bytes(int nparts) { return misc_off(nparts) + (int)sizeof(Misc) + 1024; }
};

// try_wait that may suspend the thread until the phase completes (or ~100 us pass), so a waiting
// warp does not spin through issue slots the epilogue warps of its scheduler need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with parity `parity`; false (and a counted timeout) if it never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (clock64() - t0 > kTimeoutCycles) {
            atomicAdd(&g_tq_umma_timeouts, 1u);
            if (err) atomicAdd(err, 1u);
            return false;
        }
    }
    return true;
}

// One 32-bit table entry per (bin, copy), the 32 copies of a bin side by side so that lane l
// reads copy l: one shared-memory wavefront per warp lookup. An entry is the bin's decision
// boundary m in y units (8.0: the bin holds none) with its low four mantissa bits replaced by
// the code below the boundary. That moves m by at most 15 units in the last place (under 2.3e-7
// for the |m| < 0.25 of 2- to 4-bit codebooks), far inside the settle band kRiskBand: a
// coordinate whose fast decision against the stored value could differ from the exact one is
// within the band of it and is settled exactly.
constexpr uint32_t kLutCodeMask = 15u;

// Correctly rounded x / den for fp16 x with |x| <= den, den in [1e-8, 2^20]: from the
// correctly rounded reciprocal r, two FMA corrections of the quotient (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000 processor", IBM J.
// Res. Dev. 34(1), 1990): q1 = q0 + (x - den q0) r is faithful, the remainder x - den q1
// is then exact and q1 + (x - den q1) r is the rounded quotient. Branch-free, so the
// quotients of a row pipeline. (Checked against exact rational arithmetic on the domain.)
__device__ __forceinline__ float quot_rn(float x, float den, float r) {
    const float q0 = __fmul_rn(x, r);
    const float q1 = __fmaf_rn(__fmaf_rn(-q0, den, x), r, q0);
    return __fmaf_rn(__fmaf_rn(-q1, den, x), r, q1);
}

// Exact float32 statement for one queued row, by one thread, on the stored bytes:
// the sequential sum of the squares (norm), then for each listed coordinate the
// sequential sum of Pi[i][j] * (x_j / (norm + 1e-8)) and the first-minimum nearest
// centroid, patched into the row's bit stream. Loads are 16-byte vectors; the
// input row stays in L1 across the coordinates.
template <typename TIn, int BITS>
__device__ __forceinline__ void settle_row_inline(const TqArgs& a, int64_t vi, int64_t prow, uint32_t flags,
                                               uint32_t m0, uint32_t m1, uint32_t m2, uint32_t m3, const float* cen) {
    constexpr int EPV = 16 / sizeof(TIn);  // elements per 16-byte vector
    const int nlev = 1 << BITS;
    const int P = (D * BITS) >> 3;
    const uint4* xr = (const uint4*)((const TIn*)a.input + vi * D);
    float s = 0.0f;
#pragma unroll 4
    for (int c = 0; c < D / EPV; ++c) {
        Vec16<TIn> u;
        u.u = __ldg(xr + c);
#pragma unroll
        for (int e = 0; e < EPV; ++e) {
            const float x = to_f32(u.e[e]);
            s = __fadd_rn(s, __fmul_rn(x, x));
        }
    }
    const float norm = __fsqrt_rn(s);
    if (flags & kFixNorm) ((__half*)a.norms_pool)[prow] = __float2half_rn(norm);
    const float den = __fadd_rn(norm, 1e-8f);
    uint8_t* row = (uint8_t*)a.packed_pool + prow * P;
    for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t m = (flags & kFixAll) ? 0xffffffffu : (c4 == 0 ? m0 : c4 == 1 ? m1 : c4 == 2 ? m2 : m3);
        while (m) {
            const int i = c4 * 32 + __ffs(m) - 1;
            m &= m - 1;
            const float4* pr = (const float4*)(a.rotation + i * D);
            float y = 0.0f;
#pragma unroll 2
            for (int c = 0; c < D / EPV; ++c) {
                Vec16<TIn> u;
                u.u = __ldg(xr + c);
#pragma unroll
                for (int e4 = 0; e4 < EPV / 4; ++e4) {
                    const float4 p = __ldg(pr + c * (EPV / 4) + e4);
                    y = __fadd_rn(y, __fmul_rn(p.x, __fdiv_rn(to_f32(u.e[4 * e4 + 0]), den)));
                    y = __fadd_rn(y, __fmul_rn(p.y, __fdiv_rn(to_f32(u.e[4 * e4 + 1]), den)));
                    y = __fadd_rn(y, __fmul_rn(p.z, __fdiv_rn(to_f32(u.e[4 * e4 + 2]), den)));
                    y = __fadd_rn(y, __fmul_rn(p.w, __fdiv_rn(to_f32(u.e[4 * e4 + 3]), den)));
                }
            }
            const uint32_t code = (uint32_t)nearest_centroid(y, cen, nlev);
            for (int b = 0; b < BITS; ++b) {
                const int bp = i * BITS + b;
                const uint8_t bit = (uint8_t)(0x80u >> (bp & 7));
                row[bp >> 3] = ((code >> (BITS - 1 - b)) & 1u) ? (uint8_t)(row[bp >> 3] | bit) : (uint8_t)(row[bp >> 3] & ~bit);
            }
        }
    }
}

// One queued entry, by one thread: the sequential sum of the row's
// squares (norm, rewritten when flagged), then for the entry's coordinate i the sequential
// sum of Pi[i][j] * (x_j / (norm + 1e-8)) and the first-minimum nearest centroid, whose bits
// are patched into the pool row with word atomics (entries of one row patch disjoint bits;
// threads may hold entries of the same row). FP16 inputs take the corrected-reciprocal quotient.
template <typename TIn, int BITS>
__device__ __forceinline__ void settle_entry(const TqArgs& a, const FixEntry& en, const float* cen) {
    constexpr int EPV = 16 / sizeof(TIn);  // elements per 16-byte vector
    const int nlev = 1 << BITS;
    const int P = (D * BITS) >> 3;
    const uint4* xr = (const uint4*)((const TIn*)a.input + (int64_t)en.vi * D);
    const int i = (int)(en.info & 127u);
    const float4* pr = (const float4*)(a.rotation + i * D);
    // the row and, for a coordinate, its rotation row into L1 at once: the sums below then
    // wait on one memory round trip instead of one per load
#pragma unroll
    for (int l = 0; l < D * (int)sizeof(TIn) / 128; ++l)
        asm volatile("prefetch.global.L1 [%0];" ::"l"((const char*)xr + 128 * l));
    if (en.info & kHasCoord) {
#pragma unroll
        for (int l = 0; l < D * 4 / 128; ++l) asm volatile("prefetch.global.L1 [%0];" ::"l"((const char*)pr + 128 * l));
    }
    float s = 0.0f;
#pragma unroll 4
    for (int c = 0; c < D / EPV; ++c) {
        Vec16<TIn> u;
        u.u = __ldg(xr + c);
#pragma unroll
        for (int e = 0; e < EPV; ++e) {
            const float x = to_f32(u.e[e]);
            s = __fadd_rn(s, __fmul_rn(x, x));
        }
    }
    const float norm = __fsqrt_rn(s);
    if (en.info & kFixNorm) ((__half*)a.norms_pool)[en.prow] = __float2half_rn(norm);
    if (!(en.info & kHasCoord)) return;
    const float den = __fadd_rn(norm, 1e-8f);
    const float r = __frcp_rn(den);
    float y = 0.0f;
#pragma unroll 2
    for (int c = 0; c < D / EPV; ++c) {
        Vec16<TIn> u;
        u.u = __ldg(xr + c);
#pragma unroll
        for (int e4 = 0; e4 < EPV / 4; ++e4) {
            const float4 p = __ldg(pr + c * (EPV / 4) + e4);
            const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float x = to_f32(u.e[4 * e4 + k]);
                const float qn = dtype_of<TIn>::value == FB_FP16 ? quot_rn(x, den, r) : __fdiv_rn(x, den);
                y = __fadd_rn(y, __fmul_rn(pv[k], qn));
            }
        }
    }
    const uint32_t code = (uint32_t)nearest_centroid(y, cen, nlev);
    uint32_t* roww = (uint32_t*)((uint8_t*)a.packed_pool + en.prow * P);
    for (int b = 0; b < BITS; ++b) {
        // MSB-first stream bit bp lives in byte bp >> 3 at bit 7 - (bp & 7); bytes little-endian in words
        const int bp = i * BITS + b;
        const int byte = bp >> 3;
        const uint32_t bit = 1u << (8 * (byte & 3) + 7 - (bp & 7));
        if ((code >> (BITS - 1 - b)) & 1u) atomicOr(roww + (byte >> 2), bit);
        else atomicAnd(roww + (byte >> 2), ~bit);
    }
}

// One packing word of codes (16 for 2 bits, else 8) in stream order. 4-bit: 8 codes, byte k =
// (c[2k] << 4) | c[2k+1] with bytes little-endian, so the word is stored as is; 2-bit: 16 codes,
// byte k = c[4k] .. c[4k+3] MSB first; 3-bit: 8 codes as a 24-bit value, first code on top.
template <int BITS>
__device__ __forceinline__ uint32_t pack_codes(const uint32_t (&c)[BITS == 2 ? 16 : 8]) {
    if constexpr (BITS == 4) {
        uint32_t b[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) b[k] = c[2 * k] * 16u + c[2 * k + 1];
        return ((b[3] * 256u + b[2]) * 256u + b[1]) * 256u + b[0];
    } else if constexpr (BITS == 2) {
        uint32_t b[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) b[k] = ((c[4 * k] * 4u + c[4 * k + 1]) * 4u + c[4 * k + 2]) * 4u + c[4 * k + 3];
        return ((b[3] * 256u + b[2]) * 256u + b[1]) * 256u + b[0];
    } else {
        uint32_t v = c[0];
#pragma unroll
        for (int q = 1; q < 8; ++q) v = v * 8u + c[q];
        return v;
    }
}

// One compress call of a launch, served by CTAs [cta0, cta0 + ncta) of the grid.
struct TqJob {
    TqArgs a;
    int num_tiles;
    int cta0, ncta;
    DivU32 hdiv;  // division by num_heads
};

// The kernel's parameters: one or two calls (njobs) with their input tensor maps.
struct TqLaunch {
    CUtensorMap map[2];
    TqJob job[2];
    int njobs;
};

// The work of one CTA for job `jb`: CTA `cta` of the job's `ncta` takes tiles cta, cta + ncta, ...
template <typename TIn, int NPARTS, int BITS>
__device__ __forceinline__ void compress_cta(const CUtensorMap* tmap_p, const TqJob& jb) {
    constexpr int STAGES = stages_for(NPARTS);
    const TqArgs& a = jb.a;
    const int num_tiles = jb.num_tiles;
    const int cta = (int)blockIdx.x - jb.cta0, ncta = jb.ncta;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array, so that the compiler still
    // knows every pointer derived from it addresses shared memory (plain ld/st.shared)
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sB = base;
    uint8_t* sA = base + Smem::a_off(NPARTS);
    uint32_t* lut = (uint32_t*)(base + Smem::lut_off(NPARTS));
    Misc* misc = (Misc*)(base + Smem::misc_off(NPARTS));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nlev = 1 << BITS;

    const int ntiles_cta = num_tiles > cta ? (num_tiles - 1 - cta) / ncta + 1 : 0;
    const int prefetched = ntiles_cta < STAGES ? ntiles_cta : STAGES;

    // ── prologue ─────────────────────────────────────────────────────────────
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         smem_u32(&misc->tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&misc->full[s], 1);
            mbar_init(&misc->empty[s], 1);
        }
        for (int b = 0; b < EPI_WGS; ++b) {
            mbar_init(&misc->tfull[b], 1);
            mbar_init(&misc->tempty[b], 4);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        misc->use_exact = 0;
        misc->sq_tail = 0u;
        // The first tiles are requested now, so their loads overlap the set-up below.
        for (int i = 0; i < prefetched; ++i) {
            const int tile = cta + i * ncta;
            mbar_expect_tx(&misc->full[i], TILE_BYTES);
            tma_load_2d(sA + i * TILE_BYTES, tmap_p, &misc->full[i], 0, tile * TILE);
            tma_load_2d(sA + i * TILE_BYTES + KBLK_BYTES, tmap_p, &misc->full[i], 64, tile * TILE);
        }
    }
    for (int e = threadIdx.x; e < nlev; e += THREADS) misc->cen[e] = __ldg(a.centroids + e);
    // B operand: Pi split into NPARTS parts (hi + lo [+ lo2]) in the SW128 K-major image. A
    // thread's loads of Pi (four pairs of 16 bytes at most) are all in flight before it splits.
    {
        constexpr int PER = (D * D / 8 + THREADS - 1) / THREADS;
        float4 pv[PER][2];
#pragma unroll
        for (int q = 0; q < PER; ++q) {
            const int c = threadIdx.x + q * THREADS;
            if (c < D * D / 8) {
                const int n = c >> 4, k0 = (c & 15) << 3;
                pv[q][0] = __ldg((const float4*)(a.rotation + n * D + k0));
                pv[q][1] = __ldg((const float4*)(a.rotation + n * D + k0 + 4));
            }
        }
#pragma unroll
        for (int q = 0; q < PER; ++q) {
            const int c = threadIdx.x + q * THREADS;
            if (c >= D * D / 8) break;
            const int n = c >> 4, k0 = (c & 15) << 3;
            float rem[8] = {pv[q][0].x, pv[q][0].y, pv[q][0].z, pv[q][0].w,
                            pv[q][1].x, pv[q][1].y, pv[q][1].z, pv[q][1].w};
#pragma unroll
            for (int p = 0; p < NPARTS; ++p) {
                Vec16<TIn> v;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    v.e[e] = from_f32<TIn>(rem[e]);
                    rem[e] = rem[e] - to_f32(v.e[e]);
                }
                *(uint4*)(sB + p * TILE_BYTES + sw128_offset(n, k0)) = v.u;
            }
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();

    // Decision table: boundaries m_k = (c_k + c_{k+1}) / 2, must be increasing, inside
    // the table range and farther apart than one bin plus the bands (thread NB checks).
    // Bin b covers y in [(b - kBin0 - 1/2) w, (b - kBin0 + 1/2) w) and owns the one
    // boundary within kWindowPad of that interval, if any (threads 0..NB-1, one bin
    // each); then every thread copies entries into the LUT_COPIES copies.
    {
        const float w = 1.0f / kInvW;
        if (threadIdx.x == NB) {
            bool ok = true;
            for (int k = 0; k + 1 < nlev; ++k) {
                const float m = 0.5f * (misc->cen[k] + misc->cen[k + 1]);
                if (!(misc->cen[k + 1] > misc->cen[k]) || !(fabsf(m) < 0.9f)) ok = false;
                if (k > 0) {
                    const float mp = 0.5f * (misc->cen[k - 1] + misc->cen[k]);
                    if (!(m - mp > w + 2.0f * kWindowPad + 4.0f * kRiskBand)) ok = false;
                }
            }
            if (!ok) misc->use_exact = 1;
        }
        if (threadIdx.x < NB) {
            const int bin = threadIdx.x;
            const float ylo = ((float)(bin - kBin0) - 0.5f) * w, yhi = ((float)(bin - kBin0) + 0.5f) * w;
            int below = 0, owner = -1;
            for (int k = 0; k + 1 < nlev; ++k) {
                const float m = 0.5f * (misc->cen[k] + misc->cen[k + 1]);
                if (m < ylo - kWindowPad) below = k + 1;
                if (m >= ylo - kWindowPad && m <= yhi + kWindowPad) owner = k;
            }
            misc->bin_mid[bin] = owner >= 0 ? 0.5f * (misc->cen[owner] + misc->cen[owner + 1]) : 8.0f;
            misc->bin_base[bin] = owner >= 0 ? (uint32_t)owner : (uint32_t)below;
        }
        __syncthreads();
        for (int e = threadIdx.x; e < NB * LUT_COPIES; e += THREADS)
            lut[e] = (__float_as_uint(misc->bin_mid[e / LUT_COPIES]) & ~kLutCodeMask) | misc->bin_base[e / LUT_COPIES];
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = misc->tmem_base;
    const int use_exact = misc->use_exact;
    unsigned int* err = a.err_count;

    if (warp == 0) {
        // ── TMA producer ────────────────────────────────────────────────────
        if (lane == 0) {
            int issued = prefetched;
            for (int i = prefetched; i < ntiles_cta; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&misc->empty[s], ((i / STAGES) + 1) & 1, err)) break;
                const int tile = cta + i * ncta;
                mbar_expect_tx(&misc->full[s], TILE_BYTES);
                tma_load_2d(sA + s * TILE_BYTES, tmap_p, &misc->full[s], 0, tile * TILE);
                tma_load_2d(sA + s * TILE_BYTES + KBLK_BYTES, tmap_p, &misc->full[s], 64, tile * TILE);
                ++issued;
            }
            // Loads still in flight land before the CTA exits.
            for (int i = std::max(0, issued - STAGES); i < issued; ++i)
                mbar_wait(&misc->full[i % STAGES], (i / STAGES) & 1, err);
        }
    } else if (warp == 1) {
        // ── MMA issuer ──────────────────────────────────────────────────────
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(sizeof(TIn) == 2 && dtype_of<TIn>::value == FB_BF16 ? 1u : 0u);
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            int done = 0;
            for (int i = 0; i < ntiles_cta; ++i) {
                const int s = i % STAGES, buf = i % EPI_WGS;
                if (!mbar_wait(&misc->full[s], (i / STAGES) & 1, err)) break;
                if (!mbar_wait(&misc->tempty[buf], ((i / EPI_WGS) + 1) & 1, err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * D);
                uint32_t acc = 0;
#pragma unroll
                for (int p = 0; p < NPARTS; ++p)
#pragma unroll
                    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t off = kb * KBLK_BYTES + k * 32;
                            mma_f16(d, sw128_desc(a0 + s * TILE_BYTES + off), sw128_desc(b0 + p * TILE_BYTES + off), idesc,
                                 acc);
                            acc = 1;
                        }
                umma_commit(&misc->empty[s]);
                umma_commit(&misc->tfull[buf]);
                done = i + 1;
            }
            // The last accumulations finish before TMEM is released.
            if (done > 0) mbar_wait(&misc->tfull[(done - 1) % EPI_WGS], ((done - 1) / EPI_WGS) & 1, err);
        }
    } else {
        // ── epilogue: warps 2.., warpgroup eg handles tiles i with i % EPI_WGS == eg ──
        const int eg = (warp - 2) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int P = (D * BITS) >> 3;
        const float magic = 12582912.0f;  // 1.5 * 2^23: fma(y, 1/w, magic + kBin0) holds the bin in its low bits
        const float ubias = magic + (float)kBin0;
        const uint32_t lut_lane = smem_u32(lut) + lane * 4u - (uint32_t)__float_as_uint(magic) * (LUT_COPIES * 4u);
        const int64_t nvec = a.num_tokens * a.num_heads;
        constexpr int G = (BITS == 2) ? 16 : 8;  // codes per packing word
        constexpr int CW = 16;                    // accumulator columns per TMEM load in the coding pass
        constexpr int NCH = D / CW;               // chunks per row
        constexpr int WPC = CW / G;               // packing words per chunk
        // Pool rows in two steps so that no wait falls on a load: raw_of(i) issues the slot-map or
        // block-table read for this thread's vector of tile i (kNoVec: no vector), a tile ahead of its
        // use; prow_of applies the slot rule of tq_slot to it (-1: no row; err_count bumped for a
        // slot out of range). Token and head by multiply-high division (the host keeps the vector
        // count below 2^31).
        constexpr int64_t kNoVec = INT64_MIN;  // a slot-map entry may itself be negative
        auto raw_of = [&](int i) -> int64_t {
            const int64_t v = (int64_t)(cta + i * ncta) * TILE + row;
            if (i >= ntiles_cta || v >= nvec) return kNoVec;
            const uint32_t t = divu32((uint32_t)v, jb.hdiv);
            if (a.slot_map) return __ldg(a.slot_map + t);
            if (a.block_table) return (int64_t)(uint32_t)__ldg(a.block_table + ((a.start_pos + t) >> 4));
            return 0;
        };
        auto prow_of = [&](int i, int64_t raw) -> int64_t {
            if (raw == kNoVec) return -1;
            const uint32_t v = (uint32_t)((cta + i * ncta) * TILE + row);
            const uint32_t t = divu32(v, jb.hdiv), head = v - t * (uint32_t)a.num_heads;
            const int64_t pos = a.start_pos + t;
            int64_t slot = pos;
            if (a.slot_map) {
                slot = raw;
            } else if (a.block_table) {
                const int32_t b = (int32_t)(uint32_t)raw;
                slot = b < 0 ? -1 : (int64_t)b * 16 + (pos & 15);
            }
            if (slot < 0 || slot >= a.pool_rows) {
                if (a.err_count) atomicAdd(a.err_count, 1u);
                return -1;
            }
            return slot * a.num_heads + head;
        };
        int64_t raw_next = raw_of(eg);
        for (int i = eg; i < ntiles_cta; i += EPI_WGS) {
            const int tile = cta + i * ncta;
            const int64_t vi = (int64_t)tile * TILE + row;
            const int64_t raw = raw_next;
            raw_next = raw_of(i + EPI_WGS);
            if (!mbar_wait(&misc->tfull[eg], (i / EPI_WGS) & 1, err)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (uint32_t)(eg * D) + ((uint32_t)(quarter * 32) << 16);
            // Pass 1: |Pi x|^2 = |x|^2 from the accumulator row, 16-column chunks with the next three
            // loads in flight while one is summed (paired FMAs; the exact norm is settled where
            // needed).
            float2 s2[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
            {
                constexpr int NB1 = 4;  // load buffers
                uint32_t xb[NB1][CW];
#pragma unroll
                for (int h = 0; h < NB1 - 1; ++h) tmem_ld16_issue(taddr + h * CW, xb[h]);
#pragma unroll
                for (int h = 0; h < NCH; ++h) {
                    tmem_wait_one(xb[h % NB1]);
                    if (h + NB1 - 1 < NCH) tmem_ld16_issue(taddr + (h + NB1 - 1) * CW, xb[(h + NB1 - 1) % NB1]);
#pragma unroll
                    for (int j = 0; j < CW / 2; ++j) {
                        const float2 v2 = make_float2(__uint_as_float(xb[h % NB1][2 * j]), __uint_as_float(xb[h % NB1][2 * j + 1]));
                        s2[j & 1] = __ffma2_rn(v2, v2, s2[j & 1]);
                    }
                }
            }
            const float ss = (s2[0].x + s2[0].y) + (s2[1].x + s2[1].y);
            // zero vector: y = 0 exactly for every coordinate in both statements, so the table
            // codes it exactly (the lower code at a boundary that is exactly 0, the statement's first
            // minimum); no coordinate of it needs settling
            const bool zero = ss == 0.0f;
            const bool finite = ss <= 3.402823466e38f;  // NaN or inf: the row takes the exact path
            if (__any_sync(0xffffffffu, !finite)) {
                // rare: a row of this warp holds NaN/inf (its accumulator values are not finite).
                // Its accumulator row is overwritten with zeros so that every table index of the
                // coding pass stays in range; the row is settled whole by the exact path below.
                uint32_t z[CW];
#pragma unroll 1
                for (int c = 0; c < NCH; ++c) {
                    tmem_ld16_issue(taddr + c * CW, z);
                    tmem_wait_tie(z);
#pragma unroll
                    for (int j = 0; j < CW; ++j) z[j] = finite ? z[j] : 0u;
                    tmem_st16(taddr + c * CW, z);
                }
                tmem_wait_st();
            }
            const int64_t prow = prow_of(i, raw);
            uint8_t* dst = prow >= 0 ? (uint8_t*)a.packed_pool + prow * P : nullptr;
            const float norm_f = sqrtf(ss);
            const float kr = finite ? __frcp_rn(norm_f + 1e-8f) : 0.0f;  // y = acc * kr
            const float ku = kr * kInvW;
            const float2 ku2 = make_float2(ku, ku), ub2 = make_float2(ubias, ubias);
            const bool norm_amb =
                __float2half_rn(norm_f * (1.0f - kNormBand)) != __float2half_rn(norm_f * (1.0f + kNormBand));
            // Pass 2, codes: chunks 0..NCH-1, the next load in flight while one is coded; two
            // chunks (one 32-coordinate round) are coded and stored per loop iteration. Per coordinate: its table bin
            // from the rounded fma(acc, ku, ubias) (two coordinates per paired FMA), the bin's
            // entry (boundary m, lower code in its low bits), dd = m - y, code = lower + (y > m)
            // from the sign of dd, packed big-endian (first code in the top bits) by integer
            // multiply-add; the running minimum of |dd| flags the rare chunk to list for the exact
            // settle. The accumulator goes back to the MMA warp once the last chunk is loaded.
            uint32_t mask[4] = {0u, 0u, 0u, 0u};
            uint32_t w[2 * WPC];
            uint32_t ra[CW], rb[CW];
            // one chunk: code its 16 coordinates into w[half * WPC ..], return whether a lane's
            // coordinate lies within the settle band (and list those coordinates in mk)
            auto code_chunk = [&](const uint32_t (&cur)[CW], int half, uint32_t& mk) {
                float dm[2] = {1.0f, 1.0f};
#pragma unroll
                for (int w2 = 0; w2 < WPC; ++w2) {
                    uint32_t code[G];
#pragma unroll
                    for (int q = 0; q < G; q += 2) {
                        const float2 v2 = make_float2(__uint_as_float(cur[w2 * G + q]), __uint_as_float(cur[w2 * G + q + 1]));
                        const float2 u2 = __ffma2_rn(v2, ku2, ub2);
                        const uint32_t addr0 = __float_as_uint(u2.x) * (LUT_COPIES * 4u) + lut_lane;
                        const uint32_t addr1 = __float_as_uint(u2.y) * (LUT_COPIES * 4u) + lut_lane;
                        uint32_t e0, e1;
                        asm("ld.shared.b32 %0, [%1];" : "=r"(e0) : "r"(addr0));
                        asm("ld.shared.b32 %0, [%1];" : "=r"(e1) : "r"(addr1));
                        const float dd0 = fmaf(-v2.x, kr, __uint_as_float(e0));
                        const float dd1 = fmaf(-v2.y, kr, __uint_as_float(e1));
                        float& m = dm[(q >> 1) & 1];
                        asm("min.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(m), "f"(fabsf(dd0)), "f"(fabsf(dd1)));
                        code[q] = (e0 & kLutCodeMask) + (__float_as_uint(dd0) >> 31);
                        code[q + 1] = (e1 & kLutCodeMask) + (__float_as_uint(dd1) >> 31);
                    }
                    // the word as stored: byte k holds codes of stream order MSB first, bytes
                    // little-endian (4-bit: byte k = c[2k] c[2k+1]; 2-bit: c[4k] .. c[4k+3];
                    // 3-bit: a 24-bit big-endian group, laid out by the caller)
                    w[half * WPC + w2] = pack_codes<BITS>(code);
                }
                mk = 0;
                if (fminf(dm[0], dm[1]) < kRiskBand && !zero) {
                    // rare: list this chunk's coordinates within the band
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        const float v = __uint_as_float(cur[j]);
                        const float u = fmaf(v, ku, ubias);
                        uint32_t e;
                        asm("ld.shared.b32 %0, [%1];" : "=r"(e) : "r"(__float_as_uint(u) * (LUT_COPIES * 4u) + lut_lane));
                        if (fabsf(fmaf(-v, kr, __uint_as_float(e))) < kRiskBand) mk |= 1u << j;
                    }
                }
            };
            // rounds g = 0 .. NCH/2-1 of two chunks, rolled so the hot loop stays small in the
            // instruction cache; chunk 2g is in ra, 2g + 1 in rb
            tmem_ld16_issue(taddr, ra);
#pragma unroll 1
            for (int g = 0; g < NCH / 2; ++g) {
                uint32_t mk0, mk1;
                tmem_wait_tie(ra);
                tmem_ld16_issue(taddr + (2 * g + 1) * CW, rb);
                code_chunk(ra, 0, mk0);
                tmem_wait_tie(rb);
                if (g + 1 < NCH / 2) {
                    tmem_ld16_issue(taddr + (2 * g + 2) * CW, ra);
                } else {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&misc->tempty[eg]);
                }
                code_chunk(rb, 1, mk1);
                const uint32_t mm = mk0 | (mk1 << CW);
                if (mm) {
                    if (g == 0) mask[0] = mm;
                    else if (g == 1) mask[1] = mm;
                    else if (g == 2) mask[2] = mm;
                    else mask[3] = mm;
                }
                if (dst) {
                    if constexpr (BITS == 4) {
                        *(uint4*)(dst + 16 * g) = make_uint4(w[0], w[1], w[2], w[3]);
                    } else if constexpr (BITS == 2) {
                        *(uint2*)(dst + 8 * g) = make_uint2(w[0], w[1]);
                    } else {
                        // 3-bit: each word holds 24 stream bits (bits 23..0, first code on top)
                        uint32_t* d3 = (uint32_t*)(dst + 12 * g);
                        d3[0] = __byte_perm(w[0], w[1], 0x6012);  // w0.b2 w0.b1 w0.b0 w1.b2
                        d3[1] = __byte_perm(w[1], w[2], 0x5601);  // w1.b1 w1.b0 w2.b2 w2.b1
                        d3[2] = __byte_perm(w[2], w[3], 0x4560);  // w2.b0 w3.b2 w3.b1 w3.b0
                    }
                }
            }
            if (prow < 0) continue;
            ((__half*)a.norms_pool)[prow] = __float2half_rn(norm_f);
            const uint32_t flags = ((norm_amb && !zero) ? kFixNorm : 0u) |
                                   ((use_exact || !finite) ? kFixAll | kFixNorm : 0u);
            if (!finite) mask[0] = mask[1] = mask[2] = mask[3] = 0u;
            const uint32_t ncoord = __popc(mask[0]) + __popc(mask[1]) + __popc(mask[2]) + __popc(mask[3]);
            if (flags & kFixAll) {
                // rare: a non-finite row, or no decision table; settled whole here
                settle_row_inline<TIn, BITS>(a, vi, prow, flags, 0u, 0u, 0u, 0u, misc->cen);
            } else if (flags || ncoord) {
                // one entry per listed coordinate (the first also carries the norm flag), or a
                // norm-only entry; settled after the last tile (the row's stores above stay first)
                const uint32_t nent = ncoord == 0 ? 1u : ncoord;
                const uint32_t q0 = atomicAdd(&misc->sq_tail, nent);
                if (q0 + nent > (uint32_t)SQ) {
                    // queue full: void the slots reserved below SQ and settle the row here
                    for (uint32_t q = q0; q < (uint32_t)SQ; ++q) misc->sq[q] = FixEntry{0u, kSkip, 0};
                    settle_row_inline<TIn, BITS>(a, vi, prow, flags, mask[0], mask[1], mask[2], mask[3], misc->cen);
                } else if (ncoord == 0) {
                    misc->sq[q0] = FixEntry{(uint32_t)vi, flags, prow};
                } else {
                    uint32_t k = 0, nf = flags;
#pragma unroll 1
                    for (int c4 = 0; c4 < 4; ++c4) {
                        uint32_t m = mask[c4];
                        while (m) {
                            const uint32_t ci = (uint32_t)(c4 * 32 + __ffs(m) - 1);
                            m &= m - 1;
                            misc->sq[q0 + k] = FixEntry{(uint32_t)vi, ci | kHasCoord | nf, prow};
                            nf = 0;
                            ++k;
                        }
                    }
                }
            }
        }
    }

    // Every tile is coded and stored: the queued entries, one per thread.
    __syncthreads();
    {
        const uint32_t nq = min(misc->sq_tail, (uint32_t)SQ);
        for (uint32_t e = threadIdx.x; e < nq; e += THREADS) {
            const FixEntry en = misc->sq[e];
            if (!(en.info & kSkip)) settle_entry<TIn, BITS>(a, en, misc->cen);
        }
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem_base) : "memory");
    }
}

// B0 / B1: code widths of job 0 / job 1 (equal for a single call, or for K and V of one width).
template <typename TIn, int NPARTS, int B0, int B1>
__global__ void __maxnreg__(MAX_REGS)
    tq_compress_umma_kernel(const __grid_constant__ TqLaunch L) {
    const int j = (L.njobs > 1 && (int)blockIdx.x >= L.job[1].cta0) ? 1 : 0;
    if constexpr (B0 == B1) {
        compress_cta<TIn, NPARTS, B0>(&L.map[j], L.job[j]);
    } else {
        if (j == 0) compress_cta<TIn, NPARTS, B0>(&L.map[0], L.job[0]);
        else compress_cta<TIn, NPARTS, B1>(&L.map[1], L.job[1]);
    }
}

}  // namespace umma

// ── host side ───────────────────────────────────────────────────────────────

static bool device_is_sm100() {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    return major == 10 && minor == 0;
}

static bool encode_input_map(CUtensorMap* map, const TqArgs& a, bool bf16) {
    auto encode = sm100::tensor_map_encoder();
    if (!encode) return false;
    const int64_t nvec = a.num_tokens * a.num_heads;
    const cuuint64_t dims[2] = {(cuuint64_t)umma::D, (cuuint64_t)nvec};
    const cuuint64_t strides[1] = {(cuuint64_t)umma::D * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)umma::TILE};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(a.input), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches jobs[0..njobs) (njobs 1 or 2) as one grid of at most one CTA per SM, split between
// the jobs in proportion to their tiles (each job at least one CTA, at most one per tile).
template <typename TIn, int NPARTS, int B0, int B1>
static int launch_umma(const TqArgs* jobs, int njobs, cudaStream_t s) {
    umma::TqLaunch L;
    memset(&L, 0, sizeof L);
    L.njobs = njobs;
    int64_t tiles[2] = {0, 0};
    for (int j = 0; j < njobs; ++j) {
        if (!encode_input_map(&L.map[j], jobs[j], dtype_of<TIn>::value == FB_BF16)) return (int)cudaErrorInvalidValue;
        L.job[j].a = jobs[j];
        L.job[j].hdiv = sm100::make_divu32((uint32_t)jobs[j].num_heads);
        tiles[j] = (jobs[j].num_tokens * jobs[j].num_heads + umma::TILE - 1) / umma::TILE;
        L.job[j].num_tiles = (int)tiles[j];
    }
    const int sms = num_sms();
    int n0 = (int)std::min<int64_t>(tiles[0], sms), n1 = 0;
    if (njobs == 2) {
        if (tiles[0] + tiles[1] <= sms) {
            n0 = (int)tiles[0];
            n1 = (int)tiles[1];
        } else {
            n0 = (int)((tiles[0] * sms + (tiles[0] + tiles[1]) / 2) / (tiles[0] + tiles[1]));
            n0 = std::max(1, std::min(n0, sms - 1));
            n1 = sms - n0;
            n0 = (int)std::min<int64_t>(n0, tiles[0]);
            n1 = (int)std::min<int64_t>(n1, tiles[1]);
        }
    }
    L.job[0].cta0 = 0;
    L.job[0].ncta = n0;
    L.job[1].cta0 = n0;
    L.job[1].ncta = n1;
    constexpr int smem = umma::Smem::bytes(NPARTS);
    auto kern = umma::tq_compress_umma_kernel<TIn, NPARTS, B0, B1>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    kern<<<std::max(1, n0 + n1), umma::THREADS, smem, s>>>(L);
    return (int)cudaGetLastError();
}

static bool umma_eligible(const TqArgs& a) {
    if (a.head_dim != umma::D || !(a.bits == 2 || a.bits == 3 || a.bits == 4)) return false;
    if (a.in_dtype != FB_FP16 && a.in_dtype != FB_BF16) return false;
    if (!aligned16(a.input) || !aligned16(a.packed_pool) || (((uintptr_t)a.norms_pool) & 1)) return false;
    if (((uintptr_t)a.rotation & 15) != 0) return false;
    if (a.num_tokens * a.num_heads > ((int64_t)1 << 31) - umma::TILE) return false;
    static const bool sm100 = device_is_sm100();  // thread-safe one-time initialisation
    return sm100;
}

template <typename TIn, int NPARTS>
static int launch_same_bits(const TqArgs* jobs, int njobs, int bits, cudaStream_t s) {
    if (bits == 4) return launch_umma<TIn, NPARTS, 4, 4>(jobs, njobs, s);
    if (bits == 3) return launch_umma<TIn, NPARTS, 3, 3>(jobs, njobs, s);
    return launch_umma<TIn, NPARTS, 2, 2>(jobs, njobs, s);
}

int tq_compress_umma(const TqArgs& a, cudaStream_t s, bool* handled) {
    *handled = false;
    if (!umma_eligible(a)) return 0;
    *handled = true;
    if (a.in_dtype == FB_FP16) return launch_same_bits<__half, 2>(&a, 1, a.bits, s);
    return launch_same_bits<__nv_bfloat16, 3>(&a, 1, a.bits, s);
}

// K and V of one append in one launch, when both take the tensor-core path with the same input
// type and their widths are equal or 4/2 (the reference's default key/value widths).
int tq_compress_umma_pair(const TqArgs& k, const TqArgs& v, cudaStream_t s, bool* handled) {
    *handled = false;
    if (!umma_eligible(k) || !umma_eligible(v) || k.in_dtype != v.in_dtype) return 0;
    if (k.bits != v.bits && !(k.bits == 4 && v.bits == 2)) return 0;
    *handled = true;
    const TqArgs jobs[2] = {k, v};
    const bool pair42 = k.bits != v.bits;
    if (k.in_dtype == FB_FP16)
        return pair42 ? launch_umma<__half, 2, 4, 2>(jobs, 2, s) : launch_same_bits<__half, 2>(jobs, 2, k.bits, s);
    return pair42 ? launch_umma<__nv_bfloat16, 3, 4, 2>(jobs, 2, s)
                  : launch_same_bits<__nv_bfloat16, 3>(jobs, 2, k.bits, s);
}


}  // namespace fb

namespace fb {
unsigned int tq_dequant_timeouts();
unsigned int tqa_stream_timeouts();
unsigned int tqa_timeouts();
}

extern "C" unsigned int fb_tq_timeouts(void) {
    unsigned int v = 0;
    cudaMemcpyFromSymbol(&v, fb::g_tq_umma_timeouts, sizeof(v));
    return v + fb::tq_dequant_timeouts() + fb::tqa_stream_timeouts() + fb::tqa_timeouts();
}
