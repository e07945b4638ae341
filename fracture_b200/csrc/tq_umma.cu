// TurboQuant compress on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Replaces backends/fracture-cuda/kernels/turboquant_compress.cu:27-222 for
// head_dim 128 and 2/3/4-bit codes. One persistent CTA per SM streams tiles of
// 128 head vectors:
//
//   warp 0      TMA producer: [128 vectors x 128] fp16/bf16 tile -> smem (SW128)
//   warp 1      MMA issuer:   acc[v][i] = sum_j x[v][j] * Pi[i][j] on tcgen05,
//               Pi split into 2 fp16 (or 3 bf16) parts so the product is
//               float32-accurate while x stays exact; accumulator in TMEM
//   warps 2-9   epilogue, two warpgroups on alternating TMEM buffers: one
//               thread per vector reads its row of acc from TMEM, derives the
//               norm (|Pi x| = |x|), maps each coordinate to its code through
//               a lane-private boundary table, packs the MSB-first bit stream
//               and writes it straight into its paged-pool row.
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
#include <mutex>

#include "common.cuh"
#include "tq_common.cuh"

namespace fb {

__device__ unsigned int g_tq_umma_timeouts = 0;

namespace umma {

constexpr int D = 128;              // head_dim
constexpr int TILE = 128;           // vectors per tile
constexpr int STAGES = 3;           // A-tile pipeline depth
constexpr int KBLK_BYTES = TILE * 128;    // one K-block (64 elements) of a 128-row tile, SW128
constexpr int TILE_BYTES = 2 * KBLK_BYTES;  // 32 KB
constexpr int NB = 64;              // decision-table bins over [-kRange, kRange]
constexpr float kRange = 0.54f;
constexpr float kRiskBand = 1e-6f;   // |y - boundary| below this: settle with the exact sequence
constexpr float kNormBand = 1e-6f;  // relative band around fp16 rounding ties of the norm
constexpr float kWindowPad = 1e-4f; // a bin owns the boundaries within this distance of its edges
constexpr int EPI_WGS = 3;                 // epilogue warpgroups, one TMEM accumulator each
constexpr int THREADS = 64 + EPI_WGS * 128;  // warp 0 TMA, warp 1 MMA, then the epilogue
constexpr int VCH = 32;                    // accumulator values per thread per TMEM load round
constexpr int MAX_REGS = 128;              // 14 warps: at most 4 per scheduler, 16K registers each
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// Rows whose fast-path result is not certain (a coordinate within kRiskBand of a
// decision boundary, or a norm within kNormBand of an fp16 rounding tie) are
// queued here and settled by tq_fixup_kernel with the exact float32 sequence.
struct FixEntry {
    uint32_t vi;       // vector index (token * heads + head) of the call
    uint32_t flags;    // kFixNorm: rewrite the norm; kFixAll: every coordinate
    uint32_t mask[4];  // coordinates to recompute
};
constexpr uint32_t kFixNorm = 1u, kFixAll = 2u;

struct Misc {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[EPI_WGS];
    uint64_t tempty[EPI_WGS];
    uint32_t tmem_base;
    int use_exact;  // table could not be built: every row takes the exact path
    uint32_t zero_word; // packing word of a zero vector (every code = nearest centroid of 0)
    float cen[256];
};

// Byte offsets from the 1024-aligned base of dynamic shared memory.
struct Smem {
    static constexpr int a_off(int nparts) { return nparts * TILE_BYTES; }
    static constexpr int lut_off(int nparts) { return a_off(nparts) + STAGES * TILE_BYTES; }
    static constexpr int misc_off(int nparts) { return lut_off(nparts) + NB * 32 * 8; }
    static constexpr int bytes(int nparts) { return misc_off(nparts) + (int)sizeof(Misc) + 1024; }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with parity `parity`; false (and a counted timeout) if it never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kTimeoutCycles) {
            atomicAdd(&g_tq_umma_timeouts, 1u);
            if (err) atomicAdd(err, 1u);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: D f32, A/B fp16 (fmt 0) or bf16 (fmt 1), both K-major, M=128, N=128.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t fmt) {
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(D >> 3) << 17) | ((uint32_t)(TILE >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t set_ge(float a, float b) {
    uint32_t r;
    asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(r) : "f"(a), "f"(b));
    return r;  // 0xffffffff or 0
}

// One table entry per (bin, lane): lane-private copies keep the 32 lanes of a
// warp on 32 different banks. lo/hi are in t units (t = y / (2 R) + 0.5);
// hi's low 4 mantissa bits hold the code of the lower side of the bin's boundary.
struct LutEntry {
    float mid;      // boundary in t units (4.0: the bin holds no boundary)
    uint32_t base;  // code below the boundary (the code of the whole bin when mid = 4.0)
};

// Byte offset in the SW128 K-major image of element (row n, column k) of a
// 128 x 128 tile stored as two 64-column K-blocks.
__device__ __forceinline__ int sw128_offset(int n, int k) {
    const int kb = k >> 6, kk = k & 63;
    return kb * KBLK_BYTES + n * 128 + ((((kk >> 3) ^ (n & 7))) << 4) + ((kk & 7) << 1);
}

// Exact float32 statement for one queued row, by one thread, on the stored
// bytes (used when the fixup queue is full).
template <typename TIn, int BITS>
__device__ __forceinline__ void settle_row_inline(const TqArgs& a, int64_t vi, int64_t prow, uint32_t flags,
                                               uint32_t m0, uint32_t m1, uint32_t m2, uint32_t m3, const float* cen) {
    const int nlev = 1 << BITS;
    const int P = (D * BITS) >> 3;
    const TIn* xr = (const TIn*)a.input + vi * D;
    float s = 0.0f;
    for (int j = 0; j < D; ++j) {
        const float x = to_f32(xr[j]);
        s = __fadd_rn(s, __fmul_rn(x, x));
    }
    const float norm = __fsqrt_rn(s);
    if (flags & kFixNorm) ((__half*)a.norms_pool)[prow] = __float2half_rn(norm);
    const float den = __fadd_rn(norm, 1e-8f);
    uint8_t* row = (uint8_t*)a.packed_pool + prow * P;
    for (int c = 0; c < 4; ++c) {
        uint32_t m = (flags & kFixAll) ? 0xffffffffu : (c == 0 ? m0 : c == 1 ? m1 : c == 2 ? m2 : m3);
        while (m) {
            const int i = c * 32 + __ffs(m) - 1;
            m &= m - 1;
            float y = 0.0f;
            for (int j = 0; j < D; ++j) y = __fadd_rn(y, __fmul_rn(a.rotation[i * D + j], __fdiv_rn(to_f32(xr[j]), den)));
            const uint32_t code = (uint32_t)nearest_centroid(y, cen, nlev);
            for (int b = 0; b < BITS; ++b) {
                const int bp = i * BITS + b;
                const uint8_t bit = (uint8_t)(0x80u >> (bp & 7));
                row[bp >> 3] = ((code >> (BITS - 1 - b)) & 1u) ? (uint8_t)(row[bp >> 3] | bit) : (uint8_t)(row[bp >> 3] & ~bit);
            }
        }
    }
}

template <typename TIn, int NPARTS, int BITS>
__global__ void __maxnreg__(MAX_REGS)
    tq_compress_umma_kernel(const __grid_constant__ CUtensorMap tmap, TqArgs a, int num_tiles, FixEntry* fix,
                            unsigned int* fix_count, unsigned int fix_cap) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sB = base;
    uint8_t* sA = base + Smem::a_off(NPARTS);
    LutEntry* lut = (LutEntry*)(base + Smem::lut_off(NPARTS));
    Misc* misc = (Misc*)(base + Smem::misc_off(NPARTS));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nlev = 1 << BITS;
    const float inv2r = 1.0f / (2.0f * kRange);

    // ── prologue ─────────────────────────────────────────────────────────────
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
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         smem_u32(&misc->tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    for (int e = threadIdx.x; e < nlev; e += THREADS) misc->cen[e] = __ldg(a.centroids + e);
    // B operand: Pi split into NPARTS parts (hi + lo [+ lo2]) in the SW128 K-major image.
    for (int c = threadIdx.x; c < D * D / 8; c += THREADS) {
        const int n = c >> 4, k0 = (c & 15) << 3;
        float rem[8];
        const float4 p0 = __ldg((const float4*)(a.rotation + n * D + k0));
        const float4 p1 = __ldg((const float4*)(a.rotation + n * D + k0 + 4));
        rem[0] = p0.x; rem[1] = p0.y; rem[2] = p0.z; rem[3] = p0.w;
        rem[4] = p1.x; rem[5] = p1.y; rem[6] = p1.z; rem[7] = p1.w;
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
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();

    // Decision table (all threads): boundaries m_k = (c_k + c_{k+1}) / 2, must be
    // increasing, inside the table range and farther apart than one bin plus the bands.
    {
        const float w = 2.0f * kRange / (float)(NB - 1);
        bool ok = true;
        for (int k = 0; k + 1 < nlev; ++k) {
            const float m = 0.5f * (misc->cen[k] + misc->cen[k + 1]);
            if (!(misc->cen[k + 1] > misc->cen[k]) || !(fabsf(m) < kRange - 2.0f * w)) ok = false;
            if (k > 0) {
                const float mp = 0.5f * (misc->cen[k - 1] + misc->cen[k]);
                if (!(m - mp > w + 2.0f * kWindowPad + 4.0f * kRiskBand)) ok = false;
            }
        }
        for (int e = threadIdx.x; e < NB * 32; e += THREADS) {
            const int bin = e >> 5;
            const float ylo = -kRange + ((float)bin - 0.5f) * w, yhi = -kRange + ((float)bin + 0.5f) * w;
            int below = 0, owner = -1;
            for (int k = 0; k + 1 < nlev; ++k) {
                const float m = 0.5f * (misc->cen[k] + misc->cen[k + 1]);
                if (m < ylo - kWindowPad) below = k + 1;
                if (m >= ylo - kWindowPad && m <= yhi + kWindowPad) owner = k;
            }
            LutEntry en;
            if (owner >= 0) {
                const float m = 0.5f * (misc->cen[owner] + misc->cen[owner + 1]);
                en.mid = m * inv2r + 0.5f;
                en.base = (uint32_t)owner;
            } else {
                en.mid = 4.0f;
                en.base = (uint32_t)below;
            }
            lut[e] = en;
        }
        if (threadIdx.x == 0) {
            if (!ok) misc->use_exact = 1;
            const uint32_t cz = (uint32_t)nearest_centroid(0.0f, misc->cen, nlev);
            misc->zero_word = BITS == 4 ? cz * 0x11111111u : BITS == 2 ? cz * 0x55555555u : cz * 0x249249u;
        }
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = misc->tmem_base;
    const int use_exact = misc->use_exact;
    const uint32_t zero_word = misc->zero_word;
    const int ntiles_cta = num_tiles > (int)blockIdx.x ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    unsigned int* err = a.err_count;

    if (warp == 0) {
        // ── TMA producer ────────────────────────────────────────────────────
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < ntiles_cta; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&misc->empty[s], ((i / STAGES) + 1) & 1, err)) break;
                const int tile = (int)blockIdx.x + i * (int)gridDim.x;
                mbar_expect_tx(&misc->full[s], TILE_BYTES);
                tma_load_2d(sA + s * TILE_BYTES, &tmap, &misc->full[s], 0, tile * TILE);
                tma_load_2d(sA + s * TILE_BYTES + KBLK_BYTES, &tmap, &misc->full[s], 64, tile * TILE);
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
                            umma(d, sw128_desc(a0 + s * TILE_BYTES + off), sw128_desc(b0 + p * TILE_BYTES + off), idesc,
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
        const float magic = 12582912.0f;  // 1.5 * 2^23: fma(t, NB-1, magic) holds round(t*(NB-1)) in its low bits
        const uint32_t lut_lane = smem_u32(lut) + lane * 8 - (uint32_t)__float_as_uint(magic) * 256u;
        const int64_t nvec = a.num_tokens * a.num_heads;
        constexpr int G = (BITS == 2) ? 16 : 8;  // codes per packing word
        constexpr int WPR = VCH / G;              // packing words per round
        const float band_t = kRiskBand * inv2r;
        for (int i = eg; i < ntiles_cta; i += EPI_WGS) {
            const int tile = (int)blockIdx.x + i * (int)gridDim.x;
            const int64_t vi = (int64_t)tile * TILE + row;
            // Pool row: the block-table lookup is issued before the accumulator wait.
            int64_t slot = -1;
            if (vi < nvec) slot = tq_slot(a, vi / a.num_heads);
            const int64_t prow = slot >= 0 ? slot * a.num_heads + vi % a.num_heads : -1;
            uint8_t* dst = prow >= 0 ? (uint8_t*)a.packed_pool + prow * P : nullptr;
            if (!mbar_wait(&misc->tfull[eg], (i / EPI_WGS) & 1, err)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (uint32_t)(eg * D) + ((uint32_t)(quarter * 32) << 16);
            // Pass 1: |Pi x|^2 = |x|^2 from the accumulator row (four partial sums for ILP;
            // the exact norm is settled later when needed).
            float v[VCH];
            float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
            for (int h = 0; h < D / VCH; ++h) {
                tmem_ld32_nowait(taddr + h * VCH, v);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < VCH; ++j) s4[j & 3] = fmaf(v[j], v[j], s4[j & 3]);
            }
            const float ss = (s4[0] + s4[1]) + (s4[2] + s4[3]);
            const bool zero = ss == 0.0f;  // zero vector: y = 0 for every coordinate in both statements
            const float norm_f = sqrtf(ss);
            const float kr = __frcp_rn(norm_f + 1e-8f) * inv2r;
            const bool norm_amb =
                __float2half_rn(norm_f * (1.0f - kNormBand)) != __float2half_rn(norm_f * (1.0f + kNormBand));
            // Pass 2, codes, VCH coordinates per round, stored as soon as a round is done.
            // Per coordinate: t = y/(2R) + 0.5 (saturated), its table bin, the bin's boundary
            // `mid`; code = base + (t > mid) from the sign of mid - t; packed big-endian by
            // integer multiply-add (first code in the top bits). The accumulator goes back
            // to the MMA warp as soon as the last round is in registers.
            uint32_t mask[4] = {0u, 0u, 0u, 0u};
#pragma unroll 1
            for (int h = 0; h < D / VCH; ++h) {
                float dmin = 1.0f;
                tmem_ld32_nowait(taddr + h * VCH, v);
                tmem_wait_ld();
                if (h == D / VCH - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&misc->tempty[eg]);
                }
                uint32_t w[WPR];
#pragma unroll
                for (int w2 = 0; w2 < WPR; ++w2) {
                    uint32_t wd = 0;
#pragma unroll
                    for (int q = 0; q < G; ++q) {
                        const int j = w2 * G + q;
                        float t;
                        asm("fma.rn.sat.f32 %0, %1, %2, 0f3F000000;" : "=f"(t) : "f"(v[j]), "f"(kr));
                        const float u = fmaf(t, (float)(NB - 1), magic);
                        const uint32_t addr = __float_as_uint(u) * 256u + lut_lane;
                        float mid;
                        uint32_t base;
                        asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=f"(mid), "=r"(base) : "r"(addr));
                        const float dd = mid - t;
                        dmin = fminf(dmin, fabsf(dd));
                        const uint32_t code = base + (__float_as_uint(dd) >> 31);
                        wd = wd * (1u << BITS) + code;
                    }
                    w[w2] = zero ? zero_word : wd;
                }
                if (dst) {
                    if constexpr (BITS == 4) {
                        *(uint4*)(dst + 16 * h) = make_uint4(__byte_perm(w[0], 0, 0x0123), __byte_perm(w[1], 0, 0x0123),
                                                             __byte_perm(w[2], 0, 0x0123), __byte_perm(w[3], 0, 0x0123));
                    } else if constexpr (BITS == 2) {
                        *(uint2*)(dst + 8 * h) = make_uint2(__byte_perm(w[0], 0, 0x0123), __byte_perm(w[1], 0, 0x0123));
                    } else {
                        // 3-bit: each word holds 24 stream bits (bits 23..0, first code on top)
                        uint32_t* d3 = (uint32_t*)(dst + 12 * h);
                        d3[0] = __byte_perm(w[0], w[1], 0x6012);  // w0.b2 w0.b1 w0.b0 w1.b2
                        d3[1] = __byte_perm(w[1], w[2], 0x5601);  // w1.b1 w1.b0 w2.b2 w2.b1
                        d3[2] = __byte_perm(w[2], w[3], 0x4560);  // w2.b0 w3.b2 w3.b1 w3.b0
                    }
                }
                if (dmin < band_t && !zero) {
                    // rare: list this round's coordinates within the band
                    uint32_t m = 0;
#pragma unroll
                    for (int j = 0; j < VCH; ++j) {
                        float t;
                        asm("fma.rn.sat.f32 %0, %1, %2, 0f3F000000;" : "=f"(t) : "f"(v[j]), "f"(kr));
                        const float u = fmaf(t, (float)(NB - 1), magic);
                        const uint32_t addr = __float_as_uint(u) * 256u + lut_lane;
                        float mid;
                        uint32_t base;
                        asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=f"(mid), "=r"(base) : "r"(addr));
                        if (fabsf(mid - t) < band_t) m |= 1u << j;
                    }
                    if (h == 0) mask[0] = m;
                    else if (h == 1) mask[1] = m;
                    else if (h == 2) mask[2] = m;
                    else mask[3] = m;
                }
            }
            if (prow < 0) continue;
            ((__half*)a.norms_pool)[prow] = __float2half_rn(norm_f);
            const uint32_t flags = ((norm_amb && !zero) ? kFixNorm : 0u) | (use_exact ? kFixAll | kFixNorm : 0u);
            if (flags || (mask[0] | mask[1] | mask[2] | mask[3])) {
                const uint32_t qi = atomicAdd(fix_count, 1u);
                if (qi < fix_cap) {
                    FixEntry en;
                    en.vi = (uint32_t)vi;
                    en.flags = flags;
                    en.mask[0] = mask[0];
                    en.mask[1] = mask[1];
                    en.mask[2] = mask[2];
                    en.mask[3] = mask[3];
                    fix[qi] = en;
                } else {
                    // queue full: settle the row here
                    settle_row_inline<TIn, BITS>(a, vi, prow, flags, mask[0], mask[1], mask[2], mask[3], misc->cen);
                }
            }
        }
    }

    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem_base) : "memory");
    }
}


// Settles queued rows with the exact float32 statement, one row per warp: the
// lanes form the squares, quotients x_j / (norm + 1e-8) and products in
// parallel (4 coordinates each) and lane 0 adds them up in index order, so
// every sum is the sequential float32 sum; then the first-minimum nearest
// centroid, patched into the stored bit stream, and the norm rewritten.
constexpr int FIX_WARPS = 4;

template <typename TIn, int BITS>
__global__ void __launch_bounds__(FIX_WARPS * 32) tq_fixup_kernel(TqArgs a, const FixEntry* __restrict__ fix,
                                                                  const unsigned int* __restrict__ fix_count,
                                                                  unsigned int fix_cap) {
    __shared__ float cen[256];
    __shared__ float terms[FIX_WARPS][D];
    const int nlev = 1 << BITS;
    for (int e = threadIdx.x; e < nlev; e += blockDim.x) cen[e] = __ldg(a.centroids + e);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* tw = terms[warp];
    const unsigned int n = min(*fix_count, fix_cap);
    const int P = (D * BITS) >> 3;
    for (unsigned int q = blockIdx.x * FIX_WARPS + warp; q < n; q += gridDim.x * FIX_WARPS) {
        const FixEntry en = fix[q];
        const int64_t vi = en.vi;
        const int64_t slot = tq_slot(a, vi / a.num_heads);
        if (slot < 0) continue;
        const TIn* xr = (const TIn*)a.input + vi * D + 4 * lane;
        float x[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = to_f32(xr[k]);
#pragma unroll
        for (int k = 0; k < 4; ++k) tw[4 * lane + k] = __fmul_rn(x[k], x[k]);
        __syncwarp();
        float den = 0.0f;
        if (lane == 0) {
            float s = 0.0f;
#pragma unroll 16
            for (int j = 0; j < D; ++j) s = __fadd_rn(s, tw[j]);
            const float norm = __fsqrt_rn(s);
            if (en.flags & kFixNorm)
                ((__half*)a.norms_pool)[slot * a.num_heads + vi % a.num_heads] = __float2half_rn(norm);
            den = __fadd_rn(norm, 1e-8f);
        }
        den = __shfl_sync(0xffffffffu, den, 0);
        const bool any = (en.flags & kFixAll) || (en.mask[0] | en.mask[1] | en.mask[2] | en.mask[3]);
        if (!any) {
            __syncwarp();
            continue;
        }
        float xn[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) xn[k] = __fdiv_rn(x[k], den);
        uint4* rowp = (uint4*)((uint8_t*)a.packed_pool + (slot * a.num_heads + vi % a.num_heads) * P);
        uint32_t wds[16];
        if (lane == 0) {
#pragma unroll
            for (int q4 = 0; q4 < P / 16; ++q4) {
                const uint4 t4 = rowp[q4];
                wds[4 * q4] = t4.x; wds[4 * q4 + 1] = t4.y; wds[4 * q4 + 2] = t4.z; wds[4 * q4 + 3] = t4.w;
            }
        }
        for (int c = 0; c < 4; ++c) {
            uint32_t m = (en.flags & kFixAll) ? 0xffffffffu : en.mask[c];
            while (m) {
                const int i = c * 32 + __ffs(m) - 1;
                m &= m - 1;
                const float4 p = __ldg((const float4*)(a.rotation + i * D) + lane);
                __syncwarp();
                tw[4 * lane + 0] = __fmul_rn(p.x, xn[0]);
                tw[4 * lane + 1] = __fmul_rn(p.y, xn[1]);
                tw[4 * lane + 2] = __fmul_rn(p.z, xn[2]);
                tw[4 * lane + 3] = __fmul_rn(p.w, xn[3]);
                __syncwarp();
                if (lane == 0) {
                    float y = 0.0f;
#pragma unroll 16
                    for (int j = 0; j < D; ++j) y = __fadd_rn(y, tw[j]);
                    const uint32_t code = (uint32_t)nearest_centroid(y, cen, nlev);
                    // MSB-first stream bit bp lives in byte bp>>3 at bit 7-(bp&7); bytes little-endian in words
#pragma unroll
                    for (int b = 0; b < BITS; ++b) {
                        const int bp = i * BITS + b;
                        const int byte = bp >> 3;
                        const uint32_t bit = 1u << (8 * (byte & 3) + 7 - (bp & 7));
                        const uint32_t on = (code >> (BITS - 1 - b)) & 1u;
#pragma unroll
                        for (int w2 = 0; w2 < 16; ++w2)
                            if (w2 == (byte >> 2)) wds[w2] = on ? (wds[w2] | bit) : (wds[w2] & ~bit);
                    }
                }
            }
        }
        if (lane == 0) {
#pragma unroll
            for (int q4 = 0; q4 < P / 16; ++q4)
                rowp[q4] = make_uint4(wds[4 * q4], wds[4 * q4 + 1], wds[4 * q4 + 2], wds[4 * q4 + 3]);
        }
        __syncwarp();
    }
}

}  // namespace umma

// ── host side ───────────────────────────────────────────────────────────────

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

static bool device_is_sm100() {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    return major == 10 && minor == 0;
}

// Fixup queue: one per device, grown to the largest call (24 bytes per vector), kept for the
// life of the process. The queue is consumed by the fixup kernel of the same launch sequence on
// the same stream; calls on different streams of one device must not overlap.
struct FixWorkspace {
    void* ptr = nullptr;
    size_t cap = 0;  // entries
};

static int fix_workspace(int64_t nvec, umma::FixEntry** entries, unsigned int** count, unsigned int* cap) {
    static FixWorkspace ws[64];
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    FixWorkspace& w = ws[dev];
    const size_t want = (size_t)std::max<int64_t>(nvec, 4096);
    if (w.cap < want) {
        if (w.ptr) {
            e = cudaFree(w.ptr);
            if (e != cudaSuccess) return (int)e;
        }
        w.ptr = nullptr;
        w.cap = 0;
        e = cudaMalloc(&w.ptr, 256 + want * sizeof(umma::FixEntry));
        if (e != cudaSuccess) return (int)e;
        w.cap = want;
    }
    *count = (unsigned int*)w.ptr;
    *entries = (umma::FixEntry*)((char*)w.ptr + 256);
    *cap = (unsigned int)std::min<size_t>(w.cap, 0xffffffffu);
    return 0;
}

// Fixup queue of the no-allocation entry point: a file-scope device array, so that a call
// allocates nothing. It holds the queue header (256 bytes) and one entry per vector of the
// largest call accepted, kTqNoAllocMaxVectors (524288 vectors, e.g. 65536 tokens x 8 KV heads):
// 12 MiB + 256 bytes per device, reserved when the module loads. One array per device serves
// every call on that device, so calls that overlap in time (two streams, two host threads)
// race on it.
static __device__ __align__(256) unsigned char
    g_tq_fix_scratch[256 + (size_t)kTqNoAllocMaxVectors * sizeof(umma::FixEntry)];

// Set-up, once per device with that device current: the device address of g_tq_fix_scratch.
// The first call on a device does this set-up (it may load the module), so it belongs before
// any stream capture; later calls only read the cached address.
static int static_fix_scratch(int64_t nvec, umma::FixEntry** entries, unsigned int** count, unsigned int* cap) {
    static void* addr[64];
    static std::mutex mu;
    if (nvec > kTqNoAllocMaxVectors) return (int)cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_tq_fix_scratch);
        if (e != cudaSuccess) return (int)e;
        if (!p) return (int)cudaErrorInvalidSymbol;
        addr[dev] = p;
    }
    *count = (unsigned int*)addr[dev];
    *entries = (umma::FixEntry*)((char*)addr[dev] + 256);
    *cap = (unsigned int)kTqNoAllocMaxVectors;
    return 0;
}

template <typename TIn, int NPARTS, int BITS>
static int launch_umma(const TqArgs& a, cudaStream_t s, bool static_scratch) {
    auto encode = get_encode();
    if (!encode) return (int)cudaErrorNotSupported;
    const int64_t nvec = a.num_tokens * a.num_heads;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)umma::D, (cuuint64_t)nvec};
    const cuuint64_t strides[1] = {(cuuint64_t)umma::D * sizeof(TIn)};
    const cuuint32_t box[2] = {64, (cuuint32_t)umma::TILE};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&map, dtype_of<TIn>::value == FB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, const_cast<void*>(a.input), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return (int)cudaErrorInvalidValue;
    umma::FixEntry* fix;
    unsigned int* fix_count;
    unsigned int fix_cap;
    int rc = static_scratch ? static_fix_scratch(nvec, &fix, &fix_count, &fix_cap)
                            : fix_workspace(nvec, &fix, &fix_count, &fix_cap);
    if (rc) return rc;
    // the queue counter must start at zero; the entries are written before they are read
    cudaError_t e = cudaMemsetAsync(fix_count, 0, sizeof(unsigned int), s);
    if (e != cudaSuccess) return (int)e;
    constexpr int smem = umma::Smem::bytes(NPARTS);
    auto kern = umma::tq_compress_umma_kernel<TIn, NPARTS, BITS>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    const int num_tiles = (int)((nvec + umma::TILE - 1) / umma::TILE);
    const int grid = std::max(1, std::min(num_tiles, num_sms()));
    kern<<<grid, umma::THREADS, smem, s>>>(map, a, num_tiles, fix, fix_count, fix_cap);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
    umma::tq_fixup_kernel<TIn, BITS><<<num_sms() * 16, umma::FIX_WARPS * 32, 0, s>>>(a, fix, fix_count, fix_cap);
    return (int)cudaGetLastError();
}

static int umma_dispatch(const TqArgs& a, cudaStream_t s, bool* handled, bool static_scratch) {
    *handled = false;
    if (a.head_dim != umma::D || !(a.bits == 2 || a.bits == 3 || a.bits == 4)) return 0;
    if (a.in_dtype != FB_FP16 && a.in_dtype != FB_BF16) return 0;
    if (!aligned16(a.input) || !aligned16(a.packed_pool) || (((uintptr_t)a.norms_pool) & 1)) return 0;
    if (((uintptr_t)a.rotation & 15) != 0) return 0;
    if (a.num_tokens * a.num_heads > ((int64_t)1 << 31) - umma::TILE) return 0;
    static int sm100 = -1;
    if (sm100 < 0) sm100 = device_is_sm100() ? 1 : 0;
    if (!sm100) return 0;
    *handled = true;
    if (a.in_dtype == FB_FP16) {
        if (a.bits == 4) return launch_umma<__half, 2, 4>(a, s, static_scratch);
        if (a.bits == 3) return launch_umma<__half, 2, 3>(a, s, static_scratch);
        return launch_umma<__half, 2, 2>(a, s, static_scratch);
    }
    if (a.bits == 4) return launch_umma<__nv_bfloat16, 3, 4>(a, s, static_scratch);
    if (a.bits == 3) return launch_umma<__nv_bfloat16, 3, 3>(a, s, static_scratch);
    return launch_umma<__nv_bfloat16, 3, 2>(a, s, static_scratch);
}

int tq_compress_umma(const TqArgs& a, cudaStream_t s, bool* handled) {
    return umma_dispatch(a, s, handled, false);
}

int tq_compress_umma_noalloc(const TqArgs& a, cudaStream_t s, bool* handled) {
    return umma_dispatch(a, s, handled, true);
}

}  // namespace fb

extern "C" unsigned int fb_tq_timeouts(void) {
    unsigned int v = 0;
    cudaMemcpyFromSymbol(&v, fb::g_tq_umma_timeouts, sizeof(v));
    return v;
}
