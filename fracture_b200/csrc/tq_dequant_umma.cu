// TurboQuant dequantize on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Replaces backends/fracture-cuda/kernels/turboquant_decompress.cu:21-127 for head_dim 128,
// 2/3/4-bit codes and FP16/BF16 output:
//
//   x_hat[v][i] = norm[v] * sum_j Pi[j][i] * c[idx[v][j]]
//
// One persistent CTA per SM streams tiles of 128 head vectors. A launch serves one dequantize
// call, or two (the K and V of a cache read): the grid is split between them in proportion to
// their tiles, each CTA working for one of them.
//
//   warp 0       MMA issuer: acc[v][i] = sum_j Y[v][j] * PiT[i][j] on tcgen05 with
//                Y[v][j] = c[idx[v][j]]; one fp16 pass (fp16 centroids and Pi keep the
//                output within about 1e-4 of its magnitude of the float32 statement)
//   warps 1-16   decoders: four threads per vector take their quarter of the row's codes and
//                write fp16 centroid values straight into the 128-byte-swizzled A tile,
//                through lane-private lookup tables (two 4-bit, four 2-bit or two 3-bit codes
//                per lookup)
//   warps 17-24  epilogue, two warpgroups taking tiles in turn: one thread per vector scales
//                its accumulator row (one of four TMEM accumulators) by the stored fp16
//                norm, converts, and stages it in its warp's swizzled staging area, one
//                64-column half of the warp's 32 rows at a time, each half written with one
//                TMA tensor store
//   warp 25      producer (staged calls): copies each tile's packed codes and norms into a
//                ring of shared-memory stages with bulk asynchronous copies, three tiles
//                ahead of the decoders
//
// Staged calls are those whose tiles are runs of whole tokens in at most two cache blocks
// (head count a multiple of 8 dividing 128, a block table or none, 16-byte aligned pools):
// a tile's codes are then one or two contiguous byte ranges of the pool. Other calls
// (slot maps, other head counts) have each decoder thread gather its codes from global
// memory itself, two tiles ahead of use.
//
// Pool rows follow the slot rule of tq_common.cuh; a token without a valid slot
// dequantizes to zeros (norm 0), as the CUDA-core kernel does. Every barrier wait is
// bounded; on timeout the kernel counts the event in g_tq_dequant_timeouts, abandons
// its loop and still frees its TMEM.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tq_common.cuh"
#include "tq_sm100.cuh"

namespace fb {

__device__ unsigned int g_tq_dequant_timeouts = 0;

namespace dq {

using namespace sm100;

constexpr int A_STAGES = 3;  // decoded A tiles in flight
constexpr int NACC = 4;      // TMEM accumulators (4 x 128 columns: all of TMEM)
constexpr int STG = 2;       // output staging areas (one per epilogue warpgroup)
constexpr int STG_WARP = 32 * 128;        // a warp's staging: 32 rows x 64 columns (one half), SW128
constexpr int STG_BYTES = 4 * STG_WARP;   // a warpgroup's staging area
constexpr int CSTAGES = 3;   // code stages of a staged call (tiles the producer runs ahead)
constexpr int DEC_WARPS = 16;
constexpr int TPR = DEC_WARPS * 32 / TILE;  // decoder threads per vector
constexpr int EPI_WGS = 2;                 // epilogue warpgroups, taking tiles in turn
constexpr int EPI_WARPS = 4 * EPI_WGS;
constexpr int PROD_WARP = 1 + DEC_WARPS + EPI_WARPS;
constexpr int THREADS = 32 * (PROD_WARP + 1);
constexpr int MAX_REGS = 72;  // 26 warps: up to 7 on one scheduler, 16K registers each
// Norms travel from the decoders to the epilogue through shared memory, one row of 128 per
// tile, NORM_BUF rows deep: the decoder of tile i + NORM_BUF can only start after the MMA of
// tile i + NACC, which waits for the epilogue of tile i to release its accumulator.
constexpr int NORM_BUF = A_STAGES + NACC;
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

struct Misc {
    uint64_t a_full[A_STAGES];
    uint64_t a_empty[A_STAGES];
    uint64_t tfull[NACC];
    uint64_t tempty[NACC];
    uint64_t pi_full;        // Pi (fp32) copied into the staging area for the set-up
    uint64_t code_full[CSTAGES];   // a tile's codes and norms have landed in the code stage
    uint64_t code_empty[CSTAGES];  // every decoder warp has read the code stage
    uint32_t tmem_base;
    float cen[16];
    uint64_t norm_full[NORM_BUF];  // the decoders have written norm[k] for the tile
    float norm[NORM_BUF][TILE];    // written by the decoders (h == 0), read by the epilogue
};

// Lookup tables of the decoders, lane-private so the 32 lanes of a warp hit 32 banks:
// 4-bit: byte -> half2 (2 codes), 32 copies; 2-bit: byte -> 2 x half2 (4 codes), 16 copies
// (64-bit loads, one copy per half-warp lane); 3-bit: 6 bits -> half2 (2 codes), 32 copies.
template <int BITS>
struct Table {
    static constexpr int entries = BITS == 3 ? 64 : 256;
    static constexpr int copies = BITS == 2 ? 16 : 32;
    static constexpr int entry_bytes = BITS == 2 ? 8 : 4;
    static constexpr int bytes = entries * copies * entry_bytes;
};

template <int BITS>
struct Smem {
    static constexpr int P = D * BITS / 8;                            // packed bytes per vector
    static constexpr int b_off = 0;                                   // Pi^T, fp16, SW128
    static constexpr int a_off = TILE_BYTES;                          // A_STAGES decoded tiles
    static constexpr int st_off = a_off + A_STAGES * TILE_BYTES;      // STG output staging areas
    static constexpr int tab_off = st_off + STG * STG_BYTES;
    static constexpr int code_off = tab_off + Table<BITS>::bytes;     // CSTAGES x (codes, norms)
    static constexpr int code_stage = TILE * P + TILE * 2;
    static constexpr int misc_off = code_off + CSTAGES * code_stage;
    static constexpr int bytes = misc_off + (int)sizeof(Misc) + 1024;
};

// One dequantize call of a launch, served by CTAs [cta0, cta0 + ncta) of the grid.
struct DqJob {
    TqArgs a;
    int num_tiles;
    int cta0, ncta;
    DivU32 hdiv;  // division by num_heads
};

struct DqLaunch {
    CUtensorMap omap[2];  // output tensor maps of the jobs
    DqJob job[2];
    int njobs;
};

// Bounded wait for the phase with parity `parity`; false (and a counted timeout) if it never
// completes. After a first probe the thread may be suspended until the phase completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
            : "memory");
        if (ok) return true;
        if (clock64() - t0 > kTimeoutCycles) {
            atomicAdd(&g_tq_dequant_timeouts, 1u);
            return false;
        }
    }
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

template <typename TOut>
__device__ __forceinline__ uint32_t pack_out(float a, float b) {
    if constexpr (dtype_of<TOut>::value == FB_BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}

// The work of one CTA for job `jb`: CTA `cta` of the job's `ncta` takes tiles cta, cta + ncta, ...
template <typename TOut, int BITS, bool STAGED>
__device__ __forceinline__ void dequant_cta(const CUtensorMap* omap, const DqJob& jb) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the shared array, so that the compiler still
    // knows every pointer derived from it addresses shared memory (plain ld/st.shared)
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    using L = Smem<BITS>;
    using TB = Table<BITS>;
    const TqArgs& a = jb.a;
    const int cta = (int)blockIdx.x - jb.cta0, ncta = jb.ncta;
    uint8_t* sB = base + L::b_off;
    uint8_t* sA = base + L::a_off;
    uint8_t* sST = base + L::st_off;
    uint8_t* tab = base + L::tab_off;
    uint8_t* sCode = base + L::code_off;
    Misc* misc = (Misc*)(base + L::misc_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nlev = 1 << BITS;
    constexpr int P = L::P;
    const int64_t nvec = a.num_tokens * a.num_heads;
    const int num_tiles = jb.num_tiles;
    const int ntiles_cta = num_tiles > cta ? (num_tiles - 1 - cta) / ncta + 1 : 0;

    // ── prologue ─────────────────────────────────────────────────────────────
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                         smem_u32(&misc->tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        tc_fence_before();
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < A_STAGES; ++s) {
            mbar_init(&misc->a_full[s], DEC_WARPS);
            mbar_init(&misc->a_empty[s], 1);
        }
        for (int b = 0; b < NACC; ++b) {
            mbar_init(&misc->tfull[b], 1);
            mbar_init(&misc->tempty[b], 4);
        }
        for (int c = 0; c < CSTAGES; ++c) {
            mbar_init(&misc->code_full[c], 1);
            mbar_init(&misc->code_empty[c], DEC_WARPS);
        }
        mbar_init(&misc->pi_full, 1);
        for (int k = 0; k < NORM_BUF; ++k) mbar_init(&misc->norm_full[k], DEC_WARPS);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // Pi (64 KB fp32) lands in the A stages, which are free until the first tile
        mbar_expect_tx(&misc->pi_full, D * D * 4);
        bulk_load(sA, a.rotation, D * D * 4, &misc->pi_full);
    }
    if (threadIdx.x < nlev) misc->cen[threadIdx.x] = __ldg(a.centroids + threadIdx.x);
    __syncthreads();
    // In staged calls the producer warp (the last warp) starts copying codes right away, while
    // the other warps build the tables and the B operand and meet on named barrier 1.
    constexpr int PRO_THREADS = STAGED ? THREADS - 32 : THREADS;
    if (!STAGED || warp != PROD_WARP) {
        // Decode tables (codes in MSB-first order: the first code of a byte is its high bits).
        for (int e = threadIdx.x; e < TB::entries * TB::copies; e += PRO_THREADS) {
            const int ent = e / TB::copies;
            const float* cen = misc->cen;
            if constexpr (BITS == 4) {
                ((uint32_t*)tab)[e] = h2_bits(__floats2half2_rn(cen[ent >> 4], cen[ent & 15]));
            } else if constexpr (BITS == 3) {
                ((uint32_t*)tab)[e] = h2_bits(__floats2half2_rn(cen[ent >> 3], cen[ent & 7]));
            } else {
                const __half2 h0 = __floats2half2_rn(cen[ent >> 6], cen[(ent >> 4) & 3]);
                const __half2 h1 = __floats2half2_rn(cen[(ent >> 2) & 3], cen[ent & 3]);
                ((uint2*)tab)[e] = make_uint2(h2_bits(h0), h2_bits(h1));
            }
        }
        // B operand: B[i][j] = Pi[j][i] in fp16 (K-major: the contraction index j is contiguous);
        // item (i, j0) packs Pi[j0..j0+7][i] into one 16-byte chunk.
        mbar_wait(&misc->pi_full, 0);  // a timeout is counted (B would then be garbage)
        {
            const float* pis = (const float*)sA;
            for (int it = threadIdx.x; it < D * D / 8; it += PRO_THREADS) {
                const int i = it & (D - 1), j0 = (it >> 7) * 8;
                uint32_t o[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    o[k] = h2_bits(__floats2half2_rn(pis[(j0 + 2 * k) * D + i], pis[(j0 + 2 * k + 1) * D + i]));
                *(uint4*)(sB + sw128_offset(i, j0)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
        fence_async_smem();
        if constexpr (STAGED) asm volatile("bar.sync 1, %0;" ::"r"(PRO_THREADS) : "memory");
        else __syncthreads();
    }
    tc_fence_after();
    const uint32_t tmem_base = misc->tmem_base;

    if (warp == 0) {
        // ── MMA issuer ──────────────────────────────────────────────────────
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(0u);
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            int done = 0;
            for (int i = 0; i < ntiles_cta; ++i) {
                const int s = i % A_STAGES, buf = i % NACC;
                if (!mbar_wait(&misc->a_full[s], (i / A_STAGES) & 1)) break;
                if (!mbar_wait(&misc->tempty[buf], ((i / NACC) + 1) & 1)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(buf * D);
#pragma unroll
                for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t off = kb * KBLK_BYTES + k * 32;
                        mma_f16(d, sw128_desc(a0 + s * TILE_BYTES + off), sw128_desc(b0 + off), idesc,
                                (kb | k) ? 1u : 0u);
                    }
                umma_commit(&misc->a_empty[s]);
                umma_commit(&misc->tfull[buf]);
                done = i + 1;
            }
            // The last accumulations finish before TMEM is released.
            if (done > 0) mbar_wait(&misc->tfull[(done - 1) % NACC], ((done - 1) / NACC) & 1);
        }
    } else if (warp <= DEC_WARPS) {
        // ── decoders: thread dt handles part h (codes CPT*h ..) of row r ─────
        constexpr int RPW = 32 / TPR;
        static_assert(RPW == 8, "a warp covers eight rows");
        constexpr int CPT = D / TPR;
        constexpr int NW = BITS * CPT / 32;  // 32-bit words of packed codes per part
        const int dt = threadIdx.x - 32;
        // Gathering decoders: quarter-warp q takes part q of eight consecutive rows, so its 16-byte
        // stores into the swizzled A tile fall in eight distinct bank groups. Staged decoders: lane
        // (q, j) takes row j and part (j / 2 + q) % 4, which keeps those stores conflict-free and
        // also the quarter-warp's 16-byte reads of the code stage (4-bit rows are 64 bytes).
        const int r = (dt >> 5) * RPW + (lane & 7);
        const int h = STAGED ? (((lane & 7) >> 1) + (lane >> 3)) & 3 : lane >> 3;
        const uint32_t tlane = smem_u32(tab) + (uint32_t)(lane & (TB::copies - 1)) * TB::entry_bytes;
        // One tile: wait for the stage, publish the norm, decode `wv` into the A tile, signal.
        auto decode_tile = [&](int i, const uint32_t (&wv)[NW], unsigned short nbits) -> bool {
            const int s = i % A_STAGES;
            if (!mbar_wait(&misc->a_empty[s], ((i / A_STAGES) + 1) & 1)) return false;
            if (h == 0) misc->norm[i % NORM_BUF][r] = __half2float(__ushort_as_half(nbits));
            uint8_t* dstrow = sA + s * TILE_BYTES;
#pragma unroll
            for (int c = 0; c < CPT / 8; ++c) {  // chunks of 8 values: columns CPT*h + 8c ..
                uint32_t o[4];
                if constexpr (BITS == 4) {
                    const uint32_t w = wv[c];  // 4 bytes = 8 codes, byte 0 first
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t byte = (w >> (8 * k)) & 0xffu;
                        asm("ld.shared.b32 %0, [%1];" : "=r"(o[k]) : "r"(tlane + byte * (TB::copies * 4u)));
                    }
                } else if constexpr (BITS == 2) {
                    const uint32_t w = wv[c >> 1] >> (16 * (c & 1));  // 2 bytes = 8 codes
#pragma unroll
                    for (int k = 0; k < 2; ++k) {
                        const uint32_t byte = (w >> (8 * k)) & 0xffu;
                        asm("ld.shared.v2.b32 {%0, %1}, [%2];"
                            : "=r"(o[2 * k]), "=r"(o[2 * k + 1])
                            : "r"(tlane + byte * (TB::copies * 8u)));
                    }
                } else {
                    // 3 bytes = 8 codes; stream bytes 3c, 3c+1, 3c+2 as a big-endian 24-bit value
                    const int b0 = 3 * c;
                    const uint32_t x0 = (wv[b0 >> 2] >> (8 * (b0 & 3))) & 0xffu;
                    const uint32_t x1 = (wv[(b0 + 1) >> 2] >> (8 * ((b0 + 1) & 3))) & 0xffu;
                    const uint32_t x2 = (wv[(b0 + 2) >> 2] >> (8 * ((b0 + 2) & 3))) & 0xffu;
                    const uint32_t v24 = (x0 << 16) | (x1 << 8) | x2;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint32_t six = (v24 >> (18 - 6 * k)) & 63u;
                        asm("ld.shared.b32 %0, [%1];" : "=r"(o[k]) : "r"(tlane + six * (TB::copies * 4u)));
                    }
                }
                *(uint4*)(dstrow + sw128_offset(r, CPT * h + 8 * c)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&misc->norm_full[i % NORM_BUF]);
                mbar_arrive(&misc->a_full[s]);
            }
            return true;
        };
        if constexpr (STAGED) {
            // codes and norm of tile i from code stage i % CSTAGES, filled by the producer warp
            for (int i = 0; i < ntiles_cta; ++i) {
                const int cs = i % CSTAGES;
                if (!mbar_wait(&misc->code_full[cs], (i / CSTAGES) & 1)) break;
                const uint8_t* stage = sCode + cs * L::code_stage;
                const uint8_t* src = stage + r * P + h * (P / TPR);
                uint32_t wv[NW];
                if constexpr (NW == 4) {
                    const uint4 t = *(const uint4*)src;
                    wv[0] = t.x;
                    wv[1] = t.y;
                    wv[2] = t.z;
                    wv[3] = t.w;
                } else if constexpr (NW == 2) {
                    const uint2 t = *(const uint2*)src;
                    wv[0] = t.x;
                    wv[1] = t.y;
                } else {
#pragma unroll
                    for (int k = 0; k < NW; ++k) wv[k] = ((const uint32_t*)src)[k];
                }
                const unsigned short nb = h == 0 ? ((const unsigned short*)(stage + TILE * P))[r] : (unsigned short)0;
                __syncwarp();
                if (lane == 0) mbar_arrive(&misc->code_empty[cs]);
                if (!decode_tile(i, wv, nb)) break;
            }
        } else {
            // The packed codes of tile i+2 and the block-table entry of tile i+4 are requested
            // while tile i is decoded, so the two dependent global loads overlap the pipeline.
            // Pool row of this thread's vector in tile i, in two steps so that no branch waits on
            // a load: bt_of issues the slot-map or block-table read (-1: no vector; 0 without
            // either), row_of applies the slot rule of tq_slot to it two steps later (-1: no row).
            // (32-bit division by the head count: the host keeps the vector count below 2^31.)
            // Prefetched values stay raw (the slot-map entry, or the int32 table entry zero-extended;
            // fp16 norm bits) until they are used, so no conversion waits on a load still in flight.
            auto bt_of = [&](int i) -> int64_t {
                const uint32_t vi = (uint32_t)(cta + i * ncta) * TILE + r;
                if (i >= ntiles_cta || (int64_t)vi >= nvec) return -1;
                const uint32_t tok = divu32(vi, jb.hdiv);
                if (a.slot_map) return __ldg(a.slot_map + tok);
                if (!a.block_table) return 0;
                return (int64_t)(uint32_t)__ldg(a.block_table + ((a.start_pos + tok) >> 4));
            };
            auto row_of = [&](int i, int64_t raw) -> int64_t {
                if (raw == -1) return -1;
                const uint32_t vi = (uint32_t)(cta + i * ncta) * TILE + r;
                const uint32_t tok = divu32(vi, jb.hdiv), head = vi - tok * (uint32_t)a.num_heads;
                const int64_t pos = a.start_pos + tok;
                int64_t slot = pos;
                if (a.slot_map) {
                    slot = raw;
                } else if (a.block_table) {
                    const int32_t b = (int32_t)(uint32_t)raw;
                    slot = b < 0 ? -1 : (int64_t)b * 16 + (pos & 15);
                }
                return (slot >= 0 && slot < a.pool_rows) ? slot * a.num_heads + head : -1;
            };
            auto load_codes = [&](int64_t prow, uint32_t (&wv)[NW]) {  // zeros when there is no row
#pragma unroll
                for (int k = 0; k < NW; ++k) wv[k] = 0u;
                if (prow < 0) return;
                const uint8_t* src = (const uint8_t*)a.packed_pool + prow * P + h * (P / TPR);
                if constexpr (NW % 4 == 0) {
#pragma unroll
                    for (int k = 0; k < NW / 4; ++k) {
                        const uint4 t = __ldg((const uint4*)src + k);
                        wv[4 * k] = t.x;
                        wv[4 * k + 1] = t.y;
                        wv[4 * k + 2] = t.z;
                        wv[4 * k + 3] = t.w;
                    }
                } else if constexpr (NW % 2 == 0) {
#pragma unroll
                    for (int k = 0; k < NW / 2; ++k) {
                        const uint2 t = __ldg((const uint2*)src + k);
                        wv[2 * k] = t.x;
                        wv[2 * k + 1] = t.y;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < NW; ++k) wv[k] = __ldg((const uint32_t*)src + k);
                }
            };
            auto load_norm = [&](int64_t prow) -> unsigned short {
                return (prow >= 0 && h == 0) ? __ldg((const unsigned short*)a.norms_pool + prow) : (unsigned short)0;
            };
            // Register rings, no copies between iterations: at step t the codes and norm of tile
            // t + 2 are requested (ring slot (t + 2) % 3) and the block-table entry of tile t + 4
            // (slot (t + 1) % 3, freed at step t - 1), then tile t is decoded; every load has two
            // steps to arrive before it is used.
            uint32_t w[3][NW];
            unsigned short nr[3];
            int64_t bt[3];
            bt[0] = bt_of(0);
            bt[1] = bt_of(1);
            bt[2] = bt_of(2);
            {
                const int64_t q0 = row_of(0, bt[0]), q1 = row_of(1, bt[1]);
                load_codes(q0, w[0]);
                nr[0] = load_norm(q0);
                load_codes(q1, w[1]);
                nr[1] = load_norm(q1);
            }
            bt[0] = bt_of(3);
            bool ok = true;
            for (int i = 0; i < ntiles_cta && ok; i += 3) {
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    const int t = i + k;
                    if (t >= ntiles_cta) break;
                    const int64_t q = row_of(t + 2, bt[(k + 2) % 3]);
                    load_codes(q, w[(k + 2) % 3]);
                    nr[(k + 2) % 3] = load_norm(q);
                    bt[(k + 1) % 3] = bt_of(t + 4);
                    if (!decode_tile(t, w[k], nr[k])) {
                        ok = false;
                        break;
                    }
                }
            }
        }
    } else if (warp < PROD_WARP) {
        // ── epilogue: warpgroup e takes the tiles i with i % EPI_WGS == e (accumulator i % NACC).
        // Each warp stages its own 32 rows one 64-column half at a time in its own 4 KB of the
        // warpgroup's staging area and writes the half with one TMA tensor store; before it stages
        // the next half its lane 0 waits until that store has read the area. No barrier joins the
        // four warps. ──
        const int e = (warp - 1 - DEC_WARPS) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        // 4 KB-aligned, so the SW128 pattern of the 32 x 64 box follows (lane & 7) = (row & 7)
        uint8_t* st_w = sST + e * STG_BYTES + quarter * STG_WARP;
        for (int i = e; i < ntiles_cta; i += EPI_WGS) {
            const int tile = cta + i * ncta;
            const int acc = i % NACC;
            if (!mbar_wait(&misc->tfull[acc], (i / NACC) & 1)) break;
            tc_fence_after();
            if (!mbar_wait(&misc->norm_full[i % NORM_BUF], (i / NORM_BUF) & 1)) break;
            const float nrm = misc->norm[i % NORM_BUF][row];
            const uint32_t taddr = tmem_base + (uint32_t)(acc * D) + ((uint32_t)(quarter * 32) << 16);
            // the first of this warp's rows exists (the last tile may end inside the warp's rows;
            // the store box is clipped at the tensor's end, and no store starts past it)
            const bool has_rows = (int64_t)tile * TILE + quarter * 32 < nvec;
            // 16-column chunks, the next chunk's load in flight while the current chunk is stored
            // (tcgen05.wait::ld waits for every load in flight, so a third buffer would hide no more)
            constexpr int NBE = 2;  // load buffers
            uint32_t vbuf[NBE][16];
#pragma unroll
            for (int h = 0; h < NBE - 1; ++h) tmem_ld16_issue(taddr + 16 * h, vbuf[h]);
#pragma unroll
            for (int cchunk = 0; cchunk < D / 16; ++cchunk) {
                uint32_t(&v)[16] = vbuf[cchunk % NBE];
                tmem_wait_one(v);
                if (cchunk + NBE - 1 < D / 16) {
                    tmem_ld16_issue(taddr + (cchunk + NBE - 1) * 16, vbuf[(cchunk + NBE - 1) % NBE]);
                } else if (cchunk == D / 16 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&misc->tempty[acc]);
                }
                if ((cchunk & 3) == 0) {
                    // the store of the previous half has read the staging area
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                }
#pragma unroll
                for (int g = 0; g < 2; ++g) {
                    uint32_t o[4];
#pragma unroll
                    for (int k2 = 0; k2 < 4; ++k2)
                        o[k2] = pack_out<TOut>(__uint_as_float(v[8 * g + 2 * k2]) * nrm,
                                               __uint_as_float(v[8 * g + 2 * k2 + 1]) * nrm);
                    *(uint4*)(st_w + sw128_offset(lane, (16 * cchunk + 8 * g) & 63)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
                if ((cchunk & 3) == 3) {
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0 && has_rows) {
                        tma_store_2d(omap, st_w, 64 * (cchunk >> 2), tile * TILE + quarter * 32);
                        bulk_commit();
                    }
                }
            }
        }
        if (lane == 0) bulk_wait_all();
    } else if constexpr (STAGED) {
        // ── producer: one lane copies tile i's codes and norms into code stage i % CSTAGES ──
        // A tile is TPT = 128 / H whole tokens (H a multiple of 8 dividing 128), at most two
        // cache blocks: per block one contiguous copy of codes (P bytes per vector) and one of
        // norms (2 bytes per vector). The block-table entries of 32 tiles are fetched at once,
        // one per lane, a batch ahead of use.
        const int H = a.num_heads;
        const int TPT = TILE / H;
        auto fetch = [&](int ibase, int32_t& e0, int32_t& e1) {
            const int i = ibase + lane;
            e0 = e1 = -1;
            if (i < ntiles_cta && a.block_table) {
                const int64_t tok0 = (int64_t)(cta + i * ncta) * TPT;
                const int64_t pos0 = a.start_pos + tok0;
                const int64_t ntok = min((int64_t)TPT, a.num_tokens - tok0);
                e0 = __ldg(a.block_table + (pos0 >> 4));
                if ((pos0 & 15) + ntok > 16) e1 = __ldg(a.block_table + (pos0 >> 4) + 1);
            }
        };
        int32_t c0, c1, n0, n1;
        fetch(0, c0, c1);
        fetch(32, n0, n1);
        // The pool rows of tile i's (at most two) segments, from its block-table entries.
        auto segments = [&](int i, int32_t e0, int32_t e1, int (&k0)[2], int (&nt)[2], int (&nvalid)[2],
                            int64_t (&slot0)[2]) {
            const int64_t tok0 = (int64_t)(cta + i * ncta) * TPT;
            const int ntok = (int)min((int64_t)TPT, a.num_tokens - tok0);
            const int64_t pos0 = a.start_pos + tok0;
            // tokens [0, nA) in block pos0 / 16, then [nA, ntok) in the next
            const int nA = min(ntok, 16 - (int)(pos0 & 15));
            k0[0] = 0;
            k0[1] = nA;
            nt[0] = nA;
            nt[1] = ntok - nA;
            for (int sg = 0; sg < 2; ++sg) {
                nvalid[sg] = 0;
                slot0[sg] = 0;
                if (nt[sg] <= 0) continue;
                const int64_t pos = pos0 + k0[sg];
                int64_t sl = pos;
                if (a.block_table) {
                    const int32_t ent = sg == 0 ? e0 : e1;
                    sl = ent < 0 ? -1 : (int64_t)ent * 16 + (pos & 15);
                }
                slot0[sg] = sl;
                nvalid[sg] = sl < 0 ? 0 : (int)max((int64_t)0, min((int64_t)nt[sg], a.pool_rows - sl));
            }
        };
        // entries of tile i (i < current batch + 32), from the current batch
        auto entries = [&](int i, int32_t& e0, int32_t& e1) {
            e0 = __shfl_sync(0xffffffffu, c0, i & 31);
            e1 = __shfl_sync(0xffffffffu, c1, i & 31);
        };
        bool ok = true;
        for (int i = 0; i < ntiles_cta && ok; ++i) {
            if (i > 0 && (i & 31) == 0) {
                c0 = n0;
                c1 = n1;
                fetch(i + 32, n0, n1);
            }
            int32_t e0, e1;
            entries(i, e0, e1);
            int good = 1;
            if (lane == 0) {
                const int cs = i % CSTAGES;
                good = mbar_wait(&misc->code_empty[cs], ((i / CSTAGES) + 1) & 1) ? 1 : 0;
                if (good) {
                    uint8_t* stage = sCode + cs * L::code_stage;
                    int k0[2], nt[2], nvalid[2];
                    int64_t slot0[2];
                    segments(i, e0, e1, k0, nt, nvalid, slot0);
                    // tokens without a pool row: zero codes and norm (the output row is then 0)
                    bool zeroed = false;
                    for (int sg = 0; sg < 2; ++sg) {
                        for (int t = k0[sg] + nvalid[sg]; t < k0[sg] + max(nt[sg], 0); ++t) {
                            uint4* zc = (uint4*)(stage + (size_t)t * H * P);
                            for (int q = 0; q < H * P / 16; ++q) zc[q] = make_uint4(0u, 0u, 0u, 0u);
                            uint4* zn = (uint4*)(stage + TILE * P + (size_t)t * H * 2);
                            for (int q = 0; q < H * 2 / 16; ++q) zn[q] = make_uint4(0u, 0u, 0u, 0u);
                            zeroed = true;
                        }
                    }
                    if (zeroed) fence_async_smem();  // before later bulk copies into the same bytes
                    const uint32_t bytes = (uint32_t)(nvalid[0] + nvalid[1]) * (uint32_t)H * (P + 2);
                    mbar_expect_tx(&misc->code_full[cs], bytes);
                    for (int sg = 0; sg < 2; ++sg) {
                        if (nvalid[sg] == 0) continue;
                        const uint32_t nv = (uint32_t)nvalid[sg] * (uint32_t)H;
                        bulk_load(stage + (size_t)k0[sg] * H * P, (const uint8_t*)a.packed_pool + slot0[sg] * H * P,
                                  nv * P, &misc->code_full[cs]);
                        bulk_load(stage + TILE * P + (size_t)k0[sg] * H * 2,
                                  (const uint8_t*)a.norms_pool + slot0[sg] * H * 2, nv * 2, &misc->code_full[cs]);
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, good, 0) != 0;
        }
        // copies still in flight land before the CTA exits
        if (lane == 0 && ntiles_cta > 0)
            for (int i = max(0, ntiles_cta - CSTAGES); i < ntiles_cta; ++i)
                mbar_wait(&misc->code_full[i % CSTAGES], (i / CSTAGES) & 1);
    }

    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem_base) : "memory");
    }
}

// B0 / B1: code widths of job 0 / job 1 (equal for a single call).
template <typename TOut, int B0, int B1, bool STAGED>
__global__ void __maxnreg__(MAX_REGS) tq_dequant_umma_kernel(const __grid_constant__ DqLaunch L) {
    const int j = (L.njobs > 1 && (int)blockIdx.x >= L.job[1].cta0) ? 1 : 0;
    if constexpr (B0 == B1) {
        dequant_cta<TOut, B0, STAGED>(&L.omap[j], L.job[j]);
    } else {
        if (j == 0) dequant_cta<TOut, B0, STAGED>(&L.omap[0], L.job[0]);
        else dequant_cta<TOut, B1, STAGED>(&L.omap[1], L.job[1]);
    }
}

}  // namespace dq

// ── host side ───────────────────────────────────────────────────────────────

static PFN_cuTensorMapEncodeTiled_v12000 dq_encode() {
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

static bool encode_output_map(CUtensorMap* map, const TqArgs& a) {
    auto encode = dq_encode();
    if (!encode) return false;
    const int64_t nvec = a.num_tokens * a.num_heads;
    const cuuint64_t dims[2] = {(cuuint64_t)dq::D, (cuuint64_t)nvec};
    const cuuint64_t strides[1] = {(cuuint64_t)dq::D * 2};
    const cuuint32_t box[2] = {64, 32};  // one epilogue warp's rows of one 64-column half
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, a.out_dtype == FB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  a.output, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Launches jobs[0..njobs) (njobs 1 or 2) as one grid of at most one CTA per SM, split between
// the jobs in proportion to their tiles (each job at least one CTA, at most one per tile).
template <typename TOut, int B0, int B1, bool STAGED>
static int launch_dequant(const TqArgs* jobs, int njobs, cudaStream_t s) {
    dq::DqLaunch L;
    memset(&L, 0, sizeof L);
    L.njobs = njobs;
    int64_t tiles[2] = {0, 0};
    for (int j = 0; j < njobs; ++j) {
        if (!encode_output_map(&L.omap[j], jobs[j])) return (int)cudaErrorInvalidValue;
        L.job[j].a = jobs[j];
        L.job[j].hdiv = sm100::make_divu32((uint32_t)jobs[j].num_heads);
        tiles[j] = (jobs[j].num_tokens * jobs[j].num_heads + dq::TILE - 1) / dq::TILE;
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
    constexpr int smem = std::max(dq::Smem<B0>::bytes, dq::Smem<B1>::bytes);
    auto kern = dq::tq_dequant_umma_kernel<TOut, B0, B1, STAGED>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    kern<<<std::max(1, n0 + n1), dq::THREADS, smem, s>>>(L);
    return (int)cudaGetLastError();
}

static bool dq_eligible(const TqArgs& a) {
    if (a.head_dim != dq::D || !(a.bits == 2 || a.bits == 3 || a.bits == 4)) return false;
    if (a.out_dtype != FB_FP16 && a.out_dtype != FB_BF16) return false;
    if (!aligned16(a.output) || !aligned16(a.packed_pool) || (((uintptr_t)a.norms_pool) & 1)) return false;
    if (!aligned16(a.rotation)) return false;
    if (a.num_tokens * a.num_heads > ((int64_t)1 << 31) - dq::TILE) return false;
    static const bool sm100 = [] {
        int dev = 0, major = 0, minor = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return false;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        return major == 10 && minor == 0;
    }();
    return sm100;
}

// Tiles of whole tokens in at most two cache blocks, pools that bulk copies can read.
static bool dq_stageable(const TqArgs& a) {
    return !a.slot_map && a.num_heads % 8 == 0 && dq::TILE % a.num_heads == 0 && aligned16(a.norms_pool);
}

template <typename TOut, bool STAGED>
static int launch_same_bits(const TqArgs* jobs, int njobs, int bits, cudaStream_t s) {
    if (bits == 4) return launch_dequant<TOut, 4, 4, STAGED>(jobs, njobs, s);
    if (bits == 3) return launch_dequant<TOut, 3, 3, STAGED>(jobs, njobs, s);
    return launch_dequant<TOut, 2, 2, STAGED>(jobs, njobs, s);
}

int tq_dequant_umma(const TqArgs& a, cudaStream_t s, bool* handled) {
    *handled = false;
    if (!dq_eligible(a)) return 0;
    *handled = true;
    const bool staged = dq_stageable(a);
    if (a.out_dtype == FB_FP16)
        return staged ? launch_same_bits<__half, true>(&a, 1, a.bits, s) : launch_same_bits<__half, false>(&a, 1, a.bits, s);
    return staged ? launch_same_bits<__nv_bfloat16, true>(&a, 1, a.bits, s)
                  : launch_same_bits<__nv_bfloat16, false>(&a, 1, a.bits, s);
}

// K and V of one cache read in one launch, when both take the staged tensor-core path with the
// same output type and their widths are equal or 4/2 (the reference's default key/value widths).
int tq_dequant_umma_pair(const TqArgs& k, const TqArgs& v, cudaStream_t s, bool* handled) {
    *handled = false;
    if (!dq_eligible(k) || !dq_eligible(v) || !dq_stageable(k) || !dq_stageable(v) || k.out_dtype != v.out_dtype)
        return 0;
    if (k.bits != v.bits && !(k.bits == 4 && v.bits == 2)) return 0;
    *handled = true;
    const TqArgs jobs[2] = {k, v};
    const bool pair42 = k.bits != v.bits;
    if (k.out_dtype == FB_FP16)
        return pair42 ? launch_dequant<__half, 4, 2, true>(jobs, 2, s) : launch_same_bits<__half, true>(jobs, 2, k.bits, s);
    return pair42 ? launch_dequant<__nv_bfloat16, 4, 2, true>(jobs, 2, s)
                  : launch_same_bits<__nv_bfloat16, true>(jobs, 2, k.bits, s);
}

unsigned int tq_dequant_timeouts() {
    unsigned int v = 0;
    cudaMemcpyFromSymbol(&v, g_tq_dequant_timeouts, sizeof(v));
    return v;
}

}  // namespace fb
