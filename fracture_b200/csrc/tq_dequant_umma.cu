// TurboQuant dequantize on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Replaces backends/fracture-cuda/kernels/turboquant_decompress.cu:21-127 for head_dim 128,
// 2/3/4-bit codes and FP16/BF16 output:
//
//   x_hat[v][i] = norm[v] * sum_j Pi[j][i] * c[idx[v][j]]
//
// One persistent CTA per SM streams tiles of 128 head vectors:
//
//   warp 0       MMA issuer: acc[v][i] = sum_j Y[v][j] * PiT[i][j] on tcgen05 with
//                Y[v][j] = c[idx[v][j]]; one fp16 pass (fp16 centroids and Pi keep the
//                output within about 1e-4 of its magnitude of the float32 statement)
//   warps 1-8    decoders: two threads per vector gather the packed codes of their half
//                of the row through the block table and write fp16 centroid values
//                straight into the 128-byte-swizzled A tile, through lane-private
//                lookup tables (two 4-bit, four 2-bit or two 3-bit codes per lookup)
//   warps 9-16   epilogue, two warpgroups on alternating TMEM buffers: one thread per
//                vector scales its accumulator row by the stored fp16 norm, converts,
//                stages the tile in swizzled shared memory, and one thread writes it out
//                with two TMA tensor stores
//
// Pool rows follow the slot rule of tq_common.cuh; a token without a valid slot
// dequantizes to zeros (norm 0), as the CUDA-core kernel does. Every barrier wait is
// bounded; on timeout the kernel counts the event in g_tq_dequant_timeouts, abandons
// its loop and still frees its TMEM.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tq_common.cuh"
#include "tq_sm100.cuh"

namespace fb {

__device__ unsigned int g_tq_dequant_timeouts = 0;

namespace dq {

using namespace sm100;

constexpr int A_STAGES = 2;  // A tiles in flight
constexpr int TBUF = 2;      // TMEM accumulators = epilogue warpgroups = staging tiles
constexpr int DEC_WARPS = 8;
constexpr int EPI_WARPS = 4 * TBUF;
constexpr int THREADS = 32 * (1 + DEC_WARPS + EPI_WARPS);
constexpr int MAX_REGS = 96;  // 17 warps: up to 5 on one scheduler, 16K registers each
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

struct Misc {
    uint64_t a_full[A_STAGES];
    uint64_t a_empty[A_STAGES];
    uint64_t tfull[TBUF];
    uint64_t tempty[TBUF];
    uint64_t st_free[TBUF];  // staging tile may be overwritten (its last TMA store has read it)
    uint64_t st_full[TBUF];  // staging tile written by all four warps of the warpgroup
    uint32_t tmem_base;
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
    static constexpr int b_off = 0;                                   // Pi^T, fp16, SW128
    static constexpr int a_off = TILE_BYTES;                          // A_STAGES decoded tiles
    static constexpr int st_off = a_off + A_STAGES * TILE_BYTES;      // TBUF output staging tiles
    static constexpr int tab_off = st_off + TBUF * TILE_BYTES;
    static constexpr int misc_off = tab_off + Table<BITS>::bytes;
    static constexpr int bytes = misc_off + (int)sizeof(Misc) + 1024;
};

// Bounded wait for the phase with parity `parity`; false (and a counted timeout) if it never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kTimeoutCycles) {
            atomicAdd(&g_tq_dequant_timeouts, 1u);
            return false;
        }
    }
    return true;
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

template <typename TOut, int BITS>
__global__ void __maxnreg__(MAX_REGS)
    tq_dequant_umma_kernel(const __grid_constant__ CUtensorMap omap, TqArgs a, int num_tiles) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    using L = Smem<BITS>;
    using TB = Table<BITS>;
    uint8_t* sB = base + L::b_off;
    uint8_t* sA = base + L::a_off;
    uint8_t* sST = base + L::st_off;
    uint8_t* tab = base + L::tab_off;
    Misc* misc = (Misc*)(base + L::misc_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nlev = 1 << BITS;
    const int P = (D * BITS) >> 3;
    const int64_t nvec = a.num_tokens * a.num_heads;
    const int ntiles_cta = num_tiles > (int)blockIdx.x ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    // ── prologue ─────────────────────────────────────────────────────────────
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(
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
        for (int b = 0; b < TBUF; ++b) {
            mbar_init(&misc->tfull[b], 1);
            mbar_init(&misc->tempty[b], 4);
            mbar_init(&misc->st_free[b], 1);
            mbar_init(&misc->st_full[b], 4);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // B operand: B[i][j] = Pi[j][i] in fp16 (K-major: the contraction index j is contiguous).
    for (int e = threadIdx.x; e < D * D; e += THREADS) {
        const int j = e >> 7, i = e & (D - 1);
        *(__half*)(sB + sw128_offset(i, j)) = __float2half_rn(__ldg(a.rotation + e));
    }
    // Decode tables (codes in MSB-first order: the first code of a byte is its high bits).
    for (int e = threadIdx.x; e < TB::entries * TB::copies; e += THREADS) {
        const int ent = e / TB::copies;
        if constexpr (BITS == 4) {
            const __half2 h = __floats2half2_rn(__ldg(a.centroids + (ent >> 4)), __ldg(a.centroids + (ent & 15)));
            ((uint32_t*)tab)[e] = h2_bits(h);
        } else if constexpr (BITS == 3) {
            const __half2 h = __floats2half2_rn(__ldg(a.centroids + (ent >> 3)), __ldg(a.centroids + (ent & 7)));
            ((uint32_t*)tab)[e] = h2_bits(h);
        } else {
            const __half2 h0 = __floats2half2_rn(__ldg(a.centroids + (ent >> 6)), __ldg(a.centroids + ((ent >> 4) & 3)));
            const __half2 h1 = __floats2half2_rn(__ldg(a.centroids + ((ent >> 2) & 3)), __ldg(a.centroids + (ent & 3)));
            ((uint2*)tab)[e] = make_uint2(h2_bits(h0), h2_bits(h1));
        }
    }
    (void)nlev;
    fence_async_smem();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = misc->tmem_base;

    if (warp == 0) {
        // ── MMA issuer ──────────────────────────────────────────────────────
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16(0u);
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            int done = 0;
            for (int i = 0; i < ntiles_cta; ++i) {
                const int s = i % A_STAGES, buf = i % TBUF;
                if (!mbar_wait(&misc->a_full[s], (i / A_STAGES) & 1)) break;
                if (!mbar_wait(&misc->tempty[buf], ((i / TBUF) + 1) & 1)) break;
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
            if (done > 0) mbar_wait(&misc->tfull[(done - 1) % TBUF], ((done - 1) / TBUF) & 1);
        }
    } else if (warp <= DEC_WARPS) {
        // ── decoders: thread dt handles half h of row r ─────────────────────
        const int dt = threadIdx.x - 32;
        const int r = dt >> 1, h = dt & 1;
        const uint32_t tlane = smem_u32(tab) + (uint32_t)(lane & (TB::copies - 1)) * TB::entry_bytes;
        for (int i = 0; i < ntiles_cta; ++i) {
            const int s = i % A_STAGES;
            const int tile = (int)blockIdx.x + i * (int)gridDim.x;
            const int64_t vi = (int64_t)tile * TILE + r;
            int64_t slot = -1;
            if (vi < nvec) slot = tq_slot(a, vi / a.num_heads);
            const uint8_t* src =
                slot >= 0 ? (const uint8_t*)a.packed_pool + (slot * a.num_heads + vi % a.num_heads) * P + h * (P / 2)
                          : nullptr;
            // this half-row's packed bytes (zeros when the vector has no slot)
            uint32_t wv[BITS * 2];
#pragma unroll
            for (int k = 0; k < BITS * 2; ++k) wv[k] = 0u;
            if (src) {
                if constexpr (BITS == 3) {
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        const uint2 t = __ldg((const uint2*)src + k);
                        wv[2 * k] = t.x;
                        wv[2 * k + 1] = t.y;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < BITS / 2; ++k) {
                        const uint4 t = __ldg((const uint4*)src + k);
                        wv[4 * k] = t.x;
                        wv[4 * k + 1] = t.y;
                        wv[4 * k + 2] = t.z;
                        wv[4 * k + 3] = t.w;
                    }
                }
            }
            if (!mbar_wait(&misc->a_empty[s], ((i / A_STAGES) + 1) & 1)) break;
            uint8_t* dstrow = sA + s * TILE_BYTES;
#pragma unroll
            for (int c = 0; c < 8; ++c) {  // 8 chunks of 8 values: columns 64h + 8c ..
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
                *(uint4*)(dstrow + sw128_offset(r, 64 * h + 8 * c)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&misc->a_full[s]);
        }
    } else {
        // ── epilogue: warpgroup e takes the tiles i with i % TBUF == e ──────
        const int e = (warp - 1 - DEC_WARPS) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const bool leader = ((warp - 1 - DEC_WARPS) & 3) == 0 && lane == 0;
        uint8_t* st = sST + e * TILE_BYTES;
        int n = 0;
        for (int i = e; i < ntiles_cta; i += TBUF, ++n) {
            const int tile = (int)blockIdx.x + i * (int)gridDim.x;
            const int64_t vi = (int64_t)tile * TILE + row;
            float nrm = 0.0f;
            if (vi < nvec) {
                const int64_t slot = tq_slot(a, vi / a.num_heads);
                if (slot >= 0) nrm = __half2float(((const __half*)a.norms_pool)[slot * a.num_heads + vi % a.num_heads]);
            }
            if (leader) {
                bulk_wait_read_all();  // the previous store from this staging tile has read it
                mbar_arrive(&misc->st_free[e]);
            }
            if (!mbar_wait(&misc->tfull[e], n & 1)) break;
            if (!mbar_wait(&misc->st_free[e], n & 1)) break;
            tc_fence_after();
            const uint32_t taddr = tmem_base + (uint32_t)(e * D) + ((uint32_t)(quarter * 32) << 16);
#pragma unroll
            for (int cchunk = 0; cchunk < D / 32; ++cchunk) {
                uint32_t v[32];
                tmem_ld32_issue(taddr + cchunk * 32, v);
                tmem_wait_tie(v);
                if (cchunk == D / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&misc->tempty[e]);
                }
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    uint32_t o[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        o[k] = pack_out<TOut>(__uint_as_float(v[8 * g + 2 * k]) * nrm,
                                              __uint_as_float(v[8 * g + 2 * k + 1]) * nrm);
                    *(uint4*)(st + sw128_offset(row, 32 * cchunk + 8 * g)) = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&misc->st_full[e]);
            if (leader) {
                if (!mbar_wait(&misc->st_full[e], n & 1)) break;
                tma_store_2d(&omap, st, 0, tile * TILE);
                tma_store_2d(&omap, st + KBLK_BYTES, 64, tile * TILE);
                bulk_commit();
            }
        }
        if (leader) bulk_wait_all();
    }

    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem_base) : "memory");
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

template <typename TOut, int BITS>
static int launch_dequant(const TqArgs& a, cudaStream_t s) {
    auto encode = dq_encode();
    if (!encode) return (int)cudaErrorNotSupported;
    const int64_t nvec = a.num_tokens * a.num_heads;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)dq::D, (cuuint64_t)nvec};
    const cuuint64_t strides[1] = {(cuuint64_t)dq::D * sizeof(TOut)};
    const cuuint32_t box[2] = {64, (cuuint32_t)dq::TILE};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(&map, dtype_of<TOut>::value == FB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        2, a.output, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return (int)cudaErrorInvalidValue;
    constexpr int smem = dq::Smem<BITS>::bytes;
    auto kern = dq::tq_dequant_umma_kernel<TOut, BITS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    const int num_tiles = (int)((nvec + dq::TILE - 1) / dq::TILE);
    const int grid = std::max(1, std::min(num_tiles, num_sms()));
    kern<<<grid, dq::THREADS, smem, s>>>(map, a, num_tiles);
    return (int)cudaGetLastError();
}

int tq_dequant_umma(const TqArgs& a, cudaStream_t s, bool* handled) {
    *handled = false;
    if (a.head_dim != dq::D || !(a.bits == 2 || a.bits == 3 || a.bits == 4)) return 0;
    if (a.out_dtype != FB_FP16 && a.out_dtype != FB_BF16) return 0;
    if (!aligned16(a.output) || !aligned16(a.packed_pool) || (((uintptr_t)a.norms_pool) & 1)) return 0;
    if (((uintptr_t)a.rotation & 3) != 0) return 0;
    if (a.num_tokens * a.num_heads > ((int64_t)1 << 31) - dq::TILE) return 0;
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) return 0;
    *handled = true;
    if (a.out_dtype == FB_FP16) {
        if (a.bits == 4) return launch_dequant<__half, 4>(a, s);
        if (a.bits == 3) return launch_dequant<__half, 3>(a, s);
        return launch_dequant<__half, 2>(a, s);
    }
    if (a.bits == 4) return launch_dequant<__nv_bfloat16, 4>(a, s);
    if (a.bits == 3) return launch_dequant<__nv_bfloat16, 3>(a, s);
    return launch_dequant<__nv_bfloat16, 2>(a, s);
}

unsigned int tq_dequant_timeouts() {
    unsigned int v = 0;
    cudaMemcpyFromSymbol(&v, g_tq_dequant_timeouts, sizeof(v));
    return v;
}

}  // namespace fb
