// Streamed tensor-core attention over the TurboQuant paged cache (2-, 4- and 8-bit codes), sm_100a.
//
// Replaces tqa_mma (2- and 4-bit codes) and tqa_chunk (8-bit codes) for caches with a KV-head count
// that is a multiple of 8, in this library's contiguous pools or in the reference ABI's per-block
// buffers (template PTRS: copied block by block with bulk copies). The math is the same split-K statement
// (attention_paged_tq.cu:12-17 of the reference: scores in K's rotated space, softmax, values
// summed in V's rotated space; tqa_combine adds the partials and rotates back), the operands
// decoded the same way (lane-private lookup tables feeding mma.sync m16n8k16 with FP16
// operands and FP32 accumulators). What changes is how the cache reaches the warps:
//
//   * An item is (sequence, chunk of positions, query token, group of 8 KV heads). The 16 rows
//     of a block hold all KV heads of a position side by side, so one block's K codes for the
//     group are one rectangle of the pool, fetched with one TMA box; the V codes likewise; the
//     norms of a block are one contiguous run (one bulk copy) when the pool holds 8 KV heads,
//     else a TMA box. A stage holds two blocks (one with 8-bit codes); the ring of stages runs
//     ahead across items.
//   * Two producer warps per block slot issue a stage's copies in parallel (K side / V side:
//     the issue of one copy takes long enough that one thread would not keep up), each first
//     planning the item's blocks from the block table (32 entries per load, the next item's
//     entries requested before this item's copies).
//   * Eight consumer warps: warp w takes KV head w of the group in every tile of a stage (two
//     tiles are independent work for the scheduler), keeps a running softmax for the
//     head's Q heads over the item, and writes one partial (maximum, sum, accumulator). The
//     item's rotated queries are loaded into registers one item ahead.
//   * A block's codes land as [16 rows][128-byte lines] with the 128-byte swizzle, and the value
//     MMA's k index 2t + e stands for position t + 4e, so the lanes of one shared-memory
//     wavefront read lines whose swizzle phases differ: the K and 2-bit V code loads are
//     conflict-free.
//   * The decoding tables sit at shared address 0x10000 (64 KB aligned): one byte permute of a
//     code byte and the lane's copy offset is the whole lookup address. 2-bit codes decode four
//     at a time (one 8-byte lookup, 16 lane copies), 4-bit codes two at a time (one 4-byte
//     lookup, 32 copies), 8-bit codes one at a time (two lookups and a byte permute per register). Scores carry log2(e) so the softmax uses exp2; the partial's maximum
//     is converted back to natural units.
//
// Every wait is bounded: a wait that runs out counts itself in g_tqa_stream_timeouts, raises the
// CTA's abort flag and ends the warp's work; each producer then waits (bounded) for the copies
// in flight before the CTA exits.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "tq_attention.cuh"
#include "tq_sm100.cuh"

namespace fb {

__device__ unsigned int g_tqa_stream_timeouts = 0;

namespace tqa {
namespace stream {

using namespace sm100;

constexpr int HC = 8;                    // KV heads per item
constexpr int NCW = 8;                   // consumer warps: warp w takes KV head w in every block of a stage
constexpr int MAX_NST = 8;
constexpr int MAX_SPI = 128;             // stages per item (2048 positions at one block per stage)
constexpr uint32_t TAB = 0x10000;        // shared address of the decoding tables (64 KB)
constexpr uint32_t DYN_BYTES = 232448;   // dynamic shared memory requested (the sm_100 maximum)
constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// A stage holds BPS 16-position blocks: two, or one when a side has 8-bit codes (its blocks are
// 16 KB). Producer warp p copies block slot p % BPS, side p / BPS (0: K codes and norms, 1: V).
// 8-bit codes sit line-major ([lines][16 rows][128]) so that the 128-byte swizzle phase follows
// the row; 2- and 4-bit codes row-major ([16 rows][lines][128]).
template <int KB, int VB>
struct Layout {
    static constexpr bool K8 = KB == 8, V8 = VB == 8;
    static constexpr int BPS = K8 || V8 ? 1 : 2;
    static constexpr int NPW = 2 * BPS;
    static constexpr int THREADS = (NCW + NPW) * 32;
    static constexpr int PK = D * KB / 8, PV = D * VB / 8;
    static constexpr int KBOX = HC * PK / 128, VBOX = HC * PV / 128;  // 128-byte lines per block row
    static constexpr int k_off = 0;
    static constexpr int v_off = BPS * KBOX * 2048;
    static constexpr int kn_off = v_off + BPS * VBOX * 2048;
    static constexpr int vn_off = kn_off + BPS * 16 * HC * 2;
    static constexpr int hdr_off = vn_off + BPS * 16 * HC * 2;
    static constexpr int stage_bytes = (hdr_off + 16 + 1023) / 1024 * 1024;
};

// Shared memory other than the tables and stages: barriers, the producers' plans, the
// consumers' weight tiles and, with per-block buffers (PTRS), the producers' block pointers.
template <int BPS, bool PTRS>
struct Small {
    static constexpr int NPW = 2 * BPS;
    static constexpr int bar_off = 0;                           // full[MAX_NST], empty[MAX_NST], abort flag
    static constexpr int plan_off = 256;                        // [NPW][MAX_SPI] int2
    static constexpr int p_off = plan_off + NPW * MAX_SPI * 8;  // [NCW][BPS][16 x 8] f16
    static constexpr int ptr_off = p_off + NCW * BPS * 256;     // [NPW][MAX_SPI / BPS] (codes, norms) pointers
    static constexpr int bytes = (ptr_off + (PTRS ? NPW * (MAX_SPI / BPS) * 16 : 0) + 1023) / 1024 * 1024;
};

struct Params {
    CUtensorMap kmap, vmap, knmap, vnmap;  // codes: uint8 [pool_rows][hkv * P / 128][128]; norms: f16 [pool_rows, hkv]
    AttnArgs a;
    int items, spi;                // spi: stages per item (ch = spi * blocks per stage * 16)
    int nchi, ng;                  // chunks per sequence, KV-head groups
    DivU32 dng, dqps, dnchi;
    int64_t pool_rows;
    const __half* kn;              // norm pools (bulk copies when norms_bulk)
    const __half* vn;
    int norms_bulk;                // hkv == HC: a block's norms are contiguous
    // per-block buffers (kernel template PTRS, the reference ABI's cache): block b's codes
    // [16, hkv * P] at codes[side][b], its norms [16, hkv] at norms[side][b]; side 0 K, 1 V
    const uint8_t* const* codes[2];
    const __half* const* norms[2];
};

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
            : "memory");
        if (ok) return true;
        if (*abort) return false;
        if (clock64() - t0 > kTimeoutCycles) {
            atomicAdd(&g_tqa_stream_timeouts, 1u);
            *abort = 1;
            return false;
        }
    }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            dst),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
__device__ __forceinline__ void tma_load_2d_u(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void bulk_load_u(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// Shared-memory loads the compiler may schedule freely: every address they take is derived
// from a value produced after the barrier that makes the data valid (the decoding tables are
// written before the block-wide barrier; a stage's base comes from stage_base(), which is
// ordered after that stage's wait).
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ float lds16f(uint32_t addr) {
    unsigned short v;
    asm("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return __half2float(__ushort_as_half(v));
}
// A value the compiler cannot compute before this point: loads addressed through it stay after
// the barrier wait that precedes it.
__device__ __forceinline__ uint32_t after_wait(uint32_t x) {
    uint32_t y;
    asm volatile("mov.b32 %0, %1;" : "=r"(y) : "r"(x) : "memory");
    return y;
}
__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// Table address of code byte b of word w: TAB | byte << 8 | lane offset (off = TAB | offset < 256).
__device__ __forceinline__ uint32_t tab_addr(uint32_t w, uint32_t off, int b) {
    return __byte_perm(w, off, 0x7604u | ((uint32_t)b << 4));
}

// Item index -> (sequence, chunk, query token, head group); sequence-major so that the query
// tokens of one sequence and chunk are neighbours (their CTAs read the same codes from L2).
struct Item {
    int s, c, t, hg, row, L, p0, nstg;
};
template <int BPS>
__device__ __forceinline__ Item decode_item(const Params& P, int item) {
    Item it;
    const uint32_t r1 = divu32((uint32_t)item, P.dng);
    it.hg = item - (int)r1 * P.ng;
    const uint32_t r2 = divu32(r1, P.dqps);
    it.t = (int)r1 - (int)r2 * P.a.q_per_seq;
    const uint32_t r3 = divu32(r2, P.dnchi);
    it.c = (int)r2 - (int)r3 * P.nchi;
    it.s = (int)r3;
    it.row = it.s * P.a.q_per_seq + it.t;
    it.L = causal_len(P.a, it.s, it.t);
    it.p0 = it.c * P.spi * BPS * 16;
    it.nstg = it.p0 < it.L ? min(P.spi, (it.L - it.p0 + BPS * 16 - 1) / (BPS * 16)) : 0;
    return it;
}

// Where the stages and the small region sit. The window of dynamic shared memory is
// [base, base + DYN_BYTES); the tables take [TAB, TAB + 64 KB); stages fill [base, TAB) and then
// [TAB + 64 KB, small), the small region the end of the window.
struct Places {
    uint32_t lo, hi, small;
    int n_lo, nst;
    __device__ uint32_t stage(int i, int sb) const { return i < n_lo ? lo + i * sb : hi + (i - n_lo) * sb; }
};
template <int SMALL_BYTES>
__device__ __forceinline__ Places places(uint32_t base, int sb) {
    Places pl;
    pl.lo = (base + 1023u) & ~1023u;
    pl.hi = TAB + 0x10000u;
    pl.small = ((base + DYN_BYTES) & ~1023u) - SMALL_BYTES;
    pl.n_lo = pl.lo + sb <= TAB ? (int)((TAB - pl.lo) / sb) : 0;
    const int n_hi = pl.small >= pl.hi + sb ? (int)((pl.small - pl.hi) / sb) : 0;
    pl.nst = min(MAX_NST, pl.n_lo + n_hi);
    return pl;
}

// PTRS: the cache is the reference ABI's per-block buffers, a block's rows of one head group
// copied by bulk copies into unswizzled stage rows; else the pools, copied by TMA boxes that land
// with the 128-byte swizzle.
template <int KB, int VB, bool PTRS>
__global__ void __launch_bounds__(Layout<KB, VB>::THREADS, 1) tqa_stream(const __grid_constant__ Params P) {
    pdl_trigger();  // the combine's CTAs may take SMs this grid has left and stage Pi_v meanwhile
    using Ly = Layout<KB, VB>;
    constexpr int PK = Ly::PK, PV = Ly::PV;
    constexpr int SB = Ly::stage_bytes;
    constexpr int BPS = Ly::BPS, NPW = Ly::NPW, THREADS = Ly::THREADS;
    using Sm = Small<BPS, PTRS>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t base = smem_u32(smem_raw);
    const Places pl = places<Sm::bytes>(base, SB);
    const AttnArgs& a = P.a;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.hq / a.hkv;
    // a window that does not hold the tables and two stages (not expected: the window starts
    // within the first few KB of the shared address space) ends the launch with a counted error
    if (base + 1024 > TAB || pl.nst < 2) {
        if (threadIdx.x == 0) atomicAdd(&g_tqa_stream_timeouts, 1u);
        return;
    }
    uint8_t* gsmall = smem_raw + (pl.small - base);  // generic pointer to the small region
    uint64_t* full = (uint64_t*)(gsmall + Sm::bar_off);
    uint64_t* empty = full + MAX_NST;
    volatile int* abort = (volatile int*)(empty + MAX_NST);

    if (threadIdx.x == 0) {
        for (int i = 0; i < pl.nst; ++i) {
            mbar_init(&full[i], NPW);
            mbar_init(&empty[i], NCW);
        }
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // Decoding tables (codes MSB first: the first code of a byte is its high bits). Entry e at
    // TAB + 256e. K part (+0): 8-bit, 32 copies of half2(c[e], c[e]); 4-bit, 32 copies of
    // half2(c[e >> 4], c[e & 15]); 2-bit, 16 copies of half2(c[e >> 6], c[(e >> 4) & 3]),
    // half2(c[(e >> 2) & 3], c[e & 3]) (four coordinates of one row). V part (+128): 8-bit and
    // 4-bit as for K (a 4-bit pair is one coordinate at two positions); 2-bit, 16 copies of half2(c[e >> 6], c[(e >> 2) & 3]), half2(c[(e >> 4) & 3],
    // c[e & 3]) (two coordinates, each at two positions; the index interleaves two positions'
    // code bytes).
    for (int j = threadIdx.x; j < 512; j += THREADS) {
        const int e = j >> 1;
        const bool key = (j & 1) == 0;
        const int bits = key ? KB : VB;
        const float* cen = key ? a.ck : a.cv;
        uint4 v;
        if (bits == 8) {  // one code: half2(c[e], c[e])
            const uint32_t w = pack_half2(__ldg(cen + e), __ldg(cen + e));
            v = make_uint4(w, w, w, w);
        } else if (bits == 4) {
            const uint32_t w = pack_half2(__ldg(cen + (e >> 4)), __ldg(cen + (e & 15)));
            v = make_uint4(w, w, w, w);
        } else if (key) {
            const uint32_t w0 = pack_half2(__ldg(cen + (e >> 6)), __ldg(cen + ((e >> 4) & 3)));
            const uint32_t w1 = pack_half2(__ldg(cen + ((e >> 2) & 3)), __ldg(cen + (e & 3)));
            v = make_uint4(w0, w1, w0, w1);
        } else {
            const uint32_t w0 = pack_half2(__ldg(cen + (e >> 6)), __ldg(cen + ((e >> 2) & 3)));
            const uint32_t w1 = pack_half2(__ldg(cen + ((e >> 4) & 3)), __ldg(cen + (e & 3)));
            v = make_uint4(w0, w1, w0, w1);
        }
        const uint32_t row = TAB + e * 256 + (key ? 0 : 128);
#pragma unroll
        for (int k = 0; k < 8; ++k) sts128(row + 16 * ((k + j) & 7), v);
    }
    // The tables read only the codebooks; what follows reads the rotate kernel's output.
    pdl_begin();
    __syncthreads();

    if (warp >= NCW) {
        // ── producers: warp NCW + p copies block slot p % BPS, side p / BPS (0: K codes and norms,
        // 1: V codes and norms) of every stage ──
        const int p = warp - NCW, slot = p % BPS, side = p / BPS;
        int2* plan = (int2*)(gsmall + Sm::plan_off) + p * MAX_SPI;  // per stage: (pool row, valid rows)
        int sidx = 0;
        uint32_t sph = 0;
        long long issued = 0;
        bool ok = true;
        // block-table entries of an item for this slot: lane l holds stages l, l + 32, ... (with
        // per-block buffers, also the blocks' code and norm pointers of this side)
        constexpr int NBT = MAX_SPI / BPS / 32;
        constexpr int NBP = PTRS ? NBT : 1;
        unsigned long long cp_next[NBP], np_next[NBP];
        auto fetch = [&](int item, int32_t (&bt)[NBT]) {
            Item it{};
            if (item < P.items) it = decode_item<BPS>(P, item);
#pragma unroll
            for (int i = 0; i < NBT; ++i) {
                const int st = lane + 32 * i, b = (it.p0 >> 4) + BPS * st + slot;
                bt[i] = it.nstg > 0 && st < it.nstg && b < a.max_blocks
                            ? __ldg(a.block_tables + (int64_t)it.s * a.max_blocks + b)
                            : -1;
            }
            if constexpr (PTRS) {
#pragma unroll
                for (int i = 0; i < NBT; ++i) {
                    cp_next[i] = bt[i] >= 0 ? __ldg((const unsigned long long*)P.codes[side] + bt[i]) : 0ull;
                    np_next[i] = bt[i] >= 0 ? __ldg((const unsigned long long*)P.norms[side] + bt[i]) : 0ull;
                }
            }
        };
        int32_t bt_next[NBT];
        fetch(blockIdx.x, bt_next);
        for (int item = blockIdx.x; item < P.items && ok; item += gridDim.x) {
            int32_t bt[NBT];
            unsigned long long cps[NBP], nps[NBP];
#pragma unroll
            for (int i = 0; i < NBT; ++i) bt[i] = bt_next[i];
            if constexpr (PTRS) {
#pragma unroll
                for (int i = 0; i < NBT; ++i) {
                    cps[i] = cp_next[i];
                    nps[i] = np_next[i];
                }
            }
            const Item it = decode_item<BPS>(P, item);
            fetch(item + gridDim.x, bt_next);
            if (it.nstg == 0) continue;
            // valid rows of each block from row 0: causal range, missing blocks, pool end
#pragma unroll
            for (int i = 0; i < NBT; ++i) {
                const int st = lane + 32 * i;
                const int32_t blk = bt[i];
                const int pos = it.p0 + (BPS * st + slot) * 16;
                const int64_t first = (int64_t)blk * 16;
                int n = 0;
                if (blk >= 0 && pos < it.L && first < P.pool_rows)
                    n = (int)min((int64_t)min(16, it.L - pos), P.pool_rows - first);
                plan[st] = make_int2(n > 0 ? (int)first : 0, n);
                if constexpr (PTRS)
                    ((ulonglong2*)(gsmall + Sm::ptr_off))[p * (MAX_SPI / BPS) + st] = make_ulonglong2(cps[i], nps[i]);
            }
            __syncwarp();
            if constexpr (PTRS) {
                // The group's rows of a block: with 8 KV heads the whole buffers (one bulk copy for
                // the codes, one for the norms), else 16 code rows and 16 norm rows, one copy per
                // lane. A block whose buffers are not 16-byte aligned is copied by the lanes with
                // byte loads and shared stores into the same unswizzled rows.
                const ulonglong2* pp = (const ulonglong2*)(gsmall + Sm::ptr_off) + p * (MAX_SPI / BPS);
                const uint32_t rb = HC * (side ? PV : PK);       // a stage row: the group's codes of a position
                const uint32_t cb = 16u * rb;
                const int64_t rs = (int64_t)a.hkv * (side ? PV : PK);  // a buffer row
                const int64_t ns = (int64_t)a.hkv * 2;
                const uint32_t cd0 = side ? Ly::v_off + slot * Ly::VBOX * 2048 : Ly::k_off + slot * Ly::KBOX * 2048;
                const uint32_t nd0 = (side ? Ly::vn_off : Ly::kn_off) + slot * 16 * HC * 2;
                for (int st = 0; st < it.nstg; ++st) {
                    const int2 pn = plan[st];
                    const ulonglong2 ptr = pp[st];
                    if (lane == 0) ok = wait_bar(&empty[sidx], sph ^ 1u, abort);
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok) break;
                    __syncwarp();  // every lane's writes into the stage come after lane 0's wait
                    const uint32_t stg = pl.stage(sidx, SB);
                    const uint32_t cd = stg + cd0, nd = stg + nd0;
                    const uint8_t* cs = (const uint8_t*)ptr.x + (int64_t)it.hg * rb;
                    const uint8_t* nsrc = (const uint8_t*)ptr.y + it.hg * HC * 2;
                    const bool bulk = ((ptr.x | ptr.y) & 15ull) == 0;
                    if (pn.y > 0 && !bulk) {
                        for (uint32_t e = lane; e < cb; e += 32)
                            asm volatile("st.shared.u8 [%0], %1;" ::"r"(cd + e), "h"((unsigned short)__ldg(cs + (e / rb) * rs + e % rb))
                                         : "memory");
                        for (uint32_t e = lane; e < 16u * HC * 2u; e += 32)
                            asm volatile("st.shared.u8 [%0], %1;" ::"r"(nd + e), "h"((unsigned short)__ldg(nsrc + (e >> 4) * ns + (e & 15)))
                                         : "memory");
                        fence_async_smem();  // later bulk copies into these bytes come after the stores
                    }
                    __syncwarp();
                    if (lane == 0) {
                        if (side == 0) *(int*)(smem_raw + (stg - base) + Ly::hdr_off + 4 * slot) = pn.y;
                        mbar_expect_tx(&full[sidx], pn.y > 0 && bulk ? cb + 16u * HC * 2u : 0u);
                    }
                    __syncwarp();
                    if (pn.y > 0 && bulk) {
                        if (a.hkv == HC) {
                            if (lane == 0) bulk_load_u(cd, cs, cb, &full[sidx]);
                            if (lane == 16) bulk_load_u(nd, nsrc, 16u * HC * 2u, &full[sidx]);
                        } else if (lane < 16) {
                            bulk_load_u(cd + lane * rb, cs + lane * rs, rb, &full[sidx]);
                        } else {
                            bulk_load_u(nd + (lane - 16) * 16, nsrc + (lane - 16) * ns, 16u, &full[sidx]);
                        }
                    }
                    ++issued;
                    if (++sidx == pl.nst) {
                        sidx = 0;
                        sph ^= 1u;
                    }
                }
            } else if (lane == 0) {
                for (int st = 0; st < it.nstg; ++st) {
                    const int2 pn = plan[st];
                    ok = wait_bar(&empty[sidx], sph ^ 1u, abort);
                    if (!ok) break;
                    const uint32_t stg = pl.stage(sidx, SB);
                    if (side == 0) *(int*)(smem_raw + (stg - base) + Ly::hdr_off + 4 * slot) = pn.y;
                    // norms: with one head group the block's norms are 16 rows x 16 contiguous
                    // bytes, copied as far as the pool reaches; else a TMA box (zeros past the pool)
                    const uint32_t nb = !P.norms_bulk ? 16u * HC * 2u
                                                      : (uint32_t)min((int64_t)16, P.pool_rows - pn.x) * (HC * 2u);
                    const uint32_t tx = pn.y > 0 ? (side ? Ly::VBOX : Ly::KBOX) * 2048u + nb : 0u;
                    mbar_expect_tx(&full[sidx], tx);
                    if (pn.y > 0) {
                        const uint32_t nd = stg + (side ? Ly::vn_off : Ly::kn_off) + slot * 16 * HC * 2;
                        // row-major maps take (line, row), line-major ones (8-bit codes) (row, line)
                        if (side == 0) {
                            const int l0 = it.hg * Ly::KBOX;
                            tma_load_3d(stg + Ly::k_off + slot * Ly::KBOX * 2048, &P.kmap, &full[sidx], 0,
                                        Ly::K8 ? pn.x : l0, Ly::K8 ? l0 : pn.x);
                        } else {
                            const int l0 = it.hg * Ly::VBOX;
                            tma_load_3d(stg + Ly::v_off + slot * Ly::VBOX * 2048, &P.vmap, &full[sidx], 0,
                                        Ly::V8 ? pn.x : l0, Ly::V8 ? l0 : pn.x);
                        }
                        if (P.norms_bulk)
                            bulk_load_u(nd, (side ? P.vn : P.kn) + (int64_t)pn.x * HC, nb, &full[sidx]);
                        else
                            tma_load_2d_u(nd, side ? &P.vnmap : &P.knmap, &full[sidx], it.hg * HC, pn.x);
                    }
                    ++issued;
                    if (++sidx == pl.nst) {
                        sidx = 0;
                        sph ^= 1u;
                    }
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            __syncwarp();  // lane 0 is done with the plan
        }
        // no copy may be in flight when the CTA exits: wait for the last stages filled
        if (lane == 0) {
            const int last = issued < (long long)pl.nst ? (int)issued : pl.nst;
            int i = sidx;
            uint32_t ph = sph;
            for (int k = 0; k < last; ++k) {
                if (--i < 0) {
                    i = pl.nst - 1;
                    ph ^= 1u;
                }
                const long long t0 = clock64();
                while (!mbar_try_wait(&full[i], ph))
                    if (clock64() - t0 > kTimeoutCycles) {
                        atomicAdd(&g_tqa_stream_timeouts, 1u);
                        break;
                    }
            }
        }
        return;
    }

    // ── consumers: warp hl takes KV head hl of the group in every block slot ──
    const int r = lane >> 2, t = lane & 3;
    const int hl = warp;
    // This lane's byte offsets inside a stage's block slot 0 (other slots: + the slot's size).
    // Row-major codes (2-, 4-bit): [16 rows][lines][128], the 16-byte chunk j of line L at
    // j ^ (L & 7). Line-major codes (8-bit): [lines][16 rows][128], chunk j of (line, row) at
    // j ^ (row & 7); KV head hl owns line hl. Fragment row r of the score MMA is tile row r. The
    // value MMA's k index 2t + e (+8) stands for position t + 4e (+8) with 2- and 4-bit values
    // and for position 2t + e (+8) with 8-bit ones, so that the lanes of one wavefront read
    // chunks whose swizzle phases differ. koff2 / voff2 / voff3: the second 16 bytes of a K row
    // and the other two V rows of an 8-bit lane.
    uint32_t koff, koff2 = 0, voff0, voff1;
    if constexpr (PTRS) {
        // unswizzled rows of the group: K [16 positions][8 heads x PK], V [16][8 x PV]; the same
        // bytes of a head as the swizzled layouts below give each lane
        koff = Ly::k_off + r * HC * PK + hl * PK + (PK / 4) * t;
        koff2 = koff + 16;
        const int p0 = VB == 8 ? 2 * t : t, p1 = VB == 8 ? 2 * t + 1 : t + 4;
        voff0 = Ly::v_off + p0 * HC * PV + hl * PV + (PV / 8) * r;
        voff1 = Ly::v_off + p1 * HC * PV + hl * PV + (PV / 8) * r;
    } else {
        constexpr int KL = Ly::KBOX, VL = Ly::VBOX;
        const int kc = (hl * PK) >> 7, kj = ((hl * PK) & 127) >> 4;
        if constexpr (KB == 8) {
            koff = Ly::k_off + hl * 2048 + r * 128 + (((2 * t) ^ (r & 7)) << 4);
            koff2 = Ly::k_off + hl * 2048 + r * 128 + (((2 * t + 1) ^ (r & 7)) << 4);
        } else if constexpr (KB == 4) {
            koff = Ly::k_off + r * KL * 128 + kc * 128 + (((kj + t) ^ ((r * KL + kc) & 7)) << 4);
        } else {
            koff = Ly::k_off + r * KL * 128 + kc * 128 + (((kj + (t >> 1)) ^ ((r * KL + kc) & 7)) << 4) + 8 * (t & 1);
        }
        const int vc = (hl * PV) >> 7, vj = ((hl * PV) & 127) >> 4;
        const int q0 = t, q1 = t + 4;
        const int vbase = Ly::v_off + vc * 128;
        if constexpr (VB == 8) {
            const int p0 = 2 * t, p1 = 2 * t + 1;
            voff0 = Ly::v_off + hl * 2048 + p0 * 128 + ((r ^ (p0 & 7)) << 4);
            voff1 = Ly::v_off + hl * 2048 + p1 * 128 + ((r ^ (p1 & 7)) << 4);
        } else if constexpr (VB == 2) {
            voff0 = vbase + q0 * VL * 128 + (((vj + (r >> 2)) ^ ((q0 * VL + vc) & 7)) << 4) + 4 * (r & 3);
            voff1 = vbase + q1 * VL * 128 + (((vj + (r >> 2)) ^ ((q1 * VL + vc) & 7)) << 4) + 4 * (r & 3);
        } else {
            voff0 = vbase + q0 * VL * 128 + (((vj + (r >> 1)) ^ ((q0 * VL + vc) & 7)) << 4) + 8 * (r & 1);
            voff1 = vbase + q1 * VL * 128 + (((vj + (r >> 1)) ^ ((q1 * VL + vc) & 7)) << 4) + 8 * (r & 1);
        }
    }
    constexpr uint32_t KSLOT = Ly::KBOX * 2048, VSLOT = Ly::VBOX * 2048, NSLOT = 16 * HC * 2;
    // 8 rows further: row-major (swizzled or not), 8 rows of lines; line-major, 8 rows of 128 bytes
    constexpr uint32_t KROW8 = Ly::K8 && !PTRS ? 8 * 128 : 8 * Ly::KBOX * 128;
    constexpr uint32_t VROW8 = Ly::V8 && !PTRS ? 8 * 128 : 8 * Ly::VBOX * 128;
    const uint32_t knoff = Ly::kn_off + (r * HC + hl) * 2;
    const uint32_t vnoff = Ly::vn_off + (r * HC + hl) * 2;
    const int kr = Ly::V8 ? r : 2 * (r & 3) + (r >> 2);  // the value MMA's k index of tile row r (r + 8: kr + 8)
    const uint32_t kof = TAB | (KB != 2 ? 4u * lane : 8u * (lane & 15));
    const uint32_t vof = TAB | (VB != 2 ? 128u + 4u * lane : 128u + 8u * (lane & 15));
    const uint32_t pbuf = pl.small + Sm::p_off + warp * BPS * 256;  // this warp's weight tiles
    const uint32_t pw0 = pbuf + (kr * 8 + 2 * t) * 2, pw1 = pw0 + 8 * 8 * 2;  // rows kr, kr + 8
    const uint32_t pld = pbuf + (lane & 15) * 16;                              // ldmatrix row address
    const float kscale = rsqrtf((float)D) * 1.4426950408889634f;  // 1/sqrt(d) and log2(e)

    // rotated queries (fp16) of Q head r of this KV head at coordinates 32t + 4kk .. +3, as the
    // score MMA's B registers (zeros past the group)
    auto load_q = [&](int item, uint2 (&q)[8]) {
        Item it{};
        if (item < P.items) it = decode_item<BPS>(P, item);
        const bool live = it.nstg > 0 && r < G;
        const __half* qh = (const __half*)a.qrot + ((int64_t)it.row * a.hq + (it.hg * HC + hl) * G + r) * D + 32 * t;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) q[kk] = live ? __ldg((const uint2*)(qh + 4 * kk)) : make_uint2(0u, 0u);
    };
    uint2 qn[8];
    load_q(blockIdx.x, qn);

    int sidx = 0;
    uint32_t sph = 0;
    for (int item = blockIdx.x; item < P.items; item += gridDim.x) {
        const Item it = decode_item<BPS>(P, item);
        if (it.nstg == 0) {
            load_q(item + gridDim.x, qn);
            continue;
        }
        uint2 qf[8];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) qf[kk] = qn[kk];
        load_q(item + gridDim.x, qn);  // the next item's, in flight during this one

        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // heads 2t, 2t + 1 (log2 units)
        float acc[8][4];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;

        for (int st = 0; st < it.nstg; ++st) {
            if (!__all_sync(0xffffffffu, wait_bar(&full[sidx], sph, abort))) return;
            const uint32_t sb = after_wait(pl.stage(sidx, SB));
            int2 nn;  // valid rows per slot
            asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(nn.x), "=r"(nn.y) : "r"(sb + Ly::hdr_off));
            // Both tiles are computed whatever their valid rows: a missing block's stage bytes are
            // stale but harmless (codes index the tables; scores and norms are masked below).
            float sc[BPS][4];
            float vnv[BPS][2];
#pragma unroll
            for (int j = 0; j < BPS; ++j) {
                const int n = j ? nn.y : nn.x;
                const uint32_t ks = sb + j * KSLOT, ns = sb + j * NSLOT;
                uint32_t kw[2][PK / 16];
                if constexpr (KB == 8) {  // 32 bytes of rows r and r + 8
                    const uint4 x0 = lds128(ks + koff), x1 = lds128(ks + koff2);
                    const uint4 y0 = lds128(ks + koff + KROW8), y1 = lds128(ks + koff2 + KROW8);
                    kw[0][0] = x0.x; kw[0][1] = x0.y; kw[0][2] = x0.z; kw[0][3] = x0.w;
                    kw[0][4] = x1.x; kw[0][5] = x1.y; kw[0][6] = x1.z; kw[0][7] = x1.w;
                    kw[1][0] = y0.x; kw[1][1] = y0.y; kw[1][2] = y0.z; kw[1][3] = y0.w;
                    kw[1][4] = y1.x; kw[1][5] = y1.y; kw[1][6] = y1.z; kw[1][7] = y1.w;
                } else if constexpr (KB == 4) {
                    const uint4 x = lds128(ks + koff), y = lds128(ks + koff + KROW8);
                    kw[0][0] = x.x; kw[0][1] = x.y; kw[0][2] = x.z; kw[0][3] = x.w;
                    kw[1][0] = y.x; kw[1][1] = y.y; kw[1][2] = y.z; kw[1][3] = y.w;
                } else {
                    const uint2 x = lds64(ks + koff), y = lds64(ks + koff + KROW8);
                    kw[0][0] = x.x; kw[0][1] = x.y;
                    kw[1][0] = y.x; kw[1][1] = y.y;
                }
                const bool ok0 = r < n, ok1 = r + 8 < n;
                const float kn0 = lds16f(ns + knoff), kn1 = lds16f(ns + knoff + 16 * HC);
                vnv[j][0] = ok0 ? lds16f(ns + vnoff) : 0.0f;
                vnv[j][1] = ok1 ? lds16f(ns + vnoff + 16 * HC) : 0.0f;
                // ── scores: S[16 positions x 8 heads] = K_tile . Q^T ──
                float c4[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};  // even / odd steps
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    uint32_t a0, a1, a2, a3;
                    if constexpr (KB == 8) {  // bytes 4kk .. 4kk + 3: coordinates 32t + 4kk .. +3, one code each
                        const uint32_t w0 = kw[0][kk], w1 = kw[1][kk];
                        a0 = __byte_perm(lds32(tab_addr(w0, kof, 0)), lds32(tab_addr(w0, kof, 1)), 0x7610u);
                        a2 = __byte_perm(lds32(tab_addr(w0, kof, 2)), lds32(tab_addr(w0, kof, 3)), 0x7610u);
                        a1 = __byte_perm(lds32(tab_addr(w1, kof, 0)), lds32(tab_addr(w1, kof, 1)), 0x7610u);
                        a3 = __byte_perm(lds32(tab_addr(w1, kof, 2)), lds32(tab_addr(w1, kof, 3)), 0x7610u);
                    } else if constexpr (KB == 4) {  // byte 2kk: coordinates 32t + 4kk, +1; byte 2kk + 1: +2, +3
                        const uint32_t w0 = kw[0][kk >> 1], w1 = kw[1][kk >> 1];
                        const int b = 2 * (kk & 1);
                        a0 = lds32(tab_addr(w0, kof, b));
                        a1 = lds32(tab_addr(w1, kof, b));
                        a2 = lds32(tab_addr(w0, kof, b + 1));
                        a3 = lds32(tab_addr(w1, kof, b + 1));
                    } else {  // byte kk: coordinates 32t + 4kk .. +3
                        const int b = kk & 3;
                        const uint2 x = lds64(tab_addr(kw[0][kk >> 2], kof, b));
                        const uint2 y = lds64(tab_addr(kw[1][kk >> 2], kof, b));
                        a0 = x.x;
                        a2 = x.y;
                        a1 = y.x;
                        a3 = y.y;
                    }
                    mma16816(c4[kk & 1], a0, a1, a2, a3, qf[kk].x, qf[kk].y);
                }
                const float f0 = kn0 * kscale, f1 = kn1 * kscale;
                sc[j][0] = ok0 ? (c4[0][0] + c4[1][0]) * f0 : -INFINITY;
                sc[j][1] = ok0 ? (c4[0][1] + c4[1][1]) * f0 : -INFINITY;
                sc[j][2] = ok1 ? (c4[0][2] + c4[1][2]) * f1 : -INFINITY;
                sc[j][3] = ok1 ? (c4[0][3] + c4[1][3]) * f1 : -INFINITY;
            }

            // ── running softmax over the stage's tiles: their maximum per head ──
            float t0 = fmaxf(sc[0][0], sc[0][2]), t1 = fmaxf(sc[0][1], sc[0][3]);
#pragma unroll
            for (int j = 1; j < BPS; ++j) {
                t0 = fmaxf(t0, fmaxf(sc[j][0], sc[j][2]));
                t1 = fmaxf(t1, fmaxf(sc[j][1], sc[j][3]));
            }
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
                t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
            }
            if (t0 > m0 || t1 > m1) {
                const float n0 = fmaxf(m0, t0), n1 = fmaxf(m1, t1);
                const float g0 = ex2(m0 - n0), g1 = ex2(m1 - n1);
                m0 = n0;
                m1 = n1;
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
            // a head with no valid position so far keeps m = -inf: its weights are exp2(-inf) = 0
            const float u0 = m0 == -INFINITY ? 0.0f : m0, u1 = m1 == -INFINITY ? 0.0f : m1;
#pragma unroll
            for (int j = 0; j < BPS; ++j) {
                const float e0 = ex2(sc[j][0] - u0), e1 = ex2(sc[j][1] - u1);
                const float e2 = ex2(sc[j][2] - u0), e3 = ex2(sc[j][3] - u1);
                l0 += e0 + e2;
                l1 += e1 + e3;
                sts32(pw0 + j * 256, pack_half2(e0 * vnv[j][0], e1 * vnv[j][0]));
                sts32(pw1 + j * 256, pack_half2(e2 * vnv[j][1], e3 * vnv[j][1]));
            }
            __syncwarp();

            // ── values: acc^T[128 dims x 8 heads] += V_tile^T . P per tile; MMA mt, rows r / r + 8
            // are dims 16r + 2mt / 16r + 2mt + 1 ──
#pragma unroll
            for (int j = 0; j < BPS; ++j) {
                uint32_t b0, b1;
                ldsm_x2_trans(b0, b1, pld + j * 256);
                const uint32_t vs = sb + j * VSLOT;
                if constexpr (VB == 8) {
                    // 16 bytes (dims 16r .. 16r + 15) of positions 2t, 2t + 1, 2t + 8, 2t + 9; MMA mt:
                    // dims 16r + 2mt (row r) and + 1 (row r + 8), one code per byte
                    const uint4 x0 = lds128(vs + voff0), x1 = lds128(vs + voff1);
                    const uint4 x2 = lds128(vs + voff0 + VROW8), x3 = lds128(vs + voff1 + VROW8);
                    const uint32_t v0[4] = {x0.x, x0.y, x0.z, x0.w}, v1[4] = {x1.x, x1.y, x1.z, x1.w};
                    const uint32_t v2[4] = {x2.x, x2.y, x2.z, x2.w}, v3[4] = {x3.x, x3.y, x3.z, x3.w};
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        const int wd = mt >> 1, b = 2 * (mt & 1);
                        const uint32_t a0 = __byte_perm(lds32(tab_addr(v0[wd], vof, b)), lds32(tab_addr(v1[wd], vof, b)), 0x7610u);
                        const uint32_t a1 = __byte_perm(lds32(tab_addr(v0[wd], vof, b + 1)), lds32(tab_addr(v1[wd], vof, b + 1)), 0x7610u);
                        const uint32_t a2 = __byte_perm(lds32(tab_addr(v2[wd], vof, b)), lds32(tab_addr(v3[wd], vof, b)), 0x7610u);
                        const uint32_t a3 = __byte_perm(lds32(tab_addr(v2[wd], vof, b + 1)), lds32(tab_addr(v3[wd], vof, b + 1)), 0x7610u);
                        mma16816(acc[mt], a0, a1, a2, a3, b0, b1);
                    }
                } else if constexpr (VB == 2) {
                    // words: bytes 4r..4r+3 (dims 16r..16r+15) of positions t, t + 4 (and + 8); X
                    // byte q: dims 16r + 4q, +1 at both positions of the pair; Xb: dims +2, +3
                    const uint32_t w0 = lds32(vs + voff0), w1 = lds32(vs + voff1);
                    const uint32_t w2 = lds32(vs + voff0 + VROW8), w3 = lds32(vs + voff1 + VROW8);
                    const uint32_t X = (w0 & 0xf0f0f0f0u) | ((w1 >> 4) & 0x0f0f0f0fu);
                    const uint32_t Xb = ((w0 << 4) & 0xf0f0f0f0u) | (w1 & 0x0f0f0f0fu);
                    const uint32_t Y = (w2 & 0xf0f0f0f0u) | ((w3 >> 4) & 0x0f0f0f0fu);
                    const uint32_t Yb = ((w2 << 4) & 0xf0f0f0f0u) | (w3 & 0x0f0f0f0fu);
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        const int q = mt >> 1;
                        const uint2 x = lds64(tab_addr((mt & 1) ? Xb : X, vof, q));
                        const uint2 y = lds64(tab_addr((mt & 1) ? Yb : Y, vof, q));
                        mma16816(acc[mt], x.x, x.y, y.x, y.y, b0, b1);
                    }
                } else {
                    // H byte q: the high nibbles of byte 4u + q at both positions (dim
                    // 16r + 2(4u + q)); Lo: low nibbles (dim + 1); H2 / L2: positions + 8
                    const uint2 x0 = lds64(vs + voff0), x1 = lds64(vs + voff1);
                    const uint2 x2 = lds64(vs + voff0 + VROW8), x3 = lds64(vs + voff1 + VROW8);
                    const uint32_t v0[2] = {x0.x, x0.y}, v1[2] = {x1.x, x1.y}, v2[2] = {x2.x, x2.y},
                                   v3[2] = {x3.x, x3.y};
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint32_t H = (v0[u] & 0xf0f0f0f0u) | ((v1[u] >> 4) & 0x0f0f0f0fu);
                        const uint32_t Lo = ((v0[u] << 4) & 0xf0f0f0f0u) | (v1[u] & 0x0f0f0f0fu);
                        const uint32_t H2 = (v2[u] & 0xf0f0f0f0u) | ((v3[u] >> 4) & 0x0f0f0f0fu);
                        const uint32_t L2 = ((v2[u] << 4) & 0xf0f0f0f0u) | (v3[u] & 0x0f0f0f0fu);
#pragma unroll
                        for (int b = 0; b < 4; ++b)
                            mma16816(acc[4 * u + b], lds32(tab_addr(H, vof, b)), lds32(tab_addr(Lo, vof, b)),
                                     lds32(tab_addr(H2, vof, b)), lds32(tab_addr(L2, vof, b)), b0, b1);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[sidx]);
            if (++sidx == pl.nst) {
                sidx = 0;
                sph ^= 1u;
            }
        }

        // ── the item's partial: heads 2t, 2t + 1 of KV head hg * HC + hl ──
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, o);
            l1 += __shfl_xor_sync(0xffffffffu, l1, o);
        }
        const int kvh = it.hg * HC + hl;
        constexpr float kLn2 = 0.6931471805599453f;
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
            const int h = 2 * t + h2;
            if (h >= G) continue;
            float* ph = a.part + (((int64_t)it.row * a.hq + kvh * G + h) * a.nch + it.c) * PART;
            if (r == 0) {
                const float m = h2 ? m1 : m0;
                ph[0] = m == -INFINITY ? -INFINITY : m * kLn2;
                ph[1] = h2 ? l1 : l0;
            }
#pragma unroll
            for (int mt = 0; mt < 8; ++mt)
                *(float2*)(ph + 2 + 16 * r + 2 * mt) = make_float2(acc[mt][h2], acc[mt][2 + h2]);
        }
    }
}

// ── host side ──

// Norms: f16 [rows, hkv], box of HC heads x 16 rows.
static bool encode_norms(CUtensorMap* map, const void* base, uint64_t hkv, uint64_t rows) {
    auto encode = sm100::tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)hkv, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(hkv * 2)};
    const cuuint32_t box[2] = {HC, 16};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Codes: uint8 [rows, hkv * P] seen as [rows][hkv * P / 128 lines][128 bytes]; box of `lines`
// lines (one head group) x 16 rows, 128-byte swizzle. Line-major (8-bit codes): the same bytes
// seen as [lines][rows][128] (dimension order 128, rows, lines), so the box lands line by line.
static bool encode_codes(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t lines,
                         bool line_major) {
    auto encode = sm100::tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t nl = row_bytes / 128;
    const cuuint64_t dims[3] = {128, line_major ? (cuuint64_t)rows : nl, line_major ? nl : (cuuint64_t)rows};
    const cuuint64_t strides[2] = {line_major ? (cuuint64_t)row_bytes : 128, line_major ? 128 : (cuuint64_t)row_bytes};
    const cuuint32_t box[3] = {128, line_major ? 16u : lines, line_major ? lines : 16u};
    const cuuint32_t estr[3] = {1, 1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace stream

// Positions per chunk for the streamed kernel. Of 256, 512, 1024 and 2048, the one whose items
// fill the persistent grid's waves best, the longer on a tie (chunks that would leave a query row
// more than 32 partials are skipped while a longer chunk exists: the combine reads every partial
// of a row). When that leaves SMs without an item (few query rows over a context that is short, or
// long and cut in few chunks), every power of two from 32 to 2048 whose chunk count the
// workspace's slots hold is weighed instead by an estimate of its time: waves of items, each
// taking its positions at a per-position cost plus a fixed cost (pipeline fill, partial write),
// and the partials written and read again by the combine.
static int stream_chunk(int64_t positions, int64_t rows, int ng, int hq, int sms, int64_t slots, int kb, int vb) {
    int best = 0;
    double best_eff = -1.0;
    for (int ch = 256; ch <= 2048; ch *= 2) {
        if (ch < 2048 && (positions + ch - 1) / ch > 32) continue;
        const int64_t items = (positions + ch - 1) / ch * rows * ng;
        const int64_t waves = (items + sms - 1) / sms;
        const double eff = (double)items / (double)(waves * sms) + 1e-3 * (ch / 256);
        if (eff > best_eff) {
            best_eff = eff;
            best = ch;
        }
    }
    if ((positions + best - 1) / best * rows * ng >= sms) return best;
    const double tpos = (0.5 + (kb + vb) / 12.0) / 32.0;  // us per position of an item (8 KV heads)
    const double fixed = 2.0;                            // us per item
    const double part = 2.0 * PART * 4 / 3.0e6;          // us per partial (written, read; ~3 TB/s)
    double best_t = 0.0;
    best = 0;
    for (int ch = 2048; ch >= 32; ch /= 2) {
        const int64_t nchi = (positions + ch - 1) / ch;
        if (nchi > slots) break;  // shorter chunks have more
        const int64_t waves = (nchi * rows * ng + sms - 1) / sms;
        const double t = (double)waves * (ch * tpos + fixed) + (double)(nchi * rows * hq) * part;
        if (best == 0 || t < 0.98 * best_t) {  // a shorter chunk has to win by 2 %
            best = ch;
            best_t = t;
        }
    }
    return best;
}

// Whether the streamed kernel takes this call: 2-, 4- or 8-bit codes, KV heads a multiple of 8;
// with pools, 16-byte aligned ones whose rows a TMA coordinate can reach. (Per-block buffers are
// checked block by block in the kernel: a block whose buffers are not 16-byte aligned is copied
// without the bulk copies.)
static bool stream_shape_ok(const AttnArgs& a, int kb, int vb) {
    const auto bits = [](int b) { return b == 2 || b == 4 || b == 8; };
    if (!bits(kb) || !bits(vb)) return false;
    return a.hkv % stream::HC == 0 && a.hq / a.hkv <= MAXG;
}
bool stream_ok(const AttnArgs& a, int kb, int vb, const PoolAddr& ad) {
    if (!stream_shape_ok(a, kb, vb)) return false;
    if (!aligned16(ad.kp) || !aligned16(ad.vp) || !aligned16(ad.kn) || !aligned16(ad.vn)) return false;
    return ad.pool_rows > 0 && ad.pool_rows <= INT32_MAX;
}
bool stream_ok(const AttnArgs& a, int kb, int vb, const BlockPtrAddr&) { return stream_shape_ok(a, kb, vb); }

// One of pool / ptrs is given (PTRS selects which).
template <int KB, int VB, bool PTRS>
static int stream_launch_t(AttnArgs& a, const PoolAddr* pool, const BlockPtrAddr* ptrs, cudaStream_t s) {
    using Ly = stream::Layout<KB, VB>;
    const int rows = a.num_seqs * a.q_per_seq;
    const int ng = a.hkv / stream::HC;
    const int sms = num_sms();
    const int64_t positions = (int64_t)a.nch * CH;  // the context rounded up to CH
    const int ch = stream_chunk(positions, rows, ng, a.hq, sms, std::max(a.slots, a.nch), KB, VB);
    stream::Params P;
    memset(&P, 0, sizeof P);
    if constexpr (PTRS) {
        P.codes[0] = ptrs->kp;
        P.codes[1] = ptrs->vp;
        P.norms[0] = ptrs->kn;
        P.norms[1] = ptrs->vn;
        P.pool_rows = INT64_MAX;  // every row of a listed block exists
    } else {
        const PoolAddr& ad = *pool;
        const uint64_t prow = (uint64_t)ad.pool_rows;
        if (!stream::encode_codes(&P.kmap, ad.kp, (uint64_t)a.hkv * Ly::PK, prow, Ly::KBOX, Ly::K8) ||
            !stream::encode_codes(&P.vmap, ad.vp, (uint64_t)a.hkv * Ly::PV, prow, Ly::VBOX, Ly::V8) ||
            !stream::encode_norms(&P.knmap, ad.kn, (uint64_t)a.hkv, prow) ||
            !stream::encode_norms(&P.vnmap, ad.vn, (uint64_t)a.hkv, prow))
            return (int)cudaErrorInvalidValue;
        P.pool_rows = ad.pool_rows;
        P.kn = ad.kn;
        P.vn = ad.vn;
        P.norms_bulk = a.hkv == stream::HC ? 1 : 0;
    }
    const int nchi = (int)((positions + ch - 1) / ch);
    a.ch = ch;
    a.spc = 1;
    a.nch = nchi;
    P.a = a;
    P.spi = ch / (Ly::BPS * 16);
    P.nchi = nchi;
    P.ng = ng;
    P.dng = sm100::make_divu32((uint32_t)ng);
    P.dqps = sm100::make_divu32((uint32_t)a.q_per_seq);
    P.dnchi = sm100::make_divu32((uint32_t)nchi);
    const int64_t items = (int64_t)a.num_seqs * nchi * a.q_per_seq * ng;
    if (items > INT32_MAX) return (int)cudaErrorInvalidValue;
    P.items = (int)items;
    auto kern = stream::tqa_stream<KB, VB, PTRS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)stream::DYN_BYTES);
    if (e != cudaSuccess) return (int)e;
    const int grid = (int)std::min<int64_t>(items, sms);
    launch_pdl_smem(kern, dim3(grid), dim3(Ly::THREADS), (size_t)stream::DYN_BYTES, s, P);
    return (int)cudaGetLastError();
}

template <bool PTRS>
static int stream_dispatch(AttnArgs& a, int kb, int vb, const PoolAddr* pool, const BlockPtrAddr* ptrs,
                           cudaStream_t s) {
    switch (kb * 10 + vb) {
        case 22: return stream_launch_t<2, 2, PTRS>(a, pool, ptrs, s);
        case 24: return stream_launch_t<2, 4, PTRS>(a, pool, ptrs, s);
        case 28: return stream_launch_t<2, 8, PTRS>(a, pool, ptrs, s);
        case 42: return stream_launch_t<4, 2, PTRS>(a, pool, ptrs, s);
        case 44: return stream_launch_t<4, 4, PTRS>(a, pool, ptrs, s);
        case 48: return stream_launch_t<4, 8, PTRS>(a, pool, ptrs, s);
        case 82: return stream_launch_t<8, 2, PTRS>(a, pool, ptrs, s);
        case 84: return stream_launch_t<8, 4, PTRS>(a, pool, ptrs, s);
        default: return stream_launch_t<8, 8, PTRS>(a, pool, ptrs, s);
    }
}

// Launches the streamed kernel for a call stream_ok() accepted.
int stream_launch(AttnArgs& a, int kb, int vb, const PoolAddr& ad, cudaStream_t s) {
    if (!stream_ok(a, kb, vb, ad)) return (int)cudaErrorInvalidValue;
    return stream_dispatch<false>(a, kb, vb, &ad, nullptr, s);
}
int stream_launch(AttnArgs& a, int kb, int vb, const BlockPtrAddr& ad, cudaStream_t s) {
    if (!stream_ok(a, kb, vb, ad)) return (int)cudaErrorInvalidValue;
    return stream_dispatch<true>(a, kb, vb, nullptr, &ad, s);
}

}  // namespace tqa

unsigned int tqa_stream_timeouts() {
    unsigned int v = 0;
    cudaMemcpyFromSymbol(&v, g_tqa_stream_timeouts, sizeof(v));
    return v;
}

}  // namespace fb
