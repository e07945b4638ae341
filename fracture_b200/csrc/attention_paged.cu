// Paged attention over the FP16/BF16 KV cache and the paged append, sm_100a.
//
// Replaces backends/fracture-cuda/kernels/attention_paged.cu:25-185 (one CTA per query token
// and Q head over the whole causal range, every Q head of a GQA group re-reading its KV head's
// rows, the value phase one thread per coordinate walking every position) and the per-block row
// copies of PagedKvCacheManager::append_kv (crates/fracture-engine/src/paged_kv_cache.rs:253-315).
// The math is the reference kernel's: scores q . k / sqrt(d) in float32, softmax over
// [0, min(start_pos + t + 1, kv_len)), out = sum p v. Here, split-K over 256-position chunks:
//
//   kvp_chunk    one CTA per (chunk, KV head, query token): thread p scores position p for
//                every Q head of the group from the position's key row (16-byte loads,
//                two-wide FP32 FMAs against the queries in shared memory), the CTA takes the
//                chunk's softmax maximum and sum, then warp w accumulates its 32 positions'
//                value rows (lane l: coordinates 4l..4l+3, one coalesced 8-byte load per
//                position) for every head; the chunk's (max, sum, acc) go to the workspace
//   kvp_mma      (queries 16-byte aligned, i.e. always through the Python and backend layers)
//                replaces kvp_chunk: tensor cores, persistent CTAs, chunks of 512 to 2048
//                positions; see below
//   kvp_combine  rescales and sums the chunks of each query token and head and divides
//   kvp_append   writes new key/value rows into the pool through the block table
//
// Each KV head's rows are read once per query token for its whole group of Q heads. A position
// whose block-table entry is negative, or whose pool row is out of range, is left out; a query
// token with no position gives zeros.

#include <algorithm>
#include <atomic>

#include "common.cuh"

namespace fb {

namespace kvp {

constexpr int D = 128;
constexpr int CH = 256;
constexpr int THREADS = 256;
constexpr int NWARPS = THREADS / 32;
constexpr int MAXG = 8;
constexpr int PART = D + 2;  // max, sum, acc[D]

struct Args {
    const void* q;
    int dtype;  // FB_FP16 / FB_BF16: q, cache rows and out
    int num_seqs, q_per_seq, hq, hkv;
    const int32_t* block_tables;
    int max_blocks;
    const int32_t* kv_lens;    // null: kv_len for every sequence
    const int32_t* start_pos;  // null: start for every sequence
    int kv_len, start;
    float* part;  // [rows, hq, nch, PART]
    int nch;
    int ch;   // positions per chunk
    int rnd;  // tensor-core kernel: rounds of four 16-position tiles per warp and item
    void* out;
};

// Rows of the contiguous pools ([blocks * 16, hkv, D]) or of the reference's per-block tensors.
struct PoolRows {
    const uint8_t* k;
    const uint8_t* v;
    int64_t pool_rows;
    __device__ bool locate(int32_t blk, int off, int g, int hkv, int esz, const uint8_t*& kr, const uint8_t*& vr) const {
        const int64_t row = (int64_t)blk * 16 + off;
        if (row >= pool_rows) return false;
        const int64_t o = (row * hkv + g) * (int64_t)D * esz;
        kr = k + o;
        vr = v + o;
        return true;
    }
    // Rows of block blk inside the pool (16 unless the pool ends inside the block).
    __device__ int block_rows(int32_t blk) const {
        return (int)max((int64_t)0, min((int64_t)16, pool_rows - (int64_t)blk * 16));
    }
    // KV head g of row `off` of block blk: at kb + off * hkv * D * esz (the same for V).
    __device__ void block_base(int32_t blk, int g, int hkv, int esz, const uint8_t*& kb, const uint8_t*& vb) const {
        const int64_t o = ((int64_t)blk * 16 * hkv + g) * (int64_t)D * esz;
        kb = k + o;
        vb = v + o;
    }
};
struct BlockPtrRows {
    const uint8_t* const* k;
    const uint8_t* const* v;
    __device__ bool locate(int32_t blk, int off, int g, int hkv, int esz, const uint8_t*& kr, const uint8_t*& vr) const {
        const int64_t o = ((int64_t)off * hkv + g) * D * esz;
        kr = k[blk] + o;
        vr = v[blk] + o;
        return true;
    }
    __device__ int block_rows(int32_t) const { return 16; }
    __device__ void block_base(int32_t blk, int g, int, int esz, const uint8_t*& kb, const uint8_t*& vb) const {
        kb = k[blk] + (int64_t)g * D * esz;
        vb = v[blk] + (int64_t)g * D * esz;
    }
};

__device__ __forceinline__ int causal_len(const Args& a, int s, int t) {
    const int kv = a.kv_lens ? a.kv_lens[s] : a.kv_len;
    const int st = a.start_pos ? a.start_pos[s] : a.start;
    return max(0, min(st + t + 1, kv));
}

template <typename T>
__device__ __forceinline__ float2 to_f2(uint32_t w) {
    if constexpr (dtype_of<T>::value == FB_BF16) {
        return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
    } else {
        return __half22float2(*reinterpret_cast<const __half2*>(&w));
    }
}

template <typename T, int G>
struct ChunkSmem {
    static constexpr int q_off = 0;                              // [G][D] f32 (scaled queries)
    static constexpr int acc_off = q_off + G * D * 4;            // [NWARPS][G][D] f32
    static constexpr int w_off = acc_off + NWARPS * G * D * 4;   // [CH][G] f32 weights
    static constexpr int red_off = w_off + CH * G * 4;           // [NWARPS][G]
    static constexpr int bytes = red_off + NWARPS * G * 4 + 16;
};

template <typename T, int G, typename Rows>
__global__ void __launch_bounds__(THREADS) kvp_chunk(Args a, Rows rw) {
    using S = ChunkSmem<T, G>;
    extern __shared__ __align__(16) uint8_t sm[];
    float* qs = (float*)(sm + S::q_off);
    float* accs = (float*)(sm + S::acc_off);
    float* ws = (float*)(sm + S::w_off);
    float* red = (float*)(sm + S::red_off);
    const int row = blockIdx.z, g = blockIdx.y, c = blockIdx.x;
    const int s = row / a.q_per_seq, t = row - s * a.q_per_seq;
    const int L = causal_len(a, s, t);
    const int p0 = c * CH;
    if (p0 >= L) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int GA = a.hq / a.hkv;
    const float scale = rsqrtf((float)D);
    for (int e = tid; e < G * D; e += THREADS) {
        float v = 0.0f;
        if (e < GA * D) {
            const int64_t qi = ((int64_t)row * a.hq + g * GA) * D + e;
            v = dtype_of<T>::value == FB_BF16 ? __bfloat162float(((const __nv_bfloat16*)a.q)[qi])
                                              : __half2float(((const __half*)a.q)[qi]);
        }
        qs[e] = v * scale;
    }
    __syncthreads();

    // ── scores: thread tid takes position p0 + tid ──
    const int p = p0 + tid;
    bool valid = p < L && (p >> 4) < a.max_blocks;
    const uint8_t* kr = nullptr;
    const uint8_t* vr = nullptr;
    if (valid) {
        const int32_t blk = a.block_tables[(int64_t)s * a.max_blocks + (p >> 4)];
        valid = blk >= 0 && rw.locate(blk, p & 15, g, a.hkv, (int)sizeof(T), kr, vr);
    }
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = 0.0f;
    if (valid) {
        float2 s2[G];
#pragma unroll
        for (int h = 0; h < G; ++h) s2[h] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int k = 0; k < D / 8; ++k) {  // 8 coordinates per 16-byte load (all loads issued first)
            const uint4 u = __ldg((const uint4*)kr + k);
            const float2 x0 = to_f2<T>(u.x), x1 = to_f2<T>(u.y), x2 = to_f2<T>(u.z), x3 = to_f2<T>(u.w);
#pragma unroll
            for (int h = 0; h < G; ++h) {
                const float4 qa = *(const float4*)&qs[h * D + 8 * k];
                const float4 qb = *(const float4*)&qs[h * D + 8 * k + 4];
                s2[h] = __ffma2_rn(make_float2(qa.x, qa.y), x0, s2[h]);
                s2[h] = __ffma2_rn(make_float2(qa.z, qa.w), x1, s2[h]);
                s2[h] = __ffma2_rn(make_float2(qb.x, qb.y), x2, s2[h]);
                s2[h] = __ffma2_rn(make_float2(qb.z, qb.w), x3, s2[h]);
            }
        }
#pragma unroll
        for (int h = 0; h < G; ++h) sc[h] = s2[h].x + s2[h].y;
    }

    // ── softmax over the chunk ──
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
        mx[h] = v;
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const float e = valid ? expf(sc[h] - mx[h]) : 0.0f;
        ws[tid * G + h] = e;
        float v = e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp * G + h] = v;
    }
    __syncthreads();

    // ── values: warp w takes its 32 positions, lane l coordinates 4l..4l+3 of every head ──
    float2 acc[G][2];
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h][0] = acc[h][1] = make_float2(0.0f, 0.0f);
    // warp w scored the same 32 positions it now accumulates: lane j's value-row pointer
    // travels by shuffle (0: position left out)
    const unsigned long long vrow = valid ? (unsigned long long)vr : 0ull;
    const int jn = min(32, L - (p0 + warp * 32));
    for (int j0 = 0; j0 < jn; j0 += 8) {
        // eight positions' value rows requested before any is used (a position left out, or past
        // the causal range, loads nothing and has weight 0)
        uint2 u[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const unsigned long long rp = __shfl_sync(0xffffffffu, vrow, j0 + k);
            u[k] = make_uint2(0u, 0u);
            if (j0 + k < jn && rp != 0ull) u[k] = __ldg((const uint2*)rp + lane);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float2 a0 = to_f2<T>(u[k].x), a1 = to_f2<T>(u[k].y);
            const float* wp = ws + (warp * 32 + j0 + k) * G;
#pragma unroll
            for (int h4 = 0; h4 < G; h4 += 4) {
                const float4 w4 = *(const float4*)(wp + h4);
                const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 w2 = make_float2(wv[q], wv[q]);
                    acc[h4 + q][0] = __ffma2_rn(w2, a0, acc[h4 + q][0]);
                    acc[h4 + q][1] = __ffma2_rn(w2, a1, acc[h4 + q][1]);
                }
            }
        }
    }
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

// out = (sum_c acc_c e^(m_c - M)) / (sum_c l_c e^(m_c - M)); thread i: coordinate i of every head.
template <typename T>
__global__ void __launch_bounds__(128) kvp_combine(Args a) {
    pdl_begin();
    const int row = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
    const int s = row / a.q_per_seq, t = row - s * a.q_per_seq;
    const int L = causal_len(a, s, t);
    const int nc = min((L + a.ch - 1) / a.ch, a.nch);  // kv_lens past max_kv_len: the chunks computed
    const float* ph = a.part + ((int64_t)row * a.hq + h) * a.nch * PART;
    float M = -INFINITY;
#pragma unroll 8
    for (int c = 0; c < nc; ++c) M = fmaxf(M, ph[c * PART]);
    float l = 0.0f, v = 0.0f;
    if (M > -INFINITY) {
#pragma unroll 4
        for (int c = 0; c < nc; ++c) {
            const float m = ph[c * PART];
            if (m == -INFINITY) continue;
            const float f = expf(m - M);
            l = fmaf(ph[c * PART + 1], f, l);
            v = fmaf(ph[c * PART + 2 + i], f, v);
        }
    }
    const float o = l > 0.0f ? v / l : 0.0f;
    ((T*)a.out)[((int64_t)row * a.hq + h) * D + i] = from_f32<T>(o);
}

// ── tensor-core path ──
//
// One work item = (chunk of 512 x rnd positions, KV head, query token), rnd = 1, 2 or 4 chosen
// per call (tc_chunks); persistent CTAs take items in turn. Warp w takes its 64 rnd positions of
// the chunk as rnd rounds of four 16-position tiles, one after the
// other (the next tile's rows requested into the registers the current one has finished with)
// with its own running softmax (maximum, sum, accumulator) per head, and does both
// contractions with mma.sync m16n8k16 (16-bit operands, FP32 accumulators) on operands loaded
// straight into registers:
//
//   scores   S[16 positions x 8 heads] = K_tile . Q^T: lane (r, t) = (lane / 4, lane % 4) loads
//            coordinates 32t..32t+31 of key rows r and r + 8 (four 16-byte loads each); the k
//            index 2t+e of step kk stands for coordinate 32t + 4kk + e (+2 for the upper half),
//            and the B registers hold the query of head r at the same coordinates.
//   values   acc^T[128 dims x 8 heads] += V_tile^T . P: lane (r, t) loads coordinates
//            16r..16r+15 of value rows 2t, 2t+1, 2t+8, 2t+9 and pairs the two positions of one
//            coordinate into an A register with a byte permute; the weights P go through shared
//            memory and come back transposed (ldmatrix .trans) as B registers. BF16 weights are
//            split into a high and a low part (two MMAs), which keeps them to FP32 accuracy.
//
// At the end of an item the warps' (maximum, sum, accumulator) are rescaled to the item's
// maximum and added in warp order.

namespace tc {
constexpr int TILE = 16, TPW = 4, MAX_RND = 4;  // an item: NWARPS * rnd * TPW * TILE positions, rnd <= MAX_RND

struct Smem {
    static constexpr int acc_off = 0;                                  // [NWARPS][8][D] f32
    static constexpr int p_off = acc_off + NWARPS * 8 * D * 4;         // [NWARPS][2][16][8] 16-bit
    static constexpr int mx_off = p_off + NWARPS * 2 * TILE * 8 * 2;   // [NWARPS][8] f32
    static constexpr int l_off = mx_off + NWARPS * 8 * 4;              // [NWARPS][8] f32
    static constexpr int q_off = l_off + NWARPS * 8 * 4;               // [8 steps][32 lanes] uint2
    static constexpr int bytes = q_off + 8 * 32 * 8;
};

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    if constexpr (dtype_of<T>::value == FB_BF16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ void ldsm_x2_trans(uint32_t& r0, uint32_t& r1, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr)
                 : "memory");
}

// Two floats as a 16-bit pair of type T (x in the low half), and what rounding left over.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y, float& rx, float& ry) {
    if constexpr (dtype_of<T>::value == FB_BF16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
        const float2 back = __bfloat1622float2(h);
        rx = x - back.x;
        ry = y - back.y;
        return *reinterpret_cast<const uint32_t*>(&h);
    } else {
        const __half2 h = __floats2half2_rn(x, y);
        rx = ry = 0.0f;
        return *reinterpret_cast<const uint32_t*>(&h);
    }
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float x, float y) {
    float rx, ry;
    return pack2<T>(x, y, rx, ry);
}

}  // namespace tc

template <typename T, typename Rows>
__global__ void __launch_bounds__(THREADS, 2) kvp_mma(Args a, Rows rw, int items) {
    pdl_begin();
    using namespace tc;
    constexpr bool SPLIT = dtype_of<T>::value == FB_BF16;
    extern __shared__ __align__(16) uint8_t sm[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, r = lane >> 2, t = lane & 3;
    const int GA = a.hq / a.hkv;
    float* accs = (float*)(sm + Smem::acc_off);
    uint16_t* pb = (uint16_t*)(sm + Smem::p_off) + warp * 2 * TILE * 8;
    float* rmx = (float*)(sm + Smem::mx_off);
    float* rl = (float*)(sm + Smem::l_off);
    uint2* qf = (uint2*)(sm + Smem::q_off);
    const float scale = rsqrtf((float)D);
    const int64_t rst = (int64_t)a.hkv * D * (int64_t)sizeof(T);  // bytes between a block's rows

    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int c = item % a.nch, rest = item / a.nch, g = rest % a.hkv, row = rest / a.hkv;
        const int s = row / a.q_per_seq, tq = row - s * a.q_per_seq;
        const int L = causal_len(a, s, tq);
        const int p0 = c * a.ch;
        if (p0 >= L) continue;  // the whole CTA

        // B registers of the score MMA, step kk, lane (r, t): the query of head r (zeros past
        // the group) at coordinates 32t + 4kk .. 32t + 4kk + 3, staged in shared memory in that
        // order (one conflict-free 8-byte load per lane and step); thread (kk, lane) = (warp, lane)
        {
            const uint2 u = r < GA ? __ldg((const uint2*)((const T*)a.q + ((int64_t)row * a.hq + g * GA + r) * D +
                                                          32 * t + 4 * warp))
                                   : make_uint2(0u, 0u);
            qf[warp * 32 + lane] = u;
        }
        __syncthreads();
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // heads 2t, 2t + 1
        float acc[8][4];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.0f;

#pragma unroll 1
        for (int rd = 0; rd < a.rnd; ++rd) {  // rounds of four tiles, one running softmax
            const int pw = p0 + (warp * a.rnd + rd) * TPW * TILE;
            const int lim = min(L, a.max_blocks * 16);
            // the warp's tiles: block entry and positions in the cache (a prefix of the 16)
            int32_t bk[TPW];
            int nv[TPW];
#pragma unroll
            for (int i = 0; i < TPW; ++i) {
                const int ps = pw + i * TILE;
                const int32_t blk = ps < lim ? __ldg(a.block_tables + (int64_t)s * a.max_blocks + (ps >> 4)) : -1;
                nv[i] = blk >= 0 ? min(min(TILE, L - ps), rw.block_rows(blk)) : 0;
                bk[i] = blk;
            }
            // Tile i + 1's keys are requested as soon as tile i's scores are done with the key
            // registers, its values as soon as tile i's values are done with the value registers.
            uint32_t kw[2][16], vw[4][8];
            auto load_k = [&](int i) {
                const int n = nv[i];
                const uint8_t *kb = nullptr, *vb = nullptr;
                if (n > 0) rw.block_base(bk[i], g, a.hkv, (int)sizeof(T), kb, vb);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int off = r + 8 * h;
                    const uint4* p = (const uint4*)(kb + off * rst + 64 * t);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint4 u = off < n ? __ldg(p + j) : make_uint4(0, 0, 0, 0);
                        kw[h][4 * j] = u.x;
                        kw[h][4 * j + 1] = u.y;
                        kw[h][4 * j + 2] = u.z;
                        kw[h][4 * j + 3] = u.w;
                    }
                }
            };
            auto load_v = [&](int i) {
                const int n = nv[i];
                const uint8_t *kb = nullptr, *vb = nullptr;
                if (n > 0) rw.block_base(bk[i], g, a.hkv, (int)sizeof(T), kb, vb);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int off = 2 * t + (u & 1) + 8 * (u >> 1);
                    const uint4* p = (const uint4*)(vb + off * rst + 32 * r);
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const uint4 x = off < n ? __ldg(p + j) : make_uint4(0, 0, 0, 0);
                        vw[u][4 * j] = x.x;
                        vw[u][4 * j + 1] = x.y;
                        vw[u][4 * j + 2] = x.z;
                        vw[u][4 * j + 3] = x.w;
                    }
                }
            };
            load_k(0);
            load_v(0);
#pragma unroll
            for (int i = 0; i < TPW; ++i) {
                const int n = nv[i];
                // scores of the tile
                float c4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (n > 0) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint2 b = qf[kk * 32 + lane];
                        mma16816<T>(c4, kw[0][2 * kk], kw[1][2 * kk], kw[0][2 * kk + 1], kw[1][2 * kk + 1], b.x, b.y);
                    }
                }
                if (i + 1 < TPW) load_k(i + 1);
                if (n > 0) {
                    const float s0 = r < n ? c4[0] * scale : -INFINITY, s1 = r < n ? c4[1] * scale : -INFINITY;
                    const float s2 = r + 8 < n ? c4[2] * scale : -INFINITY, s3 = r + 8 < n ? c4[3] * scale : -INFINITY;

                    // running softmax: the tile's maximum per head (row 0 of the tile is in range)
                    float t0 = fmaxf(s0, s2), t1 = fmaxf(s1, s3);
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, o));
                        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, o));
                    }
                    if (t0 > m0 || t1 > m1) {
                        const float f0 = t0 > m0 ? __expf(m0 - t0) : 1.0f, f1 = t1 > m1 ? __expf(m1 - t1) : 1.0f;
                        m0 = fmaxf(m0, t0);
                        m1 = fmaxf(m1, t1);
                        l0 *= f0;
                        l1 *= f1;
#pragma unroll
                        for (int mt = 0; mt < 8; ++mt) {
                            acc[mt][0] *= f0;
                            acc[mt][2] *= f0;
                            acc[mt][1] *= f1;
                            acc[mt][3] *= f1;
                        }
                    }
                    const float e0 = __expf(s0 - m0), e1 = __expf(s1 - m1), e2 = __expf(s2 - m0), e3 = __expf(s3 - m1);
                    l0 += e0 + e2;
                    l1 += e1 + e3;

                    // weights -> B registers (transposed through shared memory)
                    __syncwarp();
                    {
                        uint32_t* pr = (uint32_t*)(pb + r * 8 + 2 * t);
                        float x0, x1, x2, x3;
                        pr[0] = pack2<T>(e0, e1, x0, x1);
                        pr[32] = pack2<T>(e2, e3, x2, x3);  // row r + 8
                        if constexpr (SPLIT) {
                            pr[64] = pack2<T>(x0, x1);  // the low parts, rows 16..31
                            pr[96] = pack2<T>(x2, x3);
                        }
                    }
                    __syncwarp();
                    uint32_t b0, b1, b2 = 0u, b3 = 0u;
                    ldsm_x2_trans(b0, b1, (uint32_t)__cvta_generic_to_shared(pb + (lane & 15) * 8));
                    if constexpr (SPLIT) ldsm_x2_trans(b2, b3, (uint32_t)__cvta_generic_to_shared(pb + (16 + (lane & 15)) * 8));

                    // values: A register = one coordinate at two adjacent positions
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        const uint32_t a0 = __byte_perm(vw[0][mt], vw[1][mt], 0x5410u);
                        const uint32_t a1 = __byte_perm(vw[0][mt], vw[1][mt], 0x7632u);
                        const uint32_t a2 = __byte_perm(vw[2][mt], vw[3][mt], 0x5410u);
                        const uint32_t a3 = __byte_perm(vw[2][mt], vw[3][mt], 0x7632u);
                        mma16816<T>(acc[mt], a0, a1, a2, a3, b0, b1);
                        if constexpr (SPLIT) mma16816<T>(acc[mt], a0, a1, a2, a3, b2, b3);
                    }
                }
                if (i + 1 < TPW) load_v(i + 1);
            }

        }

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
        __syncthreads();  // the next item rewrites the shared sums
    }
}

// Token t of the call goes to pool row block_table[(start + t) / 16] * 16 + (start + t) % 16 (a
// negative entry or a row past the pool: skipped and counted in err_count); each thread copies
// one 16-byte piece of one token's K and V rows ([Hkv * head_dim] elements).
__global__ void kvp_append(const uint4* __restrict__ keys, const uint4* __restrict__ values, int64_t num_tokens,
                           int row_vecs, const int32_t* __restrict__ block_table, int64_t start_pos,
                           int64_t pool_rows, uint4* __restrict__ k_pool, uint4* __restrict__ v_pool,
                           unsigned int* err_count) {
    const int64_t n = num_tokens * row_vecs;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = e / row_vecs, k = e - t * row_vecs;
        const int64_t pos = start_pos + t;
        const int32_t b = block_table[pos >> 4];
        const int64_t slot = b < 0 ? -1 : (int64_t)b * 16 + (pos & 15);
        if (slot < 0 || slot >= pool_rows) {
            if (k == 0 && err_count) atomicAdd(err_count, 1u);
            continue;
        }
        k_pool[slot * row_vecs + k] = __ldg(keys + e);
        v_pool[slot * row_vecs + k] = __ldg(values + e);
    }
}

size_t workspace_bytes(int64_t rows, int hq, int nch) { return (size_t)rows * hq * nch * PART * 4; }

template <typename T, int G, typename Rows>
int launch_chunk(const Args& a, const Rows& rw, cudaStream_t s) {
    constexpr int smem = ChunkSmem<T, G>::bytes;
    auto kern = kvp_chunk<T, G, Rows>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return (int)e;
    kern<<<dim3(a.nch, a.hkv, a.num_seqs * a.q_per_seq), THREADS, smem, s>>>(a, rw);
    return (int)cudaGetLastError();
}

template <typename T, typename Rows>
int launch_tc(const Args& a, const Rows& rw, cudaStream_t s) {
    constexpr int smem = tc::Smem::bytes;
    auto kern = kvp_mma<T, Rows>;
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
    launch_pdl_smem(kern, dim3((unsigned)std::min<int64_t>(items, slots[dev].load(std::memory_order_relaxed))), dim3(THREADS), (size_t)smem, s, a, rw,
                    (int)items);
    return (int)cudaGetLastError();
}

// Items of the tensor-core kernel as long as they still fill three quarters of one wave of CTA
// slots (two CTAs per SM): long items pay the per-item cost (query staging, the warps'
// reduction, one partial) over more positions, short ones keep small batches spread over the
// SMs. (Measured at 8192-token contexts: 8 sequences, 256 items of 2048 positions, ran in 56 us
// against 72 us for 1024 items of 512; 1 sequence, 128 items of 512, in 37 us against 48 us for
// 32 items of 2048.)
inline void tc_chunks(Args& a, int64_t positions, int64_t rows) {
    int rnd = tc::MAX_RND;
    const int64_t per_round = (int64_t)NWARPS * tc::TPW * tc::TILE;
    while (rnd > 1 && (positions + per_round * rnd - 1) / (per_round * rnd) * a.hkv * rows * 4 < 3LL * 2 * num_sms())
        rnd /= 2;
    a.rnd = rnd;
    a.ch = (int)(per_round * rnd);
    a.nch = (int)((positions + a.ch - 1) / a.ch);
}

template <typename T, typename Rows>
int run_t(Args a, const Rows& rw, cudaStream_t s) {
    const int rows = a.num_seqs * a.q_per_seq;
    if (rows == 0) return 0;
    a.ch = CH;
    // the tensor-core kernel reads the queries 16 bytes at a time; a.nch counts CH-position
    // chunks (the workspace is sized for them), the tensor-core kernel takes larger ones
    if (aligned16(a.q)) {
        tc_chunks(a, (int64_t)a.nch * CH, rows);
        if (a.nch > 0) {
            const int rc = launch_tc<T>(a, rw, s);
            if (rc) return rc;
        }
    } else if (a.nch > 0) {
        const int rc = a.hq / a.hkv <= 4 ? launch_chunk<T, 4>(a, rw, s) : launch_chunk<T, 8>(a, rw, s);
        if (rc) return rc;
    }
    launch_pdl(kvp_combine<T>, dim3(rows, a.hq), dim3(128), s, a);
    return (int)cudaGetLastError();
}

template <typename Rows>
int run(const Args& a, const Rows& rw, cudaStream_t s) {
    return a.dtype == FB_BF16 ? run_t<__nv_bfloat16>(a, rw, s) : run_t<__half>(a, rw, s);
}

bool shape_ok(int hq, int hkv, int head_dim) {
    if (head_dim != D || hkv <= 0 || hq <= 0 || hq % hkv) return false;
    const int G = hq / hkv;
    return G == 1 || G == 2 || G == 4 || G == 8;
}

}  // namespace kvp

void set_last_error(const char* msg);

}  // namespace fb

using namespace fb;

extern "C" size_t fb_attention_workspace_bytes(int num_seqs, int q_per_seq, int num_q_heads, int max_kv_len) {
    if (num_seqs < 0 || q_per_seq < 0 || num_q_heads <= 0 || max_kv_len < 0) return 0;
    return kvp::workspace_bytes((int64_t)num_seqs * q_per_seq, num_q_heads, (max_kv_len + kvp::CH - 1) / kvp::CH);
}

extern "C" int fb_launch_attention_paged(const void* q, int dtype, int num_seqs, int q_per_seq, int num_q_heads,
                                         int num_kv_heads, int head_dim, const void* k_pool, const void* v_pool,
                                         int64_t num_pool_rows, const int32_t* block_tables, int max_blocks_per_seq,
                                         const int32_t* kv_lens, const int32_t* start_pos, int max_kv_len,
                                         void* workspace, size_t workspace_bytes, void* output, void* stream) {
    if ((dtype != FB_FP16 && dtype != FB_BF16) || !kvp::shape_ok(num_q_heads, num_kv_heads, head_dim))
        return (int)cudaErrorInvalidValue;
    if (num_seqs < 0 || q_per_seq < 0 || max_blocks_per_seq < 0 || max_kv_len < 0 || num_pool_rows < 0)
        return (int)cudaErrorInvalidValue;
    const int64_t rows = (int64_t)num_seqs * q_per_seq;
    if (rows == 0) return 0;
    if (!q || !output || !kv_lens || !start_pos) return (int)cudaErrorInvalidValue;
    if (max_kv_len > 0 && (!block_tables || !k_pool || !v_pool)) return (int)cudaErrorInvalidValue;
    if (!aligned16(k_pool) || !aligned16(v_pool) || !aligned16(workspace)) return (int)cudaErrorInvalidValue;
    const int nch = (max_kv_len + kvp::CH - 1) / kvp::CH;
    if (rows > 65535 || !workspace || workspace_bytes < kvp::workspace_bytes(rows, num_q_heads, nch)) {
        set_last_error("fb_launch_attention_paged: workspace missing or smaller than fb_attention_workspace_bytes(), "
                       "or more than 65535 query rows");
        return (int)cudaErrorInvalidValue;
    }
    kvp::Args a{};
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
    a.part = (float*)workspace;
    a.nch = nch;
    a.out = output;
    kvp::PoolRows rw{(const uint8_t*)k_pool, (const uint8_t*)v_pool, num_pool_rows};
    return kvp::run(a, rw, (cudaStream_t)stream);
}

// ffi.rs:186-200 (attention_paged.cu:161-185): one sequence, FP16, per-block pointer arrays
// (block b's K rows at k_block_ptrs[b], [16, Hkv, d]). Workspace: this library's, one per device
// and stream, grown to the largest call on that stream.
extern "C" int launch_paged_attention(void* output, const void* q, const int* block_table, const void** k_block_ptrs,
                                      const void** v_block_ptrs, int num_tokens, int num_q_heads, int num_kv_heads,
                                      int head_dim, int kv_len, int start_pos, int num_blocks_in_seq, void* stream) {
    if (!kvp::shape_ok(num_q_heads, num_kv_heads, head_dim) || num_tokens < 0 || num_tokens > 65535 || kv_len < 0 ||
        start_pos < 0 || num_blocks_in_seq < 0)
        return (int)cudaErrorInvalidValue;
    if (num_tokens == 0) return 0;
    if (!output || !q) return (int)cudaErrorInvalidValue;
    if (kv_len > 0 && (!block_table || !k_block_ptrs || !v_block_ptrs)) return (int)cudaErrorInvalidValue;
    const int nch = (kv_len + kvp::CH - 1) / kvp::CH;
    const size_t need = std::max<size_t>(kvp::workspace_bytes(num_tokens, num_q_heads, nch), 16);
    return with_stream_workspace(stream, need, [&](void* ws) {
        kvp::Args a{};
        a.q = q;
        a.dtype = FB_FP16;
        a.num_seqs = 1;
        a.q_per_seq = num_tokens;
        a.hq = num_q_heads;
        a.hkv = num_kv_heads;
        a.block_tables = block_table;
        a.max_blocks = num_blocks_in_seq;
        a.kv_len = kv_len;
        a.start = start_pos;
        a.part = (float*)ws;
        a.nch = nch;
        a.out = output;
        kvp::BlockPtrRows rw{(const uint8_t* const*)k_block_ptrs, (const uint8_t* const*)v_block_ptrs};
        return kvp::run(a, rw, (cudaStream_t)stream);
    });
}

// PagedKvCacheManager::append_kv's writes (paged_kv_cache.rs:290-315) in one launch: keys/values
// [num_tokens, Hkv, d] (dtype FP16/BF16/FP32, the pool's), token t at sequence position
// start_pos + t.
extern "C" int fb_launch_kv_append_paged(const void* keys, const void* values, int dtype, int64_t num_tokens,
                                         int num_kv_heads, int head_dim, const int32_t* block_table, int64_t start_pos,
                                         int64_t num_pool_rows, void* k_pool, void* v_pool, unsigned int* err_count,
                                         void* stream) {
    const int esz = dtype == FB_FP32 ? 4 : (dtype == FB_FP16 || dtype == FB_BF16) ? 2 : 0;
    if (!esz || num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || start_pos < 0 || num_pool_rows < 0)
        return (int)cudaErrorInvalidValue;
    if (num_tokens == 0) return 0;
    const int64_t row_bytes = (int64_t)num_kv_heads * head_dim * esz;
    if (row_bytes % 16 || !keys || !values || !block_table || !k_pool || !v_pool)
        return (int)cudaErrorInvalidValue;
    if (!aligned16(keys) || !aligned16(values) || !aligned16(k_pool) || !aligned16(v_pool))
        return (int)cudaErrorInvalidValue;
    const int row_vecs = (int)(row_bytes / 16);
    const int64_t n = num_tokens * row_vecs;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 16));
    kvp::kvp_append<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint4*)keys, (const uint4*)values, num_tokens,
                                                            row_vecs, block_table, start_pos, num_pool_rows,
                                                            (uint4*)k_pool, (uint4*)v_pool, err_count);
    return (int)cudaGetLastError();
}
