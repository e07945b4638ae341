// TurboQuant compress / dequantize for small calls (decode steps: up to a few thousand head
// vectors), in the exact float32 order of tq_exact.cu.
//
// The tensor-core kernels build their operands and decision table in every CTA (~10 us of
// GPU time before the first tile), which at decode sizes is the whole call. Here a CTA takes
// V vectors (V chosen so the call spreads over the SMs), copies Pi into shared memory with
// asynchronous 16-byte copies (rows padded to d + 4 floats, so that thread i reading row i
// four floats at a time, and thread i reading column i, are both free of bank conflicts),
// and thread i computes coordinate i of the CTA's vectors with their sequential sums
// interleaved (compress: two thread halves with half the vectors each where head_dim allows; a
// launch may serve the K and V of one append, its CTAs split between them). Results are the
// exact statement
// (crates/fracture-core/src/turboquant.rs:1225-1290), like tq_exact.cu, with the same slot
// rule and error counting.

#include <algorithm>

#include "common.cuh"
#include "tq_common.cuh"

namespace fb {

namespace {

constexpr int SMALL_MAX_V = 8;

// Shared layout: Pi (d rows of d + 4 floats), the V vectors ([V][d] floats), centroids (256),
// denominators or norms and pool rows (V each), codes ([V][d] bytes).
size_t small_smem(int d, int V) {
    return sizeof(float) * ((size_t)d * (d + 4) + (size_t)V * d + 256 + V) + sizeof(long long) * V + 16 +
           (size_t)V * d;
}

// Pi (row-major in global memory) into shared rows of stride d + 4: 16-byte asynchronous
// copies when rows allow it (all in flight at once; the caller waits with
// cp.async.wait_all), element copies otherwise.
__device__ __forceinline__ void stage_pi(float* dst, const float* pi, int d) {
    const int ld = d + 4;
    if ((d & 3) == 0 && ((uintptr_t)pi & 15) == 0) {
        const int q = d / 4;
        for (int e = threadIdx.x; e < d * q; e += blockDim.x) {
            const int r = e / q, c = e - r * q;
            const uint32_t sa = (uint32_t)__cvta_generic_to_shared(dst + r * ld + 4 * c);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(pi + (int64_t)r * d + 4 * c) : "memory");
        }
    } else {
        for (int e = threadIdx.x; e < d * d; e += blockDim.x) {
            const int r = e / d, c = e - r * d;
            dst[r * ld + c] = __ldg(pi + e);
        }
    }
}

__device__ __forceinline__ void stage_wait() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// exact_norm of tq_common.cuh (the same sequential sum) with the shared-memory loads issued
// eight at a time ahead of the chain.
__device__ __forceinline__ float norm_seq(const float* x, int d) {
    float s = 0.0f;
    int j = 0;
    for (; j + 8 <= d; j += 8) {
        float t[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) t[k] = x[j + k];
#pragma unroll
        for (int k = 0; k < 8; ++k) s = __fadd_rn(s, __fmul_rn(t[k], t[k]));
    }
    for (; j < d; ++j) s = __fadd_rn(s, __fmul_rn(x[j], x[j]));
    return __fsqrt_rn(s);
}

// One launch serves one compress call, or two (the K and V of an append, equal in vector count
// and head_dim): CTAs [0, nblk0) take job 0, the rest job 1.
struct SmallJobs {
    TqArgs a[2];
    unsigned nblk0;
    int njobs;
};

// NH = 2 splits the CTA's vectors between two halves of the threads (each half one thread per
// coordinate), so that a CTA runs twice the warps on the sequential sums.
template <int V, int NH>
__global__ void __launch_bounds__(256) tq_compress_small_kernel(const __grid_constant__ SmallJobs J) {
    pdl_begin();
    extern __shared__ __align__(16) float sm[];
    const int jb = (J.njobs > 1 && blockIdx.x >= J.nblk0) ? 1 : 0;
    const TqArgs& a = J.a[jb];
    const int64_t blk = (int64_t)blockIdx.x - (jb ? (int64_t)J.nblk0 : 0);
    const int d = a.head_dim, ld = d + 4, i = threadIdx.x;
    float* pis = sm;                 // pis[r * ld + j] = Pi[r][j]
    float* xs = pis + d * ld;        // [V][d]: x, then x / (norm + 1e-8)
    float* cen = xs + V * d;         // [256]
    float* den = cen + 256;          // [V]
    long long* prow_s = (long long*)(((uintptr_t)(den + V) + 7) & ~(uintptr_t)7);  // [V]
    uint8_t* idx = (uint8_t*)(prow_s + V);  // [V][d]
    const int64_t nvec = a.num_tokens * a.num_heads;
    const int64_t v0 = blk * V;
    const int nv = (int)std::min<int64_t>(V, nvec - v0);

    stage_pi(pis, a.rotation, d);  // in flight while the norms are summed
    int64_t prow = -1;
    if (i < nv) {  // the slot lookup overlaps the loads below
        const int64_t vi = v0 + i;
        const int64_t slot = tq_slot(a, vi / a.num_heads);  // once per vector
        prow = slot >= 0 ? slot * a.num_heads + vi % a.num_heads : -1;
    }
    for (int e = i; e < a.n_levels; e += blockDim.x) cen[e] = __ldg(a.centroids + e);
    for (int e = i; e < nv * d; e += blockDim.x) xs[e] = load_in_f32(a.input, a.in_dtype, v0 * d + e);
    __syncthreads();
    if (i < nv) {
        const float norm = norm_seq(xs + i * d, d);
        if (prow >= 0) ((__half*)a.norms_pool)[prow] = __float2half_rn(norm);
        prow_s[i] = prow;
        den[i] = __fadd_rn(norm, 1e-8f);
    }
    stage_wait();
    __syncthreads();
    for (int e = i; e < nv * d; e += blockDim.x) xs[e] = __fdiv_rn(xs[e], den[e / d]);
    __syncthreads();
    constexpr int VH = V / NH;  // vectors per thread
    const int tph = (int)blockDim.x / NH, half = i / tph, c = i - half * tph;  // coordinate c of half `half`
    if (c < d) {
        float acc[VH];
#pragma unroll
        for (int v = 0; v < VH; ++v) acc[v] = 0.0f;
        const float* row = pis + c * ld;
        const float* xh = xs + half * VH * d;
        if ((d & 3) == 0) {
            // row c four floats at a time (16-byte aligned: ld is a multiple of 4)
#pragma unroll 2
            for (int j = 0; j < d; j += 4) {
                const float4 p = *(const float4*)(row + j);
#pragma unroll
                for (int v = 0; v < VH; ++v) {
                    const float4 x = *(const float4*)(xh + v * d + j);
                    acc[v] = __fadd_rn(acc[v], __fmul_rn(p.x, x.x));
                    acc[v] = __fadd_rn(acc[v], __fmul_rn(p.y, x.y));
                    acc[v] = __fadd_rn(acc[v], __fmul_rn(p.z, x.z));
                    acc[v] = __fadd_rn(acc[v], __fmul_rn(p.w, x.w));
                }
            }
        } else {
            for (int j = 0; j < d; ++j) {
                const float p = row[j];
#pragma unroll
                for (int v = 0; v < VH; ++v) acc[v] = __fadd_rn(acc[v], __fmul_rn(p, xh[v * d + j]));
            }
        }
#pragma unroll
        for (int v = 0; v < VH; ++v) {
            const int vv = half * VH + v;
            if (vv < nv) idx[vv * d + c] = (uint8_t)nearest_centroid(acc[v], cen, a.n_levels);
        }
    }
    __syncthreads();
    const int P = (d * a.bits + 7) >> 3;
    for (int e = i; e < nv * P; e += blockDim.x) {
        const int v = e / P, b = e - v * P;
        if (prow_s[v] < 0) continue;
        const uint8_t* c = idx + v * d;
        uint8_t byte;
        if (a.bits == 4) byte = (uint8_t)((c[2 * b] << 4) | (2 * b + 1 < d ? c[2 * b + 1] : 0));
        else if (a.bits == 8) byte = c[b];
        else byte = pack_byte(c, d, a.bits, b);  // MSB-first stream, any width
        ((uint8_t*)a.packed_pool)[prow_s[v] * P + b] = byte;
    }
}

// x_i = (sum_j Pi[j][i] * c[idx_j] in order) * norm; a vector without a slot gives zeros.
template <typename Tout, int V>
__global__ void __launch_bounds__(256) tq_dequant_small_kernel(TqArgs a) {
    pdl_begin();
    extern __shared__ __align__(16) float sm[];
    const int d = a.head_dim, i = threadIdx.x;
    const int ld = d + 4;
    float* pi = sm;               // pi[j * ld + i] = Pi[j][i] (thread i reads column i)
    float* yh = pi + d * ld;      // [V][d] centroid values
    float* cen = yh + V * d;      // [256]
    float* nrm = cen + 256;       // [V]
    long long* prow_s = (long long*)(((uintptr_t)(nrm + V) + 7) & ~(uintptr_t)7);  // [V]
    const int64_t nvec = a.num_tokens * a.num_heads;
    const int64_t v0 = (int64_t)blockIdx.x * V;
    const int nv = (int)std::min<int64_t>(V, nvec - v0);
    const int P = (d * a.bits + 7) >> 3;
    stage_pi(pi, a.rotation, d);
    for (int e = i; e < a.n_levels; e += blockDim.x) cen[e] = __ldg(a.centroids + e);
    if (i < nv) {
        const int64_t vi = v0 + i;
        const int64_t slot = tq_slot(a, vi / a.num_heads);
        const int64_t prow = slot >= 0 ? slot * a.num_heads + vi % a.num_heads : -1;
        prow_s[i] = prow;
        nrm[i] = prow >= 0 ? __half2float(((const __half*)a.norms_pool)[prow]) : 0.0f;
    }
    __syncthreads();
    for (int e = i; e < nv * d; e += blockDim.x) {
        const int v = e / d, j = e - v * d;
        const long long prow = prow_s[v];
        yh[e] = cen[prow >= 0 ? unpack_code((const uint8_t*)a.packed_pool + prow * P, j, a.bits) : 0];
    }
    stage_wait();
    __syncthreads();
    if (i < d) {
        float acc[V];
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = 0.0f;
#pragma unroll 4
        for (int j = 0; j < d; ++j) {
            const float p = pi[j * ld + i];
#pragma unroll
            for (int v = 0; v < V; ++v) acc[v] = __fadd_rn(acc[v], __fmul_rn(p, yh[v * d + j]));
        }
#pragma unroll
        for (int v = 0; v < V; ++v)
            if (v < nv) ((Tout*)a.output)[(v0 + v) * d + i] = from_f32<Tout>(__fmul_rn(acc[v], nrm[v]));
    }
}

int small_threads(int d) { return std::max(32, ((d + 31) / 32) * 32); }

// Vectors per CTA: the smallest power of two up to SMALL_MAX_V that keeps the CTAs within
// about two per SM.
int small_v(int64_t nvec) {
    int v = 1;
    while (v < SMALL_MAX_V && nvec > (int64_t)num_sms() * 2 * v) v *= 2;
    return v;
}

template <typename K>
int launch_small(K kern, const TqArgs& a, int V, cudaStream_t s) {
    const size_t smem = small_smem(a.head_dim, V);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    const int64_t nvec = a.num_tokens * a.num_heads;
    launch_pdl_smem(kern, dim3((unsigned)((nvec + V - 1) / V)), dim3(small_threads(a.head_dim)), smem, s, a);
    return (int)cudaGetLastError();
}

// jobs[0..njobs) (njobs 1 or 2, equal head_dim) in one launch of V-vector CTAs.
template <int V>
int launch_compress_small(const TqArgs* jobs, int njobs, cudaStream_t s) {
    SmallJobs J{};
    int64_t blocks = 0;
    for (int j = 0; j < njobs; ++j) {
        J.a[j] = jobs[j];
        const int64_t nb = (jobs[j].num_tokens * jobs[j].num_heads + V - 1) / V;
        if (j == 0) J.nblk0 = (unsigned)nb;
        blocks += nb;
    }
    J.njobs = njobs;
    if (blocks == 0) return 0;
    // two thread halves (each one thread per coordinate) when the CTA has vectors to split and
    // room for twice the threads
    const int th = small_threads(jobs[0].head_dim);
    const bool split = V >= 2 && 2 * th <= 256;
    auto kern = split ? tq_compress_small_kernel<V, (V >= 2 ? 2 : 1)> : tq_compress_small_kernel<V, 1>;
    const size_t smem = small_smem(jobs[0].head_dim, V);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    launch_pdl_smem(kern, dim3((unsigned)blocks), dim3(split ? 2 * th : th), smem, s, J);
    return (int)cudaGetLastError();
}

int compress_small_jobs(const TqArgs* jobs, int njobs, cudaStream_t s) {
    int64_t nvec = 0;
    for (int j = 0; j < njobs; ++j) nvec += jobs[j].num_tokens * jobs[j].num_heads;
    if (nvec == 0) return 0;
    const int V = small_v(nvec);
    if (V == 1) return launch_compress_small<1>(jobs, njobs, s);
    if (V == 2) return launch_compress_small<2>(jobs, njobs, s);
    if (V == 4) return launch_compress_small<4>(jobs, njobs, s);
    return launch_compress_small<8>(jobs, njobs, s);
}

}  // namespace

// head_dim <= 192 (the entry points' limit): Pi and the vectors fit in shared memory.
bool tq_small_compress_call(const TqArgs& a) {
    return a.head_dim <= 192 && a.num_tokens * a.num_heads <= kTqSmallCompressVectors;
}

bool tq_small_dequant_call(const TqArgs& a) {
    return a.head_dim <= 192 && a.num_tokens * a.num_heads <= kTqSmallDequantVectors;
}

int tq_compress_small(const TqArgs& a, cudaStream_t s) { return compress_small_jobs(&a, 1, s); }

// The K and V of one append (the same tokens and head layout) in one launch.
int tq_compress_small_pair(const TqArgs& k, const TqArgs& v, cudaStream_t s) {
    const TqArgs jobs[2] = {k, v};
    return compress_small_jobs(jobs, 2, s);
}

int tq_dequant_small(const TqArgs& a, cudaStream_t s) {
    if (a.num_tokens * a.num_heads == 0) return 0;
    const int V = small_v(a.num_tokens * a.num_heads);
    return FB_DISPATCH_FLOAT(a.out_dtype, {
        if (V == 1) return launch_small(tq_dequant_small_kernel<T, 1>, a, 1, s);
        if (V == 2) return launch_small(tq_dequant_small_kernel<T, 2>, a, 2, s);
        if (V == 4) return launch_small(tq_dequant_small_kernel<T, 4>, a, 4, s);
        return launch_small(tq_dequant_small_kernel<T, 8>, a, 8, s);
    });
}

}  // namespace fb
