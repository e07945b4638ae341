// TurboQuant compress / dequantize on CUDA cores in exact float32 order.
//
// These kernels evaluate the reference's CPU statement of the algorithm
// (crates/fracture-core/src/turboquant.rs:1225-1290) operation for operation:
// sequential sums with separately rounded multiply and add (__fmul_rn /
// __fadd_rn, so nothing is contracted to an FMA), true division by
// (norm + 1e-8), nearest centroid with the first minimum winning. They serve
// every head_dim up to 192 (the limit the entry points check) and any input
// alignment; the tensor-core kernel in
// tq_umma.cu takes head_dim 128 and reuses the per-coordinate routine here to
// settle coordinates that fall near a decision boundary.
//
// Layout (shared with tq_umma.cu): token t of the call is position
// start_pos + t of the sequence; its pool row is
//   slot = block_table ? block_table[pos / 16] * 16 + pos % 16 : pos
// packed bytes of head h at packed_pool[slot * H * P + h * P ...], P = ceil(d*bits/8),
// MSB-first bit stream; the fp16 norm at norms_pool[slot * H + h].

#include <algorithm>

#include "common.cuh"
#include "tq_common.cuh"

namespace fb {

constexpr int EX_V = 4;  // vectors per CTA iteration

// One CTA of `nthreads` (>= d, multiple of 32) handles EX_V vectors at a time;
// thread i computes coordinate i of each.
template <typename Tin>
__global__ void __launch_bounds__(256) tq_compress_exact_kernel(TqArgs a) {
    extern __shared__ float smem[];
    const int d = a.head_dim;
    float* piT = smem;                  // [d][d]: piT[j*d + i] = Pi[i][j]
    float* xs = piT + d * d;            // [EX_V][d] input as float, then xn
    float* cen = xs + EX_V * d;         // [256]
    float* scal = cen + 256;            // [EX_V] denominators
    int64_t* prow_s = (int64_t*)(((uintptr_t)(scal + EX_V) + 7) & ~(uintptr_t)7);  // [EX_V] pool rows (-1: none)
    uint8_t* idx = (uint8_t*)(prow_s + EX_V);   // [EX_V][d]

    for (int e = threadIdx.x; e < d * d; e += blockDim.x) {
        const int i = e / d, j = e % d;
        piT[j * d + i] = a.rotation[e];
    }
    for (int e = threadIdx.x; e < a.n_levels; e += blockDim.x) cen[e] = a.centroids[e];
    __syncthreads();

    const int64_t nvec = a.num_tokens * a.num_heads;
    const int P = (d * a.bits + 7) >> 3;
    for (int64_t v0 = (int64_t)blockIdx.x * EX_V; v0 < nvec; v0 += (int64_t)gridDim.x * EX_V) {
        const int nv = (int)std::min<int64_t>(EX_V, nvec - v0);
        for (int e = threadIdx.x; e < nv * d; e += blockDim.x) {
            const int v = e / d, j = e % d;
            xs[v * d + j] = load_in_f32(a.input, a.in_dtype, (v0 + v) * d + j);
        }
        __syncthreads();
        if (threadIdx.x < nv) {
            const int v = threadIdx.x;
            const float norm = exact_norm(xs + v * d, d);
            const int64_t vi = v0 + v;
            const int64_t slot = tq_slot(a, vi / a.num_heads);  // once per vector (counts a miss once)
            prow_s[v] = slot >= 0 ? slot * a.num_heads + vi % a.num_heads : -1;
            if (slot >= 0) ((__half*)a.norms_pool)[prow_s[v]] = __float2half_rn(norm);
            scal[v] = __fadd_rn(norm, 1e-8f);
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nv * d; e += blockDim.x) {
            const int v = e / d;
            xs[e] = __fdiv_rn(xs[e], scal[v]);
        }
        __syncthreads();
        if (threadIdx.x < d) {
            const int i = threadIdx.x;
            float acc[EX_V];
#pragma unroll
            for (int v = 0; v < EX_V; ++v) acc[v] = 0.0f;
            for (int j = 0; j < d; ++j) {
                const float p = piT[j * d + i];
#pragma unroll
                for (int v = 0; v < EX_V; ++v) acc[v] = __fadd_rn(acc[v], __fmul_rn(p, xs[v * d + j]));
            }
            for (int v = 0; v < nv; ++v) idx[v * d + i] = (uint8_t)nearest_centroid(acc[v], cen, a.n_levels);
        }
        __syncthreads();
        for (int e = threadIdx.x; e < nv * P; e += blockDim.x) {
            const int v = e / P, byte = e % P;
            if (prow_s[v] < 0) continue;
            ((uint8_t*)a.packed_pool)[prow_s[v] * P + byte] = pack_byte(idx + v * d, d, a.bits, byte);
        }
        __syncthreads();
    }
}

// x_i = sum_j Pi[j][i] * c[idx_j] (sequential, non-fused), times the fp16 norm.
template <typename Tout>
__global__ void __launch_bounds__(256) tq_dequant_exact_kernel(TqArgs a) {
    extern __shared__ float smem[];
    const int d = a.head_dim;
    float* pi = smem;            // [d][d] row-major Pi
    float* yh = pi + d * d;      // [EX_V][d]
    float* cen = yh + EX_V * d;  // [256]
    for (int e = threadIdx.x; e < d * d; e += blockDim.x) pi[e] = a.rotation[e];
    for (int e = threadIdx.x; e < a.n_levels; e += blockDim.x) cen[e] = a.centroids[e];
    __syncthreads();
    const int64_t nvec = a.num_tokens * a.num_heads;
    const int P = (d * a.bits + 7) >> 3;
    for (int64_t v0 = (int64_t)blockIdx.x * EX_V; v0 < nvec; v0 += (int64_t)gridDim.x * EX_V) {
        const int nv = (int)std::min<int64_t>(EX_V, nvec - v0);
        for (int e = threadIdx.x; e < nv * d; e += blockDim.x) {
            const int v = e / d, i = e % d;
            const int64_t vi = v0 + v;
            const int64_t slot = tq_slot(a, vi / a.num_heads);
            int code = 0;
            if (slot >= 0)
                code = unpack_code((const uint8_t*)a.packed_pool + (slot * a.num_heads + vi % a.num_heads) * P, i, a.bits);
            yh[e] = cen[code];
        }
        __syncthreads();
        if (threadIdx.x < d) {
            const int i = threadIdx.x;
            for (int v = 0; v < nv; ++v) {
                float acc = 0.0f;
                for (int j = 0; j < d; ++j) acc = __fadd_rn(acc, __fmul_rn(pi[j * d + i], yh[v * d + j]));
                const int64_t vi = v0 + v;
                const int64_t slot = tq_slot(a, vi / a.num_heads);
                const float nrm = slot >= 0 ? __half2float(((const __half*)a.norms_pool)[slot * a.num_heads + vi % a.num_heads]) : 0.0f;
                ((Tout*)a.output)[vi * d + i] = from_f32<Tout>(__fmul_rn(acc, nrm));
            }
        }
        __syncthreads();
    }
}

static size_t exact_compress_smem(int d) {
    return sizeof(float) * ((size_t)d * d + EX_V * d + 256 + EX_V) + 8 + sizeof(int64_t) * EX_V + EX_V * d;
}

int tq_compress_exact(const TqArgs& a, cudaStream_t s) {
    const int threads = std::max(32, std::min(256, ((a.head_dim + 31) / 32) * 32));
    const size_t smem = exact_compress_smem(a.head_dim);
    cudaError_t e;
    if (a.in_dtype == FB_BF16) {
        e = cudaFuncSetAttribute(tq_compress_exact_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
    } else {
        e = cudaFuncSetAttribute(tq_compress_exact_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
    }
    const int64_t nvec = a.num_tokens * a.num_heads;
    const int64_t want = (nvec + EX_V - 1) / EX_V;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)num_sms() * 8));
    if (a.in_dtype == FB_BF16) tq_compress_exact_kernel<__nv_bfloat16><<<grid, threads, smem, s>>>(a);
    else tq_compress_exact_kernel<__half><<<grid, threads, smem, s>>>(a);
    return (int)cudaGetLastError();
}

int tq_dequant_exact(const TqArgs& a, cudaStream_t s) {
    const int threads = std::max(32, std::min(256, ((a.head_dim + 31) / 32) * 32));
    const size_t smem = sizeof(float) * ((size_t)a.head_dim * a.head_dim + EX_V * a.head_dim + 256);
    const int64_t nvec = a.num_tokens * a.num_heads;
    const int64_t want = (nvec + EX_V - 1) / EX_V;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)num_sms() * 8));
    return FB_DISPATCH_FLOAT(a.out_dtype, {
        cudaError_t e = cudaFuncSetAttribute(tq_dequant_exact_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return (int)e;
        tq_dequant_exact_kernel<T><<<grid, threads, smem, s>>>(a);
        return (int)cudaGetLastError();
    });
}

}  // namespace fb
