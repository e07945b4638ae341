// Streaming elementwise kernels of the per-layer hot path, sm_100a.
//
// Every kernel moves activations with 128-bit coalesced loads/stores (one
// 16-byte vector per thread per step, several in flight per thread) and does
// its arithmetic in float32, rounding once to the storage dtype. Scalar
// variants of the same kernels cover unaligned pointers and ragged tails.
//
// Reference kernels replaced (paths relative to the Fracture repository):
//   embedding  backends/fracture-cuda/kernels/embedding.cu:7-47
//   add        backends/fracture-cuda/kernels/add.cu:5-29
//   rmsnorm    backends/fracture-cuda/kernels/rmsnorm.cu:10-85
//   silu_mul   backends/fracture-cuda/kernels/silu_mul.cu:8-38
//   add+rmsnorm has no reference kernel (the engine issues add then rmsnorm).

#include <algorithm>
#include <map>

#include "common.cuh"

namespace fb {

int num_sms() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

std::mutex& stream_workspace_mutex() {
    static std::mutex m;
    return m;
}

StreamWorkspace& stream_workspace(int device, const void* stream) {
    static std::map<std::pair<int, uintptr_t>, StreamWorkspace> buffers;
    return buffers[{device, reinterpret_cast<uintptr_t>(stream)}];
}

// Coherent streaming load: used where the same kernel writes the buffer it
// reads (in-place residual add, in-place rope), so the non-coherent path is
// not allowed.
__device__ __forceinline__ uint4 ld_stream_rw(const void* p) {
    uint4 v;
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// silu(g) * u in float32: g / (1 + e^-g) * u with the hardware exp2 and
// reciprocal (a few ulp of float32, far below the FP16/BF16 output rounding;
// for g < -87 the quotient flushes to zero instead of ~1e-37).
__device__ __forceinline__ float silu_mul_f32(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// ─── silu_mul ────────────────────────────────────────────────────────────────

template <typename T, int UNROLL>
__global__ void __launch_bounds__(256) silu_mul_vec_kernel(T* __restrict__ out, const T* __restrict__ gate,
                                                           const T* __restrict__ up, int64_t nvec) {
    pdl_begin();
    using V = Vec16<T>;
    const int64_t base = (int64_t)blockIdx.x * (blockDim.x * UNROLL) + threadIdx.x;
    V g[UNROLL], u[UNROLL];
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
        const int64_t i = base + (int64_t)k * blockDim.x;
        if (i < nvec) {
            g[k].u = ld_stream(gate + i * V::N);
            u[k].u = ld_stream(up + i * V::N);
        }
    }
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
        const int64_t i = base + (int64_t)k * blockDim.x;
        if (i < nvec) {
            V o;
#pragma unroll
            for (int e = 0; e < V::N; ++e) o.e[e] = from_f32<T>(silu_mul_f32(to_f32(g[k].e[e]), to_f32(u[k].e[e])));
            st_stream(out + i * V::N, o.u);
        }
    }
}

template <typename T>
__global__ void silu_mul_scalar_kernel(T* out, const T* gate, const T* up, int64_t begin, int64_t n) {
    pdl_begin();
    for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = from_f32<T>(silu_mul_f32(to_f32(gate[i]), to_f32(up[i])));
}

// ─── add ─────────────────────────────────────────────────────────────────────

template <typename T, int UNROLL>
__global__ void __launch_bounds__(256) add_vec_kernel(T* out, const T* a, const T* b, int64_t nvec) {
    pdl_begin();
    using V = Vec16<T>;
    const int64_t base = (int64_t)blockIdx.x * (blockDim.x * UNROLL) + threadIdx.x;
    V x[UNROLL], y[UNROLL];
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
        const int64_t i = base + (int64_t)k * blockDim.x;
        if (i < nvec) {
            x[k].u = ld_stream_rw(a + i * V::N);
            y[k].u = ld_stream_rw(b + i * V::N);
        }
    }
#pragma unroll
    for (int k = 0; k < UNROLL; ++k) {
        const int64_t i = base + (int64_t)k * blockDim.x;
        if (i < nvec) {
            V o;
#pragma unroll
            for (int e = 0; e < V::N; ++e) o.e[e] = from_f32<T>(to_f32(x[k].e[e]) + to_f32(y[k].e[e]));
            st_plain(out + i * V::N, o.u);
        }
    }
}

template <typename T>
__global__ void add_scalar_kernel(T* out, const T* a, const T* b, int64_t begin, int64_t n) {
    pdl_begin();
    for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = from_f32<T>(to_f32(a[i]) + to_f32(b[i]));
}

// ─── embedding ───────────────────────────────────────────────────────────────

// One CTA per token row; out-of-vocabulary ids give a zero row (embedding.cu:21-25).
template <typename T>
__global__ void embedding_vec_kernel(T* __restrict__ out, const T* __restrict__ table,
                                     const uint32_t* __restrict__ ids, int64_t hidden, int64_t hvec,
                                     uint32_t vocab) {
    pdl_begin();
    using V = Vec16<T>;
    const int64_t t = blockIdx.x;
    const uint32_t id = __ldg(ids + t);
    const bool ok = id < vocab;
    const T* src = table + (int64_t)(ok ? id : 0) * hidden;
    T* dst = out + t * hidden;
    for (int64_t c = threadIdx.x; c < hvec; c += blockDim.x) {
        uint4 v = ok ? ld_keep(src + c * V::N) : make_uint4(0, 0, 0, 0);
        st_stream(dst + c * V::N, v);
    }
}

template <typename T>
__global__ void embedding_scalar_kernel(T* out, const T* table, const uint32_t* ids, int64_t hidden, uint32_t vocab) {
    pdl_begin();
    const int64_t t = blockIdx.x;
    const uint32_t id = ids[t];
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x)
        out[t * hidden + c] = id < vocab ? table[(int64_t)id * hidden + c] : from_f32<T>(0.0f);
}

// ─── rmsnorm / fused residual add + rmsnorm ─────────────────────────────────

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        float s = lane < (int)((blockDim.x + 31) >> 5) ? red[lane] : 0.0f;
        s = warp_sum(s);
        if (lane == 0) red[32] = s;
    }
    __syncthreads();
    return red[32];
}

// One CTA per row; each thread keeps VPT 16-byte vectors of the row in
// registers, so the row is read from HBM once. With ADD, h = round(h + r) is
// formed first, written back, and the norm is taken of the rounded h — the
// value a separate add kernel would have stored.
template <typename T, int VPT, bool ADD>
__global__ void __launch_bounds__(256) norm_rows_vec_kernel(const T* x, const T* __restrict__ r, T* h_out,
                                                             const T* __restrict__ w, T* out, float eps,
                                                             int64_t cols, int cols_vec) {
    pdl_begin();
    using V = Vec16<T>;
    __shared__ float red[33];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * cols;
    V v[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < cols_vec) {
            v[k].u = ld_stream_rw(xr + (int64_t)c * V::N);
            if constexpr (ADD) {
                V rr;
                rr.u = ld_stream(r + row * cols + (int64_t)c * V::N);
#pragma unroll
                for (int e = 0; e < V::N; ++e) v[k].e[e] = from_f32<T>(to_f32(v[k].e[e]) + to_f32(rr.e[e]));
            }
        } else {
            v[k].u = make_uint4(0, 0, 0, 0);
        }
    }
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
        for (int e = 0; e < V::N; ++e) {
            const float f = to_f32(v[k].e[e]);
            ss += f * f;
        }
    if constexpr (ADD) {
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const int c = threadIdx.x + k * blockDim.x;
            if (c < cols_vec) st_plain(h_out + row * cols + (int64_t)c * V::N, v[k].u);
        }
    }
    ss = block_sum<0>(ss, red);
    const float rinv = 1.0f / sqrtf(ss / (float)cols + eps);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < cols_vec) {
            V wv, o;
            wv.u = ld_keep(w + (int64_t)c * V::N);
#pragma unroll
            for (int e = 0; e < V::N; ++e) o.e[e] = from_f32<T>(to_f32(v[k].e[e]) * rinv * to_f32(wv.e[e]));
            st_stream(out + row * cols + (int64_t)c * V::N, o.u);
        }
    }
}

template <typename T, bool ADD>
__global__ void norm_rows_scalar_kernel(const T* x, const T* r, T* h_out, const T* w, T* out, float eps, int64_t cols) {
    pdl_begin();
    __shared__ float red[33];
    const int64_t row = blockIdx.x;
    float ss = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        float f = to_f32(x[row * cols + c]);
        if constexpr (ADD) {
            const T h = from_f32<T>(f + to_f32(r[row * cols + c]));
            h_out[row * cols + c] = h;
            f = to_f32(h);
        }
        ss += f * f;
    }
    ss = block_sum<0>(ss, red);
    const float rinv = 1.0f / sqrtf(ss / (float)cols + eps);
    const T* src = ADD ? h_out : x;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
        out[row * cols + c] = from_f32<T>(to_f32(src[row * cols + c]) * rinv * to_f32(w[c]));
}

// ─── host launchers ─────────────────────────────────────────────────────────

static inline int grid_for(int64_t work, int per_block) {
    int64_t g = (work + per_block - 1) / per_block;
    return (int)std::min<int64_t>(std::max<int64_t>(g, 1), 0x7fffffff);
}

static inline int64_t stride_grid(int64_t work, int threads) {
    return std::min<int64_t>(std::max<int64_t>((work + threads - 1) / threads, 1), (int64_t)num_sms() * 32);
}

template <typename T>
static int silu_mul_impl(T* out, const T* gate, const T* up, int64_t n, cudaStream_t s) {
    constexpr int N = Vec16<T>::N, UNROLL = 4, TPB = 256;
    int64_t vec_elems = 0;
    if (aligned16(out) && aligned16(gate) && aligned16(up)) {
        const int64_t nvec = n / N;
        vec_elems = nvec * N;
        if (nvec > 0) launch_pdl(silu_mul_vec_kernel<T, UNROLL>, dim3(grid_for(nvec, TPB * UNROLL)), dim3(TPB), s, out, gate, up, nvec);
    }
    if (vec_elems < n)
        launch_pdl(silu_mul_scalar_kernel<T>, dim3((int)stride_grid(n - vec_elems, 256)), dim3(256), s, out, gate, up, vec_elems, n);
    return (int)cudaGetLastError();
}

template <typename T>
static int add_impl(T* out, const T* a, const T* b, int64_t n, cudaStream_t s) {
    constexpr int N = Vec16<T>::N, UNROLL = 4, TPB = 256;
    int64_t vec_elems = 0;
    if (aligned16(out) && aligned16(a) && aligned16(b)) {
        const int64_t nvec = n / N;
        vec_elems = nvec * N;
        if (nvec > 0) launch_pdl(add_vec_kernel<T, UNROLL>, dim3(grid_for(nvec, TPB * UNROLL)), dim3(TPB), s, out, a, b, nvec);
    }
    if (vec_elems < n) launch_pdl(add_scalar_kernel<T>, dim3((int)stride_grid(n - vec_elems, 256)), dim3(256), s, out, a, b, vec_elems, n);
    return (int)cudaGetLastError();
}

template <typename T>
static int embedding_impl(T* out, const T* table, const uint32_t* ids, int64_t ntok, int64_t hidden, int64_t vocab,
                          cudaStream_t s) {
    constexpr int N = Vec16<T>::N;
    const uint32_t v32 = (uint32_t)std::min<int64_t>(vocab, 0xffffffffLL);
    if (aligned16(out) && aligned16(table) && hidden % N == 0) {
        const int64_t hvec = hidden / N;
        const int tpb = (int)std::min<int64_t>(256, ((hvec + 31) / 32) * 32);
        launch_pdl(embedding_vec_kernel<T>, dim3((unsigned)ntok), dim3(tpb), s, out, table, ids, hidden, hvec, v32);
    } else {
        const int tpb = (int)std::min<int64_t>(256, ((hidden + 31) / 32) * 32);
        launch_pdl(embedding_scalar_kernel<T>, dim3((unsigned)ntok), dim3(tpb), s, out, table, ids, hidden, v32);
    }
    return (int)cudaGetLastError();
}

template <typename T, bool ADD, int VPT>
static void launch_norm_vec(const T* x, const T* r, T* h, const T* w, T* out, float eps, int64_t rows, int64_t cols,
                            int cols_vec, cudaStream_t s) {
    int tpb = (cols_vec + VPT - 1) / VPT;
    tpb = ((tpb + 31) / 32) * 32;
    launch_pdl(norm_rows_vec_kernel<T, VPT, ADD>, dim3((unsigned)rows), dim3(tpb), s, x, r, h, w, out, eps, cols, cols_vec);
}

template <typename T, bool ADD>
static int norm_impl(const T* x, const T* r, T* h, const T* w, T* out, float eps, int64_t rows, int64_t cols,
                     cudaStream_t s) {
    constexpr int N = Vec16<T>::N;
    const bool vec_ok = aligned16(x) && aligned16(w) && aligned16(out) && (!ADD || (aligned16(r) && aligned16(h))) &&
                        cols % N == 0 && cols / N <= 2048;
    if (vec_ok) {
        const int cols_vec = (int)(cols / N);
        // <= 256 threads per row, each holding VPT vectors in registers.
        if (cols_vec <= 256) launch_norm_vec<T, ADD, 1>(x, r, h, w, out, eps, rows, cols, cols_vec, s);
        else if (cols_vec <= 512) launch_norm_vec<T, ADD, 2>(x, r, h, w, out, eps, rows, cols, cols_vec, s);
        else if (cols_vec <= 1024) launch_norm_vec<T, ADD, 4>(x, r, h, w, out, eps, rows, cols, cols_vec, s);
        else launch_norm_vec<T, ADD, 8>(x, r, h, w, out, eps, rows, cols, cols_vec, s);
    } else {
        launch_pdl(norm_rows_scalar_kernel<T, ADD>, dim3((unsigned)rows), dim3(256), s, x, r, h, w, out, eps, cols);
    }
    return (int)cudaGetLastError();
}

}  // namespace fb

using namespace fb;

// ─── C ABI ──────────────────────────────────────────────────────────────────

extern "C" int fb_launch_silu_mul(void* output, const void* gate, const void* up, int64_t n, int dtype, void* stream) {
    if (n < 0 || (n > 0 && (!output || !gate || !up))) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    return FB_DISPATCH_FLOAT(dtype, return silu_mul_impl<T>((T*)output, (const T*)gate, (const T*)up, n,
                                                           (cudaStream_t)stream););
}

extern "C" int fb_launch_add(void* output, const void* a, const void* b, int64_t n, int dtype, void* stream) {
    if (n < 0 || (n > 0 && (!output || !a || !b))) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    return FB_DISPATCH_FLOAT(dtype, return add_impl<T>((T*)output, (const T*)a, (const T*)b, n, (cudaStream_t)stream););
}

extern "C" int fb_launch_embedding(void* output, const void* table, const uint32_t* token_ids, int64_t num_tokens,
                                   int64_t hidden_dim, int64_t vocab_size, int dtype, void* stream) {
    if (num_tokens < 0 || hidden_dim < 0 || vocab_size < 0 || num_tokens > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
    if (num_tokens == 0 || hidden_dim == 0) return 0;
    if (!output || !token_ids || (vocab_size > 0 && !table)) return (int)cudaErrorInvalidValue;
    return FB_DISPATCH_FLOAT(dtype, return embedding_impl<T>((T*)output, (const T*)table, token_ids, num_tokens,
                                                            hidden_dim, vocab_size, (cudaStream_t)stream););
}

extern "C" int fb_launch_rmsnorm(void* output, const void* input, const void* weight, float eps, int64_t rows,
                                 int64_t cols, int dtype, void* stream) {
    if (rows < 0 || cols < 0 || rows > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
    if (rows == 0 || cols == 0) return 0;
    if (!output || !input || !weight) return (int)cudaErrorInvalidValue;
    return FB_DISPATCH_FLOAT(dtype, return norm_impl<T, false>((const T*)input, nullptr, nullptr, (const T*)weight,
                                                              (T*)output, eps, rows, cols, (cudaStream_t)stream););
}

extern "C" int fb_launch_add_rmsnorm(void* h_inout, const void* residual, const void* weight, void* normed_out,
                                     float eps, int64_t rows, int64_t cols, int dtype, void* stream) {
    if (rows < 0 || cols < 0 || rows > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
    if (rows == 0 || cols == 0) return 0;
    if (!h_inout || !residual || !weight || !normed_out) return (int)cudaErrorInvalidValue;
    return FB_DISPATCH_FLOAT(dtype, return norm_impl<T, true>((const T*)h_inout, (const T*)residual, (T*)h_inout,
                                                             (const T*)weight, (T*)normed_out, eps, rows, cols,
                                                             (cudaStream_t)stream););
}

// Reference ABI (FP16). Negative sizes are rejected; empty inputs are a no-op.
extern "C" int launch_silu_mul(void* output, const void* gate, const void* up, int n, void* stream) {
    return fb_launch_silu_mul(output, gate, up, n, FB_FP16, stream);
}

extern "C" int launch_add(void* output, const void* a, const void* b, int n, void* stream) {
    return fb_launch_add(output, a, b, n, FB_FP16, stream);
}

extern "C" int launch_embedding(void* output, const void* table, const uint32_t* token_ids, int num_tokens,
                                int hidden_dim, int vocab_size, void* stream) {
    return fb_launch_embedding(output, table, token_ids, num_tokens, hidden_dim, vocab_size, FB_FP16, stream);
}

extern "C" int launch_rmsnorm(void* output, const void* input, const void* weight, float eps, int rows, int cols,
                              void* stream) {
    return fb_launch_rmsnorm(output, input, weight, eps, rows, cols, FB_FP16, stream);
}
