// Rotary position embedding on Q and K in one launch, sm_100a.
//
// Replaces backends/fracture-cuda/kernels/rope.cu:20-82 (one thread per
// (token, head, pair) and two launches, fast-math cosf/sinf recomputed for
// every head). Here a thread owns 8 consecutive rotation pairs (one 16-byte
// vector of the low half and one of the high half of the head) for up to
// HG heads of one token: it evaluates the 8 angles once with the accurate
// sincosf and applies them to all of its heads, with all of its 2*HG vector
// loads in flight before the first store.
//
// angle = float(position) * freq[i] is the f32 product of the reference
// kernel (rope.cu:38); freq comes from fb_rope_freqs / fb_rope_freqs_llama3.

#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace fb {

__device__ __forceinline__ uint4 ld_rw_na(const void* p) {
    uint4 v;
    asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <typename T, int HG>
__global__ void __launch_bounds__(256) rope_vec_kernel(T* q, T* k, const uint32_t* __restrict__ positions,
                                                       const float* __restrict__ freqs, int64_t num_tokens,
                                                       int nq, int nkv, int head_dim, int ngv, int qgroups,
                                                       int kgroups) {
    pdl_begin();
    using V = Vec16<T>;
    constexpr int N = V::N;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int g = (int)(tid % ngv);
    const int64_t rest = tid / ngv;
    const int groups = qgroups + kgroups;
    const int hg = (int)(rest % groups);
    const int64_t tok = rest / groups;
    if (tok >= num_tokens) return;

    T* base;
    int nheads, h0;
    if (hg < qgroups) {
        base = q;
        nheads = nq;
        h0 = hg * HG;
    } else {
        base = k;
        nheads = nkv;
        h0 = (hg - qgroups) * HG;
    }
    const int hcount = min(HG, nheads - h0);
    const int half = head_dim >> 1;

    T* row = base + (tok * nheads + h0) * (int64_t)head_dim + g * N;
    V lo[HG], hi[HG];
#pragma unroll
    for (int h = 0; h < HG; ++h) {
        if (h < hcount) {
            lo[h].u = ld_rw_na(row + (int64_t)h * head_dim);
            hi[h].u = ld_rw_na(row + (int64_t)h * head_dim + half);
        }
    }

    const float p = (float)__ldg(positions + tok);
    float c[N], s[N];
#pragma unroll
    for (int e = 0; e < N; ++e) {
        const float ang = p * __ldg(freqs + g * N + e);
        sincosf(ang, &s[e], &c[e]);
    }

#pragma unroll
    for (int h = 0; h < HG; ++h) {
        if (h < hcount) {
            V a, b;
#pragma unroll
            for (int e = 0; e < N; ++e) {
                const float x0 = to_f32(lo[h].e[e]), x1 = to_f32(hi[h].e[e]);
                a.e[e] = from_f32<T>(x0 * c[e] - x1 * s[e]);
                b.e[e] = from_f32<T>(x0 * s[e] + x1 * c[e]);
            }
            st_plain(row + (int64_t)h * head_dim, a.u);
            st_plain(row + (int64_t)h * head_dim + half, b.u);
        }
    }
}

// Any even head_dim / alignment: one thread per (token, head, pair).
template <typename T>
__global__ void rope_scalar_kernel(T* q, T* k, const uint32_t* positions, const float* freqs, int64_t num_tokens,
                                   int nq, int nkv, int head_dim) {
    pdl_begin();
    const int half = head_dim >> 1;
    const int64_t per_tok = (int64_t)(nq + nkv) * half;
    const int64_t total = num_tokens * per_tok;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t tok = i / per_tok;
        const int64_t r = i % per_tok;
        const int head = (int)(r / half);
        const int d = (int)(r % half);
        T* vec = head < nq ? q + (tok * nq + head) * (int64_t)head_dim
                           : k + (tok * nkv + (head - nq)) * (int64_t)head_dim;
        float s, c;
        sincosf((float)positions[tok] * freqs[d], &s, &c);
        const float x0 = to_f32(vec[d]), x1 = to_f32(vec[d + half]);
        vec[d] = from_f32<T>(x0 * c - x1 * s);
        vec[d + half] = from_f32<T>(x0 * s + x1 * c);
    }
}

template <typename T>
static int rope_impl(T* q, T* k, const uint32_t* pos, const float* freqs, int64_t ntok, int nq, int nkv, int hd,
                     cudaStream_t s) {
    constexpr int N = Vec16<T>::N, HG = 8;
    const int half = hd / 2;
    const bool vec_ok = half % N == 0 && aligned16(q) && (nkv == 0 || aligned16(k));
    if (vec_ok) {
        const int ngv = half / N;
        const int qg = (nq + HG - 1) / HG, kg = (nkv + HG - 1) / HG;
        const int64_t threads = ntok * (int64_t)(qg + kg) * ngv;
        const int64_t blocks = (threads + 255) / 256;
        if (blocks > 0x7fffffffLL) return (int)cudaErrorInvalidValue;
        launch_pdl(rope_vec_kernel<T, HG>, dim3((unsigned)blocks), dim3(256), s, q, k, pos, freqs, ntok, nq, nkv, hd, ngv, qg, kg);
    } else {
        const int64_t total = ntok * (int64_t)(nq + nkv) * half;
        const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 32);
        launch_pdl(rope_scalar_kernel<T>, dim3((unsigned)std::max<int64_t>(blocks, 1)), dim3(256), s, q, k, pos, freqs,
                   ntok, nq, nkv, hd);
    }
    return (int)cudaGetLastError();
}

}  // namespace fb

using namespace fb;

extern "C" int fb_launch_rope(void* q, void* k, const uint32_t* positions, const float* freq_table,
                              int64_t num_tokens, int num_q_heads, int num_kv_heads, int head_dim, int dtype,
                              void* stream) {
    if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads < 0 || head_dim < 0 || (head_dim & 1))
        return (int)cudaErrorInvalidValue;
    if (num_tokens == 0 || head_dim == 0 || num_q_heads + num_kv_heads == 0) return 0;
    if (!positions || !freq_table || (num_q_heads > 0 && !q) || (num_kv_heads > 0 && !k))
        return (int)cudaErrorInvalidValue;
    return FB_DISPATCH_FLOAT(dtype, return rope_impl<T>((T*)q, (T*)k, positions, freq_table, num_tokens, num_q_heads,
                                                       num_kv_heads, head_dim, (cudaStream_t)stream););
}

extern "C" int launch_rope(void* q, void* k, const uint32_t* positions, const float* freq_table, int num_tokens,
                           int num_q_heads, int num_kv_heads, int head_dim, void* stream) {
    return fb_launch_rope(q, k, positions, freq_table, num_tokens, num_q_heads, num_kv_heads, head_dim, FB_FP16,
                          stream);
}

// Host tables ---------------------------------------------------------------

// CudaBackend::precompute_rope_freqs (src/lib.rs:133-138):
//   *freq = 1.0 / theta.powf(2.0 * i as f64 / head_dim as f64) as f32;
// `as` binds tighter than `/`, so the f64 power is cast to f32 and the
// reciprocal is an f32 division.
extern "C" int fb_rope_freqs(int head_dim, double theta, float* out) {
    if (head_dim <= 0 || (head_dim & 1) || !out || !(theta > 0.0)) return (int)cudaErrorInvalidValue;
    for (int i = 0; i < head_dim / 2; ++i) {
        const float p = (float)pow(theta, 2.0 * (double)i / (double)head_dim);
        out[i] = 1.0f / p;
    }
    return 0;
}

// Llama 3.1 frequency scaling (published rule; the reference has none):
// with wavelen = 2*pi/f, keep f where wavelen < orig/high_freq_factor, use
// f/factor where wavelen > orig/low_freq_factor, otherwise blend
// (1-s)*f/factor + s*f with s = (orig/wavelen - low)/(high - low).
// Evaluated in f64 on the f32 base frequencies, rounded to f32.
extern "C" int fb_rope_freqs_llama3(int head_dim, double theta, double factor, double low_freq_factor,
                                    double high_freq_factor, double original_max_position, float* out) {
    if (!(factor > 0.0) || !(low_freq_factor > 0.0) || !(high_freq_factor > low_freq_factor) ||
        !(original_max_position > 0.0))
        return (int)cudaErrorInvalidValue;
    int rc = fb_rope_freqs(head_dim, theta, out);
    if (rc) return rc;
    const double low_wavelen = original_max_position / low_freq_factor;
    const double high_wavelen = original_max_position / high_freq_factor;
    for (int i = 0; i < head_dim / 2; ++i) {
        const double f = (double)out[i];
        const double wavelen = 2.0 * M_PI / f;
        double r;
        if (wavelen < high_wavelen) {
            r = f;
        } else if (wavelen > low_wavelen) {
            r = f / factor;
        } else {
            const double sm = (original_max_position / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor);
            r = (1.0 - sm) * f / factor + sm * f;
        }
        out[i] = (float)r;
    }
    return 0;
}
