// Shared device helpers for the fracture_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <utility>

#include "fracture_b200.h"

namespace fb {

// Storage types. The enum values are the reference's DType order
// (crates/fracture-core/src/dtype.rs:5-11): FP16, FP32, BF16, INT8, INT4.
template <typename T> struct dtype_of;
template <> struct dtype_of<__half> { static constexpr int value = FB_FP16; };
template <> struct dtype_of<float> { static constexpr int value = FB_FP32; };
template <> struct dtype_of<__nv_bfloat16> { static constexpr int value = FB_BF16; };

__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(float x) { return x; }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }

// A 16-byte vector of storage elements, the unit of every HBM access in the
// streaming kernels (one 128-bit load/store per thread per step).
template <typename T> struct Vec16 {
    static constexpr int N = 16 / sizeof(T);
    union {
        uint4 u;
        T e[N];
    };
};

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint4 ld_keep(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Plain coherent load (for buffers the same kernel also writes, e.g. in-place rope).
__device__ __forceinline__ uint4 ld_rw(const void* p) {
    uint4 v;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void st_plain(void* p, uint4 v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// First statement of a kernel that launch_pdl may start early: waits until the previous kernel
// on the stream has completed and its writes are visible (a no-op for an ordinary launch). The
// elementwise kernels do not trigger their dependents early: they are scheduled as its CTAs exit,
// which measured faster under CUDA-graph replay than an early trigger (0.293 vs 0.368 ms for the
// 130-launch decode chain); the TurboQuant attention chain does (pdl_trigger below).
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next programmatic dependent launch on the stream be scheduled before this kernel's CTAs
// exit (its CTAs then take SMs as they free up and run up to their own pdl_begin()). Used by the
// TurboQuant attention chain, whose kernels do set-up that needs no predecessor output.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host-side helpers ----------------------------------------------------------

int num_sms();  // SM count of the current device (cached per device)

// Library-owned device workspace for the reference-ABI entry points that take none: one buffer per
// (device, stream), grown to the largest call on that stream and kept until exit. Calls on one
// stream run in order and share it; calls on different streams get different buffers, so they
// may overlap on the GPU. Growing frees the old buffer (cudaFree waits for the device first).
struct StreamWorkspace {
    void* ptr = nullptr;
    size_t cap = 0;
};
std::mutex& stream_workspace_mutex();
StreamWorkspace& stream_workspace(int device, const void* stream);  // with the mutex held

// Runs enqueue(ptr) with a workspace of at least `need` bytes for the current device and
// `stream`, holding the lock so that no other call regrows that buffer before the work is queued.
template <typename F>
int with_stream_workspace(const void* stream, size_t need, F&& enqueue) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    std::lock_guard<std::mutex> g(stream_workspace_mutex());
    StreamWorkspace& w = stream_workspace(dev, stream);
    if (w.cap < need) {
        if (w.ptr) {
            e = cudaFree(w.ptr);
            if (e != cudaSuccess) return (int)e;
        }
        w.ptr = nullptr;
        w.cap = 0;
        e = cudaMalloc(&w.ptr, need);
        if (e != cudaSuccess) return (int)e;
        w.cap = need;
    }
    return enqueue(w.ptr);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch for small grids (decode-sized calls, where launch latency is the
// cost): the kernel may be scheduled while the previous kernel on the stream is still running,
// and waits for it (with its memory visible) in pdl_begin() before touching memory. Grids of
// more than two CTAs per SM launch normally, so waiting CTAs never hold slots a large kernel
// still needs. Launch errors are left for cudaGetLastError(), as with <<<>>>.
template <typename... KArgs, typename... Args>
inline void launch_pdl_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    const uint64_t blocks = (uint64_t)grid.x * grid.y * grid.z;
    cfg.attrs = &attr;
    cfg.numAttrs = blocks <= 2ull * (uint64_t)num_sms() ? 1 : 0;
    (void)cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args&&... args) {
    launch_pdl_smem(kern, grid, block, 0, s, std::forward<Args>(args)...);
}

inline int dtype_size(int dt) {
    switch (dt) {
        case FB_FP16: return 2;
        case FB_BF16: return 2;
        case FB_FP32: return 4;
        case FB_INT8: return 1;
        default: return 0;
    }
}

}  // namespace fb

// Dispatch on the floating storage dtype; `body` sees a type alias `T`.
#define FB_DISPATCH_FLOAT(dt, ...)                                   \
    [&]() -> int {                                                   \
        switch (dt) {                                                \
            case FB_FP16: { using T = __half; __VA_ARGS__ }          \
            case FB_BF16: { using T = __nv_bfloat16; __VA_ARGS__ }   \
            case FB_FP32: { using T = float; __VA_ARGS__ }           \
            default: return (int)cudaErrorInvalidValue;              \
        }                                                            \
    }()
