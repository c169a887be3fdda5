// Device helpers shared by the attention kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kattn {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x with the MUFU unit (PTX ex2.approx.ftz.f32).  ex2(-inf) = +0.
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Async 16-byte global->shared copy; src_bytes = 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Vector reduction into global memory (sm_90+): four f32 adds in one request.
__device__ __forceinline__ void red_add_v4(float* gptr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gptr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}
__device__ __forceinline__ void red_add_v2(float* gptr, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(gptr), "f"(a), "f"(b) : "memory");
}

// Programmatic dependent launch.  Every kernel of this library waits for the
// grid it was launched behind to finish (and its memory to be visible) before
// touching global memory, then lets the next grid start launching: that
// grid's CTAs take SM slots as this grid drains and wait there, instead of
// paying the launch latency after it.  Both are no-ops for a normal launch.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// The two halves of pdl_enter, for a kernel whose threads do not all read
// what the grid before it wrote: pdl_launch lets the next grid start
// launching; pdl_wait blocks the calling thread until the grid before has
// finished and its memory is visible.  A kernel that calls pdl_launch first
// reads global memory only after its own pdl_wait: the grid before it may
// itself still be waiting for its predecessor.  (attn_bwd_rowdot waits
// before it launches the next grid, whose K / V staging relies on that.)
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Reductions over the 16 lanes that share a row (lane bits 0..3).
__device__ __forceinline__ float max16(float x) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}
__device__ __forceinline__ float sum16(float x) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// A row fragment of DC consecutive floats (DC = 2, 4 or 8) held in registers.
template <int DC>
struct Frag {
    float x[DC];
    __device__ __forceinline__ void load(const float* p) {
        if constexpr (DC == 2) {
            const float2 t = *reinterpret_cast<const float2*>(p);
            x[0] = t.x; x[1] = t.y;
        } else {
#pragma unroll
            for (int i = 0; i < DC; i += 4) {
                const float4 t = *reinterpret_cast<const float4*>(p + i);
                x[i] = t.x; x[i + 1] = t.y; x[i + 2] = t.z; x[i + 3] = t.w;
            }
        }
    }
    __device__ __forceinline__ void store(float* p) const {
        if constexpr (DC == 2) {
            *reinterpret_cast<float2*>(p) = make_float2(x[0], x[1]);
        } else {
#pragma unroll
            for (int i = 0; i < DC; i += 4)
                *reinterpret_cast<float4*>(p + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
        }
    }
    __device__ __forceinline__ void red_add(float* p) const {
        if constexpr (DC == 2) {
            red_add_v2(p, x[0], x[1]);
        } else {
#pragma unroll
            for (int i = 0; i < DC; i += 4) red_add_v4(p + i, x[i], x[i + 1], x[i + 2], x[i + 3]);
        }
    }
};

}  // namespace kattn
