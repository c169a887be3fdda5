// Global f32 rows -> bf16 hi/lo operand tiles for the tcgen05 kernels.
#pragma once

#include "sm100.cuh"

namespace kattn {
namespace tc {

// Two tiles of the same shape (e.g. Q and dO, or K and V) held in registers
// between their loads and their conversion, so the loads can be issued early
// and the shared-memory stores made once the destination is free.  Rows of
// W floats (64: bf16 rows of 128 bytes, 128B-swizzled; 32: rows of 64 bytes,
// 64B-swizzled); thread t handles (row, 8-float chunk) items t, t + NTH, ...
template <int R, int NTH, int W = 64>
struct Rows2 {
    static_assert(W == 64 || W == 32, "rows of 64 or 32 floats");
    static constexpr int CH = W / 8;  // 8-float chunks per row
    static_assert((R * CH) % NTH == 0, "tile items must divide evenly");
    static constexpr int ITEMS = R * CH / NTH;
    float4 a[2][ITEMS], b[2][ITEMS];

    __device__ __forceinline__ static uint32_t offset(int r, int ch) {
        if constexpr (W == 64) return sm100::sw128(r, ch);
        else return sm100::sw64(r, ch);
    }

    // V8: every row start is 32-byte aligned (base pointers and row strides),
    // so each 8-float chunk is one 256-bit load instead of two 128-bit ones.
    template <bool V8 = false>
    __device__ __forceinline__ void load(const float* g0, long ld0, const float* g1, long ld1, int row0, int T,
                                         int t) {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int i = t + it * NTH;
            const int r = i / CH;
            const int ch = i % CH;
            a[0][it] = make_float4(0.f, 0.f, 0.f, 0.f);
            b[0][it] = a[0][it];
            a[1][it] = a[0][it];
            b[1][it] = a[0][it];
            if (row0 + r < T) {
                const float* f0 = g0 + static_cast<long>(row0 + r) * ld0 + ch * 8;
                const float* f1 = g1 + static_cast<long>(row0 + r) * ld1 + ch * 8;
                if constexpr (V8) {
                    sm100::ldg_v8(f0, a[0][it], b[0][it]);
                    sm100::ldg_v8(f1, a[1][it], b[1][it]);
                } else {
                    const float4* s0 = reinterpret_cast<const float4*>(f0);
                    const float4* s1 = reinterpret_cast<const float4*>(f1);
                    a[0][it] = __ldg(s0);
                    b[0][it] = __ldg(s0 + 1);
                    a[1][it] = __ldg(s1);
                    b[1][it] = __ldg(s1 + 1);
                }
            }
        }
    }

    __device__ __forceinline__ void store(uint8_t* hi0, uint8_t* lo0, uint8_t* hi1, uint8_t* lo1, int t) const {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            uint8_t* hi = u ? hi1 : hi0;
            uint8_t* lo = u ? lo1 : lo0;
#pragma unroll
            for (int it = 0; it < ITEMS; ++it) {
                const int i = t + it * NTH;
                const int r = i / CH;
                const int ch = i % CH;
                uint4 h, l;
                sm100::split2(a[u][it].x, a[u][it].y, h.x, l.x);
                sm100::split2(a[u][it].z, a[u][it].w, h.y, l.y);
                sm100::split2(b[u][it].x, b[u][it].y, h.z, l.z);
                sm100::split2(b[u][it].z, b[u][it].w, h.w, l.w);
                const uint32_t off = offset(r, ch);
                *reinterpret_cast<uint4*>(hi + off) = h;
                *reinterpret_cast<uint4*>(lo + off) = l;
            }
        }
    }
};

// Two tiles of the same shape in one pass: all loads of both are in flight
// before the first conversion.
template <int R, int NTH, bool V8 = false, int W = 64>
__device__ __forceinline__ void stage_rows2(uint8_t* hi0, uint8_t* lo0, const float* g0, long ld0, uint8_t* hi1,
                                            uint8_t* lo1, const float* g1, long ld1, int row0, int T, int t) {
    Rows2<R, NTH, W> x;
    x.template load<V8>(g0, ld0, g1, ld1, row0, T, t);
    x.store(hi0, lo0, hi1, lo1, t);
}

// A raw f32 tile of R rows x 64 floats as a TMA box lands it (row-major,
// 256 bytes per row) -> the same bytes rewritten as bf16 hi (first R*128
// bytes) and lo (next R*128 bytes) in the 128B-swizzled layout, scaled by
// `mul`.  read() stages the thread's share in registers; the caller makes
// every thread's read() complete (a barrier over the NTH threads) before any
// write(), because the tile is converted in place.  Thread `t` of NTH handles
// float4 f = t, t + NTH, ... (row f/16, columns 4(f%16)..+3), so each group
// of eight threads reads 128 contiguous bytes and no read conflicts.
template <int R, int NTH>
struct RawTile {
    static_assert((R * 16) % NTH == 0, "tile items must divide evenly");
    static constexpr int ITEMS = R * 16 / NTH;
    float4 a[ITEMS];

    __device__ __forceinline__ void read(const uint8_t* tile, int t) {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) a[it] = reinterpret_cast<const float4*>(tile)[t + it * NTH];
    }

    __device__ __forceinline__ void write(uint8_t* tile, float mul, int t) const {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int f = t + it * NTH;
            const int r = f >> 4, c4 = f & 15;
            uint2 h, l;
            sm100::split2_x2(a[it].x * mul, a[it].y * mul, h.x, l.x);
            sm100::split2_x2(a[it].z * mul, a[it].w * mul, h.y, l.y);
            const uint32_t off = sm100::sw128(r, c4 >> 1) + (c4 & 1) * 8;
            *reinterpret_cast<uint2*>(tile + off) = h;
            *reinterpret_cast<uint2*>(tile + R * 128 + off) = l;
        }
    }
};

// A raw f32 tile of R rows x 32 floats (128 bytes per row, as a TMA box
// lands it) -> the same bytes rewritten as bf16 hi (first R*64 bytes) and lo
// (next R*64 bytes) in the 64B-swizzled UMMA layout (the forward at head_dim
// 32: K-major K, MN-major V), scaled by `mul`.  Same read / barrier / write
// protocol as RawTile; thread t handles float4 f = t, t + NTH, ... (row f/8,
// columns 4(f%8)..+3).
template <int R, int NTH>
struct RawTile32 {
    static_assert((R * 8) % NTH == 0, "tile items must divide evenly");
    static constexpr int ITEMS = R * 8 / NTH;
    float4 a[ITEMS];

    __device__ __forceinline__ void read(const uint8_t* tile, int t) {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) a[it] = reinterpret_cast<const float4*>(tile)[t + it * NTH];
    }

    __device__ __forceinline__ void write(uint8_t* tile, float mul, int t) const {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int f = t + it * NTH;
            const int r = f >> 3, c4 = f & 7;
            uint2 h, l;
            sm100::split2_x2(a[it].x * mul, a[it].y * mul, h.x, l.x);
            sm100::split2_x2(a[it].z * mul, a[it].w * mul, h.y, l.y);
            const uint32_t off = sm100::sw64(r, c4 >> 1) + (c4 & 1) * 8;
            *reinterpret_cast<uint2*>(tile + off) = h;
            *reinterpret_cast<uint2*>(tile + R * 64 + off) = l;
        }
    }
};

}  // namespace tc
}  // namespace kattn
