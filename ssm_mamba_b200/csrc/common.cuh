// Device helpers shared by the sm_100a selective-scan kernels: element conversion,
// MUFU exp2, the 128-byte TMA swizzle, TMA tensor copies and mbarriers with bounded
// waits.  Everything here is written for sm_100a only.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ssm {

constexpr float kLog2e = 1.4426950408889634f;

// Error codes a kernel can leave in the device error word.
enum DeviceError : int {
    kDevErrNone = 0,
    kDevErrTmaTimeout = 1,   // an mbarrier wait for a TMA load ran out of time
    kDevErrSmemAlign = 2,    // dynamic shared memory base not 1024-byte aligned
};

// ---------------------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return Elem<T>::to_f(v); }
template <typename T> __device__ __forceinline__ T from_f(float v) { return Elem<T>::from_f(v); }

// 2^x on the MUFU pipe (PTX ex2.approx.ftz.f32; max relative error 2^-22 per the PTX ISA).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x of two values on the FMA pipe (packed f32x2), for kernels whose MUFU pipe is the
// bottleneck: a share of their exp2 is computed here instead of by ex2.approx.
//   x = j + f, j = rint(x) by adding and subtracting 1.5 * 2^23 (round-to-nearest), |f| <= 1/2
//   2^f ~ 1 + f (c1 + f (c2 + f (c3 + f (c4 + f c5)))), coefficients fitted here for minimax
//       relative error on [-1/2, 1/2] with the constant term held at 1 (so 2^0 = 1 exactly):
//       1.1e-7 in exact arithmetic, 1.6e-7 (2^-22.6) evaluated in float32 with fused
//       multiply-adds
//   2^j is joined by adding j to the exponent field (j sits in the low bits of the rounded
//       sum, so (bits << 23) is j << 23)
// x is first clamped to >= -126, so that the exponent stays in the normal range: inputs below
// -126 give about 2^-126 (ex2.approx.ftz gives 0 there); those decays multiply states that
// the kernels' flush-to-zero arithmetic then rounds away.  Inputs are <= 0 in the callers
// (decays exp(delta * A), A < 0); for x > 127 the result would overflow the exponent.
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
    x = make_float2(fmaxf(x.x, -126.f), fmaxf(x.y, -126.f));
    const float2 magic = make_float2(12582912.f, 12582912.f);   // 1.5 * 2^23
    const float2 t = __fadd2_rn(x, magic);
    const float2 j = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));   // exact
    const float2 f = __ffma2_rn(j, make_float2(-1.f, -1.f), x);               // exact, |f| <= 1/2
    float2 p = make_float2(0x1.5cb5a6p-10f, 0x1.5cb5a6p-10f);
    p = __ffma2_rn(p, f, make_float2(0x1.3cf672p-7f, 0x1.3cf672p-7f));
    p = __ffma2_rn(p, f, make_float2(0x1.c6b4d6p-5f, 0x1.c6b4d6p-5f));
    p = __ffma2_rn(p, f, make_float2(0x1.ebf99ap-3f, 0x1.ebf99ap-3f));
    p = __ffma2_rn(p, f, make_float2(0x1.62e42cp-1f, 0x1.62e42cp-1f));
    p = __ffma2_rn(p, f, make_float2(1.f, 1.f));
    return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                       __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// softplus with threshold 20, as the reference computes it
// (csrc/selective_scan/forward_kernel.cu:155-159, built with --use_fast_math).
__device__ __forceinline__ float softplus20(float x) {
    return x <= 20.f ? log1pf(__expf(x)) : x;
}

__device__ __forceinline__ float sigmoidf_fast(float x) {
    return __fdividef(1.f, 1.f + __expf(-x));
}

// MUFU tanh (PTX tanh.approx.f32: max relative error about 2^-11)
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// logistic sigmoid for bfloat16 results: sigma(x) = (1 + tanh(x / 2)) / 2, one MUFU op
// instead of two (exp and reciprocal); its ~2^-11 relative error is below bf16 rounding.
// Float results use sigmoidf_fast.
template <typename IT>
__device__ __forceinline__ float sigmoid_io(float x) {
    if constexpr (sizeof(IT) == 2) return fmaf(0.5f, tanh_approx(0.5f * x), 0.5f);
    else return sigmoidf_fast(x);
}

// sigmoid_io of two values, the multiplications and adds packed (same results per element)
template <typename IT>
__device__ __forceinline__ float2 sigmoid_io2(float2 x) {
    if constexpr (sizeof(IT) == 2) {
        const float2 h = __fmul2_rn(make_float2(0.5f, 0.5f), x);
        return __ffma2_rn(make_float2(0.5f, 0.5f), make_float2(tanh_approx(h.x), tanh_approx(h.y)),
                          make_float2(0.5f, 0.5f));
    } else {
        return make_float2(sigmoidf_fast(x.x), sigmoidf_fast(x.y));
    }
}

// log(1 + e^x) = max(x, 0) + log1p(t), t = e^-|x| in (0, 1], with log1p(t) = 2 atanh(s),
// s = t / (2 + t) in (0, 1/3], from the series 2 atanh(s) = 2 s (1 + s^2/3 + s^4/5 + ...).
// Truncated after s^12/13 the series error is below (1/3)^14/15 ~ 1.4e-8 relative; the
// MUFU exp2 and the fast division add ~3e-7.  For x > 20 the correction rounds away and
// the result is x, as in the reference's threshold.  `t_out` returns e^-|x| for reuse.
__device__ __forceinline__ float softplus_series(float x, float* t_out = nullptr) {
    const float t = ex2(-fabsf(x) * kLog2e);
    const float s = __fdividef(t, 2.f + t);
    const float s2 = s * s;
    float p = 1.f / 13.f;
    p = fmaf(p, s2, 1.f / 11.f);
    p = fmaf(p, s2, 1.f / 9.f);
    p = fmaf(p, s2, 1.f / 7.f);
    p = fmaf(p, s2, 1.f / 5.f);
    p = fmaf(p, s2, 1.f / 3.f);
    p = fmaf(p, s2, 1.f);
    if (t_out) *t_out = t;
    return fmaxf(x, 0.f) + 2.f * s * p;
}

// softplus_series of two values with packed f32x2 arithmetic: per element the same
// operations in the same order (2 s p = (2 s) p exactly), so the same results.
__device__ __forceinline__ float2 softplus_series2(float2 x, float2* t_out = nullptr) {
    const float2 t = make_float2(ex2(-fabsf(x.x) * kLog2e), ex2(-fabsf(x.y) * kLog2e));
    if (t_out) *t_out = t;
    const float2 s = make_float2(__fdividef(t.x, 2.f + t.x), __fdividef(t.y, 2.f + t.y));
    const float2 s2 = __fmul2_rn(s, s);
    float2 p = make_float2(1.f / 13.f, 1.f / 13.f);
    p = __ffma2_rn(p, s2, make_float2(1.f / 11.f, 1.f / 11.f));
    p = __ffma2_rn(p, s2, make_float2(1.f / 9.f, 1.f / 9.f));
    p = __ffma2_rn(p, s2, make_float2(1.f / 7.f, 1.f / 7.f));
    p = __ffma2_rn(p, s2, make_float2(1.f / 5.f, 1.f / 5.f));
    p = __ffma2_rn(p, s2, make_float2(1.f / 3.f, 1.f / 3.f));
    p = __ffma2_rn(p, s2, make_float2(1.f, 1.f));
    const float2 sp = __fmul2_rn(__fmul2_rn(make_float2(2.f, 2.f), s), p);
    return __fadd2_rn(make_float2(fmaxf(x.x, 0.f), fmaxf(x.y, 0.f)), sp);
}

// logistic sigmoid from t = e^-|x| (as returned by softplus_series)
__device__ __forceinline__ float sigmoid_from_t(float x, float t) {
    const float r = __fdividef(1.f, 1.f + t);
    return x >= 0.f ? r : t * r;
}

// The SPT consecutive states a lane owns at token t of a float32 [T][NS] B/C row whose
// float4 groups are XOR-swizzled by `sw` (group q of row t sits at position q ^ sw), as
// SPT/2 packed pairs.  SPT = 2 reads half of a group, SPT >= 4 whole groups.
template <int SPT, int NS>
__device__ __forceinline__ void load_state_pairs(const float* rows, int t, int g, int sw,
                                                 float2 (&out)[SPT / 2]) {
    if constexpr (SPT == 2) {
        const int pos = t * NS + (((g >> 1) ^ sw) << 2) + ((g & 1) << 1);
        out[0] = *reinterpret_cast<const float2*>(rows + pos);
    } else {
#pragma unroll
        for (int s4 = 0; s4 < SPT / 4; s4++) {
            const int qq = g * (SPT / 4) + s4;
            const float4 v = *reinterpret_cast<const float4*>(rows + t * NS + ((qq ^ sw) << 2));
            out[2 * s4] = make_float2(v.x, v.y);
            out[2 * s4 + 1] = make_float2(v.z, v.w);
        }
    }
}

// two consecutive elements from a float2 (one 4- or 8-byte shared-memory store)
template <typename T> __device__ __forceinline__ void store_pair(void* p, float2 v);
template <> __device__ __forceinline__ void store_pair<float>(void* p, float2 v) {
    *reinterpret_cast<float2*>(p) = v;
}
template <> __device__ __forceinline__ void store_pair<__nv_bfloat16>(void* p, float2 v) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(v.x, v.y);
}

// Global stores of 4, 2 or 1 floats issued as ONE predicated instruction: no branch, so the
// code around them stays one straight-line block the compiler can schedule across.  For
// write-only buffers the kernel never reads back (no ordering against its own loads).
__device__ __forceinline__ void stg_f32x4_if(float* p, float a, float b, float c, float d, bool on) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t@q st.global.v4.f32 [%0], {%1, %2, %3, %4};\n\t}"
                 :: "l"(p), "f"(a), "f"(b), "f"(c), "f"(d), "r"((int)on));
}
__device__ __forceinline__ void stg_f32x2_if(float* p, float a, float b, bool on) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %3, 0;\n\t@q st.global.v2.f32 [%0], {%1, %2};\n\t}"
                 :: "l"(p), "f"(a), "f"(b), "r"((int)on));
}
__device__ __forceinline__ void stg_f32_if(float* p, float a, bool on) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t@q st.global.f32 [%0], %1;\n\t}"
                 :: "l"(p), "f"(a), "r"((int)on));
}

// Programmatic dependent launch (sm_90+): wait until the preceding grid in the stream has
// completed and its writes are visible (a no-op when this grid was launched without the
// programmatic-serialization attribute), and let the next grid start launching.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// L2 prefetch hint; L2 is the point of coherence, so a prefetched line is never stale
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

// two consecutive elements as float2 (from 4 or 8 bytes of shared memory)
template <typename T> __device__ __forceinline__ float2 load_pair(const void* p);
template <> __device__ __forceinline__ float2 load_pair<float>(const void* p) {
    return *reinterpret_cast<const float2*>(p);
}
template <> __device__ __forceinline__ float2 load_pair<__nv_bfloat16>(const void* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

// four consecutive elements as float (from 8 or 16 bytes of shared memory)
template <typename T> struct Vec4;
template <> struct Vec4<float> {
    static __device__ __forceinline__ void load(const void* p, float (&v)[4]) {
        const float4 x = *reinterpret_cast<const float4*>(p);
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    }
    static __device__ __forceinline__ void store(void* p, const float (&v)[4]) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <> struct Vec4<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const void* p, float (&v)[4]) {
        const uint2 x = *reinterpret_cast<const uint2*>(p);
        v[0] = __uint_as_float(x.x << 16); v[1] = __uint_as_float(x.x & 0xffff0000u);
        v[2] = __uint_as_float(x.y << 16); v[3] = __uint_as_float(x.y & 0xffff0000u);
    }
    static __device__ __forceinline__ void store(void* p, const float (&v)[4]) {
        const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
        uint2 x;
        x.x = *reinterpret_cast<const uint32_t*>(&a);
        x.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(p) = x;
    }
};

// ---------------------------------------------------------------------------------------
// 128-byte swizzle (CU_TENSOR_MAP_SWIZZLE_128B): inside each 1024-byte block of eight
// 128-byte rows, 16-byte chunk j of row r sits at chunk position j ^ (r & 7).  Tiles whose
// rows are exactly 128 bytes use it so that column-wise accesses by consecutive rows hit
// distinct banks.  Returns a byte offset.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t byte_in_row) {
    return row * 128u + ((((byte_in_row >> 4) ^ row) & 7u) << 4) + (byte_in_row & 15u);
}

// 32-byte swizzle (CU_TENSOR_MAP_SWIZZLE_32B) for 32-byte rows: 16-byte chunk j of row r
// sits at chunk position j ^ ((r >> 2) & 1) (address bit 4 ^= bit 7).
__device__ __forceinline__ uint32_t swz32(uint32_t row, uint32_t byte_in_row) {
    return row * 32u + ((((byte_in_row >> 4) ^ (row >> 2)) & 1u) << 4) + (byte_in_row & 15u);
}

// 64-byte swizzle (CU_TENSOR_MAP_SWIZZLE_64B) for 64-byte rows: 16-byte chunk j of row r
// sits at chunk position j ^ ((r >> 1) & 3) (address bits [4:5] ^= bits [7:8]).
__device__ __forceinline__ uint32_t swz64(uint32_t row, uint32_t byte_in_row) {
    return row * 64u + ((((byte_in_row >> 4) ^ (row >> 1)) & 3u) << 4) + (byte_in_row & 15u);
}

// ---------------------------------------------------------------------------------------
// shared-memory address helpers, mbarrier, TMA
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait: gives up after roughly `limit_cycles` SM clocks (about 1 s by default)
// and returns false, so that a lost copy turns into an error code instead of a hang.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit_cycles = 2000000000LL) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - start > limit_cycles) return false;
    }
    return true;
}

// Make generic-proxy writes to shared memory visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 3-D tiled TMA load, global -> shared, completion counted on `bar` (no multicast).
// 1-D bulk copy global -> shared completing on an mbarrier (both addresses 16-byte aligned,
// bytes a multiple of 16); no multicast
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}

// 4-D tiled TMA load, global -> shared, completion counted on `bar` (no multicast).
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

// 3-D tiled TMA store, shared -> global (out-of-range parts of the box are not written).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed TMA store has finished reading shared memory.
__device__ __forceinline__ void tma_store_wait_read_all() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until every committed TMA store is complete (writes visible in global memory).
__device__ __forceinline__ void tma_store_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ float4 lds128(const void* p) {
    return *reinterpret_cast<const float4*>(p);
}

}  // namespace ssm
