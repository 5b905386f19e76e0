// Single-token selective state update (decode) for sm_100a.
//
// Replaces the reference update kernel (nmquan1503/ssm-mamba, csrc/selective_update/kernel.cu:17-91):
// h' = exp(dt*A)*h + dt*x*B, out = sum_n C*h' + D*x, dt = softplus(dt + dt_bias).
// The reference runs one 32-thread CTA per (batch, channel) with one state per thread, half
// the lanes idle for d_state = 16, scalar loads, a CUB block reduction and a freshly
// allocated output state.  Here a thread owns SPT consecutive states of one (batch,
// channel) row, reads and writes them with 128-bit accesses (in place when state_out ==
// state), the LPC lanes of a row reduce C*h' with shuffles, and a 256-thread CTA covers
// 256/LPC consecutive rows, so a warp moves contiguous 512-byte state segments.  The gate
// out *= silu(z) and the optional softplus are fused.
#include "common.cuh"
#include "params.h"
#include "warp_reduce.cuh"

namespace ssm {

// SPT consecutive states of one row, as float (f32: 16-byte loads, bf16: 8-byte loads)
template <typename IT, int SPT>
__device__ __forceinline__ void load_row_vec(const IT* src, float (&v)[SPT]) {
#pragma unroll
    for (int s4 = 0; s4 < SPT; s4 += 4) {
        float q[4];
        Vec4<IT>::load(src + s4, q);
        v[s4] = q[0]; v[s4 + 1] = q[1]; v[s4 + 2] = q[2]; v[s4 + 3] = q[3];
    }
}

template <typename IT, int LPC, int SPT>
__global__ void __launch_bounds__(256) state_update_kernel(const __grid_constant__ UpdParams p) {
    // grid: x = batch rows, y = channel tiles of 256/LPC channels (consecutive CTAs share a
    // channel tile, so its A rows are reused from L2 / L1); no integer division
    constexpr int RPB = 256 / LPC;
    const int g = threadIdx.x % LPC;
    const int d = blockIdx.y * RPB + threadIdx.x / LPC;
    const int b = blockIdx.x;
    // lanes past the last channel still take part in the shuffles, with their work masked off
    const bool live = d < p.dim;
    const int dd = live ? d : 0;
    const int N = p.dstate;
    const int n0 = g * SPT;

    const float* hin = p.state + (int64_t)b * p.st_sb + (int64_t)dd * p.st_sd + n0;
    float* hout = p.state_out + (int64_t)b * p.so_sb + (int64_t)dd * p.so_sd + n0;
    const float* Ar = p.A + (int64_t)dd * p.A_sd + n0;
    const IT* Br = static_cast<const IT*>(p.B) + (int64_t)b * p.B_sb + n0;
    const IT* Cr = static_cast<const IT*>(p.C) + (int64_t)b * p.C_sb + n0;

    // With programmatic dependent launch this grid may start while the previous kernel in
    // the stream finishes: only an L2 prefetch of the state (its largest input) happens
    // before the dependency wait; then the next grid is allowed to start launching.
    if (live) prefetch_l2(hin);
    griddep_wait();
    griddep_launch_dependents();

    // issue every load before any arithmetic
    float h[SPT], a[SPT], bv[SPT], cv[SPT];
    const bool full = live && (n0 + SPT <= N);
    const bool vec = full && ((reinterpret_cast<uintptr_t>(hin) | reinterpret_cast<uintptr_t>(hout) |
                               reinterpret_cast<uintptr_t>(Ar)) & 15u) == 0 &&
                     ((reinterpret_cast<uintptr_t>(Br) | reinterpret_cast<uintptr_t>(Cr)) & (4 * sizeof(IT) - 1)) == 0;
    if (vec) {
#pragma unroll
        for (int s4 = 0; s4 < SPT; s4 += 4) {
            const float4 hv = *reinterpret_cast<const float4*>(hin + s4);
            const float4 av = __ldg(reinterpret_cast<const float4*>(Ar + s4));
            h[s4] = hv.x; h[s4 + 1] = hv.y; h[s4 + 2] = hv.z; h[s4 + 3] = hv.w;
            a[s4] = av.x; a[s4 + 1] = av.y; a[s4 + 2] = av.z; a[s4 + 3] = av.w;
        }
        load_row_vec<IT, SPT>(Br, bv);
        load_row_vec<IT, SPT>(Cr, cv);
    } else {
#pragma unroll
        for (int s = 0; s < SPT; s++) {
            const bool ok = live && n0 + s < N;
            h[s] = ok ? hin[s] : 0.f;
            a[s] = ok ? Ar[s] : 0.f;
            bv[s] = ok ? to_f(__ldg(Br + s)) : 0.f;
            cv[s] = ok ? to_f(__ldg(Cr + s)) : 0.f;
        }
    }
    float xv = 0.f, dtv = 0.f, zv = 0.f, bias = 0.f, Dv = 0.f;
    if (live) {
        xv = to_f(static_cast<const IT*>(p.x)[(int64_t)b * p.x_sb + dd]);
        dtv = to_f(static_cast<const IT*>(p.dtv)[(int64_t)b * p.dt_sb + dd]);
        if (p.z) zv = to_f(static_cast<const IT*>(p.z)[(int64_t)b * p.z_sb + dd]);
        if (p.dt_bias) bias = __ldg(p.dt_bias + dd);
        if (p.D) Dv = __ldg(p.D + dd);
    }
    const float x = dtv + bias;
    const float dl = p.dt_softplus ? softplus_series(x) : x;
    const float dx = dl * xv;
    const float dl2 = dl * kLog2e;

    float y = 0.f;
#pragma unroll
    for (int s = 0; s < SPT; s++) {
        h[s] = fmaf(ex2(dl2 * a[s]), h[s], dx * bv[s]);
        y = fmaf(cv[s], h[s], y);
    }
    y = allreduce<LPC>(y);

    if (vec) {
#pragma unroll
        for (int s4 = 0; s4 < SPT; s4 += 4)
            *reinterpret_cast<float4*>(hout + s4) = make_float4(h[s4], h[s4 + 1], h[s4 + 2], h[s4 + 3]);
    } else if (live) {
#pragma unroll
        for (int s = 0; s < SPT; s++)
            if (n0 + s < N) hout[s] = h[s];
    }
    if (live && g == 0) {
        float o = fmaf(Dv, xv, y);
        if (p.z) o = o * zv * sigmoid_io<IT>(zv);
        static_cast<IT*>(p.out)[(int64_t)b * p.out_sb + dd] = from_f<IT>(o);
    }
}

template <typename IT, int LPC, int SPT>
static cudaError_t launch_upd_t(const UpdParams& p, cudaStream_t stream) {
    constexpr int RPB = 256 / LPC;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)p.batch, (unsigned)((p.dim + RPB - 1) / RPB));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, state_update_kernel<IT, LPC, SPT>, p);
}

cudaError_t launch_state_update(const UpdParams& p, int is_bf16, int lpc, int spt, cudaStream_t stream) {
#define SSM_UPD_CASE(LPC_, SPT_)                                                  \
    if (lpc == LPC_ && spt == SPT_) {                                             \
        return is_bf16 ? launch_upd_t<__nv_bfloat16, LPC_, SPT_>(p, stream)       \
                       : launch_upd_t<float, LPC_, SPT_>(p, stream);              \
    }
    SSM_UPD_CASE(1, 4)
    SSM_UPD_CASE(2, 4)
    SSM_UPD_CASE(4, 4)
    SSM_UPD_CASE(8, 4)
    SSM_UPD_CASE(16, 4)
    SSM_UPD_CASE(32, 8)
    SSM_UPD_CASE(1, 8)
    SSM_UPD_CASE(2, 8)
    SSM_UPD_CASE(4, 8)
    SSM_UPD_CASE(8, 8)
    SSM_UPD_CASE(16, 8)
    SSM_UPD_CASE(1, 16)
    SSM_UPD_CASE(2, 16)
    SSM_UPD_CASE(4, 16)
    SSM_UPD_CASE(8, 16)
#undef SSM_UPD_CASE
    return cudaErrorInvalidValue;
}

}  // namespace ssm
