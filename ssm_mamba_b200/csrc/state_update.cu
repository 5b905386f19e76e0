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

// ---------------------------------------------------------------------------------------
// Streamed variant for contiguous layouts: persistent CTAs walk work units (batch row b,
// tile of RPB = 256 / LPC channels).  A unit's inputs are contiguous runs -- the state and
// A tiles (RPB * N floats each), the x, dt, z runs (RPB elements), the B, C rows (N
// elements) and the dt_bias, D runs (RPB floats) -- that thread 0 brings into a two-stage
// shared-memory pipeline with 1-D bulk copies completing on an mbarrier, one unit ahead of
// the compute, so state loads stay in flight across units instead of waiting for new CTAs,
// and no global load sits between a unit's wait and its arithmetic.  Needs dim % RPB == 0,
// 16-byte aligned rows and N = 8 * LPC.
// ---------------------------------------------------------------------------------------
struct UpdStreamSmem {
    uint32_t state, A, x, dt, z, B, C, bias, D, stage, total;
};

__host__ __device__ inline UpdStreamSmem upd_stream_layout(int rpb, int n, int es, int has_z) {
    UpdStreamSmem L;
    uint32_t o = 0;
    auto take = [&](uint32_t bytes) { const uint32_t at = o; o += (bytes + 15u) & ~15u; return at; };
    L.state = take((uint32_t)rpb * n * 4u);
    L.A = take((uint32_t)rpb * n * 4u);
    L.x = take((uint32_t)rpb * es);
    L.dt = take((uint32_t)rpb * es);
    L.z = take(has_z ? (uint32_t)rpb * es : 0u);
    L.B = take((uint32_t)n * es);
    L.C = take((uint32_t)n * es);
    L.bias = take((uint32_t)rpb * 4u);   // dt_bias and D runs travel with the unit: a global load
    L.D = take((uint32_t)rpb * 4u);      // of them after the wait would serialise every unit
    L.stage = o;
    L.total = 2u * o + 16u;   // two stages, then two mbarriers
    return L;
}

template <typename IT, int LPC>
__global__ void __launch_bounds__(256) state_update_stream_kernel(const __grid_constant__ UpdParams p) {
    constexpr int SPT = 8, RPB = 256 / LPC, N = SPT * LPC, ES = sizeof(IT);
    extern __shared__ __align__(16) unsigned char smem[];
    const bool has_z = p.z != nullptr;
    const UpdStreamSmem L = upd_stream_layout(RPB, N, ES, has_z ? 1 : 0);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * L.stage);
    const int tid = threadIdx.x, c = tid / LPC, g = tid % LPC, n0 = g * SPT;
    const int ntile = p.dim / RPB;
    const int nunits = p.batch * ntile;
    const bool has_bias = p.dt_bias != nullptr, has_D = p.D != nullptr;
    const uint32_t unit_bytes = 2u * RPB * N * 4u + (has_z ? 3u : 2u) * RPB * ES + 2u * N * ES +
                                ((has_bias ? 1u : 0u) + (has_D ? 1u : 0u)) * RPB * 4u;

    auto issue = [&](int u, int st) {
        const int b = u / ntile, d0 = (u - b * ntile) * RPB;
        unsigned char* sm = smem + st * L.stage;
        mbar_arrive_expect_tx(&bar[st], unit_bytes);
        bulk_load(sm + L.state, p.state + (int64_t)b * p.st_sb + (int64_t)d0 * N, RPB * N * 4, &bar[st]);
        bulk_load(sm + L.A, p.A + (int64_t)d0 * N, RPB * N * 4, &bar[st]);
        bulk_load(sm + L.x, static_cast<const IT*>(p.x) + (int64_t)b * p.x_sb + d0, RPB * ES, &bar[st]);
        bulk_load(sm + L.dt, static_cast<const IT*>(p.dtv) + (int64_t)b * p.dt_sb + d0, RPB * ES, &bar[st]);
        if (has_z) bulk_load(sm + L.z, static_cast<const IT*>(p.z) + (int64_t)b * p.z_sb + d0, RPB * ES, &bar[st]);
        bulk_load(sm + L.B, static_cast<const IT*>(p.B) + (int64_t)b * p.B_sb, N * ES, &bar[st]);
        bulk_load(sm + L.C, static_cast<const IT*>(p.C) + (int64_t)b * p.C_sb, N * ES, &bar[st]);
        if (has_bias) bulk_load(sm + L.bias, p.dt_bias + d0, RPB * 4, &bar[st]);
        if (has_D) bulk_load(sm + L.D, p.D + d0, RPB * 4, &bar[st]);
    };

    // programmatic dependent launch: everything read below may come from the previous kernel
    griddep_wait();
    griddep_launch_dependents();
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int u0 = blockIdx.x, ustep = gridDim.x;
    if (tid == 0) {
        if (u0 < nunits) issue(u0, 0);
        if (u0 + ustep < nunits) issue(u0 + ustep, 1);
    }
    int i = 0;
    for (int u = u0; u < nunits; u += ustep, i++) {
        const int st = i & 1;
        const int ok = mbar_wait_bounded(&bar[st], (uint32_t)((i >> 1) & 1)) ? 1 : 0;
        if (__syncthreads_or(!ok)) {
            // leave with the error word set, after the other stage's copies (if any) land
            if (tid == 0) {
                atomicExch(p.err, kDevErrTmaTimeout);
                if (u + ustep < nunits) mbar_wait_bounded(&bar[st ^ 1], (uint32_t)(((i + 1) >> 1) & 1));
            }
            return;
        }
        const unsigned char* sm = smem + st * L.stage;
        const int b = u / ntile, d = (u - b * ntile) * RPB + c;
        float h[SPT], a[SPT], bv[SPT], cv[SPT];
#pragma unroll
        for (int s4 = 0; s4 < SPT; s4 += 4) {
            const float4 hq = lds128(sm + L.state + ((c * N + n0 + s4) << 2));
            const float4 aq = lds128(sm + L.A + ((c * N + n0 + s4) << 2));
            h[s4] = hq.x; h[s4 + 1] = hq.y; h[s4 + 2] = hq.z; h[s4 + 3] = hq.w;
            a[s4] = aq.x; a[s4 + 1] = aq.y; a[s4 + 2] = aq.z; a[s4 + 3] = aq.w;
            float q[4];
            Vec4<IT>::load(sm + L.B + (n0 + s4) * ES, q);
            bv[s4] = q[0]; bv[s4 + 1] = q[1]; bv[s4 + 2] = q[2]; bv[s4 + 3] = q[3];
            Vec4<IT>::load(sm + L.C + (n0 + s4) * ES, q);
            cv[s4] = q[0]; cv[s4 + 1] = q[1]; cv[s4 + 2] = q[2]; cv[s4 + 3] = q[3];
        }
        const float xv = to_f(*reinterpret_cast<const IT*>(sm + L.x + c * ES));
        const float dtv = to_f(*reinterpret_cast<const IT*>(sm + L.dt + c * ES));
        const float bias = has_bias ? *reinterpret_cast<const float*>(sm + L.bias + c * 4) : 0.f;
        const float x0 = dtv + bias;
        const float dl = p.dt_softplus ? softplus_series(x0) : x0;
        const float dx = dl * xv;
        const float dl2 = dl * kLog2e;
        float y = 0.f;
#pragma unroll
        for (int k = 0; k < SPT; k++) {
            h[k] = fmaf(ex2(dl2 * a[k]), h[k], dx * bv[k]);
            y = fmaf(cv[k], h[k], y);
        }
        y = allreduce<LPC>(y);
        float* ho = p.state_out + (int64_t)b * p.so_sb + (int64_t)d * p.so_sd + n0;
#pragma unroll
        for (int s4 = 0; s4 < SPT; s4 += 4)
            *reinterpret_cast<float4*>(ho + s4) = make_float4(h[s4], h[s4 + 1], h[s4 + 2], h[s4 + 3]);
        if (g == 0) {
            float o = fmaf(has_D ? *reinterpret_cast<const float*>(sm + L.D + c * 4) : 0.f, xv, y);
            if (has_z) {
                const float zv = to_f(*reinterpret_cast<const IT*>(sm + L.z + c * ES));
                o = o * zv * sigmoid_io<IT>(zv);
            }
            static_cast<IT*>(p.out)[(int64_t)b * p.out_sb + d] = from_f<IT>(o);
        }
        __syncthreads();   // stage st is free: refill it with the unit after next
        if (tid == 0 && u + 2 * ustep < nunits) issue(u + 2 * ustep, st);
    }
}

template <typename IT, int LPC>
static cudaError_t launch_upd_stream_t(const UpdParams& p, int sms, cudaStream_t stream) {
    constexpr int RPB = 256 / LPC, N = 8 * LPC;
    const UpdStreamSmem L = upd_stream_layout(RPB, N, sizeof(IT), p.z != nullptr);
    auto kern = state_update_stream_kernel<IT, LPC>;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, L.total) != cudaSuccess || occ < 1) occ = 1;
    const int nunits = p.batch * (p.dim / RPB);
    int grid = sms * occ;
    if (grid > nunits) grid = nunits;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

// The streamed decode kernel for (lpc, states per thread 8), or cudaErrorNotSupported.
cudaError_t launch_state_update_stream(const UpdParams& p, int is_bf16, int lpc, int sms, cudaStream_t stream) {
#define SSM_UPDS_CASE(LPC_)                                                                     \
    if (lpc == LPC_) {                                                                          \
        return is_bf16 ? launch_upd_stream_t<__nv_bfloat16, LPC_>(p, sms, stream)               \
                       : launch_upd_stream_t<float, LPC_>(p, sms, stream);                      \
    }
    SSM_UPDS_CASE(1)
    SSM_UPDS_CASE(2)
    SSM_UPDS_CASE(4)
#undef SSM_UPDS_CASE
    return cudaErrorNotSupported;
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
