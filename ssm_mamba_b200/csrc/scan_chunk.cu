// Sequence-slice carries: the pieces that let one long sequence be scanned as independent
// slices (segments of one GPU's sequence, or the slices held by the ranks of a
// sequence-parallel group).  No reference counterpart: the reference scans each sequence
// serially in 128-token chunks inside one CTA (forward_kernel.cu:208-228).
//
// The recurrence h_t = a_t h_{t-1} + b_t (a_t = exp(delta_t A), b_t = delta_t u_t B_t) is
// linear in the state, so a slice q started from h_in(q) ends in
//     h_end(q) = P_q h_in(q) + h0_end(q),   P_q = prod_t a_t = exp(A * sum_t delta_t),
// where h0_end(q) is the slice's end state from a zero start.  Symmetrically, the gradient a
// slice sends back to the state before it is g0_start(q) + P_q g_out(q), where g0_start(q)
// is its dh_init computed with a zero incoming gradient.  So:
//
//   scan_chunk_kernel<.., REV = false>  h0_end and sum(delta) of every slice (one exp2 and
//                                       one FMA per token and state; no C, no outputs)
//   scan_chunk_kernel<.., REV = true>   g0_start of every slice: the reverse recurrence
//                                       dh_t = a_{t+1} dh_{t+1} + C_t dy_t from zero,
//                                       dy = dout * silu(z) with a gate
//   carry_compose_kernel                folds those per-slice carries in slice order
//                                       (forward) or reverse order (backward)
//
// after which every slice runs the ordinary forward / backward with its own h_init /
// dh_last.  Layout and thread mapping follow the forward scan kernel: a CTA owns (slice
// row, dt channels), a thread owns one channel and SPT states, tiles of 128 bytes per row
// arrive by 3-D TMA loads (128-byte swizzle, two stages) and are expanded to f32 work rows.
#include "common.cuh"
#include "params.h"
#include "scan_layout.h"

namespace ssm {

// With every exp2 on the MUFU pipe (one per token and state) the carry passes are bound by the
// queue that feeds MUFU and shared-memory instructions (XU ~83% busy, FMA ~40%): of every 4
// (token, state pair) exp2 pairs, kChunkExpOnFma are computed on the FMA pipe by exp2_fma2
// (common.cuh) instead of by ex2.approx.  Measured on B200 at config 5's segment shape: a
// quarter is the best share (issue, MUFU and FMA then 60-70% busy each); a half is slower.
constexpr int kChunkExpOnFma = 1;

__device__ __forceinline__ uint32_t chunk_stage(const uint32_t (&a)[2], int st) { return st ? a[1] : a[0]; }

template <typename IT, int LPC, int SPT, bool REV>
__global__ void __launch_bounds__(128, 4) scan_chunk_kernel(const __grid_constant__ ChunkParams p,
                                                            const __grid_constant__ CUtensorMap tm_x0,
                                                            const __grid_constant__ CUtensorMap tm_delta,
                                                            const __grid_constant__ CUtensorMap tm_z,
                                                            const __grid_constant__ CUtensorMap tm_bc) {
    constexpr int ES = sizeof(IT);
    constexpr int T = 128 / ES;              // tokens per tile
    constexpr int NS = LPC * SPT;            // padded state count
    constexpr int NP = SPT / 2;
    constexpr int Q = NS / 4;
    constexpr int QM = (Q < 8 ? Q : 8) - 1;
    constexpr int RS = T + 4;
    constexpr int G = 16;                    // tokens per unrolled group
    static_assert(T % G == 0 && (SPT == 2 || SPT % 4 == 0), "tile must hold whole groups");

    extern __shared__ __align__(1024) unsigned char smem[];
    if ((smem_u32(smem) & 1023u) != 0u) {
        if (threadIdx.x == 0) atomicExch(p.err, kDevErrSmemAlign);
        return;
    }
    const int DT = p.dt;
    const bool has_z = REV && p.z != nullptr;
    const ChunkSmem L = chunk_smem_layout(DT, NS, ES, has_z ? 1 : 0);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    float* sD = reinterpret_cast<float*>(smem + L.sD);
    float* sX = reinterpret_cast<float*>(smem + L.sX);
    float* sM = reinterpret_cast<float*>(smem + L.sM);
    float* sBias = reinterpret_cast<float*>(smem + L.bias);

    const int tid = threadIdx.x;
    const int nthr = DT * LPC;
    const int c = tid / LPC, g = tid % LPC;
    const int b = blockIdx.x / p.ntile_d;
    const int d0 = (blockIdx.x % p.ntile_d) * DT;
    const int d = d0 + c;
    const bool dvalid = d < p.dim;
    const int N = p.dstate, Lq = p.seqlen;
    const int ntiles = (Lq + T - 1) / T;

    float2 A2[NP], h[NP], an[NP];
#pragma unroll
    for (int s = 0; s < SPT; s++) {
        const int n = g * SPT + s;
        const float a = (dvalid && n < N) ? p.A[(int64_t)d * p.A_sd + n] * kLog2e : 0.f;
        if (s & 1) A2[s / 2].y = a; else A2[s / 2].x = a;
    }
#pragma unroll
    for (int q = 0; q < NP; q++) {
        h[q] = make_float2(0.f, 0.f);
        an[q] = make_float2(1.f, 1.f);   // reverse: decay of the token after the current one
    }
    float Ssum = 0.f;
    for (int i = tid; i < DT; i += nthr)
        sBias[i] = (d0 + i < p.dim && p.delta_bias) ? p.delta_bias[d0 + i] : 0.f;

    const uint32_t tile_bytes = (uint32_t)DT * 128u;
    const uint32_t stage_bytes = (has_z ? 3u : 2u) * tile_bytes + (uint32_t)N * 128u;

    // j-th tile in processing order: ascending (forward) or descending (reverse)
    auto tile_of = [&](int j) { return REV ? ntiles - 1 - j : j; };

    auto issue = [&](int j, int st) {
        const int t0 = tile_of(j) * T;
        mbar_arrive_expect_tx(&bar[st], stage_bytes);
        tma_load_3d(smem + chunk_stage(L.x0, st), &tm_x0, &bar[st], t0, d0, b);
        tma_load_3d(smem + chunk_stage(L.x1, st), &tm_delta, &bar[st], t0, d0, b);
        if (has_z) tma_load_3d(smem + chunk_stage(L.x2, st), &tm_z, &bar[st], t0, d0, b);
        tma_load_3d(smem + chunk_stage(L.x3, st), &tm_bc, &bar[st], t0, 0, b);
    };

    auto load_plain = [&](int j, int st) {
        const int t0 = tile_of(j) * T;
        const IT zero = from_f<IT>(0.f);
        for (int i = tid; i < DT * T; i += nthr) {
            const int cc = i / T, tt = i % T, dd = d0 + cc, tg = t0 + tt;
            const bool in = dd < p.dim && tg < Lq;
            const uint32_t off = swz128(cc, tt * ES);
            *reinterpret_cast<IT*>(smem + chunk_stage(L.x0, st) + off) =
                in ? static_cast<const IT*>(p.x0)[b * p.x0_sb + dd * p.x0_sd + tg] : zero;
            *reinterpret_cast<IT*>(smem + chunk_stage(L.x1, st) + off) =
                in ? static_cast<const IT*>(p.delta)[b * p.delta_sb + dd * p.delta_sd + tg] : zero;
            if (has_z)
                *reinterpret_cast<IT*>(smem + chunk_stage(L.x2, st) + off) =
                    in ? static_cast<const IT*>(p.z)[b * p.z_sb + dd * p.z_sd + tg] : zero;
        }
        for (int i = tid; i < N * T; i += nthr) {
            const int n = i / T, tt = i % T, tg = t0 + tt;
            const uint32_t off = swz128(n, tt * ES);
            *reinterpret_cast<IT*>(smem + chunk_stage(L.x3, st) + off) =
                tg < Lq ? static_cast<const IT*>(p.bc)[b * p.bc_sb + n * p.bc_sn + tg] : zero;
        }
    };

    if (p.use_tma && tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (p.use_tma && tid == 0) {
        issue(0, 0);
        if (ntiles > 1) issue(1, 1);
    }

    for (int j = 0; j < ntiles; j++) {
        const int st = j & 1;
        const int t0 = tile_of(j) * T;
        int ok = 1;
        if (p.use_tma) {
            ok = mbar_wait_bounded(&bar[st], (j >> 1) & 1) ? 1 : 0;
        } else {
            load_plain(j, st);
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicExch(p.err, kDevErrTmaTimeout);
            return;
        }

        // ---- prologue: delta and delta*u (forward) or dy (reverse), 4 tokens per item ------
        const unsigned char* s0 = smem + chunk_stage(L.x0, st);
        const unsigned char* s1 = smem + chunk_stage(L.x1, st);
        const unsigned char* s2 = smem + chunk_stage(L.x2, st);
        const bool tile_short = t0 + T > Lq;
        for (int i = tid; i < DT * (T / 4); i += nthr) {
            const int cc = i / (T / 4), t4 = (i % (T / 4)) * 4;
            const uint32_t off = swz128(cc, t4 * ES);
            float dr[4], xv[4], dl[4], xo[4];
            Vec4<IT>::load(s1 + off, dr);
            Vec4<IT>::load(s0 + off, xv);
            float zv[4];
            if (has_z) Vec4<IT>::load(s2 + off, zv);
            const float bias = sBias[cc];
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
                // token pairs in packed f32x2 arithmetic (the same operations per element)
                const float2 x = make_float2(dr[k] + bias, dr[k + 1] + bias);
                const float2 v = p.delta_softplus ? softplus_series2(x) : x;
                dl[k] = v.x;
                dl[k + 1] = v.y;
                float2 o;
                if (REV)
                    o = has_z ? __fmul2_rn(__fmul2_rn(make_float2(xv[k], xv[k + 1]), make_float2(zv[k], zv[k + 1])),
                                           make_float2(sigmoid_io<IT>(zv[k]), sigmoid_io<IT>(zv[k + 1])))
                              : make_float2(xv[k], xv[k + 1]);
                else
                    o = __fmul2_rn(v, make_float2(xv[k], xv[k + 1]));
                xo[k] = o.x;
                xo[k + 1] = o.y;
            }
            if (tile_short) {
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if (t0 + t4 + k >= Lq) { dl[k] = 0.f; xo[k] = 0.f; }
            }
            *reinterpret_cast<float4*>(sD + cc * RS + t4) = make_float4(dl[0], dl[1], dl[2], dl[3]);
            *reinterpret_cast<float4*>(sX + cc * RS + t4) = make_float4(xo[0], xo[1], xo[2], xo[3]);
        }
        const unsigned char* s3 = smem + chunk_stage(L.x3, st);
        // (two tokens per work item: one 4- or 8-byte load per state row)
        for (int i = tid; i < Q * (T / 2); i += nthr) {
            const int q = i / (T / 2), tt = 2 * (i % (T / 2));
            const bool ld0 = t0 + tt < Lq, ld1 = t0 + tt + 1 < Lq;
            float2 v[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int n = q * 4 + k;
                v[k] = n < N ? load_pair<IT>(s3 + swz128(n, tt * ES)) : make_float2(0.f, 0.f);
                if (!ld0) v[k].x = 0.f;
                if (!ld1) v[k].y = 0.f;
            }
            *reinterpret_cast<float4*>(sM + tt * NS + ((q ^ (tt & QM)) << 2)) = make_float4(v[0].x, v[1].x, v[2].x, v[3].x);
            *reinterpret_cast<float4*>(sM + (tt + 1) * NS + ((q ^ ((tt + 1) & QM)) << 2)) =
                make_float4(v[0].y, v[1].y, v[2].y, v[3].y);
        }
        __syncthreads();
        // the raw stage is consumed: refill it with the tile after next
        if (p.use_tma && tid == 0 && j + 2 < ntiles) issue(j + 2, st);

        // ---- recurrence over the tile ---------------------------------------------------------
#pragma unroll 1
        for (int gi = 0; gi < T / G; gi++) {
            const int q0 = REV ? T - G - gi * G : gi * G;
#pragma unroll
            for (int sbi = 0; sbi < G / 4; sbi++) {
                const int sb = REV ? G - 4 - sbi * 4 : sbi * 4;
                const int tl = q0 + sb;
                const float4 dl4 = lds128(sD + c * RS + tl);
                const float4 x4 = lds128(sX + c * RS + tl);
                const float dls[4] = {dl4.x, dl4.y, dl4.z, dl4.w};
                const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
                for (int jj = 0; jj < 4; jj++) {
                    const int k = REV ? 3 - jj : jj;
                    const int t = tl + k;
                    const int sw = (sb + k) & QM;   // q0 is a multiple of 16
                    const float2 dl2 = make_float2(dls[k], dls[k]);
                    const float2 x2 = make_float2(xs[k], xs[k]);
                    float2 mp[NP];
                    load_state_pairs<SPT, NS>(sM, t, g, sw, mp);
#pragma unroll
                    for (int pi = 0; pi < NP; pi++) {
                        const float2 e = __fmul2_rn(dl2, A2[pi]);
                        const float2 a = (k * NP + pi) % 4 < kChunkExpOnFma ? exp2_fma2(e)
                                                                            : make_float2(ex2(e.x), ex2(e.y));
                        if (REV) {
                            // dh_t = a_{t+1} dh_{t+1} + C_t dy_t
                            h[pi] = __ffma2_rn(an[pi], h[pi], __fmul2_rn(x2, mp[pi]));
                            an[pi] = a;
                        } else {
                            h[pi] = __ffma2_rn(a, h[pi], __fmul2_rn(x2, mp[pi]));
                        }
                    }
                }
                if (!REV) Ssum += (dls[0] + dls[1]) + (dls[2] + dls[3]);
            }
        }
        __syncthreads();   // the work rows are rewritten by the next tile's prologue
    }

    if (dvalid) {
#pragma unroll
        for (int s = 0; s < SPT; s++) {
            const int n = g * SPT + s;
            if (n >= N) continue;
            float v = (s & 1) ? h[s / 2].y : h[s / 2].x;
            if (REV) v *= (s & 1) ? an[s / 2].y : an[s / 2].x;   // gradient into the state before the slice
            p.carry[((int64_t)b * p.dim + d) * N + n] = v;
        }
        if (!REV && p.delta_sum && g == 0) p.delta_sum[(int64_t)b * p.dim + d] = Ssum;
    }
}

// Folds per-slice carries.  One thread per (row, channel, state).
//   forward: result[0] = start, result[q + 1] = exp(A * dsum[q]) * result[q] + carry[q]
//   reverse: result[S - 1] = start, result[q - 1] = exp(A * dsum[q]) * result[q] + carry[q]
// `start` may be the sum of nstart arrays spaced start_ss apart (one per rank), or null (0).
__global__ void carry_compose_kernel(const __grid_constant__ CarryParams p) {
    const int64_t per = (int64_t)p.batch * p.dim * p.dstate;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= per) return;
    const int n = (int)(i % p.dstate);
    const int64_t bd = i / p.dstate;
    const int d = (int)(bd % p.dim);
    const float a2 = p.A[(int64_t)d * p.A_sd + n] * kLog2e;
    // result does not overlap carry or delta_sum (C ABI), so each batch of U slices' inputs
    // is loaded before the batch's fold: the fold is sequential, its loads are not
    const float* __restrict__ carry = p.carry;
    const float* __restrict__ dsum = p.delta_sum;
    float* __restrict__ res = p.result;
    constexpr int U = 8;
    float h = 0.f;
    if (p.start)
        for (int r = 0; r < p.nstart; r++) h += p.start[r * p.start_ss + i];
    const int M = p.nslices;
    if (!p.reverse) {
        res[i] = h;
        for (int q0 = 0; q0 < M; q0 += U) {
            float e[U], c[U];
#pragma unroll
            for (int k = 0; k < U; k++) {
                const int q = q0 + k;
                e[k] = q < M ? dsum[q * p.dsum_ss + bd] : 0.f;
                c[k] = q < M ? carry[q * p.carry_ss + i] : 0.f;
            }
#pragma unroll
            for (int k = 0; k < U; k++) {
                const int q = q0 + k;
                if (q < M) {
                    h = fmaf(ex2(a2 * e[k]), h, c[k]);
                    res[(int64_t)(q + 1) * per + i] = h;
                }
            }
        }
    } else {
        res[(int64_t)(M - 1) * per + i] = h;
        for (int q0 = M - 1; q0 >= 1; q0 -= U) {
            float e[U], c[U];
#pragma unroll
            for (int k = 0; k < U; k++) {
                const int q = q0 - k;
                e[k] = q >= 1 ? dsum[q * p.dsum_ss + bd] : 0.f;
                c[k] = q >= 1 ? carry[q * p.carry_ss + i] : 0.f;
            }
#pragma unroll
            for (int k = 0; k < U; k++) {
                const int q = q0 - k;
                if (q >= 1) {
                    h = fmaf(ex2(a2 * e[k]), h, c[k]);
                    res[(int64_t)(q - 1) * per + i] = h;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------------------
template <typename IT, int LPC, int SPT, bool REV>
static cudaError_t launch_chunk_t(const ChunkParams& p, const CUtensorMap* maps, cudaStream_t stream) {
    auto kern = scan_chunk_kernel<IT, LPC, SPT, REV>;
    const ChunkSmem L = chunk_smem_layout(p.dt, LPC * SPT, sizeof(IT), (REV && p.z) ? 1 : 0);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    kern<<<p.batch * p.ntile_d, p.dt * LPC, L.total, stream>>>(p, maps[0], maps[1], maps[2], maps[3]);
    return cudaGetLastError();
}

#define SSM_CHUNK_TABLE(X)                                                                 \
    X(1, 4) X(2, 4) X(4, 4) X(8, 4) X(16, 4) X(32, 4) X(32, 8) X(2, 2) X(4, 2) X(8, 2) X(16, 2) \
    X(32, 2)

cudaError_t launch_scan_chunk(const ChunkParams& p, int is_bf16, int lpc, int spt, int reverse,
                              const CUtensorMap* maps, cudaStream_t stream) {
#define SSM_CHUNK_CASE(LPC_, SPT_)                                                                   \
    if (lpc == LPC_ && spt == SPT_) {                                                                \
        if (reverse)                                                                                 \
            return is_bf16 ? launch_chunk_t<__nv_bfloat16, LPC_, SPT_, true>(p, maps, stream)        \
                           : launch_chunk_t<float, LPC_, SPT_, true>(p, maps, stream);               \
        return is_bf16 ? launch_chunk_t<__nv_bfloat16, LPC_, SPT_, false>(p, maps, stream)           \
                       : launch_chunk_t<float, LPC_, SPT_, false>(p, maps, stream);                  \
    }
    SSM_CHUNK_TABLE(SSM_CHUNK_CASE)
#undef SSM_CHUNK_CASE
    return cudaErrorInvalidValue;
}

int chunk_occupancy(int is_bf16, int lpc, int spt, int reverse, int dt, int has_z) {
    const void* k = nullptr;
#define SSM_CHUNK_K(LPC_, SPT_)                                                                      \
    if (lpc == LPC_ && spt == SPT_) {                                                                \
        if (reverse)                                                                                 \
            k = is_bf16 ? (const void*)scan_chunk_kernel<__nv_bfloat16, LPC_, SPT_, true>            \
                        : (const void*)scan_chunk_kernel<float, LPC_, SPT_, true>;                   \
        else                                                                                         \
            k = is_bf16 ? (const void*)scan_chunk_kernel<__nv_bfloat16, LPC_, SPT_, false>           \
                        : (const void*)scan_chunk_kernel<float, LPC_, SPT_, false>;                  \
    }
    SSM_CHUNK_TABLE(SSM_CHUNK_K)
#undef SSM_CHUNK_K
    if (!k) return 0;
    const size_t smem = chunk_smem_layout(dt, lpc * spt, is_bf16 ? 2 : 4, (reverse && has_z) ? 1 : 0).total;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, dt * lpc, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_carry_compose(const CarryParams& p, cudaStream_t stream) {
    const int64_t per = (int64_t)p.batch * p.dim * p.dstate;
    const int64_t blocks = (per + 255) / 256;
    carry_compose_kernel<<<(unsigned)blocks, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

// ---- diagnostics: the FMA-pipe exp2 next to ex2.approx, on the same inputs ---------------
__global__ void exp2_compare_kernel(const float* __restrict__ x, float* __restrict__ y_fma,
                                    float* __restrict__ y_mufu, int64_t n) {
    const int64_t i = 2 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= n) return;
    const float2 v = make_float2(x[i], i + 1 < n ? x[i + 1] : 0.f);
    const float2 f = exp2_fma2(v);
    y_fma[i] = f.x;
    y_mufu[i] = ex2(v.x);
    if (i + 1 < n) {
        y_fma[i + 1] = f.y;
        y_mufu[i + 1] = ex2(v.y);
    }
}

cudaError_t launch_exp2_compare(const float* x, float* y_fma, float* y_mufu, int64_t n, cudaStream_t stream) {
    const int64_t pairs = (n + 1) / 2;
    const int block = 256;
    exp2_compare_kernel<<<(unsigned)((pairs + block - 1) / block), block, 0, stream>>>(x, y_fma, y_mufu, n);
    return cudaGetLastError();
}

}  // namespace ssm
