// Forward selective scan for sm_100a.
//
// Replaces the reference forward kernel (nmquan1503/ssm-mamba,
// csrc/selective_scan/forward_kernel.cu:69-264).  Same math -- delta = softplus(delta + bias),
// h_t = exp(delta*A) h_{t-1} + delta*u*B, y = D*u + sum_n C*h -- with a different shape:
//
//  * One CTA owns one batch row b and a tile of `dt` channels and walks the whole sequence
//    in tiles of T tokens (T*sizeof(elem) = 128 bytes).  The time recurrence stays in
//    registers, so there is no block scan and no per-chunk carry through shared memory.
//  * A thread owns one channel and SPT consecutive states; the LPC = NS/SPT lanes of a
//    channel are adjacent.  y_t = sum_n C h needs one reduce-scatter across those lanes
//    every G = max(16, LPC) tokens; each group of G tokens is straight-line code (in-group
//    checkpoints are predicated stores) and its reduce-scatter and epilogue overlap the
//    next group's recurrence.
//  * Each tile's u, delta, z and the (B, C) tile are brought in by 3-D TMA loads
//    (128-byte swizzle, 2 stages, mbarrier completion) and the outputs leave by TMA stores.
//    B and C are loaded once per CTA and shared by all of its channels (the reference
//    re-reads them for every channel).  Shapes whose strides TMA cannot describe use a
//    plain-load fallback into the same shared-memory layout.
//  * softplus, delta*u and the padding mask are computed once per (channel, token) in a
//    tile prologue; the inner loop is exp2 + 2 FMA + 1 MUL per (token, state).
//  * The gate out = y * silu(z) (modules/mamba.py:182 in the reference) is fused into the
//    epilogue, and the pre-gate y is optionally written for the backward.
//  * State checkpoints every ckpt_len tokens: compact (batch, nck, dim, dstate) for this
//    library's backward, or the reference's interleaved (prod, state) chunk carries
//    (selective_scan.cpp:271-274, forward_kernel.cu:224-228).
#include "common.cuh"
#include "params.h"
#include "scan_layout.h"
#include "warp_reduce.cuh"

namespace ssm {

// Offset of pipeline stage st (0 or 1) in a two-stage layout array.  A select rather than
// an index, so the layout struct stays in registers.
__device__ __forceinline__ uint32_t stage_off(const uint32_t (&a)[2], int st) { return st ? a[1] : a[0]; }

// This thread's SPT states of one compact checkpoint, at dst (its first state n0).
template <int SPT>
__device__ __forceinline__ void store_ckpt_row(float* dst, const float2 (&h)[SPT / 2], bool vec, int n0, int N) {
    if (vec) {
#pragma unroll
        for (int q = 0; q < SPT / 2; q++) *reinterpret_cast<float2*>(dst + 2 * q) = h[q];
    } else {
#pragma unroll
        for (int s = 0; s < SPT; s++)
            if (n0 + s < N) dst[s] = (s & 1) ? h[s / 2].y : h[s / 2].x;
    }
}

// Reference-layout chunk carry k of channel d: the interleaved (prod, state) pairs of
// selective_scan.cpp:271-274, prod = exp(A * sum of delta so far).  (Compact checkpoints go
// through store_ckpt_row.)  A free function rather than a capturing lambda so that h and A2
// stay in registers.
template <int SPT>
__device__ __forceinline__ void fwd_write_ckpt(const FwdParams& p, const float2 (&h)[SPT / 2],
                                               const float2 (&A2)[SPT / 2], float Ssum, int b, int d, int g,
                                               int k) {
    const int N = p.dstate;
    float* dst = p.ckpt + (((int64_t)b * p.dim + d) * p.nck + k) * 2 * N;
#pragma unroll
    for (int s = 0; s < SPT; s++) {
        const int n = g * SPT + s;
        if (n < N) {
            dst[2 * n] = ex2(((s & 1) ? A2[s / 2].y : A2[s / 2].x) * Ssum);
            dst[2 * n + 1] = (s & 1) ? h[s / 2].y : h[s / 2].x;
        }
    }
}

// store_ckpt_row as predicated stores (no branch): 16- or 8-byte stores when `vec`, else one
// store per valid state; nothing is stored unless `on`.
template <int SPT>
__device__ __forceinline__ void store_ckpt_row_if(float* dst, const float2 (&h)[SPT / 2], bool on, bool vec, int n0,
                                                  int N) {
    if constexpr (SPT % 4 == 0) {
#pragma unroll
        for (int q = 0; q < SPT / 4; q++)
            stg_f32x4_if(dst + 4 * q, h[2 * q].x, h[2 * q].y, h[2 * q + 1].x, h[2 * q + 1].y, on && vec);
    } else {
        stg_f32x2_if(dst, h[0].x, h[0].y, on && vec);
    }
#pragma unroll
    for (int s = 0; s < SPT; s++) stg_f32_if(dst + s, (s & 1) ? h[s / 2].y : h[s / 2].x, on && !vec && n0 + s < N);
}

// The recurrence over one group of G tokens, tile-local [q0, q0 + G), for this lane's SPT
// states of channel row c: yv[j] = the lane's part of y at token q0 + j.  tg0 is the group's
// first token in the sequence.  Compact checkpoints that fall inside the group (not at its
// end; their interval is a power of two >= CKMIN) are stored here with predicated stores, so
// the whole group is one straight-line block; everything at the group's end is
// fwd_group_end's.
template <int SPT, int NS, int G, int RS, int QM, int CKMIN>
__device__ __forceinline__ void fwd_group(const float* sD, const float* sDU, const float* sB, const float* sC, int c,
                                          int g, int q0, int tg0, const float2 (&A2)[SPT / 2], float2 (&h)[SPT / 2],
                                          float (&yv)[G], float& Ssum, float*& ck_ptr, bool ck_compact, bool ck_vec,
                                          int ck_mask, int64_t ck_step, int Lq, int N) {
    constexpr int NP = SPT / 2;
#pragma unroll
    for (int sb = 0; sb < G; sb += 4) {
        const int tl = q0 + sb;
        const float4 dl4 = lds128(sD + c * RS + tl);
        const float4 du4 = lds128(sDU + c * RS + tl);
        const float dls[4] = {dl4.x, dl4.y, dl4.z, dl4.w};
        const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            // q0 is a multiple of 16, so the swizzle term is a compile-time constant
            const int t = tl + j;
            const int sw = (sb + j) & QM;
            const float2 dl2 = make_float2(dls[j], dls[j]);
            const float2 du2 = make_float2(dus[j], dus[j]);
            float2 bp[NP], cp[NP];
            load_state_pairs<SPT, NS>(sB, t, g, sw, bp);
            load_state_pairs<SPT, NS>(sC, t, g, sw, cp);
            float2 y2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int pi = 0; pi < NP; pi++) {
                const float2 x = __fmul2_rn(dl2, A2[pi]);
                const float2 a = make_float2(ex2(x.x), ex2(x.y));
                h[pi] = __ffma2_rn(a, h[pi], __fmul2_rn(du2, bp[pi]));
                y2 = __ffma2_rn(cp[pi], h[pi], y2);
            }
            yv[sb + j] = y2.x + y2.y;
        }
        Ssum += (dls[0] + dls[1]) + (dls[2] + dls[3]);
        if (sb + 4 < G && (sb + 4) % CKMIN == 0) {
            const int tg_end = tg0 + sb + 4;
            const bool on = ck_compact && (tg_end & ck_mask) == 0 && tg_end <= Lq;
            store_ckpt_row_if<SPT>(ck_ptr, h, on, ck_vec, g * SPT, N);
            ck_ptr = on ? ck_ptr + ck_step : ck_ptr;
        }
    }
}

// At the end of a group (sequence token gend): the reference backward's chunk restart (in
// rechunk mode, every 128 tokens), then the checkpoint due at gend.  Both intervals are
// multiples of G, so nothing of either falls inside a group except compact checkpoints.
template <int SPT>
__device__ __forceinline__ void fwd_group_end(const FwdParams& p, float2 (&h)[SPT / 2], const float2 (&A2)[SPT / 2],
                                              float Ssum, int b, int d, int g, bool dvalid, bool rechunk,
                                              bool ck_compact, bool ck_vec, float*& ck_ptr, int64_t ck_step,
                                              int ck_mask, int gend, int Lq, int N) {
    if (rechunk && gend < Lq && (gend & 127) == 0 && dvalid) {
        const float* src = p.restart + (((int64_t)b * p.dim + d) * p.restart_nck + (gend / 128 - 1)) * 2 * N;
#pragma unroll
        for (int s = 0; s < SPT; s++) {
            const int n = g * SPT + s;
            const float v = n < N ? src[2 * n + 1] : 0.f;
            if (s & 1) h[s / 2].y = v; else h[s / 2].x = v;
        }
    }
    if ((gend & ck_mask) == 0 && gend <= Lq) {
        if (ck_compact) {
            store_ckpt_row<SPT>(ck_ptr, h, ck_vec, g * SPT, N);
            ck_ptr += ck_step;
        } else if (p.ckpt && dvalid) {
            fwd_write_ckpt<SPT>(p, h, A2, Ssum, b, d, g, (gend >> p.ckpt_shift) - 1);
        }
    }
}

// Reduce-scatter of one group's partial y over the LPC lanes of a channel, then the epilogue
// of the RL = G / LPC consecutive tokens lane g finishes: y = D u + sum_n C h, out = y silu(z).
// Branch-free, so that it can be scheduled into the next group's recurrence: without a gate
// sz points at the u tile and the gate is computed and discarded; y is stored before out, so
// that sy == so (no pre-gate output wanted) leaves out in place.
template <typename IT, int LPC, int G>
__device__ __forceinline__ void fwd_finish(float (&yv)[G], int c, int g, int q0, const unsigned char* su,
                                           const unsigned char* sz, unsigned char* so, unsigned char* sy, float Dd,
                                           bool has_z) {
    constexpr int ES = sizeof(IT);
    constexpr int RL = G / LPC;
    reduce_scatter_contig<LPC, G>(yv, g);
    if constexpr (RL >= 4) {
#pragma unroll
        for (int r4 = 0; r4 < RL; r4 += 4) {
            const int tl = q0 + g * RL + r4;
            const uint32_t off = swz128(c, tl * ES);
            float uv[4], zv[4], o[4], yt[4];
            Vec4<IT>::load(su + off, uv);
            Vec4<IT>::load(sz + off, zv);
#pragma unroll
            for (int j = 0; j < 4; j += 2) {   // token pairs, packed (same results per element)
                const float2 z2 = make_float2(zv[j], zv[j + 1]);
                const float2 y2 = __ffma2_rn(make_float2(Dd, Dd), make_float2(uv[j], uv[j + 1]),
                                             make_float2(yv[r4 + j], yv[r4 + j + 1]));
                const float2 gated = __fmul2_rn(__fmul2_rn(y2, z2), sigmoid_io2<IT>(z2));
                yt[j] = y2.x;
                yt[j + 1] = y2.y;
                o[j] = has_z ? gated.x : y2.x;
                o[j + 1] = has_z ? gated.y : y2.y;
            }
            Vec4<IT>::store(sy + off, yt);
            Vec4<IT>::store(so + off, o);
        }
    } else {
#pragma unroll
        for (int r = 0; r < RL; r++) {
            const int tl = q0 + g * RL + r;
            const uint32_t off = swz128(c, tl * ES);
            const float uv = to_f(*reinterpret_cast<const IT*>(su + off));
            const float zv = to_f(*reinterpret_cast<const IT*>(sz + off));
            const float yt = fmaf(Dd, uv, yv[r]);
            const float gated = yt * zv * sigmoid_io<IT>(zv);
            *reinterpret_cast<IT*>(sy + off) = from_f<IT>(yt);
            *reinterpret_cast<IT*>(so + off) = from_f<IT>(has_z ? gated : yt);
        }
    }
}

template <typename IT, int LPC, int SPT>
__global__ void __launch_bounds__(128, 3) scan_fwd_kernel(
    const __grid_constant__ FwdParams p, const __grid_constant__ CUtensorMap tm_u,
    const __grid_constant__ CUtensorMap tm_delta, const __grid_constant__ CUtensorMap tm_z,
    const __grid_constant__ CUtensorMap tm_B, const __grid_constant__ CUtensorMap tm_C,
    const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_y) {
    constexpr int ES = sizeof(IT);
    constexpr int T = 128 / ES;              // tokens per tile
    constexpr int NS = LPC * SPT;            // padded state count
    constexpr int NP = SPT / 2;              // state pairs per thread (packed f32x2 math)
    constexpr int G = LPC > 16 ? LPC : 16;   // tokens per group (one reduce-scatter each)
    constexpr int Q = NS / 4;                // float4 groups per B/C row
    constexpr int QM = (Q < 8 ? Q : 8) - 1;  // swizzle mask for the f32 B/C rows
    constexpr int RS = T + 4;                // padded row of sD / sDU (floats)
    // shortest compact checkpoint interval the host accepts: ssm_scan_ckpt_len(dstate)
    constexpr int CKMIN = NS > 128 ? 4 : 8;
    static_assert(T % G == 0 && (SPT == 2 || SPT % 4 == 0), "tile must hold whole groups");

    extern __shared__ __align__(1024) unsigned char smem[];
    if ((smem_u32(smem) & 1023u) != 0u) {  // the swizzled TMA tiles need a 1024-byte base
        if (threadIdx.x == 0) atomicExch(p.err, kDevErrSmemAlign);
        return;
    }
    const int DT = p.dt;
    const FwdSmem L = fwd_smem_layout(DT, NS, ES, p.z != nullptr, p.y != nullptr);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    float* sD = reinterpret_cast<float*>(smem + L.sD);
    float* sDU = reinterpret_cast<float*>(smem + L.sDU);
    float* sB = reinterpret_cast<float*>(smem + L.sB);
    float* sC = reinterpret_cast<float*>(smem + L.sC);
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
    const bool has_z = p.z != nullptr;
    const bool want_y = p.y != nullptr;
    const int ck_mask = p.ckpt_len - 1;     // checkpoint interval is a power of two
    // compact checkpoints are written in order: checkpoint k of this thread's states sits at
    // ck_ptr after k steps of ck_step floats (vector stores when the states are whole pairs)
    const bool ck_compact = p.ckpt != nullptr && p.ckpt_format == 0 && dvalid;
    // whole aligned vectors of states per lane (16-byte stores for SPT >= 4, 8-byte for 2)
    const bool ck_vec = (g * SPT + SPT <= p.dstate) && (p.dstate & 3) == 0 &&
                        (reinterpret_cast<uintptr_t>(p.ckpt) & (SPT % 4 == 0 ? 15u : 7u)) == 0;
    float* ck_ptr = ck_compact ? p.ckpt + ((int64_t)b * p.nck * p.dim + d) * p.dstate + g * SPT : nullptr;
    const int64_t ck_step = (int64_t)p.dim * p.dstate;

    int len = Lq;
    if (p.length) {
        long long v = p.length[b];
        len = v < 0 ? 0 : (v > Lq ? Lq : (int)v);
    }
    const bool has_len = p.length != nullptr;
    const bool rechunk = p.restart != nullptr;
    const bool want_out = p.out != nullptr;
    // rechunk mode loads as the reference backward does: zero-filled from len on when
    // seqlen % 128 != 0 (backward_kernel.cu:242-246)
    const int Lload = (rechunk && has_len && (Lq % 128) != 0) ? len : Lq;
    // tokens outside [mlo, mhi) are padding: identity steps
    const int mlo = (has_len && !p.padding_right) ? Lq - len : 0;
    const int mhi = (has_len && p.padding_right) ? len : Lq;

    // per-thread constants and state, packed in pairs of states
    float2 A2[NP], h[NP];
#pragma unroll
    for (int s = 0; s < SPT; s++) {
        const int n = g * SPT + s;
        const bool ok = dvalid && n < N;
        const float a = ok ? p.A[(int64_t)d * p.A_sd + n] * kLog2e : 0.f;
        const float h0 = (ok && p.h_init) ? p.h_init[((int64_t)b * p.dim + d) * N + n] : 0.f;
        if (s & 1) { A2[s / 2].y = a; h[s / 2].y = h0; } else { A2[s / 2].x = a; h[s / 2].x = h0; }
    }
    const float Dd = (dvalid && p.D) ? p.D[d] : 0.f;
    float Ssum = 0.f;  // running sum of effective delta (for reference-layout checkpoint products)
    for (int i = tid; i < DT; i += nthr)
        sBias[i] = (d0 + i < p.dim && p.delta_bias) ? p.delta_bias[d0 + i] : 0.f;

    const uint32_t tile_bytes = (uint32_t)DT * 128u;
    const uint32_t bc_bytes = (uint32_t)N * 128u;
    const uint32_t stage_bytes = (has_z ? 3u : 2u) * tile_bytes + 2u * bc_bytes;

    auto issue = [&](int tile, int st) {
        const int t0 = tile * T;
        mbar_arrive_expect_tx(&bar[st], stage_bytes);
        tma_load_3d(smem + stage_off(L.u, st), &tm_u, &bar[st], t0, d0, b);
        tma_load_3d(smem + stage_off(L.delta, st), &tm_delta, &bar[st], t0, d0, b);
        if (has_z) tma_load_3d(smem + stage_off(L.z, st), &tm_z, &bar[st], t0, d0, b);
        tma_load_3d(smem + stage_off(L.B, st), &tm_B, &bar[st], t0, 0, b);
        tma_load_3d(smem + stage_off(L.C, st), &tm_C, &bar[st], t0, 0, b);
    };

    // plain-load fallback into the same swizzled layout (zero fill out of range)
    auto load_plain = [&](int tile, int st) {
        const int t0 = tile * T;
        for (int i = tid; i < DT * T; i += nthr) {
            const int cc = i / T, tt = i % T, dd = d0 + cc, tg = t0 + tt;
            const bool in = dd < p.dim && tg < Lq;
            const uint32_t off = swz128(cc, tt * ES);
            const IT zero = from_f<IT>(0.f);
            *reinterpret_cast<IT*>(smem + stage_off(L.u, st) + off) =
                in ? static_cast<const IT*>(p.u)[b * p.u_sb + dd * p.u_sd + tg] : zero;
            *reinterpret_cast<IT*>(smem + stage_off(L.delta, st) + off) =
                in ? static_cast<const IT*>(p.delta)[b * p.delta_sb + dd * p.delta_sd + tg] : zero;
            if (has_z)
                *reinterpret_cast<IT*>(smem + stage_off(L.z, st) + off) =
                    in ? static_cast<const IT*>(p.z)[b * p.z_sb + dd * p.z_sd + tg] : zero;
        }
        for (int i = tid; i < N * T; i += nthr) {
            const int n = i / T, tt = i % T, tg = t0 + tt;
            const bool in = tg < Lq;
            const uint32_t off = swz128(n, tt * ES);
            const IT zero = from_f<IT>(0.f);
            *reinterpret_cast<IT*>(smem + stage_off(L.B, st) + off) =
                in ? static_cast<const IT*>(p.B)[b * p.B_sb + n * p.B_sn + tg] : zero;
            *reinterpret_cast<IT*>(smem + stage_off(L.C, st) + off) =
                in ? static_cast<const IT*>(p.C)[b * p.C_sb + n * p.C_sn + tg] : zero;
        }
    };

    auto hval = [&](int s) -> float { return (s & 1) ? h[s / 2].y : h[s / 2].x; };
    auto aval = [&](int s) -> float { return (s & 1) ? A2[s / 2].y : A2[s / 2].x; };

    if (p.use_tma && tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
        prefetch_tensormap(&tm_u);
        prefetch_tensormap(&tm_delta);
        prefetch_tensormap(&tm_B);
        prefetch_tensormap(&tm_C);
    }
    __syncthreads();
    if (p.use_tma && tid == 0 && !p.test_withhold) {
        issue(0, 0);
        if (ntiles > 1) issue(1, 1);
    }

    for (int it = 0; it < ntiles; it++) {
        const int st = it & 1;
        const int t0 = it * T;
        int ok = 1;
        if (p.use_tma) {
            ok = mbar_wait_bounded(&bar[st], (it >> 1) & 1) ? 1 : 0;
        } else {
            load_plain(it, st);
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicExch(p.err, kDevErrTmaTimeout);
            return;
        }

        // ---- prologue: 4 tokens of one channel per work item ------------------------------
        const unsigned char* su = smem + stage_off(L.u, st);
        const unsigned char* sdl = smem + stage_off(L.delta, st);
        const bool tile_masked = (t0 + T > Lload) || (t0 < mlo) || (t0 + T > mhi);
        for (int i = tid; i < DT * (T / 4); i += nthr) {
            const int cc = i / (T / 4), t4 = (i % (T / 4)) * 4;
            const uint32_t off = swz128(cc, t4 * ES);
            float dr[4], uv[4], dl[4], du[4];
            Vec4<IT>::load(sdl + off, dr);
            Vec4<IT>::load(su + off, uv);
            const float bias = sBias[cc];
            if (tile_masked) {
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (t0 + t4 + j >= Lload) { dr[j] = 0.f; uv[j] = 0.f; }
            }
#pragma unroll
            for (int j = 0; j < 4; j += 2) {
                const float2 x = make_float2(dr[j] + bias, dr[j + 1] + bias);
                const float2 v = p.delta_softplus ? softplus_series2(x) : x;
                dl[j] = v.x;
                dl[j + 1] = v.y;
                du[j] = dl[j] * uv[j];
                du[j + 1] = dl[j + 1] * uv[j + 1];
            }
            if (tile_masked) {
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int tg = t0 + t4 + j;
                    if (tg >= Lq || tg < mlo || tg >= mhi) { dl[j] = 0.f; du[j] = 0.f; }
                }
            }
            *reinterpret_cast<float4*>(sD + cc * RS + t4) = make_float4(dl[0], dl[1], dl[2], dl[3]);
            *reinterpret_cast<float4*>(sDU + cc * RS + t4) = make_float4(du[0], du[1], du[2], du[3]);
        }
        const unsigned char* sBr = smem + stage_off(L.B, st);
        const unsigned char* sCr = smem + stage_off(L.C, st);
        // (two tokens per work item: one 4- or 8-byte load per state row and stream)
        for (int i = tid; i < Q * (T / 2); i += nthr) {
            const int q = i / (T / 2), tt = 2 * (i % (T / 2));
            const bool ld0 = t0 + tt < Lload, ld1 = t0 + tt + 1 < Lload;
            float2 vb[4], vc[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int n = q * 4 + k;
                const uint32_t off = swz128(n, tt * ES);
                vb[k] = n < N ? load_pair<IT>(sBr + off) : make_float2(0.f, 0.f);
                vc[k] = n < N ? load_pair<IT>(sCr + off) : make_float2(0.f, 0.f);
                if (!ld0) { vb[k].x = 0.f; vc[k].x = 0.f; }
                if (!ld1) { vb[k].y = 0.f; vc[k].y = 0.f; }
            }
            const int pos0 = tt * NS + ((q ^ (tt & QM)) << 2);
            const int pos1 = (tt + 1) * NS + ((q ^ ((tt + 1) & QM)) << 2);
            *reinterpret_cast<float4*>(sB + pos0) = make_float4(vb[0].x, vb[1].x, vb[2].x, vb[3].x);
            *reinterpret_cast<float4*>(sC + pos0) = make_float4(vc[0].x, vc[1].x, vc[2].x, vc[3].x);
            *reinterpret_cast<float4*>(sB + pos1) = make_float4(vb[0].y, vb[1].y, vb[2].y, vb[3].y);
            *reinterpret_cast<float4*>(sC + pos1) = make_float4(vc[0].y, vc[1].y, vc[2].y, vc[3].y);
        }
        // the previous tile's TMA stores must be done reading the output tiles
        if (p.use_tma && tid == 0) tma_store_wait_read_all();
        __syncthreads();

        // ---- scan: groups of G tokens ---------------------------------------------------
        // The reduce-scatter and epilogue of group k are issued after the recurrence of
        // group k + 1 in the same straight-line block, so their shuffle and MUFU latencies
        // overlap it; the group-end work that needs branches comes last.
        const unsigned char* sz = has_z ? smem + stage_off(L.z, st) : su;
        unsigned char* so = smem + L.out;
        unsigned char* sy = want_y ? smem + L.y : so;
        if constexpr (G <= 16) {
            float yp[G];
            fwd_group<SPT, NS, G, RS, QM, CKMIN>(sD, sDU, sB, sC, c, g, 0, t0, A2, h, yp, Ssum, ck_ptr, ck_compact, ck_vec,
                                          ck_mask, ck_step, Lq, N);
            fwd_group_end<SPT>(p, h, A2, Ssum, b, d, g, dvalid, rechunk, ck_compact, ck_vec, ck_ptr, ck_step,
                               ck_mask, t0 + G, Lq, N);
#pragma unroll 2
            for (int q0 = G; q0 < T; q0 += G) {
                float yv[G];
                fwd_group<SPT, NS, G, RS, QM, CKMIN>(sD, sDU, sB, sC, c, g, q0, t0 + q0, A2, h, yv, Ssum, ck_ptr,
                                              ck_compact, ck_vec, ck_mask, ck_step, Lq, N);
                fwd_finish<IT, LPC, G>(yp, c, g, q0 - G, su, sz, so, sy, Dd, has_z);
#pragma unroll
                for (int j = 0; j < G; j++) yp[j] = yv[j];
                fwd_group_end<SPT>(p, h, A2, Ssum, b, d, g, dvalid, rechunk, ck_compact, ck_vec, ck_ptr, ck_step,
                                   ck_mask, t0 + q0 + G, Lq, N);
            }
            fwd_finish<IT, LPC, G>(yp, c, g, T - G, su, sz, so, sy, Dd, has_z);
        } else {
            // 32-token groups (32 lanes per channel): two groups' partial sums do not fit in
            // registers next to the states, so each group finishes before the next starts
#pragma unroll 1
            for (int q0 = 0; q0 < T; q0 += G) {
                float yv[G];
                fwd_group<SPT, NS, G, RS, QM, CKMIN>(sD, sDU, sB, sC, c, g, q0, t0 + q0, A2, h, yv, Ssum, ck_ptr,
                                              ck_compact, ck_vec, ck_mask, ck_step, Lq, N);
                fwd_finish<IT, LPC, G>(yv, c, g, q0, su, sz, so, sy, Dd, has_z);
                fwd_group_end<SPT>(p, h, A2, Ssum, b, d, g, dvalid, rechunk, ck_compact, ck_vec, ck_ptr, ck_step,
                                   ck_mask, t0 + q0 + G, Lq, N);
            }
        }
        __syncthreads();

        // ---- store the output tiles, refill this stage ------------------------------------
        if (p.use_tma) {
            if (tid == 0) {
                if (want_out) {
                    fence_proxy_async_smem();
                    tma_store_3d(&tm_out, so, t0, d0, b);
                    if (want_y) tma_store_3d(&tm_y, sy, t0, d0, b);
                    tma_store_commit();
                }
                if (it + 2 < ntiles) issue(it + 2, st);
            }
        } else {
            for (int i = tid; i < DT * T && want_out; i += nthr) {
                const int cc = i / T, tt = i % T, dd = d0 + cc, tg = t0 + tt;
                if (dd >= p.dim || tg >= Lq) continue;
                const uint32_t off = swz128(cc, tt * ES);
                static_cast<IT*>(p.out)[b * p.out_sb + dd * p.out_sd + tg] =
                    *reinterpret_cast<const IT*>(so + off);
                if (want_y)
                    static_cast<IT*>(p.y)[b * p.y_sb + dd * p.y_sd + tg] =
                        *reinterpret_cast<const IT*>(sy + off);
            }
            __syncthreads();
        }
    }

    // the last checkpoint of a sequence whose length is not a multiple of ckpt_len
    if (p.ckpt && (Lq & ck_mask) != 0 && dvalid) {
        if (ck_compact) store_ckpt_row<SPT>(ck_ptr, h, ck_vec, g * SPT, N);
        else fwd_write_ckpt<SPT>(p, h, A2, Ssum, b, d, g, p.nck - 1);
    }
    if (p.h_last && dvalid) {
#pragma unroll
        for (int s = 0; s < SPT; s++) {
            const int n = g * SPT + s;
            if (n < N) p.h_last[((int64_t)b * p.dim + d) * N + n] = hval(s);
        }
    }
    if (p.use_tma && tid == 0) tma_store_wait_all();
}

// ---------------------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------------------
template <typename IT, int LPC, int SPT>
static cudaError_t launch_fwd_t(const FwdParams& p, const CUtensorMap* maps, cudaStream_t stream) {
    auto kern = scan_fwd_kernel<IT, LPC, SPT>;
    const FwdSmem L = fwd_smem_layout(p.dt, LPC * SPT, sizeof(IT), p.z != nullptr, p.y != nullptr);
    const size_t smem = L.total;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int grid = p.batch * p.ntile_d;
    kern<<<grid, p.dt * LPC, smem, stream>>>(p, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5],
                                            maps[6]);
    return cudaGetLastError();
}

// states-per-thread / lanes-per-channel for a padded state count
cudaError_t launch_scan_fwd(const FwdParams& p, int is_bf16, int lpc, int spt, const CUtensorMap* maps,
                            cudaStream_t stream) {
#define SSM_FWD_CASE(LPC_, SPT_)                                                        \
    if (lpc == LPC_ && spt == SPT_) {                                                   \
        return is_bf16 ? launch_fwd_t<__nv_bfloat16, LPC_, SPT_>(p, maps, stream)       \
                       : launch_fwd_t<float, LPC_, SPT_>(p, maps, stream);              \
    }
    SSM_FWD_CASE(1, 4)
    SSM_FWD_CASE(2, 4)
    SSM_FWD_CASE(4, 4)
    SSM_FWD_CASE(8, 4)
    SSM_FWD_CASE(16, 4)
    SSM_FWD_CASE(32, 4)
    SSM_FWD_CASE(32, 8)
    SSM_FWD_CASE(2, 2)
    SSM_FWD_CASE(4, 2)
    SSM_FWD_CASE(8, 2)
    SSM_FWD_CASE(16, 2)
    SSM_FWD_CASE(32, 2)
#undef SSM_FWD_CASE
    return cudaErrorInvalidValue;
}

// Resident CTAs per SM for a CTA of dt channels (registers, shared memory, threads).
int fwd_occupancy(int is_bf16, int lpc, int spt, int dt, int has_z, int has_y) {
    const void* k = nullptr;
#define SSM_FWD_K(LPC_, SPT_)                                                                 \
    if (lpc == LPC_ && spt == SPT_) {                                                        \
        k = is_bf16 ? (const void*)scan_fwd_kernel<__nv_bfloat16, LPC_, SPT_>                \
                    : (const void*)scan_fwd_kernel<float, LPC_, SPT_>;                       \
    }
    SSM_FWD_K(1, 4) SSM_FWD_K(2, 4) SSM_FWD_K(4, 4) SSM_FWD_K(8, 4) SSM_FWD_K(16, 4) SSM_FWD_K(32, 4) SSM_FWD_K(32, 8)
    SSM_FWD_K(2, 2) SSM_FWD_K(4, 2) SSM_FWD_K(8, 2) SSM_FWD_K(16, 2) SSM_FWD_K(32, 2)
#undef SSM_FWD_K
    if (!k) return 0;
    const size_t smem = fwd_smem_layout(dt, lpc * spt, is_bf16 ? 2 : 4, has_z, has_y).total;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, dt * lpc, smem) != cudaSuccess) return 0;
    return n;
}

}  // namespace ssm
