// Backward selective scan for sm_100a, plus the deterministic reduction of its partials.
//
// Replaces the reference backward kernel (nmquan1503/ssm-mamba,
// csrc/selective_scan/backward_kernel.cu:89-478).  Same gradients -- recompute the states,
// run dh_t = exp(delta_{t+1} A) dh_{t+1} + C_t dout_t backwards, and form du, ddelta, dA,
// dB, dC, dD, ddelta_bias, dh_init -- with a different organisation:
//
//  * Same CTA / thread layout as the forward: a CTA owns (batch row, `dt` channels), a
//    thread owns one channel and SPT states, and walks the sequence backwards in tiles of
//    32 tokens, each split into sub-tiles of K tokens.
//  * Every sub-tile restarts from a state checkpoint the forward saved K tokens earlier,
//    recomputes its K states into registers (one exp2 per token and state), then runs the
//    reverse recurrence over them.  There is no block scan and no second exp pass.
//  * dB and dC (sums over channels) are reduced in registers: the lanes of the channels in a
//    warp hold their states in an XOR-rotated order (lane r keeps state 4g + (s ^ r) in
//    register s), so the 4-lane transpose-reduce is three shuffles and three adds with no
//    selects.  Warps combine through shared memory, CTAs through a per-channel-tile
//    workspace that ssm_scan_reduce_kernel sums in a fixed order.  No floating-point atomics
//    (the reference issues one atomicAdd per (token, state, channel), backward_kernel.cu:395-400).
//  * du / ddelta need sums over states: a reduce-scatter across the state lanes leaves each
//    lane with whole tokens to finish (skip term, softplus derivative, dD, ddelta_bias).
//  * Inputs arrive by one TMA stage that is refilled for the next tile as soon as the tile
//    prologue has consumed it; du, ddelta, dz leave by TMA stores.
//  * With `length` the reference's rules are reproduced exactly (backward_kernel.cu:225-400):
//    chunks of 128 tokens starting at or after len are skipped, loads are zero-filled from
//    len on when seqlen % 128 != 0, padded tokens are identity steps without C*dout, and only
//    tokens t < len feed ddelta, dA, dB and dC.
#include "common.cuh"
#include "params.h"
#include "scan_layout.h"
#include "warp_reduce.cuh"

#include <type_traits>

namespace ssm {

template <typename IT, int LPC, int SPT, int K>
__global__ void __launch_bounds__(128, 3) scan_bwd_kernel(
    const __grid_constant__ BwdParams p, const __grid_constant__ CUtensorMap tm_u,
    const __grid_constant__ CUtensorMap tm_delta, const __grid_constant__ CUtensorMap tm_dout,
    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_y,
    const __grid_constant__ CUtensorMap tm_B, const __grid_constant__ CUtensorMap tm_C,
    const __grid_constant__ CUtensorMap tm_du, const __grid_constant__ CUtensorMap tm_ddelta,
    const __grid_constant__ CUtensorMap tm_dz) {
    constexpr int ES = sizeof(IT);
    constexpr int TB = kBwdTile;
    constexpr int NS = LPC * SPT;
    constexpr int CPW = 32 / LPC;                 // channel lanes per warp
    // XOR-rotated state order across SPT channel lanes (SPT = 2 or 4) for the dB/dC sums
    constexpr bool ROT = (CPW >= SPT) && (SPT == 2 || SPT == 4);
    constexpr int NROT = ROT ? SPT : 1;
    constexpr int Q = NS / 4;
    constexpr int QM = (Q < 8 ? Q : 8) - 1;
    constexpr int NSUB = TB / K;
    constexpr int RS = TB + 4;
    constexpr int V = 2 * K;                      // S1 and S2 per sub-tile token
    static_assert(TB % K == 0 && K % 4 == 0, "sub-tiles must be whole float4 groups");
    static_assert(SPT == 2 || SPT % 4 == 0, "states per thread: 2 or a multiple of 4");

    extern __shared__ __align__(1024) unsigned char smem[];
    if ((smem_u32(smem) & 1023u) != 0u) {
        if (threadIdx.x == 0) atomicExch(p.err, kDevErrSmemAlign);
        return;
    }
    const int DT = p.dt;
    const int tid = threadIdx.x, nthr = DT * LPC;
    const int lane = tid & 31, warp = tid >> 5;
    const int c = tid / LPC, g = tid % LPC;
    const int cw = lane / LPC;
    const int rot = ROT ? (cw & (SPT - 1)) : 0;
    const int rot_n = (tid % LPC) * SPT + rot;   // state whose dB/dC channel sum this lane stores
    const bool rot_ok = ROT && rot_n < p.dstate;
    const int b = blockIdx.x / p.ntile_d, tile_d = blockIdx.x % p.ntile_d;
    const int d0 = tile_d * DT, d = d0 + c;
    const bool dvalid = d < p.dim;
    const int N = p.dstate, Lq = p.seqlen;
    const bool has_z = p.z != nullptr;
    const BwdSmem S = bwd_smem_layout(DT, NS, N, ES, NROT, nthr / 32, has_z ? 1 : 0, K);
    float* sD = reinterpret_cast<float*>(smem + S.sD);
    float* sDU = reinterpret_cast<float*>(smem + S.sDU);
    float* sG = reinterpret_cast<float*>(smem + S.sG);
    float* sSP = reinterpret_cast<float*>(smem + S.sSP);
    float* sU = reinterpret_cast<float*>(smem + S.sU);
    float* sB = reinterpret_cast<float*>(smem + S.sB);
    float* sC = reinterpret_cast<float*>(smem + S.sC);
    float* slots = reinterpret_cast<float*>(smem + S.slots);
    float* xch = reinterpret_cast<float*>(smem + S.xch);
    float* xwarp = xch + (tid >> 5) * 32 * (int)S.xch_stride;   // this warp's exchange area
    float* xmine = xwarp + (tid & 31) * (int)S.xch_stride;      // this lane's block
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S.bar);

    // ---- per-batch length rules (reference semantics when length is given) ----------------
    const bool ref = p.length != nullptr;
    int len = Lq;
    if (ref) {
        long long v = p.length[b];
        len = v < 0 ? 0 : (v > Lq ? Lq : (int)v);
    }
    const int Lload = (ref && (Lq % 128) != 0) ? len : Lq;           // zero-fill from here
    const int Rskip = ref ? min(Lq, ((len + 127) / 128) * 128) : Lq;  // skipped chunks
    const int mlo = (ref && !p.padding_right) ? Lq - len : 0;         // masked: t < mlo
    const int mhi = (ref && p.padding_right) ? len : Lq;              //      or t >= mhi

    // ---- per-thread constants, packed in pairs of states ---------------------------------------
    constexpr int NP = SPT / 2;
    float2 A2[NP], An[NP], Gp[NP], anp[NP], dAp[NP];
    int nidx[SPT];
#pragma unroll
    for (int s = 0; s < SPT; s++) {
        const int n = g * SPT + (s ^ rot);
        nidx[s] = n;
        const bool ok = dvalid && n < N;
        const float a = ok ? p.A[(int64_t)d * p.A_sd + n] : 0.f;
        const float gl = (ok && p.dh_last) ? p.dh_last[((int64_t)b * p.dim + d) * N + n] : 0.f;
        if (s & 1) {
            An[s / 2].y = a; A2[s / 2].y = a * kLog2e; Gp[s / 2].y = gl;
        } else {
            An[s / 2].x = a; A2[s / 2].x = a * kLog2e; Gp[s / 2].x = gl;
        }
    }
#pragma unroll
    for (int q = 0; q < NP; q++) {
        anp[q] = make_float2(1.f, 1.f);
        dAp[q] = make_float2(0.f, 0.f);
    }
    const float Dd = (dvalid && p.D) ? p.D[d] : 0.f;
    float dD_acc = 0.f, db_acc = 0.f;
    float* sBias = reinterpret_cast<float*>(smem + S.bias);
    for (int i = tid; i < DT; i += nthr)
        sBias[i] = (d0 + i < p.dim && p.delta_bias) ? p.delta_bias[d0 + i] : 0.f;

    // this thread's channel in checkpoint 0 (checkpoints are dim * dstate floats apart) and
    // in the initial state
    const float* const ck_thread = p.ckpt + ((int64_t)b * p.nck * p.dim + (dvalid ? d : 0)) * N;
    const int64_t ck_stride = (int64_t)p.dim * N;
    const float* const hi_thread = p.h_init ? p.h_init + ((int64_t)b * p.dim + (dvalid ? d : 0)) * N : nullptr;
    auto load_ckpt = [&](int ts, float2 (&hv)[NP]) {
        const float* row = ts == 0 ? hi_thread : ck_thread + (int64_t)(ts / K - 1) * ck_stride;
#pragma unroll
        for (int s = 0; s < SPT; s++) {
            const int n = nidx[s];
            const float v = (row != nullptr && dvalid && n < N) ? row[n] : 0.f;
            if (s & 1) hv[s / 2].y = v; else hv[s / 2].x = v;
        }
    };

    const int ntiles = (Lq + TB - 1) / TB;
    // this CTA's dB/dC partial rows in the workspace: (2, dstate, seqlen) floats
    float* const ws_bc_row = p.ws_bc + (((int64_t)tile_d * p.batch + b) * 2) * N * (int64_t)Lq;
    const uint32_t tile_bytes = (uint32_t)DT * TB * ES;
    const uint32_t bc_bytes = (uint32_t)N * TB * ES;
    const uint32_t stage_bytes = (has_z ? 5u : 3u) * tile_bytes + 2u * bc_bytes;

    auto issue = [&](int tile) {
        const int t0 = tile * TB;
        mbar_arrive_expect_tx(bar, stage_bytes);
        tma_load_3d(smem + S.u, &tm_u, bar, t0, d0, b);
        tma_load_3d(smem + S.delta, &tm_delta, bar, t0, d0, b);
        tma_load_3d(smem + S.dout, &tm_dout, bar, t0, d0, b);
        if (has_z) {
            tma_load_3d(smem + S.z, &tm_z, bar, t0, d0, b);
            tma_load_3d(smem + S.y, &tm_y, bar, t0, d0, b);
        }
        tma_load_3d(smem + S.B, &tm_B, bar, t0, 0, b);
        tma_load_3d(smem + S.C, &tm_C, bar, t0, 0, b);
    };

    auto load_plain = [&](int tile) {
        const int t0 = tile * TB;
        const IT zero = from_f<IT>(0.f);
        for (int i = tid; i < DT * TB; i += nthr) {
            const int cc = i / TB, tt = i % TB, dd = d0 + cc, tg = t0 + tt;
            const bool in = dd < p.dim && tg < Lq;
            const uint32_t off = (uint32_t)(cc * TB + tt) * ES;
            *reinterpret_cast<IT*>(smem + S.u + off) =
                in ? static_cast<const IT*>(p.u)[b * p.u_sb + dd * p.u_sd + tg] : zero;
            *reinterpret_cast<IT*>(smem + S.delta + off) =
                in ? static_cast<const IT*>(p.delta)[b * p.delta_sb + dd * p.delta_sd + tg] : zero;
            *reinterpret_cast<IT*>(smem + S.dout + off) =
                in ? static_cast<const IT*>(p.dout)[b * p.dout_sb + dd * p.dout_sd + tg] : zero;
            if (has_z) {
                *reinterpret_cast<IT*>(smem + S.z + off) =
                    in ? static_cast<const IT*>(p.z)[b * p.z_sb + dd * p.z_sd + tg] : zero;
                *reinterpret_cast<IT*>(smem + S.y + off) =
                    in ? static_cast<const IT*>(p.y)[b * p.y_sb + dd * p.y_sd + tg] : zero;
            }
        }
        for (int i = tid; i < N * TB; i += nthr) {
            const int n = i / TB, tt = i % TB, tg = t0 + tt;
            const bool in = tg < Lq;
            const uint32_t off = (uint32_t)(n * TB + tt) * ES;
            *reinterpret_cast<IT*>(smem + S.B + off) =
                in ? static_cast<const IT*>(p.B)[b * p.B_sb + n * p.B_sn + tg] : zero;
            *reinterpret_cast<IT*>(smem + S.C + off) =
                in ? static_cast<const IT*>(p.C)[b * p.C_sb + n * p.C_sn + tg] : zero;
        }
    };

    // byte offset of (channel row, token) in a swizzled output tile
    auto out_off = [&](int row, int t) -> uint32_t {
        return ES == 2 ? swz32(row, t * ES) : swz64(row, t * ES);
    };

    if (p.use_tma && tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (p.use_tma && tid == 0 && !p.test_withhold) issue(ntiles - 1);

    // checkpoint of the first sub-tile processed, then prefetched one sub-tile ahead
    float2 h0[NP], h0n[NP];
    load_ckpt(((Lq - 1) / K) * K, h0);

    for (int it = ntiles - 1; it >= 0; it--) {
        const int t0 = it * TB;
        int ok = 1;
        if (p.use_tma) {
            if (tid == 0) tma_store_wait_read_all();  // previous tile's output tiles are free
            ok = mbar_wait_bounded(bar, (uint32_t)((ntiles - 1 - it) & 1)) ? 1 : 0;
        } else {
            load_plain(it);
        }
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicExch(p.err, kDevErrTmaTimeout);
            return;
        }

        // ---- prologue: 4 tokens of one channel per work item ------------------------------
        const bool tile_short = t0 + TB > Lload;
        for (int i = tid; i < DT * (TB / 4); i += nthr) {
            const int cc = i / (TB / 4), t4 = (i % (TB / 4)) * 4;
            const uint32_t off = (uint32_t)(cc * TB + t4) * ES;
            float uv[4], dr[4], dv[4];
            Vec4<IT>::load(smem + S.u + off, uv);
            Vec4<IT>::load(smem + S.delta + off, dr);
            Vec4<IT>::load(smem + S.dout + off, dv);
            if (tile_short) {
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (t0 + t4 + j >= Lload) { uv[j] = 0.f; dr[j] = 0.f; dv[j] = 0.f; }
            }
            const float bias = sBias[cc];
            float dl[4], du[4], spg[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float x = dr[j] + bias;
                if (p.delta_softplus) {
                    float t;
                    dl[j] = softplus_series(x, &t);
                    spg[j] = sigmoid_from_t(x, t);
                } else {
                    dl[j] = x;
                    spg[j] = 1.f;
                }
                du[j] = dl[j] * uv[j];
            }
            if (has_z) {
                float zv[4], yv[4], dz[4];
                Vec4<IT>::load(smem + S.z + off, zv);
                Vec4<IT>::load(smem + S.y + off, yv);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float sg = sigmoid_io<IT>(zv[j]);
                    dz[j] = t0 + t4 + j < Rskip ? dv[j] * yv[j] * sg * (1.f + zv[j] * (1.f - sg)) : 0.f;
                    dv[j] = dv[j] * zv[j] * sg;
                }
                Vec4<IT>::store(smem + S.dz + out_off(cc, t4), dz);
            }
            *reinterpret_cast<float4*>(sD + cc * RS + t4) = make_float4(dl[0], dl[1], dl[2], dl[3]);
            *reinterpret_cast<float4*>(sDU + cc * RS + t4) = make_float4(du[0], du[1], du[2], du[3]);
            *reinterpret_cast<float4*>(sG + cc * RS + t4) = make_float4(dv[0], dv[1], dv[2], dv[3]);
            *reinterpret_cast<float4*>(sSP + cc * RS + t4) = make_float4(spg[0], spg[1], spg[2], spg[3]);
            *reinterpret_cast<float4*>(sU + cc * RS + t4) = make_float4(uv[0], uv[1], uv[2], uv[3]);
        }
        for (int i = tid; i < Q * TB; i += nthr) {
            const int q = i / TB, tt = i % TB, tg = t0 + tt;
            const bool ld = tg < Lload;
            float vb[4], vc[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int n = q * 4 + k;
                const uint32_t off = (uint32_t)(n * TB + tt) * ES;
                vb[k] = (ld && n < N) ? to_f(*reinterpret_cast<const IT*>(smem + S.B + off)) : 0.f;
                vc[k] = (ld && n < N) ? to_f(*reinterpret_cast<const IT*>(smem + S.C + off)) : 0.f;
            }
#pragma unroll
            for (int r = 0; r < NROT; r++) {
                const int pos = r * (int)S.rot_stride + tt * NS + ((q ^ (tt & QM)) << 2);
                *reinterpret_cast<float4*>(sB + pos) =
                    make_float4(vb[0 ^ r], vb[1 ^ r], vb[2 ^ r], vb[3 ^ r]);
                *reinterpret_cast<float4*>(sC + pos) =
                    make_float4(vc[0 ^ r], vc[1 ^ r], vc[2 ^ r], vc[3 ^ r]);
            }
        }
        __syncthreads();
        if (p.use_tma && tid == 0 && it > 0 && !p.test_withhold) issue(it - 1);  // raw tiles consumed

        // ---- sub-tiles, last to first -------------------------------------------------------
        unsigned char* odu = smem + S.du;
        unsigned char* odd = smem + S.ddelta;
        float* wslot = slots + warp * S.slot_stride;
        // dB/dC slot row of the state this lane sums in the rotated order (ROT only)
        float* const rot_dst = wslot + rot_n * (TB + 1);
        const float* sBr = sB + rot * (int)S.rot_stride;
        const float* sCr = sC + rot * (int)S.rot_stride;
        // swizzle term of token t = tl0 + k of a sub-tile: sub-tiles start at multiples of K,
        // so when K is a multiple of the swizzle period it depends on k alone (a constant)
        auto swz_of = [](int k, int t) { return (K % (QM + 1) == 0) ? (k & QM) : (t & QM); };
#pragma unroll 1
        for (int sub = NSUB - 1; sub >= 0; sub--) {
            const int tl0 = sub * K;
            const int ts = t0 + tl0;
            if (ts >= Lq) continue;  // past the end of the sequence: nothing to do
            // prefetch the checkpoint of the next sub-tile (one step earlier in time)
            if (ts > 0) load_ckpt(ts - K, h0n);
            const bool skipped = ts >= Rskip;

            float v[LPC <= K ? 1 : V];
            if (skipped) {
                // reference: a 128-token chunk that starts at or after len is skipped
                if constexpr (LPC <= K) {
#pragma unroll
                    for (int k = 0; k < K; k += 2)
                        *reinterpret_cast<float4*>(xmine + 2 * k) = make_float4(0.f, 0.f, 0.f, 0.f);
                } else {
#pragma unroll
                    for (int j = 0; j < V; j++) v[j] = 0.f;
                }
#pragma unroll
                for (int k = 0; k < K; k++) {
                    if (ROT) {
                        if (rot_ok) {
                            rot_dst[tl0 + k] = 0.f;
                            rot_dst[NS * (TB + 1) + tl0 + k] = 0.f;
                        }
                    } else if (cw == 0) {
#pragma unroll
                        for (int s = 0; s < SPT; s++) {
                            const int n = nidx[s];
                            if (n < N) {
                                wslot[n * (TB + 1) + tl0 + k] = 0.f;
                                wslot[(NS + n) * (TB + 1) + tl0 + k] = 0.f;
                            }
                        }
                    }
                }
            } else {
                const bool general = (ts + K > Lq) || (ref && !(ts + K <= len && ts >= mlo && ts + K <= mhi));
                auto body = [&](auto gen_tag) {
                    constexpr bool GEN = decltype(gen_tag)::value;
                    float2 av[K][NP], hv[K][NP];
                    // recompute the K states from the checkpoint
#pragma unroll
                    for (int k4 = 0; k4 < K; k4 += 4) {
                        const float4 dl4 = lds128(sD + c * RS + tl0 + k4);
                        const float4 du4 = lds128(sDU + c * RS + tl0 + k4);
                        const float dls[4] = {dl4.x, dl4.y, dl4.z, dl4.w};
                        const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int k = k4 + j, t = tl0 + k;
                            bool msk = false;
                            if (GEN) {
                                const int tg = ts + k;
                                msk = tg >= Lq || tg < mlo || tg >= mhi;
                            }
                            const float2 dl2 = make_float2(dls[j], dls[j]);
                            const float2 du2 = make_float2(dus[j], dus[j]);
                            float2 bp[NP];
                            load_state_pairs<SPT, NS>(sBr, t, g, swz_of(k, t), bp);
#pragma unroll
                            for (int pi = 0; pi < NP; pi++) {
                                const float2 prev = k == 0 ? h0[pi] : hv[k - 1][pi];
                                const float2 x = __fmul2_rn(dl2, A2[pi]);
                                float2 a = make_float2(ex2(x.x), ex2(x.y));
                                float2 bb = __fmul2_rn(du2, bp[pi]);
                                if (GEN && msk) {
                                    a = make_float2(1.f, 1.f);
                                    bb = make_float2(0.f, 0.f);
                                }
                                av[k][pi] = a;
                                hv[k][pi] = __ffma2_rn(a, prev, bb);
                            }
                        }
                    }
                    // reverse recurrence and gradient terms
                    float2 s_odd = make_float2(0.f, 0.f);
#pragma unroll
                    for (int k4 = K - 4; k4 >= 0; k4 -= 4) {
                        const float4 dl4 = lds128(sD + c * RS + tl0 + k4);
                        const float4 du4 = lds128(sDU + c * RS + tl0 + k4);
                        const float4 dg4 = lds128(sG + c * RS + tl0 + k4);
                        const float dls[4] = {dl4.x, dl4.y, dl4.z, dl4.w};
                        const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
                        const float dgs[4] = {dg4.x, dg4.y, dg4.z, dg4.w};
#pragma unroll
                        for (int j = 3; j >= 0; j--) {
                            const int k = k4 + j, t = tl0 + k;
                            bool msk = false, vld = true;
                            if (GEN) {
                                const int tg = ts + k;
                                msk = tg >= Lq || tg < mlo || tg >= mhi;
                                vld = tg < len;
                            }
                            const float2 dg2 = make_float2(dgs[j], dgs[j]);
                            const float2 du2 = make_float2(dus[j], dus[j]);
                            const float2 ndu2 = make_float2(-dus[j], -dus[j]);
                            const float dlv = (GEN && !vld) ? 0.f : dls[j];
                            const float2 dl2 = make_float2(dlv, dlv);
                            float2 s12 = make_float2(0.f, 0.f), s22 = make_float2(0.f, 0.f);
                            float dBv[SPT], dCv[SPT];
                            float2 bp[NP], cp[NP];
                            load_state_pairs<SPT, NS>(sBr, t, g, swz_of(k, t), bp);
                            load_state_pairs<SPT, NS>(sCr, t, g, swz_of(k, t), cp);
#pragma unroll
                            for (int pi = 0; pi < NP; pi++) {
                                float2 inj = __fmul2_rn(dg2, cp[pi]);
                                if (GEN && msk) inj = make_float2(0.f, 0.f);
                                const float2 Gs = __ffma2_rn(anp[pi], Gp[pi], inj);
                                Gp[pi] = Gs;
                                anp[pi] = av[k][pi];
                                // q = h_t - delta*u*B (the reference's at_ht); without padding it
                                // equals decay * h_{t-1}, one multiply
                                const float2 qv = GEN ? __ffma2_rn(ndu2, bp[pi], hv[k][pi])
                                                      : __fmul2_rn(av[k][pi], k == 0 ? h0[pi] : hv[k - 1][pi]);
                                s12 = __ffma2_rn(Gs, bp[pi], s12);
                                const float2 w = __fmul2_rn(Gs, qv);
                                s22 = __ffma2_rn(An[pi], w, s22);
                                dAp[pi] = __ffma2_rn(dl2, w, dAp[pi]);
                                float2 db = __fmul2_rn(Gs, du2);
                                float2 dc = __fmul2_rn(dg2, hv[k][pi]);
                                if (GEN && !vld) {
                                    db = make_float2(0.f, 0.f);
                                    dc = make_float2(0.f, 0.f);
                                }
                                dBv[pi * 2] = db.x; dBv[pi * 2 + 1] = db.y;
                                dCv[pi * 2] = dc.x; dCv[pi * 2 + 1] = dc.y;
                            }
                            {
                                const float s1t = s12.x + s12.y;
                                const float s2t = (GEN && !vld) ? 0.f : s22.x + s22.y;
                                if constexpr (LPC <= K) {
                                    // this lane's partial sums of tokens k, k + 1 (k even), as
                                    // (S1_k, S2_k, S1_k+1, S2_k+1); the odd token comes first
                                    if (j & 1) {
                                        s_odd = make_float2(s1t, s2t);
                                    } else {
                                        *reinterpret_cast<float4*>(xmine + 2 * k) = make_float4(s1t, s2t, s_odd.x, s_odd.y);
                                    }
                                } else {
                                    v[k] = s1t;
                                    v[K + k] = s2t;
                                }
                            }
                            // dB, dC: sum over the channels of this warp
                            if (ROT) {
                                float2 r2 = make_float2(dBv[0], dCv[0]);
#pragma unroll
                                for (int i = 1; i < SPT; i++)
                                    r2 = __fadd2_rn(r2, make_float2(__shfl_xor_sync(0xffffffffu, dBv[i], LPC * i),
                                                                    __shfl_xor_sync(0xffffffffu, dCv[i], LPC * i)));
#pragma unroll
                                for (int m = SPT; m < CPW; m *= 2)
                                    r2 = __fadd2_rn(r2, make_float2(__shfl_xor_sync(0xffffffffu, r2.x, LPC * m),
                                                                    __shfl_xor_sync(0xffffffffu, r2.y, LPC * m)));
                                // lanes cw and cw ^ SPT hold the same sums: both store them
                                if (rot_ok) {
                                    rot_dst[t] = r2.x;
                                    rot_dst[NS * (TB + 1) + t] = r2.y;
                                }
                            } else {
#pragma unroll
                                for (int m = 1; m < CPW; m *= 2) {
#pragma unroll
                                    for (int s = 0; s < SPT; s++) {
                                        dBv[s] += __shfl_xor_sync(0xffffffffu, dBv[s], LPC * m);
                                        dCv[s] += __shfl_xor_sync(0xffffffffu, dCv[s], LPC * m);
                                    }
                                }
                                if (cw == 0) {
#pragma unroll
                                    for (int s = 0; s < SPT; s++) {
                                        const int n = nidx[s];
                                        if (n < N) {
                                            wslot[n * (TB + 1) + t] = dBv[s];
                                            wslot[(NS + n) * (TB + 1) + t] = dCv[s];
                                        }
                                    }
                                }
                            }
                        }
                    }
                };
                if (general) body(std::true_type{}); else body(std::false_type{});
            }
            // gradient of the initial state: decay of token 0 times dh_0 (dh_last when the
            // whole row was skipped)
            if (ts == 0 && p.dh_init != nullptr && dvalid) {
#pragma unroll
                for (int s = 0; s < SPT; s++) {
                    const int n = nidx[s];
                    const float val = (s & 1) ? anp[s / 2].y * Gp[s / 2].y : anp[s / 2].x * Gp[s / 2].x;
                    if (n < N) p.dh_init[((int64_t)b * p.dim + d) * N + n] = val;
                }
            }

            // ---- per-token sums over states, then finish the tokens this lane owns ---------
            auto finish = [&](int k, float s1, float s2) {
                const int t = tl0 + k, tg = ts + k;
                float du = 0.f, ddl = 0.f;
                if (!skipped) {
                    const float dl = sD[c * RS + t], dg = sG[c * RS + t], uv = sU[c * RS + t];
                    du = fmaf(Dd, dg, dl * s1);
                    ddl = tg < len ? fmaf(uv, s1, s2) * sSP[c * RS + t] : 0.f;
                    dD_acc = fmaf(dg, uv, dD_acc);
                    db_acc += ddl;
                }
                *reinterpret_cast<IT*>(odu + out_off(c, t)) = from_f<IT>(du);
                *reinterpret_cast<IT*>(odd + out_off(c, t)) = from_f<IT>(ddl);
            };
            // tokens k, k + 1 (k even) at once: 8-byte row loads, one store of both outputs
            auto finish2 = [&](int k, float4 sv) {
                const int t = tl0 + k, tg = ts + k;
                float2 du = make_float2(0.f, 0.f), ddl = make_float2(0.f, 0.f);
                if (!skipped) {
                    const float2 dl = *reinterpret_cast<const float2*>(sD + c * RS + t);
                    const float2 dg = *reinterpret_cast<const float2*>(sG + c * RS + t);
                    const float2 uv = *reinterpret_cast<const float2*>(sU + c * RS + t);
                    const float2 sp = *reinterpret_cast<const float2*>(sSP + c * RS + t);
                    du.x = fmaf(Dd, dg.x, dl.x * sv.x);
                    du.y = fmaf(Dd, dg.y, dl.y * sv.z);
                    ddl.x = tg < len ? fmaf(uv.x, sv.x, sv.y) * sp.x : 0.f;
                    ddl.y = tg + 1 < len ? fmaf(uv.y, sv.z, sv.w) * sp.y : 0.f;
                    dD_acc = fmaf(dg.x, uv.x, fmaf(dg.y, uv.y, dD_acc));
                    db_acc += ddl.x + ddl.y;
                }
                store_pair<IT>(odu + out_off(c, t), du);
                store_pair<IT>(odd + out_off(c, t), ddl);
            };
            if constexpr (LPC <= K) {
                // each lane stored its partial (S1, S2) of every token pair at xmine; the lanes of
                // a channel swap them through this warp's exchange area and lane g sums the LPC
                // partials of the RK consecutive tokens g*RK ... and finishes them
                constexpr int RK = K / LPC;
                __syncwarp();
                if constexpr (RK >= 2) {
                    float4 sr[RK / 2];
#pragma unroll
                    for (int r = 0; r < RK / 2; r++) sr[r] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int gg = 0; gg < LPC; gg++) {
                        const float* src = xwarp + ((lane & ~(LPC - 1)) + gg) * (int)S.xch_stride + 2 * g * RK;
#pragma unroll
                        for (int r = 0; r < RK / 2; r++) {
                            const float4 x = *reinterpret_cast<const float4*>(src + 4 * r);
                            sr[r].x += x.x; sr[r].y += x.y; sr[r].z += x.z; sr[r].w += x.w;
                        }
                    }
                    __syncwarp();
#pragma unroll
                    for (int r = 0; r < RK / 2; r++) finish2(g * RK + 2 * r, sr[r]);
                } else {
                    float2 sr = make_float2(0.f, 0.f);
#pragma unroll
                    for (int gg = 0; gg < LPC; gg++) {
                        const float* src = xwarp + ((lane & ~(LPC - 1)) + gg) * (int)S.xch_stride + 2 * g;
                        sr = __fadd2_rn(sr, *reinterpret_cast<const float2*>(src));
                    }
                    __syncwarp();
                    finish(g, sr.x, sr.y);
                }
            } else {
                reduce_scatter<LPC, V>(v, g);
                const float other = __shfl_xor_sync(0xffffffffu, v[0], K);
                if (g < K) finish(g, v[0], other);
            }
            if (ts > 0) {
#pragma unroll
                for (int q = 0; q < NP; q++) h0[q] = h0n[q];
            }
        }
        __syncthreads();

        // ---- CTA sum of the warp dB/dC slots -> workspace; store du, ddelta, dz -------------
        {
            // rows r = q * N + n of TB tokens; thread (tid % TB) sums token t of rows
            // tid / TB, tid / TB + nthr / TB, ... over the (at most 4) warps
            const int nw = nthr >> 5;
            const int t = tid % TB;
            const int rstep = nthr / TB;
            if (t0 + t < Lq) {
                float* dst = ws_bc_row + (int64_t)(tid / TB) * Lq + t0 + t;
                const int64_t dstep = (int64_t)rstep * Lq;
                const int sstride = (int)S.slot_stride;
                for (int r = tid / TB; r < 2 * N; r += rstep, dst += dstep) {
                    const int q = r >= N ? 1 : 0, n = r - q * N;
                    const float* src = slots + (q * NS + n) * (TB + 1) + t;
                    float acc = src[0];
#pragma unroll
                    for (int w = 1; w < 4; w++)
                        if (w < nw) acc += src[w * sstride];
                    *dst = acc;
                }
            }
        }
        if (p.use_tma) {
            if (tid == 0) {
                fence_proxy_async_smem();
                tma_store_3d(&tm_du, odu, t0, d0, b);
                tma_store_3d(&tm_ddelta, odd, t0, d0, b);
                if (has_z) tma_store_3d(&tm_dz, smem + S.dz, t0, d0, b);
                tma_store_commit();
            }
        } else {
            for (int i = tid; i < DT * TB; i += nthr) {
                const int cc = i / TB, tt = i % TB, dd = d0 + cc, tg = t0 + tt;
                if (dd >= p.dim || tg >= Lq) continue;
                const uint32_t off = out_off(cc, tt);
                static_cast<IT*>(p.du)[b * p.du_sb + dd * p.du_sd + tg] =
                    *reinterpret_cast<const IT*>(odu + off);
                static_cast<IT*>(p.ddelta)[b * p.ddelta_sb + dd * p.ddelta_sd + tg] =
                    *reinterpret_cast<const IT*>(odd + off);
                if (has_z)
                    static_cast<IT*>(p.dz)[b * p.dz_sb + dd * p.dz_sd + tg] =
                        *reinterpret_cast<const IT*>(smem + S.dz + off);
            }
            __syncthreads();
        }
    }

    // ---- per-(batch, channel) partials of dA, dD, ddelta_bias ----------------------------------
#pragma unroll
    for (int s = 0; s < SPT; s++) {
        const int n = nidx[s];
        const float val = (s & 1) ? dAp[s / 2].y : dAp[s / 2].x;
        if (dvalid && n < N) p.ws_a[((int64_t)b * p.dim + d) * N + n] = val;
    }
    dD_acc = allreduce<LPC>(dD_acc);
    db_acc = allreduce<LPC>(db_acc);
    if (g == 0 && dvalid) {
        p.ws_dd[((int64_t)b * p.dim + d) * 2 + 0] = dD_acc;
        p.ws_dd[((int64_t)b * p.dim + d) * 2 + 1] = db_acc;
    }
    if (p.use_tma && tid == 0) tma_store_wait_all();
}

// Deterministic final sums: dB/dC over channel tiles, dA/dD/ddelta_bias over the batch.
__global__ void scan_reduce_kernel(const __grid_constant__ ReduceParams p) {
    // blocks [0, nbc_blocks): dB / dC, block = (token block, state, quantity * batch + b),
    // thread = one token; the rest: dA, then dD and ddelta_bias, one value per thread
    const int tblocks = (p.seqlen + 255) / 256;
    const int nbc_blocks = tblocks * p.dstate * 2 * p.batch;
    const int j = blockIdx.x;
    if (j < nbc_blocks) {
        const int tb = j % tblocks;
        const int rest = j / tblocks;
        const int n = rest % p.dstate, qb = rest / p.dstate;
        const int q = qb & 1, b = qb >> 1;
        const int t = tb * 256 + threadIdx.x;
        if (t >= p.seqlen) return;
        const int64_t plane = (int64_t)p.dstate * p.seqlen;
        const float* src = p.ws_bc + ((int64_t)b * 2 + q) * plane + (int64_t)n * p.seqlen + t;
        const int64_t tile_step = (int64_t)p.batch * 2 * plane;
        float acc = 0.f;
        for (int tile = 0; tile < p.ntile_d; tile++, src += tile_step) acc += *src;
        void* dst = q == 0 ? p.dB : p.dC;
        const int64_t sb = q == 0 ? p.dB_sb : p.dC_sb, sn = q == 0 ? p.dB_sn : p.dC_sn;
        const int64_t o = b * sb + n * sn + t;
        if (p.bc_dtype == 1)
            static_cast<__nv_bfloat16*>(dst)[o] = __float2bfloat16_rn(acc);
        else
            static_cast<float*>(dst)[o] = acc;
        return;
    }
    const int na = p.dim * p.dstate;
    const int i = (j - nbc_blocks) * 256 + threadIdx.x;
    if (i < na) {
        float acc = 0.f;
        for (int bb = 0; bb < p.batch; bb++) acc += p.ws_a[(int64_t)bb * na + i];
        p.dA[i] = acc;
    } else if (i < na + p.dim) {
        const int dd = i - na;
        float a0 = 0.f, a1 = 0.f;
        for (int bb = 0; bb < p.batch; bb++) {
            a0 += p.ws_dd[((int64_t)bb * p.dim + dd) * 2 + 0];
            a1 += p.ws_dd[((int64_t)bb * p.dim + dd) * 2 + 1];
        }
        if (p.dD) p.dD[dd] = a0;
        if (p.ddelta_bias) p.ddelta_bias[dd] = a1;
    }
}

// ---------------------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------------------
template <typename IT, int LPC, int SPT, int K>
static cudaError_t launch_bwd_t(const BwdParams& p, const CUtensorMap* maps, cudaStream_t stream) {
    auto kern = scan_bwd_kernel<IT, LPC, SPT, K>;
    constexpr int CPW = 32 / LPC;
    constexpr int NROT = ((CPW >= SPT) && (SPT == 2 || SPT == 4)) ? SPT : 1;
    const BwdSmem L = bwd_smem_layout(p.dt, LPC * SPT, p.dstate, sizeof(IT), NROT,
                                      p.dt * LPC / 32, p.z != nullptr, K);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return e;
    kern<<<p.batch * p.ntile_d, p.dt * LPC, L.total, stream>>>(p, maps[0], maps[1], maps[2], maps[3],
                                                              maps[4], maps[5], maps[6], maps[7],
                                                              maps[8], maps[9]);
    return cudaGetLastError();
}

size_t bwd_smem_bytes(int is_bf16, int lpc, int spt, int dt, int dstate, int has_z);

int bwd_occupancy(int is_bf16, int lpc, int spt, int dt, int dstate, int has_z) {
    const void* k = nullptr;
#define SSM_BWD_K(LPC_, SPT_, K_)                                                             \
    if (lpc == LPC_ && spt == SPT_) {                                                        \
        k = is_bf16 ? (const void*)scan_bwd_kernel<__nv_bfloat16, LPC_, SPT_, K_>            \
                    : (const void*)scan_bwd_kernel<float, LPC_, SPT_, K_>;                   \
    }
    SSM_BWD_K(1, 4, 8) SSM_BWD_K(2, 4, 8) SSM_BWD_K(4, 4, 8) SSM_BWD_K(8, 4, 8) SSM_BWD_K(16, 4, 8)
    SSM_BWD_K(32, 4, 8) SSM_BWD_K(32, 8, 4) SSM_BWD_K(2, 2, 8) SSM_BWD_K(4, 2, 8) SSM_BWD_K(8, 2, 8) SSM_BWD_K(16, 2, 8)
    SSM_BWD_K(32, 2, 8)
#undef SSM_BWD_K
    if (!k) return 0;
    const size_t smem = bwd_smem_bytes(is_bf16, lpc, spt, dt, dstate, has_z);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, dt * lpc, smem) != cudaSuccess) return 0;
    return n;
}

size_t bwd_smem_bytes(int is_bf16, int lpc, int spt, int dt, int dstate, int has_z) {
    const int cpw = 32 / lpc;
    const int nrot = (cpw >= spt && (spt == 2 || spt == 4)) ? spt : 1;
    const int ksub = spt == 8 ? 4 : 8;
    return bwd_smem_layout(dt, lpc * spt, dstate, is_bf16 ? 2 : 4, nrot, dt * lpc / 32, has_z, ksub).total;
}

cudaError_t launch_scan_bwd(const BwdParams& p, int is_bf16, int lpc, int spt, const CUtensorMap* maps,
                            cudaStream_t stream) {
#define SSM_BWD_CASE(LPC_, SPT_, K_)                                                     \
    if (lpc == LPC_ && spt == SPT_) {                                                    \
        return is_bf16 ? launch_bwd_t<__nv_bfloat16, LPC_, SPT_, K_>(p, maps, stream)    \
                       : launch_bwd_t<float, LPC_, SPT_, K_>(p, maps, stream);           \
    }
    SSM_BWD_CASE(1, 4, 8)
    SSM_BWD_CASE(2, 4, 8)
    SSM_BWD_CASE(4, 4, 8)
    SSM_BWD_CASE(8, 4, 8)
    SSM_BWD_CASE(16, 4, 8)
    SSM_BWD_CASE(32, 4, 8)
    SSM_BWD_CASE(32, 8, 4)
    SSM_BWD_CASE(2, 2, 8)
    SSM_BWD_CASE(4, 2, 8)
    SSM_BWD_CASE(8, 2, 8)
    SSM_BWD_CASE(16, 2, 8)
    SSM_BWD_CASE(32, 2, 8)
#undef SSM_BWD_CASE
    return cudaErrorInvalidValue;
}

cudaError_t launch_scan_reduce(const ReduceParams& p, cudaStream_t stream) {
    const int64_t nbc_blocks = (int64_t)((p.seqlen + 255) / 256) * p.dstate * 2 * p.batch;
    const int64_t rest_blocks = ((int64_t)p.dim * p.dstate + p.dim + 255) / 256;
    if (nbc_blocks + rest_blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    scan_reduce_kernel<<<(unsigned)(nbc_blocks + rest_blocks), 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace ssm
