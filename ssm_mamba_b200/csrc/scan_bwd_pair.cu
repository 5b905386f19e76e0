// Backward selective scan for sm_100a: the path for d_state 16 without `length` (every
// benchmark config), beside the general kernel of scan_bwd.cu.
//
// Same gradients as the reference backward (nmquan1503/ssm-mamba,
// csrc/selective_scan/backward_kernel.cu:212-452) and as scan_bwd_kernel, organised to move
// fewer bytes through shared memory and shuffles per (token, state, channel) element:
//
//  * A warp owns 8 * CPL channels x 16 states.  Lane (cw, g) -- channel lane cw = lane / 4,
//    state lane g = lane % 4 -- holds states 4g .. 4g+3 of CPL channels (cw, and cw + 8 when
//    CPL = 2).  With two channels the per-token B and C loads serve 8 elements instead of 4
//    and dB / dC are summed over the lane's two channels in registers before the cross-lane
//    reduction; one channel keeps twice the warps for shapes with few rows (config 2).
//  * dB / dC (sums over channels): the lane keeps its states in an XOR-rotated order (state
//    4g + (s ^ (cw & 3)) in register s; B and C are staged in 4 rotated copies), so the
//    transpose-reduce over the 8 channel lanes is shuffles with no selects; warps combine
//    through shared memory, CTAs through a per-channel-tile workspace summed by
//    scan_reduce_kernel in a fixed order.  No floating-point atomics.
//  * du / ddelta (sums over states): the per-lane partials (S1, S2) are reduce-scattered over
//    the 4 state lanes by shuffles -- per token pair (CPL = 2) or per 4-token quad (CPL = 1)
//    -- and each lane finishes one token (skip term, softplus derivative, dD, ddelta_bias).
//  * Registers hold the decays, states and B values of one quad (4 tokens).  Checkpoints are
//    every 8 tokens: the second quad of an 8-token sub-tile is reached by recomputing the
//    first quad without keeping it (1.5 exp2 per element, which the MUFU pipe affords).  The
//    two checkpoints a tile restarts from arrive by TMA with the tile (a 4-D box of the
//    checkpoint tensor), double-buffered, so no register holds a prefetch.
//  * Tiles of 16 tokens arrive by one TMA stage (with 2 channels per lane swizzled like the
//    output tiles, so the prologue's reads and row stores are free of bank conflicts),
//    refilled as soon as the tile prologue has consumed it; du, ddelta, dz leave by TMA
//    stores.  Tokens past the end of the sequence are identity steps with zero inputs (the
//    prologue zeroes their delta, delta*u, dout and softplus slope), so a ragged last tile
//    needs no other case.
#include "common.cuh"
#include "params.h"
#include "scan_layout.h"
#include "warp_reduce.cuh"
#include "bwd_prologue.cuh"

namespace ssm {

namespace {
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kPairNS = 16;   // states (exactly 16)
constexpr int kPairK = 8;     // checkpoint interval (tokens)
}  // namespace

template <typename IT, int CPL>
__global__ void __launch_bounds__(128) scan_bwd_pair_kernel(
    const __grid_constant__ BwdParams p, const __grid_constant__ CUtensorMap tm_u,
    const __grid_constant__ CUtensorMap tm_delta, const __grid_constant__ CUtensorMap tm_dout,
    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_y,
    const __grid_constant__ CUtensorMap tm_B, const __grid_constant__ CUtensorMap tm_C,
    const __grid_constant__ CUtensorMap tm_du, const __grid_constant__ CUtensorMap tm_ddelta,
    const __grid_constant__ CUtensorMap tm_dz, const __grid_constant__ CUtensorMap tm_ck) {
    constexpr int ES = sizeof(IT);
    constexpr int TB = kBwdTile;
    constexpr int NS = kPairNS;
    constexpr int K = kPairK;
    constexpr int RS = TB + 4;
    constexpr int CPW = 8 * CPL;                // channels per warp
    constexpr bool SWZ = CPL == 2;              // input tiles swizzled (see the prologue)
    static_assert(TB == 2 * K && K == 8, "tiles of two 8-token sub-tiles");
    static_assert(CPL == 1 || CPL == 2, "one or two channels per lane");

    extern __shared__ __align__(1024) unsigned char smem[];
    if ((smem_u32(smem) & 1023u) != 0u) {
        if (threadIdx.x == 0) atomicExch(p.err, kDevErrSmemAlign);
        return;
    }
    const int DT = p.dt;                        // channels per CTA, a multiple of CPW
    const int nthr = DT * 4 / CPL;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int cw = lane >> 2, g = lane & 3, rot = cw & 3;
    const int lc0 = warp * CPW + cw;            // this lane's channels: lc0 (+ 8) (CTA-local)
    const int b = blockIdx.x / p.ntile_d, tile_d = blockIdx.x % p.ntile_d;
    const int d0 = tile_d * DT;
    const int Lq = p.seqlen, Dm = p.dim;
    const bool has_z = p.z != nullptr;
    const BwdPairSmem S = bwd_pair_smem_layout(DT, nthr / 32, ES, has_z ? 1 : 0);
    float* sD = reinterpret_cast<float*>(smem + S.sD);
    float* sDU = reinterpret_cast<float*>(smem + S.sDU);
    float* sG = reinterpret_cast<float*>(smem + S.sG);
    float* sSP = reinterpret_cast<float*>(smem + S.sSP);
    float* sU = reinterpret_cast<float*>(smem + S.sU);
    float* sB = reinterpret_cast<float*>(smem + S.sB);
    float* sC = reinterpret_cast<float*>(smem + S.sC);
    float* slots = reinterpret_cast<float*>(smem + S.slots);
    float* sBias = reinterpret_cast<float*>(smem + S.bias);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S.bar);

    // ---- per-lane constants: 2 channels x 2 pairs of states, in the rotated order ----------
    int dch[CPL];
    bool dv[CPL];
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        dch[c] = d0 + lc0 + 8 * c;
        dv[c] = dch[c] < Dm;
    }
    float2 A2[CPL][2], Gp[CPL][2], anp[CPL][2], dAp[CPL][2];
#pragma unroll
    for (int c = 0; c < CPL; c++) {
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const int n = 4 * g + (s ^ rot);
            const float a = dv[c] ? p.A[(int64_t)dch[c] * p.A_sd + n] * kLog2e : 0.f;
            const float gl = (dv[c] && p.dh_last) ? p.dh_last[((int64_t)b * Dm + dch[c]) * NS + n] : 0.f;
            if (s & 1) { A2[c][s / 2].y = a; Gp[c][s / 2].y = gl; }
            else { A2[c][s / 2].x = a; Gp[c][s / 2].x = gl; }
        }
#pragma unroll
        for (int q = 0; q < 2; q++) {
            anp[c][q] = make_float2(1.f, 1.f);
            dAp[c][q] = make_float2(0.f, 0.f);
        }
    }
    // the finishing role of this lane: with 2 channels, token fo of every token pair of
    // channel lc0 + 8 * fc; with 1 channel, token g of every quad
    const int fc = CPL == 2 ? g >> 1 : 0, fo = CPL == 2 ? (g & 1) : g;
    const int fin_lc = lc0 + 8 * fc;
    const int fin_d = fc ? dch[CPL - 1] : dch[0];
    const bool fin_ok = fc ? dv[CPL - 1] : dv[0];
    const float Dd = (fin_ok && p.D) ? p.D[fin_d] : 0.f;
    float dD_acc = 0.f, db_acc = 0.f;
    for (int i = tid; i < DT; i += nthr) sBias[i] = (d0 + i < Dm && p.delta_bias) ? p.delta_bias[d0 + i] : 0.f;

    const int ntiles = (Lq + TB - 1) / TB;
    float* const ws_bc_row = p.ws_bc + (((int64_t)tile_d * p.batch + b) * 2) * NS * (int64_t)Lq;
    const uint32_t tile_bytes = (uint32_t)DT * TB * ES;
    const uint32_t bc_bytes = (uint32_t)NS * TB * ES;
    const uint32_t ck_bytes = 2u * (uint32_t)DT * NS * 4u;
    const uint32_t stage_bytes = (has_z ? 5u : 3u) * tile_bytes + 2u * bc_bytes + ck_bytes;

    // tile `tile`: its raw tiles, and the checkpoints its two sub-tiles restart from (the
    // states after tokens t0 - 1 and t0 + 7: checkpoints t0/8 - 1 and t0/8; index -1, before
    // the sequence, reads as zeros) into checkpoint buffer tile % 2
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
        tma_load_4d(smem + ((tile & 1) ? S.ck[1] : S.ck[0]), &tm_ck, bar, 0, d0, tile * 2 - 1, b);
    };
    // byte offset of (channel row, token) in a swizzled output tile
    auto out_off = [](int row, int t) -> uint32_t { return ES == 2 ? swz32(row, t * ES) : swz64(row, t * ES); };
    // ... and in an input tile: swizzled like the outputs when SWZ, else dense rows
    auto raw_off = [&](int row, int t) -> uint32_t { return SWZ ? out_off(row, t) : (uint32_t)(row * TB + t) * ES; };

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0 && !p.test_withhold) issue(ntiles - 1);

    for (int it = ntiles - 1; it >= 0; it--) {
        const int t0 = it * TB;
        if (tid == 0) tma_store_wait_read_all();   // the previous tile's output tiles are free
        const int ok = mbar_wait_bounded(bar, (uint32_t)((ntiles - 1 - it) & 1)) ? 1 : 0;
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicExch(p.err, kDevErrTmaTimeout);
            return;
        }

        // ---- prologue: 4 tokens of one channel per work item.  With 2 channels per lane (SWZ)
        // the 8 lanes of a quarter warp take 8 channels at the same tokens, so their 16-byte row
        // stores (stride RS) hit 8 distinct bank groups and their reads of the swizzled raw
        // tiles 8 distinct banks; with 1 channel per lane, 4 lanes per channel and unswizzled
        // raw tiles measured faster (config 2: 0.615 vs 0.628 ms) ----------------------------
        const bool tile_short = t0 + TB > Lq;
        for (int i = tid; i < DT * (TB / 4); i += nthr) {
            const int cc = SWZ ? (i & 7) + ((i >> 5) << 3) : i / (TB / 4);
            const int t4 = SWZ ? ((i >> 3) & 3) * 4 : (i % (TB / 4)) * 4;
            bwd_prologue_item<IT, RS>(smem, S, cc, t4, raw_off(cc, t4), out_off(cc, t4), sBias[cc], has_z,
                                      p.delta_softplus != 0, tile_short, t0 + t4, Lq);
        }
        // B, C as float32 rows [token][16 states] in 4 XOR-rotated copies (copy r holds the
        // states of float4 group q in the order s ^ r), float4 groups swizzled by token
        // (SWZ: item i -> group q, token tt such that a quarter warp's 8 stores land in 8
        // distinct 16-byte bank groups)
        for (int i = tid; i < 4 * TB; i += nthr) {
            const int q = SWZ ? ((i >> 2) & 1) + 2 * (i >> 5) : i / TB;
            const int tt = SWZ ? (i & 3) + 4 * ((i >> 3) & 3) : i % TB;
            float vb[4], vc[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t off = raw_off(q * 4 + k, tt);
                vb[k] = to_f(*reinterpret_cast<const IT*>(smem + S.B + off));
                vc[k] = to_f(*reinterpret_cast<const IT*>(smem + S.C + off));
            }
#pragma unroll
            for (int r = 0; r < 4; r++) {
                const int pos = r * (int)S.rot_stride + tt * NS + ((q ^ (tt & 3)) << 2);
                *reinterpret_cast<float4*>(sB + pos) = make_float4(vb[0 ^ r], vb[1 ^ r], vb[2 ^ r], vb[3 ^ r]);
                *reinterpret_cast<float4*>(sC + pos) = make_float4(vc[0 ^ r], vc[1 ^ r], vc[2 ^ r], vc[3 ^ r]);
            }
        }
        __syncthreads();
        if (tid == 0 && it > 0 && !p.test_withhold) issue(it - 1);   // raw tiles consumed

        unsigned char* odu = smem + S.du;
        unsigned char* odd = smem + S.ddelta;
        float* const wslot = slots + warp * (int)S.slot_stride;
        float* const rot_dst = wslot + (4 * g + cw) * (TB + 1);   // lanes cw < 4: state 4g + cw
        const float* const sBr = sB + rot * (int)S.rot_stride;
        const float* const sCr = sC + rot * (int)S.rot_stride;
        const float* const ckb = reinterpret_cast<const float*>(smem + ((it & 1) ? S.ck[1] : S.ck[0]));

        // one quad of 4 tokens (tile tokens tq .. tq+3) from hs, the state before it:
        // recompute (decays and states into registers), reverse recurrence, dB/dC into the
        // warp slots, and per token pair the sums over states and du / ddelta of one token
        auto quad = [&](int tq, const float2 (&hs)[CPL][2]) {
            float4 dl4[CPL], du4[CPL], dg4[CPL];
#pragma unroll
            for (int c = 0; c < CPL; c++) {
                const int lc = lc0 + 8 * c;
                dl4[c] = lds128(sD + lc * RS + tq);
                du4[c] = lds128(sDU + lc * RS + tq);
                dg4[c] = lds128(sG + lc * RS + tq);
            }
            float2 av[4][CPL][2], hv[4][CPL][2], bq[4][2];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                load_state_pairs<4, NS>(sBr, tq + j, g, j, bq[j]);   // tq % 4 == 0: swizzle term j
#pragma unroll
                for (int c = 0; c < CPL; c++) {
                    const float dl = j == 0 ? dl4[c].x : j == 1 ? dl4[c].y : j == 2 ? dl4[c].z : dl4[c].w;
                    const float du = j == 0 ? du4[c].x : j == 1 ? du4[c].y : j == 2 ? du4[c].z : du4[c].w;
                    const float2 dl2 = make_float2(dl, dl), du2 = make_float2(du, du);
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        const float2 x = __fmul2_rn(dl2, A2[c][q]);
                        const float2 a = make_float2(ex2(x.x), ex2(x.y));
                        const float2 prev = j == 0 ? hs[c][q] : hv[j - 1][c][q];
                        av[j][c][q] = a;
                        hv[j][c][q] = __ffma2_rn(a, prev, __fmul2_rn(du2, bq[j][q]));
                    }
                }
            }
            // (S1, S2) partials: 2 channels -> of a token pair, [channel][even, odd][S1, S2];
            // 1 channel -> of the quad, [token][S1, S2]
            float v[8];
#pragma unroll
            for (int j = 3; j >= 0; j--) {
                const int t = tq + j;
                float2 cp[2];
                load_state_pairs<4, NS>(sCr, t, g, j, cp);
                float2 dbp[2], dcp[2];
#pragma unroll
                for (int c = 0; c < CPL; c++) {
                    const float dl = j == 0 ? dl4[c].x : j == 1 ? dl4[c].y : j == 2 ? dl4[c].z : dl4[c].w;
                    const float du = j == 0 ? du4[c].x : j == 1 ? du4[c].y : j == 2 ? du4[c].z : du4[c].w;
                    const float dg = j == 0 ? dg4[c].x : j == 1 ? dg4[c].y : j == 2 ? dg4[c].z : dg4[c].w;
                    const float2 dl2 = make_float2(dl, dl), du2 = make_float2(du, du), dg2 = make_float2(dg, dg);
                    float2 s12 = make_float2(0.f, 0.f), s22 = make_float2(0.f, 0.f);
#pragma unroll
                    for (int q = 0; q < 2; q++) {
                        const float2 Gs = __ffma2_rn(anp[c][q], Gp[c][q], __fmul2_rn(dg2, cp[q]));
                        Gp[c][q] = Gs;
                        anp[c][q] = av[j][c][q];
                        const float2 prev = j == 0 ? hs[c][q] : hv[j - 1][c][q];
                        const float2 w = __fmul2_rn(Gs, __fmul2_rn(av[j][c][q], prev));
                        s12 = __ffma2_rn(Gs, bq[j][q], s12);
                        s22 = __ffma2_rn(A2[c][q], w, s22);
                        dAp[c][q] = __ffma2_rn(dl2, w, dAp[c][q]);
                        if (c == 0) {
                            dbp[q] = __fmul2_rn(Gs, du2);
                            dcp[q] = __fmul2_rn(dg2, hv[j][c][q]);
                        } else {
                            dbp[q] = __ffma2_rn(Gs, du2, dbp[q]);
                            dcp[q] = __ffma2_rn(dg2, hv[j][c][q], dcp[q]);
                        }
                    }
                    const int vi = CPL == 2 ? 4 * c + 2 * (j & 1) : 2 * j;
                    v[vi] = s12.x + s12.y;
                    v[vi + 1] = s22.x + s22.y;
                }
                // dB, dC of this token summed over the warp's channels: lane (cw, g) sums
                // state 4g + (cw & 3), which channel lane cw ^ i holds in its register i
                float2 r2 = make_float2(dbp[0].x, dcp[0].x);
                const float2 x1 = make_float2(__shfl_xor_sync(0xffffffffu, dbp[0].y, 4),
                                              __shfl_xor_sync(0xffffffffu, dcp[0].y, 4));
                const float2 x2 = make_float2(__shfl_xor_sync(0xffffffffu, dbp[1].x, 8),
                                              __shfl_xor_sync(0xffffffffu, dcp[1].x, 8));
                const float2 x3 = make_float2(__shfl_xor_sync(0xffffffffu, dbp[1].y, 12),
                                              __shfl_xor_sync(0xffffffffu, dcp[1].y, 12));
                r2 = __fadd2_rn(__fadd2_rn(r2, x1), __fadd2_rn(x2, x3));
                r2 = __fadd2_rn(r2, make_float2(__shfl_xor_sync(0xffffffffu, r2.x, 16),
                                                __shfl_xor_sync(0xffffffffu, r2.y, 16)));
                if (cw < 4) {
                    rot_dst[t] = r2.x;
                    rot_dst[NS * (TB + 1) + t] = r2.y;
                }
                if (CPL == 2 ? (j & 1) == 0 : j == 0) {
                    // sums over the 4 state lanes: lane g keeps block g -- with 2 channels
                    // (channel g / 2, odd token if g % 2) of this token pair, with 1 channel
                    // token g of the quad -- then finishes that token
                    reduce_scatter_contig<4, 8>(v, g);
                    const int tf = t + fo;
                    const float dlf = sD[fin_lc * RS + tf], dgf = sG[fin_lc * RS + tf];
                    const float uf = sU[fin_lc * RS + tf], spf = sSP[fin_lc * RS + tf];
                    const float duo = fmaf(Dd, dgf, dlf * v[0]);
                    const float ddo = fmaf(uf, v[0], kLn2 * v[1]) * spf;   // v[1]: sum of A*log2(e)*w
                    dD_acc = fmaf(dgf, uf, dD_acc);
                    db_acc += ddo;
                    *reinterpret_cast<IT*>(odu + out_off(fin_lc, tf)) = from_f<IT>(duo);
                    *reinterpret_cast<IT*>(odd + out_off(fin_lc, tf)) = from_f<IT>(ddo);
                }
            }
        };

        // ---- 8-token sub-tiles, last to first (unrolled: every shared-memory offset of a
        // token is then a compile-time constant) ------------------------------------------------
#pragma unroll
        for (int sub = TB / K - 1; sub >= 0; sub--) {
            const int tl0 = sub * K;
            const int ts = t0 + tl0;
            if (ts >= Lq) continue;   // past the end of the sequence: nothing to do
            // the state before the sub-tile: its checkpoint (staged with the tile), or h_init
            float2 h0[CPL][2];
            const float* ck = ckb + sub * DT * NS;
#pragma unroll
            for (int c = 0; c < CPL; c++) {
                const float* row = ck + (lc0 + 8 * c) * NS;
                const bool from_init = ts == 0 && p.h_init != nullptr;
                const float* src = from_init ? p.h_init + ((int64_t)b * Dm + (dv[c] ? dch[c] : 0)) * NS : row;
#pragma unroll
                for (int s = 0; s < 4; s++) {
                    const float v = (!from_init || dv[c]) ? src[4 * g + (s ^ rot)] : 0.f;
                    if (s & 1) h0[c][s / 2].y = v; else h0[c][s / 2].x = v;
                }
            }
            // the state before the second quad: run the first quad's 4 tokens without keeping them
            float2 hm[CPL][2];
            {
                float4 dlA[CPL], duA[CPL];
#pragma unroll
                for (int c = 0; c < CPL; c++) {
                    dlA[c] = lds128(sD + (lc0 + 8 * c) * RS + tl0);
                    duA[c] = lds128(sDU + (lc0 + 8 * c) * RS + tl0);
#pragma unroll
                    for (int q = 0; q < 2; q++) hm[c][q] = h0[c][q];
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float2 bp[2];
                    load_state_pairs<4, NS>(sBr, tl0 + j, g, j, bp);
#pragma unroll
                    for (int c = 0; c < CPL; c++) {
                        const float dl = j == 0 ? dlA[c].x : j == 1 ? dlA[c].y : j == 2 ? dlA[c].z : dlA[c].w;
                        const float du = j == 0 ? duA[c].x : j == 1 ? duA[c].y : j == 2 ? duA[c].z : duA[c].w;
                        const float2 dl2 = make_float2(dl, dl), du2 = make_float2(du, du);
#pragma unroll
                        for (int q = 0; q < 2; q++) {
                            const float2 x = __fmul2_rn(dl2, A2[c][q]);
                            const float2 a = make_float2(ex2(x.x), ex2(x.y));
                            hm[c][q] = __ffma2_rn(a, hm[c][q], __fmul2_rn(du2, bp[q]));
                        }
                    }
                }
            }
            quad(tl0 + 4, hm);
            quad(tl0, h0);
            // gradient of the initial state: decay of token 0 times dh_0
            if (ts == 0 && p.dh_init != nullptr) {
#pragma unroll
                for (int c = 0; c < CPL; c++) {
                    if (!dv[c]) continue;
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        const float val = (s & 1) ? anp[c][s / 2].y * Gp[c][s / 2].y : anp[c][s / 2].x * Gp[c][s / 2].x;
                        p.dh_init[((int64_t)b * Dm + dch[c]) * NS + 4 * g + (s ^ rot)] = val;
                    }
                }
            }
        }
        __syncthreads();

        // ---- CTA sum of the warp dB/dC slots -> workspace; store du, ddelta, dz -------------
        {
            const int nw = nthr >> 5;
            const int t = tid % TB;
            const int rstep = nthr / TB;
            if (t0 + t < Lq) {
                float* dst = ws_bc_row + (int64_t)(tid / TB) * Lq + t0 + t;
                const int64_t dstep = (int64_t)rstep * Lq;
                const int sstride = (int)S.slot_stride;
                for (int r = tid / TB; r < 2 * NS; r += rstep, dst += dstep) {
                    const float* src = slots + r * (TB + 1) + t;
                    float acc = src[0];
#pragma unroll
                    for (int w = 1; w < 4; w++)
                        if (w < nw) acc += src[w * sstride];
                    *dst = acc;
                }
            }
        }
        if (tid == 0) {
            fence_proxy_async_smem();
            tma_store_3d(&tm_du, odu, t0, d0, b);
            tma_store_3d(&tm_ddelta, odd, t0, d0, b);
            if (has_z) tma_store_3d(&tm_dz, smem + S.dz, t0, d0, b);
            tma_store_commit();
        }
    }

    // ---- per-(batch, channel) partials of dA, dD, ddelta_bias --------------------------------
#pragma unroll
    for (int c = 0; c < CPL; c++) {
        if (!dv[c]) continue;
#pragma unroll
        for (int s = 0; s < 4; s++) {
            const float val = (s & 1) ? dAp[c][s / 2].y : dAp[c][s / 2].x;
            p.ws_a[((int64_t)b * Dm + dch[c]) * NS + 4 * g + (s ^ rot)] = val;
        }
    }
    // the lanes that finished tokens of the same channel: g and g ^ 1 (2 channels), all 4 (1)
    dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, 1);
    db_acc += __shfl_xor_sync(0xffffffffu, db_acc, 1);
    if (CPL == 1) {
        dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, 2);
        db_acc += __shfl_xor_sync(0xffffffffu, db_acc, 2);
    }
    if (fo == 0 && fin_ok) {
        p.ws_dd[((int64_t)b * Dm + fin_d) * 2 + 0] = dD_acc;
        p.ws_dd[((int64_t)b * Dm + fin_d) * 2 + 1] = db_acc;
    }
    if (tid == 0) tma_store_wait_all();
}

// ---------------------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------------------
size_t bwd_pair_smem_bytes(int is_bf16, int cpl, int dt, int has_z) {
    return bwd_pair_smem_layout(dt, dt * 4 / cpl / 32, is_bf16 ? 2 : 4, has_z).total;
}

template <typename IT, int CPL>
static const void* pair_kernel() { return (const void*)scan_bwd_pair_kernel<IT, CPL>; }

int bwd_pair_occupancy(int is_bf16, int cpl, int dt, int has_z) {
    const void* k = cpl == 2 ? (is_bf16 ? pair_kernel<__nv_bfloat16, 2>() : pair_kernel<float, 2>())
                             : (is_bf16 ? pair_kernel<__nv_bfloat16, 1>() : pair_kernel<float, 1>());
    const size_t smem = bwd_pair_smem_bytes(is_bf16, cpl, dt, has_z);
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, dt * 4 / cpl, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_scan_bwd_pair(const BwdParams& p, int is_bf16, int cpl, const CUtensorMap* maps,
                                 cudaStream_t stream) {
    if (p.dstate != kPairNS || (cpl != 1 && cpl != 2) || p.dt % (8 * cpl) != 0 || p.dt < 8 * cpl ||
        p.dt * 4 / cpl > 128 || !p.use_tma || p.length)
        return cudaErrorInvalidValue;
    const size_t smem = bwd_pair_smem_bytes(is_bf16, cpl, p.dt, p.z != nullptr);
    auto run = [&](auto kern) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        kern<<<p.batch * p.ntile_d, p.dt * 4 / cpl, smem, stream>>>(p, maps[0], maps[1], maps[2], maps[3], maps[4],
                                                                   maps[5], maps[6], maps[7], maps[8], maps[9],
                                                                   maps[10]);
        return cudaGetLastError();
    };
    if (cpl == 2) return is_bf16 ? run(scan_bwd_pair_kernel<__nv_bfloat16, 2>) : run(scan_bwd_pair_kernel<float, 2>);
    return is_bf16 ? run(scan_bwd_pair_kernel<__nv_bfloat16, 1>) : run(scan_bwd_pair_kernel<float, 1>);
}

}  // namespace ssm
