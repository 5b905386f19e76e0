// Backward selective scan for sm_100a, d_state 16 without `length`: the lane layout for
// shapes with few rows (config 2: 12 288 rows), beside scan_bwd_pair_kernel.
//
// Same gradients as the reference backward (nmquan1503/ssm-mamba,
// csrc/selective_scan/backward_kernel.cu:212-452) and as scan_bwd_pair_kernel, whose tile
// pipeline (TMA stage per 16-token tile, checkpoints every 8 tokens staged with the tile,
// 1.5 exp2 per element, warp slots + per-CTA workspace for dB / dC) this kernel shares.  What
// differs is the lane layout, chosen to move fewer bytes through shared memory and shuffles
// per element while keeping one warp per 8 channels:
//
//  * Lane (cp, g) -- channel pair cp = lane / 8, state pair g = lane % 8 -- holds states
//    2g, 2g+1 of two channels of the warp's 8 (cp and cp + 4).  A token's B and C values are
//    then 8-byte loads serving 4 elements (scan_bwd_pair_kernel with one channel per lane:
//    16-byte loads of 4 states, from 4 rotated copies, for 4 elements), and dB / dC are summed
//    over the lane's two channels in registers before crossing 4 lanes instead of 8.
//  * dB / dC: register s of a lane holds state 2g + (s ^ r), r = cp % 2 (B and C are staged
//    in 2 copies with the pairs in either order), so the transpose-reduce over the 4 channel
//    pairs is one select-free shuffle stage and one all-reduce stage.
//  * du / ddelta (sums over the 16 states = 8 lanes): slot c of a lane holds channel
//    cp + 4 (c ^ (g / 4)), so the first of the three reduction stages (lanes g, g ^ 4) sends
//    slot 1 and keeps slot 0 without selects; the other two reduce-scatter the quad's tokens.
//    Each lane then finishes one (channel, token) of the quad.
#include "common.cuh"
#include "params.h"
#include "scan_layout.h"
#include "warp_reduce.cuh"
#include "bwd_prologue.cuh"

namespace ssm {

namespace {
constexpr float kLn2s = 0.6931471805599453f;
constexpr int kSplitNS = 16;   // states (exactly 16)
constexpr int kSplitK = 8;     // checkpoint interval (tokens)

__device__ __forceinline__ float2 lds64(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float pick4(const float4& v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}
}  // namespace

template <typename IT>
__global__ void __launch_bounds__(128) scan_bwd_split_kernel(
    const __grid_constant__ BwdParams p, const __grid_constant__ CUtensorMap tm_u,
    const __grid_constant__ CUtensorMap tm_delta, const __grid_constant__ CUtensorMap tm_dout,
    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_y,
    const __grid_constant__ CUtensorMap tm_B, const __grid_constant__ CUtensorMap tm_C,
    const __grid_constant__ CUtensorMap tm_du, const __grid_constant__ CUtensorMap tm_ddelta,
    const __grid_constant__ CUtensorMap tm_dz, const __grid_constant__ CUtensorMap tm_ck) {
    constexpr int ES = sizeof(IT);
    constexpr int TB = kBwdTile;
    constexpr int NS = kSplitNS;
    constexpr int K = kSplitK;
    constexpr int RS = TB + 4;
    static_assert(TB == 2 * K && K == 8, "tiles of two 8-token sub-tiles");

    extern __shared__ __align__(1024) unsigned char smem[];
    if ((smem_u32(smem) & 1023u) != 0u) {
        if (threadIdx.x == 0) atomicExch(p.err, kDevErrSmemAlign);
        return;
    }
    const int DT = p.dt;                        // channels per CTA, a multiple of 8
    const int nthr = DT * 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane & 7, cp = lane >> 3;
    const int r = cp & 1;                       // state order within the lane's pair
    const int sw = g >> 2;                      // channel order of the lane's two slots
    int lc[2];                                  // CTA-local channel rows of slots 0, 1
    lc[0] = warp * 8 + cp + 4 * sw;
    lc[1] = warp * 8 + cp + 4 * (sw ^ 1);
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

    // ---- per-lane constants: 2 channels x 1 pair of states (x: state 2g + r, y: 2g + 1 - r) --
    const int n0 = 2 * g + r, n1 = 2 * g + (r ^ 1);
    int dch[2];
    bool dv[2];
    float2 A2[2], Gp[2], anp[2], dAp[2];
#pragma unroll
    for (int c = 0; c < 2; c++) {
        dch[c] = d0 + lc[c];
        dv[c] = dch[c] < Dm;
        const float* Arow = p.A + (int64_t)(dv[c] ? dch[c] : 0) * p.A_sd;
        A2[c] = dv[c] ? make_float2(Arow[n0] * kLog2e, Arow[n1] * kLog2e) : make_float2(0.f, 0.f);
        const float* gl = p.dh_last ? p.dh_last + ((int64_t)b * Dm + (dv[c] ? dch[c] : 0)) * NS : nullptr;
        Gp[c] = (dv[c] && gl) ? make_float2(gl[n0], gl[n1]) : make_float2(0.f, 0.f);
        anp[c] = make_float2(1.f, 1.f);
        dAp[c] = make_float2(0.f, 0.f);
    }
    // the finishing role of this lane: token g % 4 of every quad, of the channel in slot 0
    const int fin_lc = lc[0], fin_d = dch[0];
    const bool fin_ok = dv[0];
    const float Dd = (fin_ok && p.D) ? p.D[fin_d] : 0.f;
    float dD_acc = 0.f, db_acc = 0.f;
    for (int i = tid; i < DT; i += nthr) sBias[i] = (d0 + i < Dm && p.delta_bias) ? p.delta_bias[d0 + i] : 0.f;

    const int ntiles = (Lq + TB - 1) / TB;
    float* const ws_bc_row = p.ws_bc + (((int64_t)tile_d * p.batch + b) * 2) * NS * (int64_t)Lq;
    const uint32_t tile_bytes = (uint32_t)DT * TB * ES;
    const uint32_t bc_bytes = (uint32_t)NS * TB * ES;
    const uint32_t ck_bytes = 2u * (uint32_t)DT * NS * 4u;
    const uint32_t stage_bytes = (has_z ? 5u : 3u) * tile_bytes + 2u * bc_bytes + ck_bytes;

    // tile `tile`: its raw tiles (dense rows) and the checkpoints its two sub-tiles restart
    // from (checkpoints t0/8 - 1 and t0/8; index -1 reads as zeros) into buffer tile % 2
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
    auto out_off = [](int row, int t) -> uint32_t { return ES == 2 ? swz32(row, t * ES) : swz64(row, t * ES); };
    auto raw_off = [](int row, int t) -> uint32_t { return (uint32_t)(row * TB + t) * ES; };

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

        // ---- prologue: 4 tokens of one channel per work item -------------------------------
        const bool tile_short = t0 + TB > Lq;
        for (int i = tid; i < DT * (TB / 4); i += nthr) {
            const int cc = i / (TB / 4), t4 = (i % (TB / 4)) * 4;
            bwd_prologue_item<IT, RS>(smem, S, cc, t4, raw_off(cc, t4), out_off(cc, t4), sBias[cc], has_z,
                                      p.delta_softplus != 0, tile_short, t0 + t4, Lq);
        }
        // B, C as float32 rows [token][16 states] in 2 copies: copy r holds each pair of
        // states in the order s ^ r.  Copy 1 starts 16 floats (64 bytes) past a multiple of
        // 32 banks from copy 0, so a half warp's 8-byte loads of one token's row from both
        // copies (128 bytes) fall in distinct banks.
        for (int i = tid; i < 4 * TB; i += nthr) {
            const int q = i & 3, tt = i >> 2;
            float vb[4], vc[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t off = raw_off(q * 4 + k, tt);
                vb[k] = to_f(*reinterpret_cast<const IT*>(smem + S.B + off));
                vc[k] = to_f(*reinterpret_cast<const IT*>(smem + S.C + off));
            }
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int pos = rr * (int)S.rot_stride + tt * NS + 4 * q;
                *reinterpret_cast<float4*>(sB + pos) = make_float4(vb[0 ^ rr], vb[1 ^ rr], vb[2 ^ rr], vb[3 ^ rr]);
                *reinterpret_cast<float4*>(sC + pos) = make_float4(vc[0 ^ rr], vc[1 ^ rr], vc[2 ^ rr], vc[3 ^ rr]);
            }
        }
        __syncthreads();
        if (tid == 0 && it > 0 && !p.test_withhold) issue(it - 1);   // raw tiles consumed

        unsigned char* odu = smem + S.du;
        unsigned char* odd = smem + S.ddelta;
        float* const wslot = slots + warp * (int)S.slot_stride;
        float* const rot_dst = wslot + (2 * g + cp) * (TB + 1);   // lanes cp < 2: state 2g + cp
        const float* const sBr = sB + r * (int)S.rot_stride + 2 * g;
        const float* const sCr = sC + r * (int)S.rot_stride + 2 * g;
        const float* const ckb = reinterpret_cast<const float*>(smem + ((it & 1) ? S.ck[1] : S.ck[0]));

        // one quad of 4 tokens (tile tokens tq .. tq+3) from hs, the state before it:
        // recompute (decays and states into registers), reverse recurrence, dB/dC into the
        // warp slots, then the quad's sums over states and du / ddelta of one token per lane
        auto quad = [&](int tq, const float2 (&hs)[2]) {
            float4 dl4[2], du4[2], dg4[2];
#pragma unroll
            for (int c = 0; c < 2; c++) {
                dl4[c] = lds128(sD + lc[c] * RS + tq);
                du4[c] = lds128(sDU + lc[c] * RS + tq);
                dg4[c] = lds128(sG + lc[c] * RS + tq);
            }
            float2 av[4][2], hv[4][2], bq[4];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                bq[j] = lds64(sBr + (tq + j) * NS);
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const float dl = pick4(dl4[c], j), du = pick4(du4[c], j);
                    const float2 x = __fmul2_rn(make_float2(dl, dl), A2[c]);
                    const float2 a = make_float2(ex2(x.x), ex2(x.y));
                    const float2 prev = j == 0 ? hs[c] : hv[j - 1][c];
                    av[j][c] = a;
                    hv[j][c] = __ffma2_rn(a, prev, __fmul2_rn(make_float2(du, du), bq[j]));
                }
            }
            // (S1, S2) partials of the quad: v[8c + 2j + k], slot c, token j
            float v[16];
#pragma unroll
            for (int j = 3; j >= 0; j--) {
                const int t = tq + j;
                const float2 cq = lds64(sCr + t * NS);
                float2 dbp, dcp;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const float dl = pick4(dl4[c], j), du = pick4(du4[c], j), dg = pick4(dg4[c], j);
                    const float2 dl2 = make_float2(dl, dl), du2 = make_float2(du, du), dg2 = make_float2(dg, dg);
                    const float2 Gs = __ffma2_rn(anp[c], Gp[c], __fmul2_rn(dg2, cq));
                    Gp[c] = Gs;
                    anp[c] = av[j][c];
                    const float2 prev = j == 0 ? hs[c] : hv[j - 1][c];
                    const float2 w = __fmul2_rn(Gs, __fmul2_rn(av[j][c], prev));
                    const float2 s12 = __fmul2_rn(Gs, bq[j]);
                    const float2 s22 = __fmul2_rn(A2[c], w);
                    dAp[c] = __ffma2_rn(dl2, w, dAp[c]);
                    if (c == 0) {
                        dbp = __fmul2_rn(Gs, du2);
                        dcp = __fmul2_rn(dg2, hv[j][c]);
                    } else {
                        dbp = __ffma2_rn(Gs, du2, dbp);
                        dcp = __ffma2_rn(dg2, hv[j][c], dcp);
                    }
                    v[8 * c + 2 * j] = s12.x + s12.y;
                    v[8 * c + 2 * j + 1] = s22.x + s22.y;
                }
                // dB, dC of this token summed over the warp's 8 channels: register 0 of lane
                // (cp, g) is state 2g + r, which its xor-8 partner (other r) holds in register 1
                float2 r2 = make_float2(dbp.x + __shfl_xor_sync(0xffffffffu, dbp.y, 8),
                                        dcp.x + __shfl_xor_sync(0xffffffffu, dcp.y, 8));
                r2 = __fadd2_rn(r2, make_float2(__shfl_xor_sync(0xffffffffu, r2.x, 16),
                                                __shfl_xor_sync(0xffffffffu, r2.y, 16)));
                if (cp < 2) {
                    rot_dst[t] = r2.x;
                    rot_dst[NS * (TB + 1) + t] = r2.y;
                }
            }
            // sums over the 8 state lanes: lanes g and g ^ 4 hold the same two channels in
            // opposite slots, so slot 1 goes to the partner's slot 0; then lane g keeps token
            // g % 4 of its slot-0 channel
            float w8[8];
#pragma unroll
            for (int i = 0; i < 8; i++) w8[i] = v[i] + __shfl_xor_sync(0xffffffffu, v[8 + i], 4);
            reduce_scatter_contig<4, 8>(w8, g);
            const int tf = tq + (g & 3);
            const float dlf = sD[fin_lc * RS + tf], dgf = sG[fin_lc * RS + tf];
            const float uf = sU[fin_lc * RS + tf], spf = sSP[fin_lc * RS + tf];
            const float duo = fmaf(Dd, dgf, dlf * w8[0]);
            const float ddo = fmaf(uf, w8[0], kLn2s * w8[1]) * spf;   // w8[1]: sum of A*log2(e)*w
            dD_acc = fmaf(dgf, uf, dD_acc);
            db_acc += ddo;
            *reinterpret_cast<IT*>(odu + out_off(fin_lc, tf)) = from_f<IT>(duo);
            *reinterpret_cast<IT*>(odd + out_off(fin_lc, tf)) = from_f<IT>(ddo);
        };

        // ---- 8-token sub-tiles, last to first -----------------------------------------------
#pragma unroll
        for (int sub = TB / K - 1; sub >= 0; sub--) {
            const int tl0 = sub * K;
            const int ts = t0 + tl0;
            if (ts >= Lq) continue;   // past the end of the sequence: nothing to do
            // the state before the sub-tile: its checkpoint (staged with the tile), or h_init
            float2 h0[2];
            const float* ck = ckb + sub * DT * NS;
#pragma unroll
            for (int c = 0; c < 2; c++) {
                const bool from_init = ts == 0 && p.h_init != nullptr;
                const float* src = from_init ? p.h_init + ((int64_t)b * Dm + (dv[c] ? dch[c] : 0)) * NS
                                             : ck + lc[c] * NS;
                const bool okc = !from_init || dv[c];
                h0[c] = okc ? make_float2(src[n0], src[n1]) : make_float2(0.f, 0.f);
            }
            // the state before the second quad: run the first quad's 4 tokens without keeping them
            float2 hm[2];
            {
                float4 dlA[2], duA[2];
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    dlA[c] = lds128(sD + lc[c] * RS + tl0);
                    duA[c] = lds128(sDU + lc[c] * RS + tl0);
                    hm[c] = h0[c];
                }
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 bp = lds64(sBr + (tl0 + j) * NS);
#pragma unroll
                    for (int c = 0; c < 2; c++) {
                        const float dl = pick4(dlA[c], j), du = pick4(duA[c], j);
                        const float2 x = __fmul2_rn(make_float2(dl, dl), A2[c]);
                        const float2 a = make_float2(ex2(x.x), ex2(x.y));
                        hm[c] = __ffma2_rn(a, hm[c], __fmul2_rn(make_float2(du, du), bp));
                    }
                }
            }
            quad(tl0 + 4, hm);
            quad(tl0, h0);
            // gradient of the initial state: decay of token 0 times dh_0
            if (ts == 0 && p.dh_init != nullptr) {
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    if (!dv[c]) continue;
                    float* dst = p.dh_init + ((int64_t)b * Dm + dch[c]) * NS;
                    dst[n0] = anp[c].x * Gp[c].x;
                    dst[n1] = anp[c].y * Gp[c].y;
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
                for (int rw = tid / TB; rw < 2 * NS; rw += rstep, dst += dstep) {
                    const float* src = slots + rw * (TB + 1) + t;
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
    for (int c = 0; c < 2; c++) {
        if (!dv[c]) continue;
        float* dst = p.ws_a + ((int64_t)b * Dm + dch[c]) * NS;
        dst[n0] = dAp[c].x;
        dst[n1] = dAp[c].y;
    }
    // the lanes that finished tokens of the same channel: g, g ^ 1, g ^ 2, g ^ 3
    dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, 1);
    db_acc += __shfl_xor_sync(0xffffffffu, db_acc, 1);
    dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, 2);
    db_acc += __shfl_xor_sync(0xffffffffu, db_acc, 2);
    if ((g & 3) == 0 && fin_ok) {
        p.ws_dd[((int64_t)b * Dm + fin_d) * 2 + 0] = dD_acc;
        p.ws_dd[((int64_t)b * Dm + fin_d) * 2 + 1] = db_acc;
    }
    if (tid == 0) tma_store_wait_all();
}

// ---------------------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------------------
int bwd_split_occupancy(int is_bf16, int dt, int has_z) {
    const void* k = is_bf16 ? (const void*)scan_bwd_split_kernel<__nv_bfloat16> : (const void*)scan_bwd_split_kernel<float>;
    const size_t smem = bwd_pair_smem_layout(dt, dt * 4 / 32, is_bf16 ? 2 : 4, has_z).total;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, dt * 4, smem) != cudaSuccess) return 0;
    return n;
}

cudaError_t launch_scan_bwd_split(const BwdParams& p, int is_bf16, const CUtensorMap* maps, cudaStream_t stream) {
    if (p.dstate != kSplitNS || p.dt % 8 != 0 || p.dt < 8 || p.dt * 4 > 128 || !p.use_tma || p.length)
        return cudaErrorInvalidValue;
    const size_t smem = bwd_pair_smem_layout(p.dt, p.dt * 4 / 32, is_bf16 ? 2 : 4, p.z != nullptr).total;
    auto run = [&](auto kern) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        kern<<<p.batch * p.ntile_d, p.dt * 4, smem, stream>>>(p, maps[0], maps[1], maps[2], maps[3], maps[4], maps[5],
                                                             maps[6], maps[7], maps[8], maps[9], maps[10]);
        return cudaGetLastError();
    };
    return is_bf16 ? run(scan_bwd_split_kernel<__nv_bfloat16>) : run(scan_bwd_split_kernel<float>);
}

}  // namespace ssm
