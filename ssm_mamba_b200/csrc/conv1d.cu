// Causal depthwise conv1d + SiLU for sm_100a: the step in front of the selective scan.
//
// Replaces, in the reference (nmquan1503/ssm-mamba, modules/mamba.py):
//   prefill  hidden_states = silu(self.conv(hidden_states)[..., :seq_len])      (:137-139)
//            -- nn.Conv1d(groups=dim, padding=width-1) truncated to the first seqlen outputs,
//               i.e. out[t] = bias + sum_k w[k] x[t - (width-1) + k], x[< 0] = 0
//   context  the last width-1 inputs of every row (respecting `lengths`), kept for decode
//            (:114-133)
//   decode   conv_context = cat(context, x); out = silu(sum_k context[k] w[k] + bias);
//            context shifted by one (:203-213)
// and the backward of the prefill (autograd of the above in the reference).
//
// All three are HBM-bound streams.  A warp owns 32 consecutive 16-byte vectors of one
// (batch, channel) row (256 bf16 / 128 f32 tokens); each lane loads its vector and the
// previous one (the width-1 halo, an L2 hit), so every warp access is a contiguous
// 512-byte segment.  The backward recomputes the pre-activation from x (width FMAs) and
// also reads the next vector of x and dout for the forward halo of dx; dweight and dbias are
// summed over the lanes of a warp with shuffles and over warps through a workspace that a
// second kernel reduces in a fixed order (deterministic, no floating-point atomics).
#include "common.cuh"
#include "params.h"

namespace ssm {


template <typename IT, int VT>
__device__ __forceinline__ void load_vec(const IT* p, float (&v)[VT]) {
    if constexpr (VT == 8) {          // 8 bf16 = 16 bytes
        const uint4 r = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    } else if constexpr (VT == 4) {   // 4 f32 = 16 bytes
        const float4 r = *reinterpret_cast<const float4*>(p);
        v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
    } else {
        v[0] = to_f(*p);
    }
}

template <typename IT, int VT>
__device__ __forceinline__ void store_vec(IT* p, const float (&v)[VT]) {
    if constexpr (VT == 8) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    } else if constexpr (VT == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
        *p = from_f<IT>(v[0]);
    }
}

template <typename IT>
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_io<IT>(x); }

// xw[j] = row[t0 + lo + j] for j in [0, NW), zero outside [0, seqlen).  VT > 1: the window
// is covered by the 16-byte vectors v-1, v, v+1 (lo >= -VT, lo + NW <= 2 VT; seqlen is a
// multiple of VT); VT == 1: element loads.
template <typename IT, int VT, int NW>
__device__ __forceinline__ void load_window(const IT* row, int t0, int lo, int seqlen, float (&xw)[NW]) {
    if constexpr (VT == 1) {
#pragma unroll
        for (int j = 0; j < NW; j++) {
            const int t = t0 + lo + j;
            xw[j] = (t >= 0 && t < seqlen) ? to_f(row[t]) : 0.f;
        }
    } else {
        float prev[VT], cur[VT], next[VT];
        const bool need_prev = lo < 0, need_next = lo + NW > VT;
        load_vec<IT, VT>(row + t0, cur);
#pragma unroll
        for (int i = 0; i < VT; i++) prev[i] = next[i] = 0.f;
        if (need_prev && t0 > 0) load_vec<IT, VT>(row + t0 - VT, prev);
        if (need_next && t0 + VT < seqlen) load_vec<IT, VT>(row + t0 + VT, next);
#pragma unroll
        for (int j = 0; j < NW; j++) {
            const int q = lo + j;   // offset from t0, in [-VT, 2 VT)
            xw[j] = q < 0 ? prev[q + VT] : (q < VT ? cur[q] : next[q - VT]);
        }
    }
}

// Vectors per lane: a warp covers kConvRows * 32 consecutive vectors of one row, so the
// per-row setup (indices, weights) and the backward's weight-gradient partials are shared
// by kConvRows vectors.
constexpr int kConvRows = 4;

// out[t] = act(bias + sum_k w[k] x[t - (K-1) + k]).  Grid: x = blocks of 8 rows (one warp
// per row, row = b * dim + d), y = chunks of 32 * kConvRows vectors; lane = every 32nd vector.
template <typename IT, int VT, int K>
__global__ void __launch_bounds__(256) conv1d_fwd_kernel(const __grid_constant__ ConvParams p) {
    const int lane = threadIdx.x & 31;
    const int nvec = (p.seqlen + VT - 1) / VT;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= p.batch * p.dim) return;
    const int b = row / p.dim, d = row - b * p.dim;
    const IT* xr = static_cast<const IT*>(p.x) + b * p.x_sb + d * p.x_sd;
    IT* outr = static_cast<IT*>(p.out) + b * p.out_sb + d * p.out_sd;
    float w[K];
#pragma unroll
    for (int k = 0; k < K; k++) w[k] = __ldg(p.w + d * p.w_sd + k);
    const float bias = p.bias ? __ldg(p.bias + d) : 0.f;
    const int vbase = blockIdx.y * 32 * kConvRows + lane;
#pragma unroll
    for (int r = 0; r < kConvRows; r++) {
        const int v = vbase + 32 * r;
        if (v < nvec) {
            const int t0 = v * VT;
            float xw[VT + K - 1];   // x[t0 - (K-1) .. t0 + VT - 1]
            load_window<IT, VT, VT + K - 1>(xr, t0, -(K - 1), p.seqlen, xw);
            float o[VT];
#pragma unroll
            for (int i = 0; i < VT; i++) {
                float acc = bias;
#pragma unroll
                for (int k = 0; k < K; k++) acc = fmaf(w[k], xw[i + k], acc);
                o[i] = p.silu ? silu_f<IT>(acc) : acc;
            }
            store_vec<IT, VT>(outr + t0, o);
        }
    }
    // the decode context: inputs at [len - (K-1), len), zero before the row start; lane 0
    // of the warps of chunk 0
    if (p.state && blockIdx.y == 0 && lane == 0) {
        int len = p.seqlen;
        if (p.length) {
            const long long l = p.length[b];
            len = l < 0 ? 0 : (l > p.seqlen ? p.seqlen : (int)l);
        }
        IT* sr = static_cast<IT*>(p.state) + b * p.st_sb + d * p.st_sd;
#pragma unroll
        for (int j = 0; j < K - 1; j++) {
            const int t = len - (K - 1) + j;
            sr[j] = t >= 0 ? xr[t] : from_f<IT>(0.f);
        }
    }
}

// g[i] = dout[t0 + i] * act'(pre[t0 + i]) for the N tokens from t0, all inside the row,
// with xw = x[t0 - (K-1) .. t0 + N - 1] and dw = dout[t0 .. t0 + N - 1].
template <typename IT, int K, int N>
__device__ __forceinline__ void conv_grad_tokens(const float (&w)[K], float bias, bool silu, const float* xw,
                                                 const float* dw, float (&g)[N]) {
#pragma unroll
    for (int i = 0; i < N; i++) {
        float pre = bias;
#pragma unroll
        for (int k = 0; k < K; k++) pre = fmaf(w[k], xw[i + k], pre);
        float gi = dw[i];
        if (silu) {
            const float s = sigmoid_io<IT>(pre);
            gi *= s * (1.f + pre * (1.f - s));
        }
        g[i] = gi;
    }
}

// Backward.  g[t] = dout[t] * act'(pre[t]); dx[t] = sum_k w[k] g[t + (K-1) - k];
// dw[k] = sum g[t] x[t - (K-1) + k]; dbias = sum g[t].  The warp's partials of dw, dbias go
// to ws[(chunk * batch + b), d, :].
//
// With 16-byte vectors a lane computes g only for its own VT tokens; the K-1 tokens of g
// after them (the halo dx needs) are the first tokens of the next vector, which the next
// lane owns in the same round -- or, for lane 31, lane 0 in the next round.  So every round
// finishes the dx of the PREVIOUS round's vector, taking its halo by shuffles, and after the
// last round lane 31 computes the halo of the vector after the chunk itself.
template <typename IT, int VT, int K>
__global__ void __launch_bounds__(256) conv1d_bwd_kernel(const __grid_constant__ ConvParams p) {
    if constexpr (VT > 1) {
        const int lane = threadIdx.x & 31;
        const int nvec = p.seqlen / VT;
        const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
        if (row >= p.batch * p.dim) return;   // whole warps: the shuffles below see full warps
        const int b = row / p.dim, d = row - b * p.dim;
        const IT* xr = static_cast<const IT*>(p.x) + b * p.x_sb + d * p.x_sd;
        const IT* gr = static_cast<const IT*>(p.dout) + b * p.dout_sb + d * p.dout_sd;
        IT* dxr = static_cast<IT*>(p.dx) + b * p.dx_sb + d * p.dx_sd;
        float w[K];
#pragma unroll
        for (int k = 0; k < K; k++) w[k] = __ldg(p.w + d * p.w_sd + k);
        const float bias = p.bias ? __ldg(p.bias + d) : 0.f;
        float part[K + 1];
#pragma unroll
        for (int k = 0; k <= K; k++) part[k] = 0.f;
        const int vbase = blockIdx.y * 32 * kConvRows + lane;
        float gp[VT];                        // g of this lane's vector of the previous round
        // dx of the vector v from its g and the K-1 following values of g
        auto finish = [&](int v, const float (&gv)[VT], const float (&halo)[K - 1]) {
            if (v >= nvec) return;
            float dxv[VT];
#pragma unroll
            for (int i = 0; i < VT; i++) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < K; k++) {
                    const int j = i + (K - 1) - k;
                    acc = fmaf(w[k], j < VT ? gv[j] : halo[j - VT], acc);
                }
                dxv[i] = acc;
            }
            store_vec<IT, VT>(dxr + v * VT, dxv);
        };
#pragma unroll
        for (int r = 0; r < kConvRows; r++) {
            const int v = vbase + 32 * r;
            float g[VT];
            if (v < nvec) {
                const int t0 = v * VT;
                float xw[VT + K - 1];        // x[t0 - (K-1) .. t0 + VT - 1]
                float dv[VT];
                load_window<IT, VT, VT + K - 1>(xr, t0, -(K - 1), p.seqlen, xw);
                load_vec<IT, VT>(gr + t0, dv);
                conv_grad_tokens<IT, K, VT>(w, bias, p.silu, xw, dv, g);
#pragma unroll
                for (int i = 0; i < VT; i++) {
#pragma unroll
                    for (int k = 0; k < K; k++) part[k] = fmaf(g[i], xw[i + k], part[k]);
                    part[K] += g[i];
                }
            } else {
#pragma unroll
                for (int i = 0; i < VT; i++) g[i] = 0.f;
            }
            if (r > 0) {
                // halo of the previous round's vector: the next lane's previous g, or for
                // lane 31 lane 0's current g
                float halo[K - 1];
#pragma unroll
                for (int i = 0; i < K - 1; i++) {
                    const float nb = __shfl_down_sync(0xffffffffu, gp[i], 1);
                    const float l0 = __shfl_sync(0xffffffffu, g[i], 0);
                    halo[i] = lane == 31 ? l0 : nb;
                }
                finish(v - 32, gp, halo);
            }
#pragma unroll
            for (int i = 0; i < VT; i++) gp[i] = g[i];
        }
        {
            // the last round: lanes 0..30 take the next lane's g; lane 31 needs the first K-1
            // tokens after this chunk, computed here
            float halo[K - 1];
#pragma unroll
            for (int i = 0; i < K - 1; i++) halo[i] = __shfl_down_sync(0xffffffffu, gp[i], 1);
            const int vl = vbase + 32 * (kConvRows - 1);
            if (lane == 31 && vl + 1 < nvec) {
                const int t1 = (vl + 1) * VT;
                float xh[2 * K - 2];         // x[t1 - (K-1) .. t1 + K - 2]
                float dh[K - 1];
#pragma unroll
                for (int j = 0; j < 2 * K - 2; j++) xh[j] = to_f(xr[t1 - (K - 1) + j]);
#pragma unroll
                for (int j = 0; j < K - 1; j++) dh[j] = to_f(gr[t1 + j]);
                conv_grad_tokens<IT, K, K - 1>(w, bias, p.silu, xh, dh, halo);
            } else if (lane == 31) {
#pragma unroll
                for (int i = 0; i < K - 1; i++) halo[i] = 0.f;
            }
            finish(vl, gp, halo);
        }
#pragma unroll
        for (int k = 0; k <= K; k++) {
#pragma unroll
            for (int m = 16; m >= 1; m >>= 1) part[k] += __shfl_xor_sync(0xffffffffu, part[k], m);
        }
        if (lane == 0) {
            float* dst = p.ws + (((int64_t)blockIdx.y * p.batch + b) * p.dim + d) * (K + 1);
#pragma unroll
            for (int k = 0; k <= K; k++) dst[k] = part[k];
        }
        return;
    }
    // one token per lane (rows that are not 16-byte aligned): recompute the halo of g
    const int lane = threadIdx.x & 31;
    const int nvec = (p.seqlen + VT - 1) / VT;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= p.batch * p.dim) return;   // whole warps: the shuffles below see full warps
    const int b = row / p.dim, d = row - b * p.dim;
    const IT* xr = static_cast<const IT*>(p.x) + b * p.x_sb + d * p.x_sd;
    const IT* gr = static_cast<const IT*>(p.dout) + b * p.dout_sb + d * p.dout_sd;
    IT* dxr = static_cast<IT*>(p.dx) + b * p.dx_sb + d * p.dx_sd;
    float w[K];
#pragma unroll
    for (int k = 0; k < K; k++) w[k] = __ldg(p.w + d * p.w_sd + k);
    const float bias = p.bias ? __ldg(p.bias + d) : 0.f;
    float part[K + 1];
#pragma unroll
    for (int k = 0; k <= K; k++) part[k] = 0.f;
    const int vbase = blockIdx.y * 32 * kConvRows + lane;
#pragma unroll
    for (int r = 0; r < kConvRows; r++) {
        const int v = vbase + 32 * r;
        if (v < nvec) {
            const int t0 = v * VT;
            constexpr int NG = VT + K - 1;          // tokens t0 .. t0 + VT + K - 2
            float xw[NG + K - 1];                   // x[t0 - (K-1) .. t0 + VT + K - 2]
            float gw[NG];                           // dout[t0 .. t0 + VT + K - 2]
            load_window<IT, VT, NG + K - 1>(xr, t0, -(K - 1), p.seqlen, xw);
            load_window<IT, VT, NG>(gr, t0, 0, p.seqlen, gw);
            float g[NG];
#pragma unroll
            for (int i = 0; i < NG; i++) {
                float pre = bias;
#pragma unroll
                for (int k = 0; k < K; k++) pre = fmaf(w[k], xw[i + k], pre);
                float gi = gw[i];
                if (p.silu) {
                    const float s = sigmoid_io<IT>(pre);
                    gi *= s * (1.f + pre * (1.f - s));
                }
                g[i] = (t0 + i < p.seqlen) ? gi : 0.f;
            }
            float dxv[VT];
#pragma unroll
            for (int i = 0; i < VT; i++) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < K; k++) acc = fmaf(w[k], g[i + (K - 1) - k], acc);
                dxv[i] = acc;
#pragma unroll
                for (int k = 0; k < K; k++) part[k] = fmaf(g[i], xw[i + k], part[k]);
                part[K] += g[i];
            }
            store_vec<IT, VT>(dxr + t0, dxv);
        }
    }
#pragma unroll
    for (int k = 0; k <= K; k++) {
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) part[k] += __shfl_xor_sync(0xffffffffu, part[k], m);
    }
    if (lane == 0) {
        float* dst = p.ws + (((int64_t)blockIdx.y * p.batch + b) * p.dim + d) * (K + 1);
#pragma unroll
        for (int k = 0; k <= K; k++) dst[k] = part[k];
    }
}

// dweight[d, k] and dbias[d]: sums of the nparts partials, one warp per value; lane j sums
// partials j, j + 32, ... and the warp adds the lanes in a fixed tree (deterministic).
__global__ void conv1d_reduce_kernel(const float* __restrict__ ws, int nparts, int dim, int width,
                                     float* __restrict__ dw, int64_t dw_sd, float* __restrict__ dbias) {
    const int lane = threadIdx.x & 31;
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);   // (d, k) flat
    if (i >= dim * (width + 1)) return;
    const int d = i / (width + 1), k = i - d * (width + 1);
    float acc = 0.f;
    for (int q = lane; q < nparts; q += 32) acc += ws[((int64_t)q * dim + d) * (width + 1) + k];
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
    if (lane == 0) {
        if (k < width) dw[d * dw_sd + k] = acc;
        else if (dbias) dbias[d] = acc;
    }
}

// One decode step: out = act(sum_{k < K-1} state[k] w[k] + x w[K-1] + bias); the state
// shifts by one and takes x.  Thread per (batch, channel); state may be updated in place.
template <typename IT, int K>
__global__ void __launch_bounds__(256) conv1d_update_kernel(const __grid_constant__ ConvParams p) {
    // grid: x = batch rows, y = tiles of 256 channels
    const int b = blockIdx.x, d = blockIdx.y * 256 + threadIdx.x;
    if (d < p.dim) {
        IT* sr = static_cast<IT*>(p.state) + b * p.st_sb + d * p.st_sd;
        const float x = to_f(static_cast<const IT*>(p.x)[b * p.x_sb + d * p.x_sd]);
        float win[K];
#pragma unroll
        for (int k = 0; k < K - 1; k++) win[k] = to_f(sr[k]);
        win[K - 1] = x;
        float acc = p.bias ? __ldg(p.bias + d) : 0.f;
#pragma unroll
        for (int k = 0; k < K; k++) acc = fmaf(__ldg(p.w + d * p.w_sd + k), win[k], acc);
#pragma unroll
        for (int k = 0; k < K - 1; k++) sr[k] = from_f<IT>(win[k + 1]);
        static_cast<IT*>(p.out)[b * p.out_sb + d * p.out_sd] = from_f<IT>(p.silu ? silu_f<IT>(acc) : acc);
    }
}

// ---------------------------------------------------------------------------------------
// launch
// ---------------------------------------------------------------------------------------
template <typename IT, int VT>
static cudaError_t launch_conv_vt(const ConvParams& p, int width, int kind, int sms, cudaStream_t s) {
    (void)sms;
    const dim3 grid((unsigned)((p.batch * p.dim + 7) / 8), (unsigned)p.nchunk);
#define SSM_CONV_K(K_)                                                                         \
    if (width == K_) {                                                                         \
        if (kind == 0) conv1d_fwd_kernel<IT, VT, K_><<<grid, 256, 0, s>>>(p);                  \
        else conv1d_bwd_kernel<IT, VT, K_><<<grid, 256, 0, s>>>(p);                            \
        return cudaGetLastError();                                                             \
    }
    SSM_CONV_K(2) SSM_CONV_K(3) SSM_CONV_K(4)
#undef SSM_CONV_K
    return cudaErrorInvalidValue;
}

// kind 0 forward, 1 backward; vec: 16-byte vectors along the sequence (else one token per lane)
cudaError_t launch_conv1d(const ConvParams& p, int is_bf16, int width, int kind, int vec, int sms,
                          cudaStream_t stream) {
    if (is_bf16)
        return vec ? launch_conv_vt<__nv_bfloat16, 8>(p, width, kind, sms, stream)
                   : launch_conv_vt<__nv_bfloat16, 1>(p, width, kind, sms, stream);
    return vec ? launch_conv_vt<float, 4>(p, width, kind, sms, stream)
               : launch_conv_vt<float, 1>(p, width, kind, sms, stream);
}

cudaError_t launch_conv1d_reduce(const float* ws, int nparts, int dim, int width, float* dw, int64_t dw_sd,
                                 float* dbias, int sms, cudaStream_t stream) {
    (void)sms;
    const int warps = dim * (width + 1);
    conv1d_reduce_kernel<<<(warps + 7) / 8, 256, 0, stream>>>(ws, nparts, dim, width, dw, dw_sd, dbias);
    return cudaGetLastError();
}

cudaError_t launch_conv1d_update(const ConvParams& p, int is_bf16, int width, int sms, cudaStream_t stream) {
    (void)sms;
    const dim3 grid((unsigned)p.batch, (unsigned)((p.dim + 255) / 256));
#define SSM_CONVU_K(K_)                                                                          \
    if (width == K_) {                                                                           \
        if (is_bf16) conv1d_update_kernel<__nv_bfloat16, K_><<<grid, 256, 0, stream>>>(p);       \
        else conv1d_update_kernel<float, K_><<<grid, 256, 0, stream>>>(p);                       \
        return cudaGetLastError();                                                               \
    }
    SSM_CONVU_K(2) SSM_CONVU_K(3) SSM_CONVU_K(4)
#undef SSM_CONVU_K
    return cudaErrorInvalidValue;
}

}  // namespace ssm
