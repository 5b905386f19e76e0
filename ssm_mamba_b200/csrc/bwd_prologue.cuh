// The tile prologue shared by the pair-family backward kernels (scan_bwd_pair.cu,
// scan_bwd_split.cu): one work item is 4 consecutive tokens of one channel row of the staged
// raw tiles.  It computes delta = softplus(delta + bias) with its slope (the sigmoid), delta*u,
// and -- with a gate -- the gated output gradient dout * silu(z) and dz = dout * y * silu'(z)
// (stored to the dz output tile), then writes the float32 work rows.  Pairs of tokens go
// through packed f32x2 arithmetic with the same operations per element as the scalar forms.
#pragma once
#include "common.cuh"
#include "scan_layout.h"

namespace ssm {

template <typename IT, int RS>
__device__ __forceinline__ void bwd_prologue_item(unsigned char* smem, const BwdPairSmem& S, int cc, int t4,
                                                  uint32_t off_in, uint32_t off_dz, float bias, bool has_z,
                                                  bool softplus, bool tile_short, int tok0, int Lq) {
    float uv[4], dr[4], dg[4];
    Vec4<IT>::load(smem + S.u + off_in, uv);
    Vec4<IT>::load(smem + S.delta + off_in, dr);
    Vec4<IT>::load(smem + S.dout + off_in, dg);
    float dl[4], du[4], spg[4];
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
        const float2 x = make_float2(dr[j] + bias, dr[j + 1] + bias);
        float2 v = x, sl = make_float2(1.f, 1.f);
        if (softplus) {
            float2 t;
            v = softplus_series2(x, &t);
            sl = make_float2(sigmoid_from_t(x.x, t.x), sigmoid_from_t(x.y, t.y));
        }
        const float2 w = __fmul2_rn(v, make_float2(uv[j], uv[j + 1]));
        dl[j] = v.x; dl[j + 1] = v.y;
        spg[j] = sl.x; spg[j + 1] = sl.y;
        du[j] = w.x; du[j + 1] = w.y;
    }
    if (has_z) {
        float zv[4], yv[4], dz[4];
        Vec4<IT>::load(smem + S.z + off_in, zv);
        Vec4<IT>::load(smem + S.y + off_in, yv);
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const float2 z2 = make_float2(zv[j], zv[j + 1]);
            const float2 sg = make_float2(sigmoid_io<IT>(zv[j]), sigmoid_io<IT>(zv[j + 1]));
            const float2 g2 = make_float2(dg[j], dg[j + 1]);
            // dz = dout y sg (1 + z (1 - sg)),  dout * silu(z) = dout z sg
            const float2 slope = __ffma2_rn(z2, __fadd2_rn(make_float2(1.f, 1.f), make_float2(-sg.x, -sg.y)),
                                            make_float2(1.f, 1.f));
            const float2 d = __fmul2_rn(__fmul2_rn(__fmul2_rn(g2, make_float2(yv[j], yv[j + 1])), sg), slope);
            const float2 gg = __fmul2_rn(__fmul2_rn(g2, z2), sg);
            dz[j] = d.x; dz[j + 1] = d.y;
            dg[j] = gg.x; dg[j + 1] = gg.y;
        }
        Vec4<IT>::store(smem + S.dz + off_dz, dz);
    }
    if (tile_short) {
        // past the end of the sequence: identity steps that add nothing
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (tok0 + j >= Lq) { dl[j] = 0.f; du[j] = 0.f; dg[j] = 0.f; spg[j] = 0.f; uv[j] = 0.f; }
    }
    float* row = reinterpret_cast<float*>(smem) + cc * RS + t4;
    *reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(row) + S.sD) = make_float4(dl[0], dl[1], dl[2], dl[3]);
    *reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(row) + S.sDU) = make_float4(du[0], du[1], du[2], du[3]);
    *reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(row) + S.sG) = make_float4(dg[0], dg[1], dg[2], dg[3]);
    *reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(row) + S.sSP) = make_float4(spg[0], spg[1], spg[2], spg[3]);
    *reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(row) + S.sU) = make_float4(uv[0], uv[1], uv[2], uv[3]);
}

}  // namespace ssm
