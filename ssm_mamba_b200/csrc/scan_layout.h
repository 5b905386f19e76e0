// Shared-memory layouts of the scan kernels, computed identically on host (to size the
// launch) and device (to carve the buffer).  Offsets are bytes from a 1024-aligned base.
#pragma once

#include <stdint.h>

namespace ssm {

__host__ __device__ inline uint32_t align_up(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }

// ---- forward: 2 raw stages of 128-byte rows (TMA 128B swizzle), f32 work rows ----------
struct FwdSmem {
    uint32_t u[2], delta[2], z[2], B[2], C[2];
    uint32_t out, y, sD, sDU, sB, sC, bias, bar, total;
};

__host__ __device__ inline FwdSmem fwd_smem_layout(int dt, int ns, int es, int has_z, int has_y) {
    FwdSmem L;
    const int T = 128 / es;
    const uint32_t tile = align_up((uint32_t)dt * 128u, 1024u);
    const uint32_t bc = align_up((uint32_t)ns * 128u, 1024u);
    uint32_t o = 0;
    for (int s = 0; s < 2; s++) {
        L.u[s] = o; o += tile;
        L.delta[s] = o; o += tile;
        L.z[s] = o; o += has_z ? tile : 0u;
        L.B[s] = o; o += bc;
        L.C[s] = o; o += bc;
    }
    L.out = o; o += tile;
    L.y = o; o += has_y ? tile : 0u;
    const uint32_t rows = align_up((uint32_t)dt * (T + 4) * 4u, 128u);
    L.sD = o; o += rows;
    L.sDU = o; o += rows;
    L.sB = o; o += (uint32_t)T * ns * 4u;
    L.sC = o; o += (uint32_t)T * ns * 4u;
    L.bias = o; o += align_up((uint32_t)dt * 4u, 16u);
    L.bar = align_up(o, 8u); o = L.bar + 16u;
    L.total = o;
    return L;
}

// ---- sequence-slice carries (scan_chunk.cu): 2 raw stages, f32 work rows ---------------
// forward: raw tiles x0 = u, x1 = delta, x3 = B (state rows);
// reverse: raw tiles x0 = dout, x1 = delta, x2 = z (optional), x3 = C (state rows).
struct ChunkSmem {
    uint32_t x0[2], x1[2], x2[2], x3[2];
    uint32_t sD, sX, sM, bias, bar, total;
};

__host__ __device__ inline ChunkSmem chunk_smem_layout(int dt, int ns, int es, int has_z) {
    ChunkSmem L;
    const int T = 128 / es;
    const uint32_t tile = align_up((uint32_t)dt * 128u, 1024u);
    const uint32_t bc = align_up((uint32_t)ns * 128u, 1024u);
    uint32_t o = 0;
    for (int s = 0; s < 2; s++) {
        L.x0[s] = o; o += tile;
        L.x1[s] = o; o += tile;
        L.x2[s] = o; o += has_z ? tile : 0u;
        L.x3[s] = o; o += bc;
    }
    const uint32_t rows = align_up((uint32_t)dt * (T + 4) * 4u, 128u);
    L.sD = o; o += rows;
    L.sX = o; o += rows;
    L.sM = o; o += (uint32_t)T * ns * 4u;
    L.bias = o; o += align_up((uint32_t)dt * 4u, 16u);
    L.bar = align_up(o, 8u); o = L.bar + 16u;
    L.total = o;
    return L;
}

// ---- backward: one raw stage of 32-token tiles, f32 work rows, rotated B/C copies ------
constexpr int kBwdTile = 16;   // tokens per backward tile

struct BwdSmem {
    uint32_t du, ddelta, dz;                          // output tiles (TMA store, swizzled)
    uint32_t u, delta, dout, z, y, B, C;              // raw tiles (TMA load, dense rows)
    uint32_t sD, sDU, sG, sSP, sU;                    // f32 [dt][TB+4]
    uint32_t sB, sC;                                  // f32 [nrot][TB*ns + 16]
    uint32_t slots;                                   // f32 [nwarps][2][ns][TB+1]
    uint32_t xch;                                     // f32 [nwarps][32][xch_stride]
    uint32_t bias;                                    // f32 [dt]
    uint32_t bar, total;
    uint32_t rot_stride;                              // floats between rotated copies
    uint32_t slot_stride;                             // floats between warp slots
    uint32_t xch_stride;                              // floats per lane in the exchange area
};

__host__ __device__ inline BwdSmem bwd_smem_layout(int dt, int ns, int n, int es, int nrot,
                                                   int nwarps, int has_z, int ksub) {
    BwdSmem L;
    const int TB = kBwdTile;
    const uint32_t row = (uint32_t)TB * es;               // 64 (bf16) or 128 (f32) bytes
    const uint32_t otile = align_up((uint32_t)dt * row, 512u);
    const uint32_t tile = align_up((uint32_t)dt * row, 128u);
    const uint32_t bc = align_up((uint32_t)n * row, 128u);
    uint32_t o = 0;
    L.du = o; o += otile;
    L.ddelta = o; o += otile;
    L.dz = o; o += has_z ? otile : 0u;
    L.u = o; o += tile;
    L.delta = o; o += tile;
    L.dout = o; o += tile;
    L.z = o; o += has_z ? tile : 0u;
    L.y = o; o += has_z ? tile : 0u;
    L.B = o; o += bc;
    L.C = o; o += bc;
    const uint32_t rows = align_up((uint32_t)dt * (TB + 4) * 4u, 128u);
    L.sD = o; o += rows;
    L.sDU = o; o += rows;
    L.sG = o; o += rows;
    L.sSP = o; o += rows;
    L.sU = o; o += rows;
    L.rot_stride = (uint32_t)TB * ns + 16u;
    L.sB = o; o += align_up((uint32_t)nrot * L.rot_stride * 4u, 128u);
    L.sC = o; o += align_up((uint32_t)nrot * L.rot_stride * 4u, 128u);
    L.slot_stride = 2u * ns * (TB + 1);
    L.slots = o; o += align_up((uint32_t)nwarps * L.slot_stride * 4u, 128u);
    // (S1, S2) of ksub tokens per lane, written as 16-byte token pairs; a stride of 20 floats
    // (ksub = 8) makes both the 16-byte writes and the 16-byte reads of the 4 lanes of a
    // channel bank-conflict free
    L.xch_stride = 2u * ksub + 4u;
    L.xch = o; o += align_up((uint32_t)nwarps * 32u * L.xch_stride * 4u, 128u);
    L.bias = o; o += align_up((uint32_t)dt * 4u, 16u);
    L.bar = align_up(o, 8u); o = L.bar + 8u;
    L.total = o;
    return L;
}

// ---- backward, two channels per lane (scan_bwd_pair.cu): one raw stage of 16-token tiles,
// f32 work rows, 4 rotated B/C copies, and the tile's two state checkpoints, double-buffered
// (the checkpoints of tile i-1 arrive with its raw tiles while tile i still reads its own) ---
struct BwdPairSmem {
    uint32_t du, ddelta, dz;                          // output tiles (TMA store, swizzled)
    uint32_t u, delta, dout, z, y, B, C;              // raw tiles (TMA load, dense rows)
    uint32_t sD, sDU, sG, sSP, sU;                    // f32 [dt][TB+4]
    uint32_t sB, sC;                                  // f32 [4][TB*16 + 16]
    uint32_t slots;                                   // f32 [nwarps][2][16][TB+1]
    uint32_t ck[2];                                   // f32 [2 checkpoints][dt][16], two buffers
    uint32_t bias, bar, total;
    uint32_t rot_stride, slot_stride;
};

__host__ __device__ inline BwdPairSmem bwd_pair_smem_layout(int dt, int nwarps, int es, int has_z) {
    BwdPairSmem L;
    const int TB = kBwdTile, NS = 16;
    const uint32_t row = (uint32_t)TB * es;
    // every TMA tile, loads included, is swizzled (32B for bf16 rows, 64B for f32 rows):
    // 512-byte aligned bases
    const uint32_t otile = align_up((uint32_t)dt * row, 512u);
    const uint32_t tile = otile;
    const uint32_t bc = align_up((uint32_t)NS * row, 512u);
    uint32_t o = 0;
    L.du = o; o += otile;
    L.ddelta = o; o += otile;
    L.dz = o; o += has_z ? otile : 0u;
    L.u = o; o += tile;
    L.delta = o; o += tile;
    L.dout = o; o += tile;
    L.z = o; o += has_z ? tile : 0u;
    L.y = o; o += has_z ? tile : 0u;
    L.B = o; o += bc;
    L.C = o; o += bc;
    const uint32_t rows = align_up((uint32_t)dt * (TB + 4) * 4u, 128u);
    L.sD = o; o += rows;
    L.sDU = o; o += rows;
    L.sG = o; o += rows;
    L.sSP = o; o += rows;
    L.sU = o; o += rows;
    L.rot_stride = (uint32_t)TB * NS + 16u;
    L.sB = o; o += align_up(4u * L.rot_stride * 4u, 128u);
    L.sC = o; o += align_up(4u * L.rot_stride * 4u, 128u);
    L.slot_stride = 2u * NS * (TB + 1);
    L.slots = o; o += align_up((uint32_t)nwarps * L.slot_stride * 4u, 128u);
    for (int i = 0; i < 2; i++) {
        L.ck[i] = o;
        o += align_up(2u * (uint32_t)dt * NS * 4u, 128u);
    }
    L.bias = o; o += align_up((uint32_t)dt * 4u, 16u);
    L.bar = align_up(o, 8u); o = L.bar + 8u;
    L.total = o;
    return L;
}

}  // namespace ssm
