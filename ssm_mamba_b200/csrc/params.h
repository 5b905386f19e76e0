// Kernel parameter blocks (host and device).  Built by capi.cu from the C-ABI argument
// structs after validation; strides are in elements.
#pragma once

#include <stdint.h>

namespace ssm {

struct FwdParams {
    int batch, dim, seqlen, dstate;
    int dt;              // channels per CTA
    int ntile_d;         // ceil(dim / dt)
    int use_tma;         // 1: TMA tensor-map path, 0: plain-load fallback
    int delta_softplus, padding_right;
    int ckpt_format;     // 0 compact, 1 reference
    int ckpt_len, ckpt_shift, nck;   // ckpt_len = 1 << ckpt_shift
    const void* u; int64_t u_sb, u_sd;
    const void* delta; int64_t delta_sb, delta_sd;
    const float* A; int64_t A_sd;
    const void* B; int64_t B_sb, B_sn;
    const void* C; int64_t C_sb, C_sn;
    const float* D;
    const void* z; int64_t z_sb, z_sd;
    const float* delta_bias;
    const float* h_init;
    const int64_t* length;
    void* out; int64_t out_sb, out_sd;
    void* y; int64_t y_sb, y_sd;
    float* ckpt;
    float* h_last;
    // rechunk mode (reference-format chunk states -> compact checkpoints, with the
    // reference backward's load rules): restart the state from `restart` every
    // `restart_len` tokens and zero-fill loads from token len on when seqlen % 128 != 0
    const float* restart;
    int restart_len, restart_nck;
    int* err;            // device error word
    int test_withhold;   // test hook: never issue the TMA loads, so the first bounded wait runs out
};

struct BwdParams {
    int batch, dim, seqlen, dstate;
    int dt, ntile_d;
    int use_tma;
    int delta_softplus, padding_right;
    int ref_len;         // reproduce the reference backward's length semantics
    int ckpt_format, ckpt_len, nck;
    const void* u; int64_t u_sb, u_sd;
    const void* delta; int64_t delta_sb, delta_sd;
    const float* A; int64_t A_sd;
    const void* B; int64_t B_sb, B_sn;
    const void* C; int64_t C_sb, C_sn;
    const float* D;
    const void* z; int64_t z_sb, z_sd;
    const float* delta_bias;
    const float* h_init;
    const int64_t* length;
    const void* y; int64_t y_sb, y_sd;
    const float* ckpt;
    const void* dout; int64_t dout_sb, dout_sd;
    const float* dh_last;
    void* du; int64_t du_sb, du_sd;
    void* ddelta; int64_t ddelta_sb, ddelta_sd;
    void* dz; int64_t dz_sb, dz_sd;
    float* dh_init;
    // workspace partials
    float* ws_bc;        // (ntile_d, batch, 2, dstate, seqlen): per channel-tile dB, dC sums
    float* ws_a;         // (batch, dim, dstate): per-batch dA
    float* ws_dd;        // (batch, dim, 2): per-batch dD, ddelta_bias
    int* err;
    int test_withhold;   // test hook: never issue the TMA loads, so the first bounded wait runs out
};

struct ReduceParams {
    int batch, dim, seqlen, dstate, ntile_d;
    int bc_dtype;        // 0 f32, 1 bf16
    const float* ws_bc; const float* ws_a; const float* ws_dd;
    void* dB; void* dC;
    int64_t dB_sb, dB_sn, dC_sb, dC_sn;   // element strides of dB, dC
    float* dA; float* dD; float* ddelta_bias;
};

// Sequence-slice carries: the state a slice reaches from a zero start (forward) or the
// gradient it sends back to the state before it (reverse).
struct ChunkParams {
    int batch, dim, seqlen, dstate;
    int dt, ntile_d;
    int use_tma;
    int delta_softplus;
    const void* x0; int64_t x0_sb, x0_sd;   // forward: u; reverse: dout
    const void* delta; int64_t delta_sb, delta_sd;
    const void* z; int64_t z_sb, z_sd;      // reverse only, may be null
    const void* bc; int64_t bc_sb, bc_sn;   // forward: B; reverse: C
    const float* A; int64_t A_sd;
    const float* delta_bias;
    float* carry;        // (batch, dim, dstate): h_end (forward) or g_start (reverse)
    float* delta_sum;    // (batch, dim): sum of the effective delta (forward only, may be null)
    int* err;
};

struct CarryParams {
    int batch, dim, dstate, nslices, reverse;
    const float* A; int64_t A_sd;
    const float* carry; int64_t carry_ss;
    const float* delta_sum; int64_t dsum_ss;
    const float* start; int64_t start_ss; int nstart;
    float* result;       // forward: (nslices + 1, batch, dim, dstate); reverse: (nslices, ...)
};

// Causal depthwise conv1d (conv1d.cu).
struct ConvParams {
    int batch, dim, seqlen;
    int silu;
    const void* x; int64_t x_sb, x_sd;
    const float* w; int64_t w_sd;        // (dim, width)
    const float* bias;                   // (dim) or null
    void* out; int64_t out_sb, out_sd;
    // forward only: the last width-1 inputs of every row, before token length[b] (or seqlen)
    const int64_t* length;
    void* state; int64_t st_sb, st_sd;
    // backward only
    const void* dout; int64_t dout_sb, dout_sd;
    void* dx; int64_t dx_sb, dx_sd;
    float* ws;                           // (nchunk * batch, dim, width + 1) partials
    int nchunk;                          // warps (chunks of 32 vectors) per row
};

struct UpdParams {
    int batch, dim, dstate;
    int dt_softplus;
    const float* state; int64_t st_sb, st_sd;
    float* state_out; int64_t so_sb, so_sd;
    const void* x; int64_t x_sb;
    const void* dtv; int64_t dt_sb;
    const float* A; int64_t A_sd;
    const void* B; int64_t B_sb;
    const void* C; int64_t C_sb;
    const float* D;
    const void* z; int64_t z_sb;
    const float* dt_bias;
    void* out; int64_t out_sb;
    int pdl;             // launch with programmatic dependent launch
    int* err;            // device error word (streamed kernel's bounded waits)
};

}  // namespace ssm
