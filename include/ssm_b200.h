/*
 * ssm_b200 -- C ABI of the B200 (sm_100a) selective-scan library.
 *
 * Plain C: pointers, sizes and int64 strides, no torch or CUDA types.  Every pointer
 * argument named as a tensor is a DEVICE pointer on the current CUDA device; `stream`
 * is a cudaStream_t passed as void* (NULL = legacy default stream).  All entry points
 * are asynchronous with respect to the host unless stated, and return SSM_OK (0) or an
 * error code; ssm_last_error() gives the message of the last failure on this thread.
 *
 * The entry points replace the native half of the reference (nmquan1503/ssm-mamba):
 *   ssm_scan_fwd      <- selective_scan.forward   (csrc/selective_scan/selective_scan.cpp:212-292,
 *                                                  forward_kernel.cu:246-264)
 *   ssm_scan_bwd      <- selective_scan.backward  (csrc/selective_scan/selective_scan.cpp:294-380,
 *                                                  backward_kernel.cu:456-478)
 *   ssm_state_update  <- selective_update.apply   (csrc/selective_update/selective_update.cpp:78-130,
 *                                                  kernel.cu:74-91)
 * The reference binds those through pybind (csrc/selective_scan/bindings.cpp:5-8,
 * csrc/selective_update/bindings.cpp:5-7); here they are plain C so that any FFI
 * (ctypes, cffi, a torch extension) can bind them.
 *
 * Shapes (element strides; the innermost dimension always has stride 1):
 *   u, delta, z, out, y, dout, du, ddelta, dz : (batch, dim, seqlen)
 *   A, dA                                     : (dim, dstate)        float32
 *   B, C, dB, dC                              : (batch, dstate, seqlen)
 *   D, delta_bias, dD, ddelta_bias            : (dim)                float32
 *   h_init, h_last, dh_last, dh_init          : (batch, dim, dstate) float32, contiguous
 *   length                                    : (batch)              int64
 */
#ifndef SSM_B200_H
#define SSM_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SSM_API __attribute__((visibility("default")))
#else
#define SSM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types of the streaming tensors (u, delta, z, B, C, out, y and their grads) */
#define SSM_F32 0
#define SSM_BF16 1

/* status codes */
#define SSM_OK 0
#define SSM_ERR_INVALID 1     /* bad shape, stride, alignment, dtype or missing pointer */
#define SSM_ERR_CUDA 2        /* CUDA runtime error (launch, attribute, driver entry point) */
#define SSM_ERR_WORKSPACE 3   /* workspace too small */
#define SSM_ERR_DEVICE 4      /* a kernel reported a bounded wait that ran out */

/* checkpoint layouts written by ssm_scan_fwd and read by ssm_scan_bwd */
#define SSM_CKPT_COMPACT 0    /* (batch, nchunks, dim, dstate) states only */
#define SSM_CKPT_REFERENCE 1  /* (batch, dim, nchunks, 2*dstate) interleaved (prod, state):
                                 the reference's `h` (selective_scan.cpp:271-274) */

typedef struct ssm_scan_fwd_args {
    int64_t batch, dim, seqlen, dstate;
    int32_t dtype;                 /* SSM_F32 or SSM_BF16, for u, delta, z, B, C, out, y */
    int32_t delta_softplus;        /* 1: delta = softplus(delta + bias), threshold 20 */
    int32_t padding_right;         /* length handling: 1 right padding, 0 left padding */
    int32_t _pad0;
    const void* u;      int64_t u_batch_stride, u_dim_stride;
    const void* delta;  int64_t delta_batch_stride, delta_dim_stride;
    const float* A;     int64_t A_dim_stride;
    const void* B;      int64_t B_batch_stride, B_state_stride;
    const void* C;      int64_t C_batch_stride, C_state_stride;
    const float* D;                /* may be NULL (no skip term) */
    const void* z;      int64_t z_batch_stride, z_dim_stride;     /* may be NULL (no gate) */
    const float* delta_bias;       /* may be NULL */
    const float* h_init;           /* may be NULL (zero initial state) */
    const int64_t* length;         /* may be NULL (every row has seqlen tokens) */
    void* out;          int64_t out_batch_stride, out_dim_stride;
    void* y;            int64_t y_batch_stride, y_dim_stride;     /* may be NULL: pre-gate output */
    float* ckpt;                   /* may be NULL: state checkpoints for the backward */
    int32_t ckpt_format;           /* SSM_CKPT_COMPACT or SSM_CKPT_REFERENCE */
    int32_t _pad1;
    int64_t ckpt_len;              /* tokens per checkpoint, a power of two: for SSM_CKPT_COMPACT
                                      >= ssm_scan_ckpt_len(dstate), for SSM_CKPT_REFERENCE >= 32
                                      (the reference uses 128) */
    float* h_last;                 /* may be NULL: final state (batch, dim, dstate) */
} ssm_scan_fwd_args;

typedef struct ssm_scan_bwd_args {
    int64_t batch, dim, seqlen, dstate;
    int32_t dtype;
    int32_t delta_softplus;
    int32_t padding_right;
    int32_t reference_length_semantics; /* must be 1 when length != NULL: the backward then
                                           reproduces the reference's handling of `length`
                                           (backward_kernel.cu:225-400) */
    const void* u;      int64_t u_batch_stride, u_dim_stride;
    const void* delta;  int64_t delta_batch_stride, delta_dim_stride;
    const float* A;     int64_t A_dim_stride;
    const void* B;      int64_t B_batch_stride, B_state_stride;
    const void* C;      int64_t C_batch_stride, C_state_stride;
    const float* D;
    const void* z;      int64_t z_batch_stride, z_dim_stride;
    const float* delta_bias;
    const float* h_init;
    const int64_t* length;
    const void* y;      int64_t y_batch_stride, y_dim_stride;     /* pre-gate output; needed iff z */
    const float* ckpt;
    int32_t ckpt_format;
    int32_t _pad1;
    int64_t ckpt_len;
    const void* dout;   int64_t dout_batch_stride, dout_dim_stride;
    const float* dh_last;          /* may be NULL (zero) */
    void* du;           int64_t du_batch_stride, du_dim_stride;
    void* ddelta;       int64_t ddelta_batch_stride, ddelta_dim_stride;
    void* dz;           int64_t dz_batch_stride, dz_dim_stride;   /* needed iff z */
    float* dA;                     /* (dim, dstate) contiguous */
    void* dB;                      /* (batch, dstate, seqlen) contiguous, dtype */
    void* dC;                      /* (batch, dstate, seqlen) contiguous, dtype */
    float* dD;                     /* may be NULL */
    float* ddelta_bias;            /* may be NULL */
    float* dh_init;                /* may be NULL; written iff h_init != NULL */
    /* element strides of dB and dC; 0 and 0 mean contiguous (dstate * seqlen, seqlen) */
    int64_t dB_batch_stride, dB_state_stride;
    int64_t dC_batch_stride, dC_state_stride;
} ssm_scan_bwd_args;

/* Folding of per-slice carries (ssm_scan_carry_compose). */
typedef struct ssm_carry_args {
    int64_t batch, dim, dstate;
    int64_t nslices;               /* slices in sequence order */
    int32_t reverse;               /* 0: states (forward), 1: gradients (backward) */
    int32_t nstart;                /* number of `start` arrays summed (0 when start is NULL) */
    const float* A;      int64_t A_dim_stride;
    const float* carry;  int64_t carry_slice_stride;      /* (nslices, batch, dim, dstate) */
    const float* delta_sum; int64_t delta_sum_slice_stride; /* (nslices, batch, dim) */
    const float* start;  int64_t start_stride;            /* nstart x (batch, dim, dstate) */
    float* result;                 /* forward: (nslices + 1, batch, dim, dstate);
                                      reverse: (nslices, batch, dim, dstate); contiguous;
                                      must not overlap carry or delta_sum */
} ssm_carry_args;

typedef struct ssm_state_update_args {
    int64_t batch, dim, dstate;
    int32_t dtype;                 /* for x, dt, z, B, C, out */
    int32_t dt_softplus;
    const float* state;  int64_t state_batch_stride, state_dim_stride;  /* read */
    float* state_out;    int64_t state_out_batch_stride, state_out_dim_stride; /* written;
                                      may equal `state` (in place) */
    const void* x;       int64_t x_batch_stride;
    const void* dt;      int64_t dt_batch_stride;
    const float* A;      int64_t A_dim_stride;
    const void* B;       int64_t B_batch_stride;
    const void* C;       int64_t C_batch_stride;
    const float* D;                /* may be NULL */
    const void* z;       int64_t z_batch_stride;   /* may be NULL */
    const float* dt_bias;          /* may be NULL */
    void* out;           int64_t out_batch_stride;
    int32_t launch_flags;          /* bit 0 (SSM_LAUNCH_PDL): programmatic dependent launch --
                                      the kernel may start while the previous kernel in the
                                      stream finishes; it prefetches its state into L2, then
                                      waits for that kernel before reading any input */
    int32_t _pad1;
} ssm_state_update_args;

#define SSM_LAUNCH_PDL 1

/* Message of the last failed call on the calling thread ("" if none). */
SSM_API const char* ssm_last_error(void);

/* Library version string. */
SSM_API const char* ssm_version(void);

/* Number of state checkpoints a forward with these sizes writes: ceil(seqlen / ckpt_len). */
SSM_API int64_t ssm_scan_num_ckpt(int64_t seqlen, int64_t ckpt_len);

/* Checkpoint interval (tokens) ssm_scan_bwd needs: the forward feeding a backward must
 * write SSM_CKPT_COMPACT checkpoints every ssm_scan_ckpt_len(dstate) tokens (8 for
 * dstate <= 128, 4 above). */
SSM_API int64_t ssm_scan_ckpt_len(int64_t dstate);

/* Forward selective scan (replaces selective_scan.forward).  Writes out, optionally y
 * (pre-gate output, needed by the backward when z is given), the state checkpoints and
 * the final state. */
SSM_API int ssm_scan_fwd(const ssm_scan_fwd_args* args, void* stream);

/* Rebuilds the compact checkpoints ssm_scan_bwd needs from the reference's chunk states
 * `ref_ckpt` (SSM_CKPT_REFERENCE layout, 128-token chunks, as selective_scan.forward
 * returns them in `h`), recomputing every chunk from its start state with the reference
 * backward's load rules (backward_kernel.cu:242-246, 345-353).  args->ckpt must be a
 * SSM_CKPT_COMPACT buffer with ckpt_len = ssm_scan_ckpt_len(dstate); args->out and args->y
 * must be NULL.  No reference counterpart: the reference backward recomputes inside
 * its own kernel. */
SSM_API int ssm_scan_ckpt_from_reference(const ssm_scan_fwd_args* args, const float* ref_ckpt,
                                 void* stream);

/* Bytes of device workspace ssm_scan_bwd needs for these arguments. */
SSM_API size_t ssm_scan_bwd_workspace_size(const ssm_scan_bwd_args* args);

/* Backward selective scan (replaces selective_scan.backward).  Overwrites every gradient
 * output (no pre-zeroing needed).  Deterministic: no floating-point atomics.  The
 * workspace must hold ssm_scan_bwd_workspace_size(args) bytes and be 256-byte aligned. */
SSM_API int ssm_scan_bwd(const ssm_scan_bwd_args* args, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Backward selective scan that allocates nothing.  No counterpart in the reference.
 * For callers that cannot allocate device memory where they run the backward: a framework
 * or runtime whose own allocator owns all device memory, or a host-language binding that
 * reaches this library through a plain C FFI with no device-allocation API.  Instead of a
 * caller-provided workspace it uses a 16 MiB scratch array compiled into the library (held
 * on every GPU that loads the library until exit).  Shapes whose
 * ssm_scan_bwd_workspace_size exceeds 16 MiB - 256 bytes are rejected with
 * SSM_ERR_WORKSPACE.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make it before any stream capture.  Every call on a device shares
 * the array: calls whose kernels overlap on the GPU race and must be serialised.  A bounded
 * wait that runs out inside its kernels is reported by ssm_check_device_error, like those
 * of the other entry points. */
SSM_API int ssm_scan_bwd_noalloc(const ssm_scan_bwd_args* args, void* stream);

/* One decode step (replaces selective_update.apply).  state_out may alias state.
 * Contiguous operands (state, state_out and A with a dim stride of dstate; 16-byte
 * aligned pointers and batch strides, dt_bias and D included) with dstate 8, 16 or 32 and
 * dim a multiple of 256 / (dstate / 8) take the streamed kernel (persistent CTAs, bulk
 * copies); any other layout takes the per-CTA kernel.  Both compute the same arithmetic in
 * the same order.  With launch_flags & SSM_LAUNCH_PDL the kernel is launched with
 * programmatic dependent launch and waits for the previous kernel in the stream before
 * reading any input. */
SSM_API int ssm_state_update(const ssm_state_update_args* args, void* stream);

/* ---- sequence slices ---------------------------------------------------------------------
 * A long sequence can be scanned as S independent slices -- segments of one GPU's
 * sequence viewed as a batch of S rows (batch stride = segment length), or the slices the
 * ranks of a sequence-parallel group hold -- because the recurrence is linear in the state:
 *   1. ssm_scan_chunk_state_fwd: every slice's end state from a zero start and its sum of
 *      delta (its decay is exp(A * delta_sum));
 *   2. ssm_scan_carry_compose (reverse = 0): the state entering every slice;
 *   3. ssm_scan_fwd per slice with h_init = that state;
 * and for the backward
 *   4. ssm_scan_chunk_state_bwd: every slice's gradient into the state before it, from a
 *      zero incoming gradient;
 *   5. ssm_scan_carry_compose (reverse = 1): the gradient leaving every slice's end;
 *   6. ssm_scan_bwd per slice with dh_last = that gradient and h_init from step 2.
 * None of these has a reference counterpart: the reference scans each sequence serially
 * (forward_kernel.cu:208-228, backward_kernel.cu:341-366). */

/* Step 1.  Uses u, delta, A, B, delta_bias, delta_softplus and their strides from args;
 * C, D and z are ignored; out, y, ckpt, h_init, h_last and length must be NULL.
 * Writes h_end (batch, dim, dstate) and delta_sum (batch, dim), both float32 contiguous. */
SSM_API int ssm_scan_chunk_state_fwd(const ssm_scan_fwd_args* args, float* h_end, float* delta_sum,
                                     void* stream);

/* Step 4.  Uses delta, A, C, dout, z, delta_bias, delta_softplus and their strides; u, B,
 * y, ckpt and the gradient outputs are ignored; length must be NULL.  Writes g_start
 * (batch, dim, dstate) float32 contiguous. */
SSM_API int ssm_scan_chunk_state_bwd(const ssm_scan_bwd_args* args, float* g_start, void* stream);

/* Steps 2 and 5.  Forward: result[0] = start (h_init, or 0), result[q + 1] =
 * exp(A * delta_sum[q]) * result[q] + carry[q] (carry = h_end); result[nslices] is the
 * final state.  Reverse: result[nslices - 1] = start (dh_last, or 0), result[q - 1] =
 * exp(A * delta_sum[q]) * result[q] + carry[q] (carry = g_start). */
SSM_API int ssm_scan_carry_compose(const ssm_carry_args* args, void* stream);

/* ---- causal depthwise conv1d (+ SiLU): the step in front of the scan ------------------------
 * Replaces, in the reference's Mamba module (modules/mamba.py), the prefill
 * silu(conv(x)[..., :seqlen]) with conv = nn.Conv1d(groups=dim, padding=width-1) (:137-139),
 * the gather of the decode context (the last width-1 inputs before `lengths`, :114-133), its
 * backward (torch autograd in the reference) and the decode step (:203-213):
 *   out[b, d, t] = act(bias[d] + sum_k weight[d, k] x[b, d, t - (width-1) + k]), x[< 0] = 0
 * width is 2, 3 or 4; act is SiLU or the identity. */
typedef struct ssm_conv1d_args {
    int64_t batch, dim, seqlen, width;
    int32_t dtype;                 /* SSM_F32 or SSM_BF16, for x, out, state, dout, dx */
    int32_t silu;                  /* 1: SiLU after the convolution */
    const void* x;       int64_t x_batch_stride, x_dim_stride;     /* (batch, dim, seqlen);
                                      ssm_conv1d_update: (batch, dim) */
    const float* weight; int64_t weight_dim_stride;                 /* (dim, width) */
    const float* bias;             /* (dim) or NULL */
    void* out;           int64_t out_batch_stride, out_dim_stride;
    const int64_t* length;         /* forward: (batch) or NULL; the context ends at length[b] */
    void* state;         int64_t state_batch_stride, state_dim_stride; /* (batch, dim, width-1),
                                      unit innermost stride; forward output (may be NULL),
                                      ssm_conv1d_update input and output (in place) */
    const void* dout;    int64_t dout_batch_stride, dout_dim_stride;   /* backward */
    void* dx;            int64_t dx_batch_stride, dx_dim_stride;       /* backward */
    float* dweight;      int64_t dweight_dim_stride;                   /* backward, (dim, width) */
    float* dbias;                  /* backward, (dim) or NULL */
} ssm_conv1d_args;

SSM_API int ssm_conv1d_fwd(const ssm_conv1d_args* args, void* stream);
/* Bytes of device workspace ssm_conv1d_bwd needs (per-warp dweight/dbias partials). */
SSM_API size_t ssm_conv1d_bwd_workspace_size(const ssm_conv1d_args* args);
/* Backward: dx, dweight, dbias from x and dout (the gradient of out).  Overwrites them;
 * deterministic (fixed-order sums, no floating-point atomics). */
SSM_API int ssm_conv1d_bwd(const ssm_conv1d_args* args, void* workspace, size_t workspace_bytes,
                           void* stream);
/* One decode step: x (batch, dim) joins the context `state`, which shifts by one in place;
 * out (batch, dim) = act(bias + sum_k weight[k] window[k]). */
SSM_API int ssm_conv1d_update(const ssm_conv1d_args* args, void* stream);

/* Reads and clears the device-side error words of the current device -- the library's own
 * and the one in ssm_scan_bwd_noalloc's static scratch -- (synchronizes `stream`; allocates
 * nothing).  Returns SSM_OK with *code = 0, or SSM_ERR_DEVICE with *code set to the
 * kernel's code (1: a bounded wait for a TMA copy ran out; 2: misaligned shared memory). */
SSM_API int ssm_check_device_error(int* code, void* stream);

/* Diagnostics: evaluates, for n float32 inputs x on the device, the exp2 that the carry passes
 * (ssm_scan_chunk_state_fwd / _bwd) compute on the FMA pipe for a share of their elements
 * (into y_fma) and the MUFU ex2.approx.ftz that the other elements use (into y_mufu), so
 * that a test can hold the former to the latter's error bound.  No reference counterpart. */
SSM_API int ssm_exp2_compare(const float* x, float* y_fma, float* y_mufu, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SSM_B200_H */
