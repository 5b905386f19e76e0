// C ABI of the library (include/ssm_b200.h): argument validation, TMA tensor maps, CTA
// sizing and launches.  Mirrors the checks of the reference host glue
// (nmquan1503/ssm-mamba, csrc/selective_scan/selective_scan.cpp:15-32, 229-268, 314-351;
// csrc/selective_update/selective_update.cpp:11-21, 184-206): shapes, the 256-state limit
// and dtypes -- here reported as status codes plus ssm_last_error() instead of exceptions.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/ssm_b200.h"
#include "params.h"
#include "scan_layout.h"
#include <nvtx3/nvToolsExt.h>

namespace {
// NVTX range around each entry point (named after it), for nsys / ncu timelines; a no-op
// unless a tool is attached
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace

namespace ssm {
cudaError_t launch_scan_fwd(const FwdParams& p, int is_bf16, int lpc, int spt, const CUtensorMap* maps,
                            cudaStream_t stream);
cudaError_t launch_scan_bwd(const BwdParams& p, int is_bf16, int lpc, int spt, const CUtensorMap* maps,
                            cudaStream_t stream);
cudaError_t launch_scan_reduce(const ReduceParams& p, cudaStream_t stream);
cudaError_t launch_state_update(const UpdParams& p, int is_bf16, int lpc, int spt, cudaStream_t stream);
cudaError_t launch_state_update_stream(const UpdParams& p, int is_bf16, int lpc, int sms, cudaStream_t stream);
cudaError_t launch_scan_chunk(const ChunkParams& p, int is_bf16, int lpc, int spt, int reverse,
                              const CUtensorMap* maps, cudaStream_t stream);
int chunk_occupancy(int is_bf16, int lpc, int spt, int reverse, int dt, int has_z);
cudaError_t launch_carry_compose(const CarryParams& p, cudaStream_t stream);
cudaError_t launch_conv1d(const ConvParams& p, int is_bf16, int width, int kind, int vec, int sms,
                          cudaStream_t stream);
cudaError_t launch_conv1d_reduce(const float* ws, int nparts, int dim, int width, float* dw, int64_t dw_sd,
                                 float* dbias, int sms, cudaStream_t stream);
cudaError_t launch_conv1d_update(const ConvParams& p, int is_bf16, int width, int sms, cudaStream_t stream);
size_t bwd_smem_bytes(int is_bf16, int lpc, int spt, int dt, int dstate, int has_z);
cudaError_t launch_scan_bwd_pair(const BwdParams& p, int is_bf16, int cpl, const CUtensorMap* maps,
                                 cudaStream_t stream);
int bwd_pair_occupancy(int is_bf16, int cpl, int dt, int has_z);
cudaError_t launch_exp2_compare(const float* x, float* y_fma, float* y_mufu, int64_t n, cudaStream_t stream);
cudaError_t launch_scan_bwd_split(const BwdParams& p, int is_bf16, const CUtensorMap* maps, cudaStream_t stream);
int bwd_split_occupancy(int is_bf16, int dt, int has_z);
int* noalloc_error_word();
int fwd_occupancy(int is_bf16, int lpc, int spt, int dt, int has_z, int has_y);
int bwd_occupancy(int is_bf16, int lpc, int spt, int dt, int dstate, int has_z);
}  // namespace ssm

using namespace ssm;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(SSM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---- lanes per channel / states per thread / backward sub-tile for a state count ----------
struct StateSplit { int lpc, spt, k; };

// Backward checkpoint interval (and the scan kernels' split above 128 states).
StateSplit split_states(int64_t n) {
    if (n > 128) return {32, 8, 4};
    int ns = 4;
    while (ns < n) ns *= 2;
    return {ns / 4, 4, 8};
}

// Decode kernel: SPT states per thread.  8 states per thread for small state counts (half
// the per-row scalar work per state of 4, and 32 bytes of state per thread in flight);
// SSM_DEC_SPT (4, 8, 16) overrides for experiments.
StateSplit decode_split(int64_t n) {
    if (n > 128) return {32, 8, 4};
    int ns = 4;
    while (ns < n) ns *= 2;
    int spt = ns >= 8 ? 8 : 4;
    if (const char* e = getenv("SSM_DEC_SPT")) {
        const int v = atoi(e);
        if ((v == 4 || v == 8 || v == 16) && v <= ns && ns / v <= 16) spt = v;
    }
    return {ns / spt, spt, 8};
}

// Scan kernels: 4 states per thread; 2 only when 4 would leave fewer than 4 warps per SM
// (measured on B200 at config 2: 4 states per thread is 1.5x faster than 2 at 10 warps per
// SM -- the extra per-state reductions outweigh the extra warps).  The environment
// variable named by `env` (SSM_FWD_SPT / SSM_BWD_SPT) may force 2 or 4 for experiments.
// The backward's checkpoint interval k depends on dstate only, so forward and backward
// always agree.
StateSplit scan_split(int64_t n, int64_t rows, int sms, const char* env) {
    if (n > 128) return {32, 8, 4};
    int ns = 4;
    while (ns < n) ns *= 2;
    const StateSplit s4{ns / 4, 4, 8};
    const StateSplit s2{ns / 2, 2, 8};
    const bool s2_ok = ns / 2 <= 32;
    const char* e = getenv(env);
    if (e && e[0] == '2' && s2_ok) return s2;
    if (e && e[0] == '4') return s4;
    if (e && e[0] == '8' && ns >= 16 && strcmp(env, "SSM_FWD_SPT") == 0) return {ns / 8, 8, 8};
    const double warps4 = (double)rows * (ns / 4) / 32.0 / (sms > 0 ? sms : 148);
    return (warps4 < 4.0 && s2_ok) ? s2 : s4;
}

// ---- device attributes and the per-device error word ----------------------------------------
struct DevInfo {
    int sms = 0;
    int* err = nullptr;
};
std::mutex g_mu;
DevInfo g_dev[64];

// The current device's DevInfo if an entry point has set it up, else nullptr (allocates
// nothing: no kernel can have written an error word that does not exist yet).
DevInfo* device_info_if_ready() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    return g_dev[dev].sms != 0 ? &g_dev[dev] : nullptr;
}

int device_info(DevInfo** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(SSM_ERR_CUDA, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    DevInfo& di = g_dev[dev];
    if (di.sms == 0) {
        e = cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        e = cudaMalloc(&di.err, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(error word)");
        e = cudaMemset(di.err, 0, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error word)");
    }
    *out = &di;
    return SSM_OK;
}

// ---- TMA tensor maps ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder() {
    if (g_encode) return SSM_OK;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode) return SSM_OK;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(SSM_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return SSM_OK;
}

// Can a (dim2, dim1, inner) tensor with these element strides be a TMA source/target?
bool tma_ok(const void* ptr, int64_t s1, int64_t s2, int64_t es) {
    if (!ptr) return true;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return false;
    if (((s1 * es) & 15) != 0 || ((s2 * es) & 15) != 0) return false;
    if (s1 * es >= (int64_t(1) << 40) || s2 * es >= (int64_t(1) << 40)) return false;
    return true;
}

// 3-D map of a (d2, d1, d0=inner) tensor with element strides (s2, s1, 1); box (b0, b1, 1).
int encode3d(CUtensorMap* map, const void* ptr, int is_bf16, int64_t d0, int64_t d1, int64_t d2,
             int64_t s1, int64_t s2, int b0, int b1, CUtensorMapSwizzle swz) {
    if (!ptr) {
        memset(map, 0, sizeof(*map));
        return SSM_OK;
    }
    const int64_t es = is_bf16 ? 2 : 4;
    // a size-1 outer dimension may have any stride; give TMA a valid one
    if (d1 == 1) s1 = d0;
    if (d2 == 1) s2 = s1 * d1;
    cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)(s1 * es), (cuuint64_t)(s2 * es)};
    cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, 1u};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    CUresult r = g_encode(map, is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                          const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SSM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SSM_OK;
}

// 4-D float32 map of a (d3, d2, d1, d0=inner) tensor with element strides (s3, s2, s1, 1);
// box (b0, b1, b2, 1), no swizzle.
int encode4d_f32(CUtensorMap* map, const void* ptr, int64_t d0, int64_t d1, int64_t d2, int64_t d3, int64_t s1,
                 int64_t s2, int64_t s3, int b0, int b1, int b2) {
    cuuint64_t dims[4] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2, (cuuint64_t)d3};
    cuuint64_t strides[3] = {(cuuint64_t)(s1 * 4), (cuuint64_t)(s2 * 4), (cuuint64_t)(s3 * 4)};
    cuuint32_t box[4] = {(cuuint32_t)b0, (cuuint32_t)b1, (cuuint32_t)b2, 1u};
    cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(SSM_ERR_CUDA, "cuTensorMapEncodeTiled (4-D) failed (%d)", (int)r);
    return SSM_OK;
}

// ---- CTA sizing: channels per CTA ---------------------------------------------------------------
// Picks dt (a multiple of the channels a warp holds, at most 128 threads per CTA) that
// minimises the estimated time on the busiest SM: CTAs are spread evenly over the SMs and
// run `res` at a time (res from the occupancy calculator), an SM is assumed to reach full
// throughput at 8 resident warps, and every CTA pays a fixed cost worth `ovh` channels
// (staging B and C for its batch row; in the backward also its dB/dC partials).  For the
// scan forward and backward ovh is 8: measured on B200, the forward at 4 x 5120 x 2048
// takes 420 us with 32 channels per CTA and 433 us with 16, which an overhead of 4 ranked
// the other way round.  Results are cached per shape.
template <typename OccFn>
int choose_dt(int64_t batch, int64_t dim, int lpc, int sms, double ovh, OccFn occupancy) {
    const int cpw = 32 / lpc;
    const int dtmax = 128 / lpc;
    int best = -1;
    double best_t = 1e300;
    for (int dt = cpw; dt <= dtmax; dt += cpw) {
        const int res = occupancy(dt);
        if (res < 1) continue;
        const int warps = dt * lpc / 32;
        const int64_t ctas = batch * ((dim + dt - 1) / dt);
        const int64_t per_sm = (ctas + sms - 1) / sms;
        double t = 0;
        for (int64_t left = per_sm; left > 0; left -= res) {
            const int64_t m = left < res ? left : res;
            const double thr = (m * warps) >= 8 ? 1.0 : (double)(m * warps) / 8.0;
            t += (double)m * (dt + ovh) / thr;
        }
        t *= (double)(((dim + dt - 1) / dt) * dt) / (double)dim;  // ragged last channel tile
        if (t < best_t * 0.999) {
            best_t = t;
            best = dt;
        }
    }
    return best;
}

struct DtKey {
    int dev, kind, is_bf16, lpc, spt, dstate, has_z, has_y;
    int64_t batch, dim;
    bool operator==(const DtKey& o) const { return memcmp(this, &o, sizeof(*this)) == 0; }
};
std::mutex g_dt_mu;
DtKey g_dt_keys[64];
int g_dt_vals[64];
int g_dt_n = 0;

template <typename OccFn>
int cached_dt(DtKey key, int sms, OccFn occ) {
    {
        std::lock_guard<std::mutex> lk(g_dt_mu);
        for (int i = 0; i < g_dt_n; i++)
            if (g_dt_keys[i] == key) return g_dt_vals[i];
    }
    const int dt = choose_dt(key.batch, key.dim, key.lpc, sms, (key.kind <= 1 || key.kind >= 5) ? 8.0 : 4.0, occ);
    std::lock_guard<std::mutex> lk(g_dt_mu);
    const int slot = g_dt_n < 64 ? g_dt_n++ : (int)(key.dim % 64);
    g_dt_keys[slot] = key;
    g_dt_vals[slot] = dt;
    return dt;
}

bool valid_dtype(int32_t t) { return t == SSM_F32 || t == SSM_BF16; }

}  // namespace

extern "C" {

const char* ssm_last_error(void) { return g_err.c_str(); }

const char* ssm_version(void) { return "ssm_b200 0.1.0 (sm_100a)"; }

int64_t ssm_scan_num_ckpt(int64_t seqlen, int64_t ckpt_len) {
    if (seqlen <= 0 || ckpt_len <= 0) return 0;
    return (seqlen + ckpt_len - 1) / ckpt_len;
}

// Checkpoint interval (tokens) the backward needs from the forward's compact checkpoints.
int64_t ssm_scan_ckpt_len(int64_t dstate) { return split_states(dstate).k; }

static int fwd_impl(const ssm_scan_fwd_args* a, const float* restart, void* stream_) {
    if (!a) return fail(SSM_ERR_INVALID, "ssm_scan_fwd: args is NULL");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (a->batch < 1 || a->dim < 1 || a->seqlen < 1 || a->dstate < 1)
        return fail(SSM_ERR_INVALID, "ssm_scan_fwd: sizes must be positive (batch=%lld dim=%lld seqlen=%lld dstate=%lld)",
                    (long long)a->batch, (long long)a->dim, (long long)a->seqlen, (long long)a->dstate);
    if (a->dstate > 256) return fail(SSM_ERR_INVALID, "selective_scan only supports state_dim <= 256");
    if (a->seqlen > (1 << 30) || a->dim > (1 << 30) || a->batch > (1 << 30))
        return fail(SSM_ERR_INVALID, "ssm_scan_fwd: sizes too large");
    if (!valid_dtype(a->dtype)) return fail(SSM_ERR_INVALID, "ssm_scan_fwd: dtype must be SSM_F32 or SSM_BF16");
    if (!a->u || !a->delta || !a->A || !a->B || !a->C || (!a->out && !restart))
        return fail(SSM_ERR_INVALID, "ssm_scan_fwd: u, delta, A, B, C and out are required");
    if (restart && (!a->ckpt || a->ckpt_format != SSM_CKPT_COMPACT || a->out || a->y))
        return fail(SSM_ERR_INVALID, "ssm_scan_ckpt_from_reference: needs a compact ckpt and no out / y");
    if (a->ckpt) {
        if (a->ckpt_format != SSM_CKPT_COMPACT && a->ckpt_format != SSM_CKPT_REFERENCE)
            return fail(SSM_ERR_INVALID, "ssm_scan_fwd: unknown checkpoint format");
        if (a->ckpt_len < 4 || (a->ckpt_len & (a->ckpt_len - 1)) != 0 || a->ckpt_len > (1 << 20))
            return fail(SSM_ERR_INVALID, "ssm_scan_fwd: ckpt_len must be a power of two >= 4");
        // the forward writes reference-layout carries only at the ends of its token groups
        if (a->ckpt_format == SSM_CKPT_REFERENCE && a->ckpt_len < 32)
            return fail(SSM_ERR_INVALID, "ssm_scan_fwd: SSM_CKPT_REFERENCE needs ckpt_len >= 32");
        if (a->ckpt_format == SSM_CKPT_COMPACT && a->ckpt_len < ssm_scan_ckpt_len(a->dstate))
            return fail(SSM_ERR_INVALID, "ssm_scan_fwd: SSM_CKPT_COMPACT needs ckpt_len >= ssm_scan_ckpt_len(dstate) = %lld",
                        (long long)ssm_scan_ckpt_len(a->dstate));
    }
    const int is_bf16 = a->dtype == SSM_BF16;
    const int64_t es = is_bf16 ? 2 : 4;
    DevInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc) return rc;
    const StateSplit sp = scan_split(a->dstate, a->batch * a->dim, di->sms, "SSM_FWD_SPT");
    const int T = (int)(128 / es);

    FwdParams p;
    memset(&p, 0, sizeof(p));
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.seqlen = (int)a->seqlen; p.dstate = (int)a->dstate;
    p.delta_softplus = a->delta_softplus; p.padding_right = a->padding_right;
    p.ckpt_format = a->ckpt_format;
    p.ckpt_len = a->ckpt ? (int)a->ckpt_len : 4;
    while ((1 << p.ckpt_shift) < p.ckpt_len) p.ckpt_shift++;
    p.nck = a->ckpt ? (int)ssm_scan_num_ckpt(a->seqlen, a->ckpt_len) : 0;
    p.u = a->u; p.u_sb = a->u_batch_stride; p.u_sd = a->u_dim_stride;
    p.delta = a->delta; p.delta_sb = a->delta_batch_stride; p.delta_sd = a->delta_dim_stride;
    p.A = a->A; p.A_sd = a->A_dim_stride;
    p.B = a->B; p.B_sb = a->B_batch_stride; p.B_sn = a->B_state_stride;
    p.C = a->C; p.C_sb = a->C_batch_stride; p.C_sn = a->C_state_stride;
    p.D = a->D; p.z = a->z; p.z_sb = a->z_batch_stride; p.z_sd = a->z_dim_stride;
    p.delta_bias = a->delta_bias; p.h_init = a->h_init; p.length = a->length;
    p.out = a->out; p.out_sb = a->out_batch_stride; p.out_sd = a->out_dim_stride;
    p.y = a->y; p.y_sb = a->y_batch_stride; p.y_sd = a->y_dim_stride;
    p.ckpt = a->ckpt; p.h_last = a->h_last; p.err = di->err;
    p.restart = restart;
    p.restart_len = 128;
    p.restart_nck = (int)ssm_scan_num_ckpt(a->seqlen, 128);

    const int has_z = a->z != nullptr, has_y = a->y != nullptr;
    int dev = 0;
    cudaGetDevice(&dev);
    DtKey key;
    memset(&key, 0, sizeof(key));
    key.dev = dev; key.kind = 0; key.is_bf16 = is_bf16; key.lpc = sp.lpc; key.spt = sp.spt; key.dstate = 0;
    key.has_z = has_z; key.has_y = has_y; key.batch = a->batch; key.dim = a->dim;
    p.dt = cached_dt(key, di->sms, [&](int dt) { return fwd_occupancy(is_bf16, sp.lpc, sp.spt, dt, has_z, has_y); });
    if (p.dt < 1) return fail(SSM_ERR_INVALID, "ssm_scan_fwd: no CTA shape fits shared memory");
    p.ntile_d = (int)((a->dim + p.dt - 1) / p.dt);

    p.use_tma = tma_ok(a->u, a->u_dim_stride, a->u_batch_stride, es) &&
                tma_ok(a->delta, a->delta_dim_stride, a->delta_batch_stride, es) &&
                tma_ok(a->z, a->z_dim_stride, a->z_batch_stride, es) &&
                tma_ok(a->B, a->B_state_stride, a->B_batch_stride, es) &&
                tma_ok(a->C, a->C_state_stride, a->C_batch_stride, es) &&
                tma_ok(a->out, a->out_dim_stride, a->out_batch_stride, es) &&
                tma_ok(a->y, a->y_dim_stride, a->y_batch_stride, es);
    CUtensorMap maps[7];
    memset(maps, 0, sizeof(maps));
    if (p.use_tma) {
        if ((rc = get_encoder())) return rc;
        const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
        if ((rc = encode3d(&maps[0], a->u, is_bf16, a->seqlen, a->dim, a->batch, a->u_dim_stride, a->u_batch_stride, T, p.dt, sw)) ||
            (rc = encode3d(&maps[1], a->delta, is_bf16, a->seqlen, a->dim, a->batch, a->delta_dim_stride, a->delta_batch_stride, T, p.dt, sw)) ||
            (rc = encode3d(&maps[2], a->z, is_bf16, a->seqlen, a->dim, a->batch, a->z_dim_stride, a->z_batch_stride, T, p.dt, sw)) ||
            (rc = encode3d(&maps[3], a->B, is_bf16, a->seqlen, a->dstate, a->batch, a->B_state_stride, a->B_batch_stride, T, (int)a->dstate, sw)) ||
            (rc = encode3d(&maps[4], a->C, is_bf16, a->seqlen, a->dstate, a->batch, a->C_state_stride, a->C_batch_stride, T, (int)a->dstate, sw)) ||
            (rc = encode3d(&maps[5], a->out, is_bf16, a->seqlen, a->dim, a->batch, a->out_dim_stride, a->out_batch_stride, T, p.dt, sw)) ||
            (rc = encode3d(&maps[6], a->y, is_bf16, a->seqlen, a->dim, a->batch, a->y_dim_stride, a->y_batch_stride, T, p.dt, sw)))
            return rc;
    }
    // test hook for failure detection: with SSM_TEST_WITHHOLD_TMA set the forward issues no
    // TMA load, its first bounded mbarrier wait (~1 s) runs out, and every CTA leaves with
    // device error kDevErrTmaTimeout (read by ssm_check_device_error); nothing is in flight
    // when the CTAs exit and the context stays usable
    p.test_withhold = p.use_tma && getenv("SSM_TEST_WITHHOLD_TMA") != nullptr;
    cudaError_t e = launch_scan_fwd(p, is_bf16, sp.lpc, sp.spt, maps, stream);
    if (e != cudaSuccess) return cuda_fail(e, "scan_fwd launch");
    return SSM_OK;
}

int ssm_scan_fwd(const ssm_scan_fwd_args* a, void* stream) {
    NvtxRange r_("ssm_scan_fwd");
    return fwd_impl(a, nullptr, stream);
}

int ssm_scan_ckpt_from_reference(const ssm_scan_fwd_args* a, const float* ref_ckpt, void* stream) {
    NvtxRange r_("ssm_scan_ckpt_from_reference");
    if (!ref_ckpt) return fail(SSM_ERR_INVALID, "ssm_scan_ckpt_from_reference: ref_ckpt is NULL");
    return fwd_impl(a, ref_ckpt, stream);
}

// Shape checks and CTA sizing of the backward; touches no device memory.
// Backward kernels, for d_state 16 without `length` when every stream is a TMA source/target:
// scan_bwd_pair_kernel (scan_bwd_pair.cu) with two channels per lane when the rows give it at
// least 32 warps per SM (rows >= 512 * SMs), else scan_bwd_split_kernel (scan_bwd_split.cu,
// two channels x two states per lane, twice the warps); scan_bwd_kernel for everything else.
// SSM_BWD_KERNEL=general forces the latter (for comparisons); SSM_BWD_PAIR_CPL (1: the pair
// kernel with one channel per lane, 2, 3: split) and SSM_BWD_PAIR_DT override the choice.
static bool bwd_pair_shape(const ssm_scan_bwd_args* a) {
    const char* e = getenv("SSM_BWD_KERNEL");
    if (e && strcmp(e, "general") == 0) return false;
    return a->dstate == 16 && a->length == nullptr;
}

// Channels per CTA of both backward kernels for these sizes: *dt for scan_bwd_kernel and
// *dt_pair / *cpl for scan_bwd_pair_kernel (dt_pair 0 when the shape does not take it).
// The workspace is sized for the smaller dt (more channel tiles), so it fits either kernel.
static int bwd_shape(const ssm_scan_bwd_args* a, int sms, StateSplit* sp, int* dt, int* dt_pair, int* cpl) {
    if (a->batch < 1 || a->dim < 1 || a->seqlen < 1 || a->dstate < 1)
        return fail(SSM_ERR_INVALID, "ssm_scan_bwd: sizes must be positive");
    if (a->dstate > 256) return fail(SSM_ERR_INVALID, "selective_scan only supports state_dim <= 256");
    if (a->seqlen > (1 << 30) || a->dim > (1 << 30) || a->batch > (1 << 30))
        return fail(SSM_ERR_INVALID, "ssm_scan_bwd: sizes too large");
    if (!valid_dtype(a->dtype)) return fail(SSM_ERR_INVALID, "ssm_scan_bwd: dtype must be SSM_F32 or SSM_BF16");
    *sp = scan_split(a->dstate, a->batch * a->dim, sms, "SSM_BWD_SPT");
    const int is_bf16 = a->dtype == SSM_BF16;
    const int has_z = a->z != nullptr;
    const StateSplit s = *sp;
    int dev = 0;
    cudaGetDevice(&dev);
    DtKey key;
    memset(&key, 0, sizeof(key));
    key.dev = dev; key.kind = 1; key.is_bf16 = is_bf16; key.lpc = s.lpc; key.spt = s.spt; key.dstate = (int)a->dstate;
    key.has_z = has_z; key.has_y = 0; key.batch = a->batch; key.dim = a->dim;
    *dt = cached_dt(key, sms, [&](int d) { return bwd_occupancy(is_bf16, s.lpc, s.spt, d, (int)a->dstate, has_z); });
    if (*dt < 1) return fail(SSM_ERR_INVALID, "ssm_scan_bwd: no CTA shape fits shared memory");
    *dt_pair = 0;
    *cpl = 1;
    if (bwd_pair_shape(a)) {
        // measured on B200: 20480 rows (4 x 5120): one channel per lane 1.07 ms, two 1.26 ms,
        // split 1.03 ms; 12288 rows (config 2): one 0.617 ms, split 0.596 ms; 163840 rows
        // (config 5 as 32 segments): one 13.6 ms, two 12.9 ms
        int c = (a->batch * a->dim >= (int64_t)512 * (sms > 0 ? sms : 148)) ? 2 : 3;
        if (const char* e = getenv("SSM_BWD_PAIR_CPL")) {
            const int v = atoi(e);
            if (v == 1 || v == 2 || v == 3) c = v;
        }
        // c = 3: scan_bwd_split_kernel (2 channels x 2 states per lane, 8 channels per warp)
        const int cw = c == 3 ? 1 : c;
        auto occ = [&](int dd) {
            return c == 3 ? bwd_split_occupancy(is_bf16, dd, has_z) : bwd_pair_occupancy(is_bf16, c, dd, has_z);
        };
        // 8 channels per warp per channel a lane holds: choose_dt's channel step for
        // 4 / c lanes per channel
        key.kind = c == 3 ? 6 : 5; key.lpc = 4 / cw; key.spt = 8;
        int d = cached_dt(key, sms, occ);
        if (const char* e = getenv("SSM_BWD_PAIR_DT")) {
            const int v = atoi(e);
            if (v >= 8 * cw && v * 4 / cw <= 128 && v % (8 * cw) == 0 && occ(v) > 0) d = v;
        }
        *dt_pair = d > 0 ? d : 0;
        *cpl = c;
    }
    return SSM_OK;
}

static int bwd_common(const ssm_scan_bwd_args* a, DevInfo** di, StateSplit* sp, int* dt, int* dt_pair, int* cpl) {
    int rc = device_info(di);
    if (rc) return rc;
    return bwd_shape(a, (*di)->sms, sp, dt, dt_pair, cpl);
}

static int ws_dt(int dt, int dt_pair) { return dt_pair > 0 && dt_pair < dt ? dt_pair : dt; }

struct WsLayout { size_t bc, a, dd, total; };

static WsLayout ws_layout(const ssm_scan_bwd_args* a, int dt) {
    WsLayout w;
    const int64_t ntile = (a->dim + dt - 1) / dt;
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    w.bc = 0;
    size_t o = al((size_t)ntile * a->batch * 2 * a->dstate * a->seqlen * sizeof(float));
    w.a = o;
    o += al((size_t)a->batch * a->dim * a->dstate * sizeof(float));
    w.dd = o;
    o += al((size_t)a->batch * a->dim * 2 * sizeof(float));
    w.total = o;
    return w;
}

size_t ssm_scan_bwd_workspace_size(const ssm_scan_bwd_args* a) {
    if (!a) return 0;
    DevInfo* di;
    StateSplit sp;
    int dt, dt_pair, cpl;
    if (bwd_common(a, &di, &sp, &dt, &dt_pair, &cpl)) return 0;
    return ws_layout(a, ws_dt(dt, dt_pair)).total;
}

}  // extern "C"

namespace ssm {

// Workspace bytes of the backward for these arguments on a device with `sms` SMs (0 on a
// shape error); touches no device memory.
size_t scan_bwd_workspace_bytes(const ssm_scan_bwd_args* a, int sms) {
    StateSplit sp;
    int dt, dt_pair, cpl;
    if (!a || bwd_shape(a, sms, &sp, &dt, &dt_pair, &cpl)) return 0;
    return ws_layout(a, ws_dt(dt, dt_pair)).total;
}

// The backward proper: validation, tensor maps and the two launches, with the caller's
// workspace and device error word.  Allocates nothing.
int scan_bwd_run(const ssm_scan_bwd_args* a, void* workspace, size_t ws_bytes, int* err_word, int sms,
                 void* stream_) {
    if (!a) return fail(SSM_ERR_INVALID, "ssm_scan_bwd: args is NULL");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    StateSplit sp;
    int dt, dt_pair, cpl;
    int rc = bwd_shape(a, sms, &sp, &dt, &dt_pair, &cpl);
    if (rc) return rc;
    if (!a->u || !a->delta || !a->A || !a->B || !a->C || !a->dout || !a->ckpt || !a->du ||
        !a->ddelta || !a->dA || !a->dB || !a->dC)
        return fail(SSM_ERR_INVALID, "ssm_scan_bwd: u, delta, A, B, C, dout, ckpt, du, ddelta, dA, dB, dC are required");
    if (a->z && (!a->y || !a->dz))
        return fail(SSM_ERR_INVALID, "ssm_scan_bwd: with z, the pre-gate output y and dz are required");
    if (a->ckpt_format != SSM_CKPT_COMPACT || a->ckpt_len != sp.k)
        return fail(SSM_ERR_INVALID, "ssm_scan_bwd: needs compact checkpoints every %d tokens (got format %d, len %lld)",
                    sp.k, (int)a->ckpt_format, (long long)a->ckpt_len);
    if (a->length && !a->reference_length_semantics)
        return fail(SSM_ERR_INVALID, "ssm_scan_bwd: `length` is only supported with the reference's semantics");
    const WsLayout w = ws_layout(a, ws_dt(dt, dt_pair));
    if (!workspace || ws_bytes < w.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return fail(SSM_ERR_WORKSPACE, "ssm_scan_bwd: workspace needs %zu bytes, 256-byte aligned", w.total);
    const int is_bf16 = a->dtype == SSM_BF16;
    const int64_t es = is_bf16 ? 2 : 4;
    unsigned char* ws = static_cast<unsigned char*>(workspace);

    BwdParams p;
    memset(&p, 0, sizeof(p));
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.seqlen = (int)a->seqlen; p.dstate = (int)a->dstate;
    p.dt = dt; p.ntile_d = (int)((a->dim + dt - 1) / dt);
    p.delta_softplus = a->delta_softplus; p.padding_right = a->padding_right;
    p.ref_len = a->length != nullptr;
    p.ckpt_format = a->ckpt_format; p.ckpt_len = (int)a->ckpt_len;
    p.nck = (int)ssm_scan_num_ckpt(a->seqlen, a->ckpt_len);
    p.u = a->u; p.u_sb = a->u_batch_stride; p.u_sd = a->u_dim_stride;
    p.delta = a->delta; p.delta_sb = a->delta_batch_stride; p.delta_sd = a->delta_dim_stride;
    p.A = a->A; p.A_sd = a->A_dim_stride;
    p.B = a->B; p.B_sb = a->B_batch_stride; p.B_sn = a->B_state_stride;
    p.C = a->C; p.C_sb = a->C_batch_stride; p.C_sn = a->C_state_stride;
    p.D = a->D; p.z = a->z; p.z_sb = a->z_batch_stride; p.z_sd = a->z_dim_stride;
    p.delta_bias = a->delta_bias; p.h_init = a->h_init; p.length = a->length;
    p.y = a->y; p.y_sb = a->y_batch_stride; p.y_sd = a->y_dim_stride;
    p.ckpt = a->ckpt;
    p.dout = a->dout; p.dout_sb = a->dout_batch_stride; p.dout_sd = a->dout_dim_stride;
    p.dh_last = a->dh_last;
    p.du = a->du; p.du_sb = a->du_batch_stride; p.du_sd = a->du_dim_stride;
    p.ddelta = a->ddelta; p.ddelta_sb = a->ddelta_batch_stride; p.ddelta_sd = a->ddelta_dim_stride;
    p.dz = a->dz; p.dz_sb = a->dz_batch_stride; p.dz_sd = a->dz_dim_stride;
    p.dh_init = a->h_init ? a->dh_init : nullptr;
    p.ws_bc = reinterpret_cast<float*>(ws + w.bc);
    p.ws_a = reinterpret_cast<float*>(ws + w.a);
    p.ws_dd = reinterpret_cast<float*>(ws + w.dd);
    p.err = err_word;

    p.use_tma = tma_ok(a->u, a->u_dim_stride, a->u_batch_stride, es) &&
                tma_ok(a->delta, a->delta_dim_stride, a->delta_batch_stride, es) &&
                tma_ok(a->dout, a->dout_dim_stride, a->dout_batch_stride, es) &&
                tma_ok(a->z, a->z_dim_stride, a->z_batch_stride, es) &&
                tma_ok(a->y, a->y_dim_stride, a->y_batch_stride, es) &&
                tma_ok(a->B, a->B_state_stride, a->B_batch_stride, es) &&
                tma_ok(a->C, a->C_state_stride, a->C_batch_stride, es) &&
                tma_ok(a->du, a->du_dim_stride, a->du_batch_stride, es) &&
                tma_ok(a->ddelta, a->ddelta_dim_stride, a->ddelta_batch_stride, es) &&
                tma_ok(a->dz, a->dz_dim_stride, a->dz_batch_stride, es);
    const bool pair = dt_pair > 0 && p.use_tma && (reinterpret_cast<uintptr_t>(a->ckpt) & 15u) == 0;
    if (pair) {
        dt = dt_pair;
        p.dt = dt;
        p.ntile_d = (int)((a->dim + dt - 1) / dt);
    }
    CUtensorMap maps[11];
    memset(maps, 0, sizeof(maps));
    if (p.use_tma) {
        if ((rc = get_encoder())) return rc;
        const int TB = kBwdTile;
        // the pair kernel stages each tile's two checkpoints by TMA: the compact checkpoints
        // (batch, nck, dim, 16) as a 4-D tensor, box (16 states, dt channels, 2 checkpoints)
        if (pair && (rc = encode4d_f32(&maps[10], a->ckpt, a->dstate, a->dim, p.nck, a->batch, a->dstate,
                                       a->dim * a->dstate, (int64_t)p.nck * a->dim * a->dstate, (int)a->dstate,
                                       dt, 2)))
            return rc;
        // output rows are TB * element bytes: 32 (bf16) or 64 (f32) bytes; the pair kernel with
        // two channels per lane loads its input tiles with the same swizzle (the others read
        // them unswizzled)
        const CUtensorMapSwizzle osw = is_bf16 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
        const CUtensorMapSwizzle none = (pair && cpl == 2) ? osw : CU_TENSOR_MAP_SWIZZLE_NONE;
        const int64_t L = a->seqlen, Dm = a->dim, Bs = a->batch, N = a->dstate;
        if ((rc = encode3d(&maps[0], a->u, is_bf16, L, Dm, Bs, a->u_dim_stride, a->u_batch_stride, TB, dt, none)) ||
            (rc = encode3d(&maps[1], a->delta, is_bf16, L, Dm, Bs, a->delta_dim_stride, a->delta_batch_stride, TB, dt, none)) ||
            (rc = encode3d(&maps[2], a->dout, is_bf16, L, Dm, Bs, a->dout_dim_stride, a->dout_batch_stride, TB, dt, none)) ||
            (rc = encode3d(&maps[3], a->z, is_bf16, L, Dm, Bs, a->z_dim_stride, a->z_batch_stride, TB, dt, none)) ||
            (rc = encode3d(&maps[4], a->y, is_bf16, L, Dm, Bs, a->y_dim_stride, a->y_batch_stride, TB, dt, none)) ||
            (rc = encode3d(&maps[5], a->B, is_bf16, L, N, Bs, a->B_state_stride, a->B_batch_stride, TB, (int)N, none)) ||
            (rc = encode3d(&maps[6], a->C, is_bf16, L, N, Bs, a->C_state_stride, a->C_batch_stride, TB, (int)N, none)) ||
            (rc = encode3d(&maps[7], a->du, is_bf16, L, Dm, Bs, a->du_dim_stride, a->du_batch_stride, TB, dt, osw)) ||
            (rc = encode3d(&maps[8], a->ddelta, is_bf16, L, Dm, Bs, a->ddelta_dim_stride, a->ddelta_batch_stride, TB, dt, osw)) ||
            (rc = encode3d(&maps[9], a->dz, is_bf16, L, Dm, Bs, a->dz_dim_stride, a->dz_batch_stride, TB, dt, osw)))
            return rc;
    }
    // the forward's failure-detection test hook (SSM_TEST_WITHHOLD_TMA), for the backward
    p.test_withhold = p.use_tma && getenv("SSM_TEST_WITHHOLD_TMA") != nullptr;
    cudaError_t e = !pair     ? launch_scan_bwd(p, is_bf16, sp.lpc, sp.spt, maps, stream)
                    : cpl == 3 ? launch_scan_bwd_split(p, is_bf16, maps, stream)
                               : launch_scan_bwd_pair(p, is_bf16, cpl, maps, stream);
    if (e != cudaSuccess) return cuda_fail(e, "scan_bwd launch");

    ReduceParams r;
    memset(&r, 0, sizeof(r));
    r.batch = p.batch; r.dim = p.dim; r.seqlen = p.seqlen; r.dstate = p.dstate; r.ntile_d = p.ntile_d;
    r.bc_dtype = is_bf16;
    r.ws_bc = p.ws_bc; r.ws_a = p.ws_a; r.ws_dd = p.ws_dd;
    r.dB = a->dB; r.dC = a->dC; r.dA = a->dA; r.dD = a->dD; r.ddelta_bias = a->ddelta_bias;
    const bool bc_default = a->dB_batch_stride == 0 && a->dB_state_stride == 0;
    const bool cc_default = a->dC_batch_stride == 0 && a->dC_state_stride == 0;
    r.dB_sb = bc_default ? a->dstate * a->seqlen : a->dB_batch_stride;
    r.dB_sn = bc_default ? a->seqlen : a->dB_state_stride;
    r.dC_sb = cc_default ? a->dstate * a->seqlen : a->dC_batch_stride;
    r.dC_sn = cc_default ? a->seqlen : a->dC_state_stride;
    e = launch_scan_reduce(r, stream);
    if (e != cudaSuccess) return cuda_fail(e, "scan_reduce launch");
    return SSM_OK;
}

void set_last_error(const char* msg) { g_err = msg; }

}  // namespace ssm

extern "C" {

int ssm_scan_bwd(const ssm_scan_bwd_args* a, void* workspace, size_t ws_bytes, void* stream) {
    NvtxRange r_("ssm_scan_bwd");
    if (!a) return fail(SSM_ERR_INVALID, "ssm_scan_bwd: args is NULL");
    DevInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc) return rc;
    return scan_bwd_run(a, workspace, ws_bytes, di->err, di->sms, stream);
}

int ssm_state_update(const ssm_state_update_args* a, void* stream_) {
    NvtxRange r_("ssm_state_update");
    if (!a) return fail(SSM_ERR_INVALID, "ssm_state_update: args is NULL");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (a->batch < 1 || a->dim < 1 || a->dstate < 1)
        return fail(SSM_ERR_INVALID, "ssm_state_update: sizes must be positive");
    if (a->dstate > 256) return fail(SSM_ERR_INVALID, "selective_update only supports state_dim <= 256");
    if (!valid_dtype(a->dtype)) return fail(SSM_ERR_INVALID, "ssm_state_update: dtype must be SSM_F32 or SSM_BF16");
    if (!a->state || !a->state_out || !a->x || !a->dt || !a->A || !a->B || !a->C || !a->out)
        return fail(SSM_ERR_INVALID, "ssm_state_update: state, state_out, x, dt, A, B, C and out are required");
    const StateSplit sp = decode_split(a->dstate);
    if (a->batch > (1 << 30) || (a->dim + (256 / sp.lpc) - 1) / (256 / sp.lpc) > 65535)
        return fail(SSM_ERR_INVALID, "ssm_state_update: dim must be <= 65535 * %d", 256 / sp.lpc);
    UpdParams p;
    memset(&p, 0, sizeof(p));
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.dstate = (int)a->dstate;
    p.dt_softplus = a->dt_softplus;
    p.state = a->state; p.st_sb = a->state_batch_stride; p.st_sd = a->state_dim_stride;
    p.state_out = a->state_out; p.so_sb = a->state_out_batch_stride; p.so_sd = a->state_out_dim_stride;
    p.x = a->x; p.x_sb = a->x_batch_stride;
    p.dtv = a->dt; p.dt_sb = a->dt_batch_stride;
    p.A = a->A; p.A_sd = a->A_dim_stride;
    p.B = a->B; p.B_sb = a->B_batch_stride;
    p.C = a->C; p.C_sb = a->C_batch_stride;
    p.D = a->D; p.z = a->z; p.z_sb = a->z_batch_stride;
    p.dt_bias = a->dt_bias;
    p.out = a->out; p.out_sb = a->out_batch_stride;
    p.pdl = (a->launch_flags & SSM_LAUNCH_PDL) != 0;
    // Streamed kernel (bulk-copy pipeline over persistent CTAs) for contiguous, 16-byte
    // aligned layouts with dstate 8, 16 or 32 and dim a multiple of its channel tile.
    // Measured on B200 at batch 64 x 5120 x 16 (CUDA graph, 8 rotating states): bf16
    // 9.4-9.5 us/step streamed vs 11.8-12.0 per-CTA; float32 10.2-10.3 vs 10.5-10.7.
    // SSM_DEC_STREAM=0 turns it off.
    {
        const int64_t N = a->dstate, es = a->dtype == SSM_BF16 ? 2 : 4;
        const int lpc = (int)(N / 8), rpb = lpc > 0 ? 256 / lpc : 0;
        auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
        const char* env = getenv("SSM_DEC_STREAM");
        const bool want = !(env && env[0] == '0');
        const bool ok = (N == 8 || N == 16 || N == 32) && a->dim % rpb == 0 && want &&
                        a->state_dim_stride == N && a->state_out_dim_stride == N && a->A_dim_stride == N &&
                        ((a->state_batch_stride * 4) & 15) == 0 && ((a->state_out_batch_stride * 4) & 15) == 0 &&
                        ((a->x_batch_stride * es) & 15) == 0 && ((a->dt_batch_stride * es) & 15) == 0 &&
                        (!a->z || ((a->z_batch_stride * es) & 15) == 0) && ((a->B_batch_stride * es) & 15) == 0 &&
                        ((a->C_batch_stride * es) & 15) == 0 && al(a->state) && al(a->state_out) && al(a->A) &&
                        al(a->x) && al(a->dt) && (!a->z || al(a->z)) && al(a->B) && al(a->C) &&
                        (!a->dt_bias || al(a->dt_bias)) && (!a->D || al(a->D));
        if (ok) {
            DevInfo* di = nullptr;
            int rc = device_info(&di);
            if (rc) return rc;
            p.err = di->err;
            cudaError_t e = launch_state_update_stream(p, a->dtype == SSM_BF16, lpc, di->sms, stream);
            if (e != cudaSuccess) return cuda_fail(e, "state_update_stream launch");
            return SSM_OK;
        }
    }
    cudaError_t e = launch_state_update(p, a->dtype == SSM_BF16, sp.lpc, sp.spt, stream);
    if (e != cudaSuccess) return cuda_fail(e, "state_update launch");
    return SSM_OK;
}

// ---- sequence slices ------------------------------------------------------------------------
// Shared launch path of the two chunk-state kernels.  x0 = u (forward) or dout (reverse);
// bc = B (forward) or C (reverse); z only in reverse.
static int chunk_impl(const char* name, int reverse, int64_t batch, int64_t dim, int64_t seqlen, int64_t dstate,
                      int32_t dtype, int32_t softplus, const void* x0, int64_t x0_sb, int64_t x0_sd,
                      const void* delta, int64_t delta_sb, int64_t delta_sd, const void* z, int64_t z_sb,
                      int64_t z_sd, const void* bc, int64_t bc_sb, int64_t bc_sn, const float* A, int64_t A_sd,
                      const float* delta_bias, float* carry, float* delta_sum, cudaStream_t stream) {
    if (batch < 1 || dim < 1 || seqlen < 1 || dstate < 1)
        return fail(SSM_ERR_INVALID, "%s: sizes must be positive", name);
    if (dstate > 256) return fail(SSM_ERR_INVALID, "selective_scan only supports state_dim <= 256");
    if (seqlen > (1 << 30) || dim > (1 << 30) || batch > (1 << 30))
        return fail(SSM_ERR_INVALID, "%s: sizes too large", name);
    if (!valid_dtype(dtype)) return fail(SSM_ERR_INVALID, "%s: dtype must be SSM_F32 or SSM_BF16", name);
    if (!x0 || !delta || !bc || !A || !carry)
        return fail(SSM_ERR_INVALID, "%s: a required pointer is NULL", name);
    const int is_bf16 = dtype == SSM_BF16;
    const int64_t es = is_bf16 ? 2 : 4;
    DevInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc) return rc;
    const StateSplit sp = scan_split(dstate, batch * dim, di->sms, "SSM_FWD_SPT");
    const int has_z = z != nullptr;
    ChunkParams p;
    memset(&p, 0, sizeof(p));
    p.batch = (int)batch; p.dim = (int)dim; p.seqlen = (int)seqlen; p.dstate = (int)dstate;
    p.delta_softplus = softplus;
    p.x0 = x0; p.x0_sb = x0_sb; p.x0_sd = x0_sd;
    p.delta = delta; p.delta_sb = delta_sb; p.delta_sd = delta_sd;
    p.z = z; p.z_sb = z_sb; p.z_sd = z_sd;
    p.bc = bc; p.bc_sb = bc_sb; p.bc_sn = bc_sn;
    p.A = A; p.A_sd = A_sd; p.delta_bias = delta_bias;
    p.carry = carry; p.delta_sum = delta_sum; p.err = di->err;
    int dev = 0;
    cudaGetDevice(&dev);
    DtKey key;
    memset(&key, 0, sizeof(key));
    key.dev = dev; key.kind = 2 + reverse; key.is_bf16 = is_bf16; key.lpc = sp.lpc; key.spt = sp.spt;
    key.has_z = has_z; key.batch = batch; key.dim = dim;
    p.dt = cached_dt(key, di->sms, [&](int dt) { return chunk_occupancy(is_bf16, sp.lpc, sp.spt, reverse, dt, has_z); });
    if (p.dt < 1) return fail(SSM_ERR_INVALID, "%s: no CTA shape fits shared memory", name);
    p.ntile_d = (int)((dim + p.dt - 1) / p.dt);
    p.use_tma = tma_ok(x0, x0_sd, x0_sb, es) && tma_ok(delta, delta_sd, delta_sb, es) &&
                tma_ok(z, z_sd, z_sb, es) && tma_ok(bc, bc_sn, bc_sb, es);
    CUtensorMap maps[4];
    memset(maps, 0, sizeof(maps));
    if (p.use_tma) {
        if ((rc = get_encoder())) return rc;
        const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
        const int T = (int)(128 / es);
        if ((rc = encode3d(&maps[0], x0, is_bf16, seqlen, dim, batch, x0_sd, x0_sb, T, p.dt, sw)) ||
            (rc = encode3d(&maps[1], delta, is_bf16, seqlen, dim, batch, delta_sd, delta_sb, T, p.dt, sw)) ||
            (rc = encode3d(&maps[2], z, is_bf16, seqlen, dim, batch, z_sd, z_sb, T, p.dt, sw)) ||
            (rc = encode3d(&maps[3], bc, is_bf16, seqlen, dstate, batch, bc_sn, bc_sb, T, (int)dstate, sw)))
            return rc;
    }
    cudaError_t e = launch_scan_chunk(p, is_bf16, sp.lpc, sp.spt, reverse, maps, stream);
    if (e != cudaSuccess) return cuda_fail(e, "scan_chunk launch");
    return SSM_OK;
}

int ssm_scan_chunk_state_fwd(const ssm_scan_fwd_args* a, float* h_end, float* delta_sum, void* stream) {
    NvtxRange r_("ssm_scan_chunk_state_fwd");
    if (!a) return fail(SSM_ERR_INVALID, "ssm_scan_chunk_state_fwd: args is NULL");
    if (a->out || a->y || a->ckpt || a->h_init || a->h_last || a->length)
        return fail(SSM_ERR_INVALID, "ssm_scan_chunk_state_fwd: out, y, ckpt, h_init, h_last and length must be NULL");
    if (!h_end || !delta_sum) return fail(SSM_ERR_INVALID, "ssm_scan_chunk_state_fwd: h_end and delta_sum are required");
    return chunk_impl("ssm_scan_chunk_state_fwd", 0, a->batch, a->dim, a->seqlen, a->dstate, a->dtype,
                      a->delta_softplus, a->u, a->u_batch_stride, a->u_dim_stride, a->delta,
                      a->delta_batch_stride, a->delta_dim_stride, nullptr, 0, 0, a->B, a->B_batch_stride,
                      a->B_state_stride, a->A, a->A_dim_stride, a->delta_bias, h_end, delta_sum,
                      static_cast<cudaStream_t>(stream));
}

int ssm_scan_chunk_state_bwd(const ssm_scan_bwd_args* a, float* g_start, void* stream) {
    NvtxRange r_("ssm_scan_chunk_state_bwd");
    if (!a) return fail(SSM_ERR_INVALID, "ssm_scan_chunk_state_bwd: args is NULL");
    if (a->length) return fail(SSM_ERR_INVALID, "ssm_scan_chunk_state_bwd: length must be NULL");
    if (!g_start) return fail(SSM_ERR_INVALID, "ssm_scan_chunk_state_bwd: g_start is required");
    return chunk_impl("ssm_scan_chunk_state_bwd", 1, a->batch, a->dim, a->seqlen, a->dstate, a->dtype,
                      a->delta_softplus, a->dout, a->dout_batch_stride, a->dout_dim_stride, a->delta,
                      a->delta_batch_stride, a->delta_dim_stride, a->z, a->z_batch_stride, a->z_dim_stride, a->C,
                      a->C_batch_stride, a->C_state_stride, a->A, a->A_dim_stride, a->delta_bias, g_start, nullptr,
                      static_cast<cudaStream_t>(stream));
}

int ssm_scan_carry_compose(const ssm_carry_args* a, void* stream) {
    NvtxRange r_("ssm_scan_carry_compose");
    if (!a) return fail(SSM_ERR_INVALID, "ssm_scan_carry_compose: args is NULL");
    if (a->batch < 1 || a->dim < 1 || a->dstate < 1 || a->nslices < 1 || a->nslices > (1 << 20))
        return fail(SSM_ERR_INVALID, "ssm_scan_carry_compose: sizes must be positive");
    if (a->batch * a->dim * a->dstate >= (int64_t(1) << 40))
        return fail(SSM_ERR_INVALID, "ssm_scan_carry_compose: sizes too large");
    if (!a->A || !a->carry || !a->delta_sum || !a->result)
        return fail(SSM_ERR_INVALID, "ssm_scan_carry_compose: A, carry, delta_sum and result are required");
    if (a->start && a->nstart < 1) return fail(SSM_ERR_INVALID, "ssm_scan_carry_compose: nstart must be >= 1 with start");
    CarryParams p;
    memset(&p, 0, sizeof(p));
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.dstate = (int)a->dstate; p.nslices = (int)a->nslices;
    p.reverse = a->reverse != 0;
    p.A = a->A; p.A_sd = a->A_dim_stride;
    p.carry = a->carry; p.carry_ss = a->carry_slice_stride;
    p.delta_sum = a->delta_sum; p.dsum_ss = a->delta_sum_slice_stride;
    p.start = a->start; p.start_ss = a->start_stride; p.nstart = a->start ? a->nstart : 0;
    p.result = a->result;
    cudaError_t e = launch_carry_compose(p, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "carry_compose launch");
    return SSM_OK;
}

// ---- causal depthwise conv1d -------------------------------------------------------------------
static int conv_common(const char* name, const ssm_conv1d_args* a, bool seq, bool need_out = true) {
    if (!a) return fail(SSM_ERR_INVALID, "%s: args is NULL", name);
    if (a->batch < 1 || a->dim < 1 || (seq && a->seqlen < 1))
        return fail(SSM_ERR_INVALID, "%s: sizes must be positive", name);
    if (a->batch > (1 << 30) || a->dim > (1 << 30) || a->seqlen > (1 << 30))
        return fail(SSM_ERR_INVALID, "%s: sizes too large", name);
    if (a->batch * a->dim >= (int64_t(1) << 31) || a->seqlen > (int64_t)65535 * 32)
        return fail(SSM_ERR_INVALID, "%s: batch * dim must be < 2^31 and seqlen <= 2097120", name);
    if (a->width < 2 || a->width > 4) return fail(SSM_ERR_INVALID, "%s: width must be 2, 3 or 4", name);
    if (!valid_dtype(a->dtype)) return fail(SSM_ERR_INVALID, "%s: dtype must be SSM_F32 or SSM_BF16", name);
    if (!a->x || !a->weight || (need_out && !a->out))
        return fail(SSM_ERR_INVALID, "%s: x, weight%s are required", name, need_out ? " and out" : "");
    return SSM_OK;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 16-byte vectors along the sequence: every row start 16-byte aligned and seqlen a multiple
// of the vector
static bool conv_vec_ok(const ssm_conv1d_args* a, bool bwd) {
    const int64_t es = a->dtype == SSM_BF16 ? 2 : 4, vt = 16 / es;
    auto ok = [&](const void* p, int64_t sb, int64_t sd) {
        return p == nullptr || (aligned16(p) && ((sb * es) & 15) == 0 && ((sd * es) & 15) == 0);
    };
    return (a->seqlen % vt) == 0 && ok(a->x, a->x_batch_stride, a->x_dim_stride) &&
           ok(a->out, a->out_batch_stride, a->out_dim_stride) &&
           (!bwd || (ok(a->dout, a->dout_batch_stride, a->dout_dim_stride) &&
                     ok(a->dx, a->dx_batch_stride, a->dx_dim_stride)));
}

static ConvParams conv_params(const ssm_conv1d_args* a) {
    ConvParams p;
    memset(&p, 0, sizeof(p));
    p.batch = (int)a->batch; p.dim = (int)a->dim; p.seqlen = (int)a->seqlen; p.silu = a->silu;
    p.x = a->x; p.x_sb = a->x_batch_stride; p.x_sd = a->x_dim_stride;
    p.w = a->weight; p.w_sd = a->weight_dim_stride; p.bias = a->bias;
    p.out = a->out; p.out_sb = a->out_batch_stride; p.out_sd = a->out_dim_stride;
    p.length = a->length;
    p.state = a->state; p.st_sb = a->state_batch_stride; p.st_sd = a->state_dim_stride;
    p.dout = a->dout; p.dout_sb = a->dout_batch_stride; p.dout_sd = a->dout_dim_stride;
    p.dx = a->dx; p.dx_sb = a->dx_batch_stride; p.dx_sd = a->dx_dim_stride;
    return p;
}

// chunks of 32 lanes x 4 vectors along a row (kConvRows in conv1d.cu)
static int conv_nchunk(const ssm_conv1d_args* a, bool vec) {
    const int64_t vt = vec ? (a->dtype == SSM_BF16 ? 8 : 4) : 1;
    const int64_t nvec = (a->seqlen + vt - 1) / vt;
    return (int)((nvec + 127) / 128);
}

int ssm_conv1d_fwd(const ssm_conv1d_args* a, void* stream) {
    NvtxRange r_("ssm_conv1d_fwd");
    int rc = conv_common("ssm_conv1d_fwd", a, true);
    if (rc) return rc;
    DevInfo* di = nullptr;
    if ((rc = device_info(&di))) return rc;
    const bool vec = conv_vec_ok(a, false);
    ConvParams p = conv_params(a);
    p.dout = nullptr; p.dx = nullptr;
    p.nchunk = conv_nchunk(a, vec);
    cudaError_t e = launch_conv1d(p, a->dtype == SSM_BF16, (int)a->width, 0, vec, di->sms,
                                  static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "conv1d_fwd launch");
    return SSM_OK;
}

size_t ssm_conv1d_bwd_workspace_size(const ssm_conv1d_args* a) {
    if (conv_common("ssm_conv1d_bwd", a, true, false)) return 0;
    const bool vec = conv_vec_ok(a, true);
    return (size_t)conv_nchunk(a, vec) * a->batch * a->dim * (a->width + 1) * sizeof(float);
}

int ssm_conv1d_bwd(const ssm_conv1d_args* a, void* workspace, size_t ws_bytes, void* stream) {
    NvtxRange r_("ssm_conv1d_bwd");
    int rc = conv_common("ssm_conv1d_bwd", a, true, false);
    if (rc) return rc;
    if (!a->dout || !a->dx || !a->dweight)
        return fail(SSM_ERR_INVALID, "ssm_conv1d_bwd: dout, dx and dweight are required");
    const bool vec = conv_vec_ok(a, true);
    const size_t need = (size_t)conv_nchunk(a, vec) * a->batch * a->dim * (a->width + 1) * sizeof(float);
    if (!workspace || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u))
        return fail(SSM_ERR_WORKSPACE, "ssm_conv1d_bwd: workspace needs %zu bytes, 16-byte aligned", need);
    DevInfo* di = nullptr;
    if ((rc = device_info(&di))) return rc;
    ConvParams p = conv_params(a);
    p.state = nullptr;
    p.nchunk = conv_nchunk(a, vec);
    p.ws = static_cast<float*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = launch_conv1d(p, a->dtype == SSM_BF16, (int)a->width, 1, vec, di->sms, s);
    if (e != cudaSuccess) return cuda_fail(e, "conv1d_bwd launch");
    e = launch_conv1d_reduce(p.ws, p.nchunk * p.batch, p.dim, (int)a->width, a->dweight, a->dweight_dim_stride,
                             a->dbias, di->sms, s);
    if (e != cudaSuccess) return cuda_fail(e, "conv1d_reduce launch");
    return SSM_OK;
}

int ssm_conv1d_update(const ssm_conv1d_args* a, void* stream) {
    NvtxRange r_("ssm_conv1d_update");
    int rc = conv_common("ssm_conv1d_update", a, false);
    if (rc) return rc;
    if (!a->state) return fail(SSM_ERR_INVALID, "ssm_conv1d_update: state is required");
    DevInfo* di = nullptr;
    if ((rc = device_info(&di))) return rc;
    ConvParams p = conv_params(a);
    cudaError_t e = launch_conv1d_update(p, a->dtype == SSM_BF16, (int)a->width, di->sms,
                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "conv1d_update launch");
    return SSM_OK;
}

int ssm_exp2_compare(const float* x, float* y_fma, float* y_mufu, int64_t n, void* stream) {
    NvtxRange r_("ssm_exp2_compare");
    if (!x || !y_fma || !y_mufu || n < 1 || n > ((int64_t)1 << 31))
        return fail(SSM_ERR_INVALID, "ssm_exp2_compare: x, y_fma, y_mufu must be non-NULL and 1 <= n <= 2^31");
    DevInfo* di = nullptr;
    int rc = device_info(&di);
    if (rc) return rc;
    cudaError_t e = launch_exp2_compare(x, y_fma, y_mufu, n, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "exp2_compare launch");
    return SSM_OK;
}

int ssm_check_device_error(int* code, void* stream_) {
    // two words can hold a code: the library's per-device word (every entry point but
    // ssm_scan_bwd_noalloc) and the one at the end of ssm_scan_bwd_noalloc's static
    // scratch; both are read, and a word that holds a code is cleared.  Allocates nothing.
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    int* words[2] = {nullptr, ssm::noalloc_error_word()};
    if (DevInfo* di = device_info_if_ready()) words[0] = di->err;
    int v[2] = {0, 0};
    for (int i = 0; i < 2; i++) {
        if (!words[i]) continue;
        cudaError_t e = cudaMemcpyAsync(&v[i], words[i], sizeof(int), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e, "ssm_check_device_error");
        if (v[i] != 0) {
            e = cudaMemsetAsync(words[i], 0, sizeof(int), stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return cuda_fail(e, "ssm_check_device_error (clear)");
        }
    }
    const int c = v[0] != 0 ? v[0] : v[1];
    if (code) *code = c;
    if (c != 0) return fail(SSM_ERR_DEVICE, "a kernel reported device error %d", c);
    return SSM_OK;
}

}  // extern "C"
